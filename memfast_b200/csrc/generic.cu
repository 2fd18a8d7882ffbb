// Generic SIMT engine for the sliced product: every configuration, every mode.
//
//   ideal_kernel     ideal devices whose ADC counts are exact integer digit dots
//                    (reference.py:81-115 with V and G reduced to digits): digit
//                    planes staged in shared memory 4 rows per word, dp4a dots,
//                    min(dot, adc_max) counts, signed reconstruction in registers.
//   restore_kernel   per-cell conductances with write variation, drift, stuck-at
//                    faults and shared read variation (reference.py:10-51).
//   physical_kernel  explicit FP32/FP64 currents in ascending row order with
//                    voltage noise, slice-pair and output read modes and the
//                    S-shaped ADC (reference.py:63-117).
// Both product kernels end in the same fused epilogue: per read, the reconstructed
// total is scaled fl(fl(T*xs)*ws) (or restore_scales in FP64, simulator.py:57-66)
// and summed over reads in PyTorch's CPU cascade order (simulator.py:585), so
// partials never leave registers.
#include "common.cuh"
#include "kernels.cuh"

namespace mf {

namespace {

constexpr int IDEAL_TV = 32;      // vectors per CTA
constexpr int IDEAL_TC = 64;      // output columns per CTA
constexpr int PHYS_TV = 16;
constexpr int PHYS_TC = 64;
constexpr int PHYS_RCH = 32;      // rows staged per chunk
constexpr int ST_TV = 32;         // staged physical kernel: vectors per CTA (2 per thread)
constexpr int ST_TC = 64;         // staged physical kernel: output columns per CTA (4 per thread)
constexpr size_t ST_SMEM_MAX = 200 * 1024;
constexpr int THREADS = 256;

template <typename OutT, typename ScaleT, typename TotT>
__device__ __forceinline__ OutT scaled_partial(TotT total, ScaleT xs, ScaleT ws);

template <>
__device__ __forceinline__ float scaled_partial<float, float, long long>(long long t, float xs, float ws) {
    return __fmul_rn(__fmul_rn(__ll2float_rn(t), xs), ws);
}
template <>
__device__ __forceinline__ float scaled_partial<float, float, int>(int t, float xs, float ws) {
    return __fmul_rn(__fmul_rn(__int2float_rn(t), xs), ws);
}
template <>
__device__ __forceinline__ double scaled_partial<double, double, long long>(long long t, double xs, double ws) {
    return restore_scales(__ll2double_rn(t), xs, ws);
}
template <>
__device__ __forceinline__ double scaled_partial<double, double, int>(int t, double xs, double ws) {
    return restore_scales((double)t, xs, ws);
}
// Non-finite FP32 rerun of a narrow config: partials were FP32 (reference.py:116-117).
template <>
__device__ __forceinline__ double scaled_partial<double, float, long long>(long long t, float xs, float ws) {
    return restore_scales((double)__ll2float_rn(t), (double)xs, (double)ws);
}
template <>
__device__ __forceinline__ double scaled_partial<double, float, int>(int t, float xs, float ws) {
    return restore_scales((double)__int2float_rn(t), (double)xs, (double)ws);
}

template <typename CodeT>
__device__ __forceinline__ uint32_t digit_of(CodeT code, int shift, int mask) {
    return (uint32_t)(((long long)code >> shift) & mask);
}

// Restricts a launch to the output tiles a tensor-core kernel flagged for an
// exact rerun: flags[(col - tile_begin * C) / cols][row / rows] != 0.  A null
// `flags` runs every tile.
struct TileFilter {
    const unsigned* flags;
    int rows, cols, row_tiles, col_tiles;
};

// ------------------------------------------------------------ ideal kernel --
template <typename CodeT, typename TotT, typename OutT, typename ScaleT>
__global__ void __launch_bounds__(THREADS) ideal_kernel(Layout L, MMArgs a, int power, long long full,
                                                        TileFilter filter, int grid_x, int grid_y) {
    extern __shared__ __align__(16) uint32_t smem[];
    const int R4 = (L.rows + 3) >> 2;
    uint32_t* sA = smem;                               // [n_in][32][R4]
    uint32_t* sW = smem + L.n_in * IDEAL_TV * R4;      // [n_w][R4][64]
    const CodeT* codes = static_cast<const CodeT*>(a.codes);
    const CodeT* packed = static_cast<const CodeT*>(a.packed);
    const ScaleT* xscale = static_cast<const ScaleT*>(a.xscale);
    const ScaleT* wscale = static_cast<const ScaleT*>(a.wscale);
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    const long long col_end = (long long)a.tile_end * L.C;
    const int MR = a.m * L.reads;
    const long long row_stride = (long long)a.m * L.R;
    // Work items: for a full launch the blocks of the (grid_x x grid_y) grid, one per
    // CTA; for a filtered launch the filter's tiles, over which a few CTAs step, each
    // running the blocks of a flagged tile and skipping the others after one flag read.
    const int sub_x = filter.flags ? filter.rows / IDEAL_TV : 1;
    const int sub_y = filter.flags ? filter.cols / IDEAL_TC : 1;
    const long long items = filter.flags ? (long long)filter.row_tiles * filter.col_tiles : (long long)grid_x * grid_y;
    for (long long item = blockIdx.x + (long long)blockIdx.y * gridDim.x; item < items;
         item += (long long)gridDim.x * gridDim.y) {
        long long bx0 = item % grid_x, by0 = item / grid_x;
        if (filter.flags) {
            if (!filter.flags[item]) continue;   // uniform across the CTA
            bx0 = (item % filter.row_tiles) * sub_x;
            by0 = (item / filter.row_tiles) * sub_y;
        }
        for (int sb = 0; sb < sub_x * sub_y; ++sb) {
            const long long bx = bx0 + sb % sub_x, by = by0 + sb / sub_x;
            if (bx >= grid_x || by >= grid_y) continue;
            const long long v0 = bx * IDEAL_TV;
            const long long col0 = (long long)a.tile_begin * L.C + by * IDEAL_TC;

            Cascade<OutT> acc[2][4];
#pragma unroll
            for (int e = 0; e < 2; ++e)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[e][j].init();

            for (int i = 0; i < MR; ++i) {
                const int arr = i / L.reads, g = i % L.reads;
                const int r0 = g * L.rows;
                const int len = L.rows < L.R - r0 ? L.rows : L.R - r0;
                __syncthreads();
                for (int idx = tid; idx < L.n_in * IDEAL_TV * R4; idx += THREADS) {
                    const int r4 = idx % R4, v = (idx / R4) % IDEAL_TV, s = idx / (R4 * IDEAL_TV);
                    const long long vec = v0 + v;
                    uint32_t word = 0;
                    if (vec < a.n) {
                        const CodeT* row = codes + vec * row_stride + (long long)arr * L.R + r0;
#pragma unroll
                        for (int b = 0; b < 4; ++b) {
                            const int r = 4 * r4 + b;
                            if (r < len) word |= digit_of(row[r], L.in_shift[s], L.in_mask[s]) << (8 * b);
                        }
                    }
                    sA[(s * IDEAL_TV + v) * R4 + r4] = word;
                }
                for (int idx = tid; idx < L.n_w * R4 * IDEAL_TC; idx += THREADS) {
                    const int c = idx % IDEAL_TC, r4 = (idx / IDEAL_TC) % R4, s = idx / (IDEAL_TC * R4);
                    const long long col = col0 + c;
                    uint32_t word = 0;
                    if (col < col_end) {
                        const long long t = col / L.C, cc = col % L.C;
                        const CodeT* base = packed + (((long long)arr * a.p + t) * L.R + r0) * L.C + cc;
#pragma unroll
                        for (int b = 0; b < 4; ++b) {
                            const int r = 4 * r4 + b;
                            if (r < len) word |= digit_of(base[(long long)r * L.C], L.w_shift[s], L.w_mask[s]) << (8 * b);
                        }
                    }
                    sW[(s * R4 + r4) * IDEAL_TC + c] = word;
                }
                __syncthreads();

                TotT total[2][4];
#pragma unroll
                for (int e = 0; e < 2; ++e)
#pragma unroll
                    for (int j = 0; j < 4; ++j) total[e][j] = 0;
                for (int sa = 0; sa < L.n_in; ++sa) {
                    const uint32_t* pa0 = sA + (sa * IDEAL_TV + ty) * R4;
                    const uint32_t* pa1 = pa0 + 16 * R4;
                    for (int sw = 0; sw < L.n_w; ++sw) {
                        const uint32_t* pw = sW + sw * R4 * IDEAL_TC + 4 * tx;
                        uint32_t dot[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
                        for (int r4 = 0; r4 < R4; ++r4) {
                            const uint32_t x0 = pa0[r4], x1 = pa1[r4];
                            const uint4 wv = *reinterpret_cast<const uint4*>(pw + r4 * IDEAL_TC);
                            dot[0][0] = __dp4a(x0, wv.x, dot[0][0]);
                            dot[0][1] = __dp4a(x0, wv.y, dot[0][1]);
                            dot[0][2] = __dp4a(x0, wv.z, dot[0][2]);
                            dot[0][3] = __dp4a(x0, wv.w, dot[0][3]);
                            dot[1][0] = __dp4a(x1, wv.x, dot[1][0]);
                            dot[1][1] = __dp4a(x1, wv.y, dot[1][1]);
                            dot[1][2] = __dp4a(x1, wv.z, dot[1][2]);
                            dot[1][3] = __dp4a(x1, wv.w, dot[1][3]);
                        }
                        const uint32_t maxw = (uint32_t)L.adc_max[sw];
                        const TotT factor = (TotT)(L.in_factor[sa] * L.w_factor[sw]);
#pragma unroll
                        for (int e = 0; e < 2; ++e)
#pragma unroll
                            for (int j = 0; j < 4; ++j)
                                total[e][j] += (TotT)(dot[e][j] < maxw ? dot[e][j] : maxw) * factor;
                    }
                }
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const long long vec = v0 + ty + 16 * e;
                    if (vec >= a.n) continue;
                    const ScaleT xs = xscale[vec * MR + i];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const long long col = col0 + 4 * tx + j;
                        if (col >= col_end) continue;
                        const long long t = col / L.C, cc = col % L.C;
                        const ScaleT ws = wscale[((long long)i * a.p + t) * L.C + cc];
                        cascade_push(acc[e][j], scaled_partial<OutT, ScaleT, TotT>(total[e][j], xs, ws), i, power, full);
                    }
                }
            }
            OutT* out = static_cast<OutT*>(a.out);
            const ScaleT* bias = static_cast<const ScaleT*>(a.bias);
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const long long vec = v0 + ty + 16 * e;
                if (vec >= a.n) continue;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const long long col = col0 + 4 * tx + j;
                    if (col >= col_end || col >= a.out_features) continue;
                    OutT value = cascade_finish(acc[e][j]);
                    if (bias) value = add_rn(value, (OutT)bias[col]);
                    out[vec * a.ldo + col] = value;
                    // Peer outputs of a row-sharded product (the packed kernel's exact rerun).
                    for (int g = 0; g < a.n_peers; ++g) static_cast<OutT*>(a.peer_out[g])[vec * a.ldo + col] = value;
                }
            }
            if (a.n_peers) __threadfence_system();
        }
    }
}

// ---------------------------------------------------------- restore kernel --
template <typename CurT>
__global__ void restore_kernel(Layout L, Physics P, const void* packed_raw, int wide_codes, int m,
                               int p, int begin, int width, uint32_t seed, uint64_t event, CurT* g) {
    const long long cells = (long long)m * width * L.n_w * L.R * L.C;
    const uint64_t read_seed = event_seed(seed, event);
    for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < cells;
         idx += (long long)gridDim.x * blockDim.x) {
        long long rest = idx;
        const int c = rest % L.C; rest /= L.C;
        const int r = rest % L.R; rest /= L.R;
        const int w = rest % L.n_w; rest /= L.n_w;
        const int tw = rest % width;
        const int arr = (int)(rest / width);
        const int tile = begin + tw;
        const long long address = ((((long long)arr * p + tile) * L.n_w + w) * L.R + r) * L.C + c;
        const long long pi = (((long long)arr * p + tile) * L.R + r) * L.C + c;
        const long long code = wide_codes ? static_cast<const long long*>(packed_raw)[pi]
                                          : (long long)static_cast<const uint8_t*>(packed_raw)[pi];
        const long long state = (code >> L.w_shift[w]) & L.w_mask[w];
        CurT raw;
        if (sizeof(CurT) == 4) {
            raw = (CurT)restored_conductance_f32(P, state, L.w_mask[w], address, seed, read_seed);
        } else {
            double d;
            if (L.w_mask[w] == 1) d = state ? P.high : P.low;
            else d = __dadd_rn(P.low, __dmul_rn(P.span, __ddiv_rn((double)state, (double)L.w_mask[w])));
            if (P.write_var != 0)
                d = __dmul_rn(d, (double)expf(__fmul_rn((float)P.write_var, rng_normal(address, seed, 10))));
            d = __dmul_rn(d, P.drift);
            if (P.saf_cut != 0) {
                const float u = rng_uniform(address, seed, 30);
                const float lo = (float)P.saf_low, hi = (float)P.saf_cut;
                if (u < lo) d = P.low;
                if (u >= lo && u < hi) d = P.high;
            }
            if (P.read_mode == 0 && P.read_var != 0)
                d = __dmul_rn(d, (double)expf(__fmul_rn((float)P.read_var, rng_normal(address, read_seed, 20))));
            raw = (CurT)d;
        }
        g[idx] = raw;
    }
}

// ------------------------------------------------------------ ADC counts --
__device__ __forceinline__ long long adc_count(float current, int maxw, float amw, const Physics& P) {
    float value = __fmul_rn(__fmul_rn(current, amw), (float)P.inv_unit);
    if (P.nonlinear != 0) {
        const float slope = (float)(P.nonlinear / maxw);
        value = __fdiv_rn(value, __fadd_rn(1.0f, fabsf(__fmul_rn(slope, value))));
    }
    value = value < 0.0f ? 0.0f : value;
    value = value > (float)maxw ? (float)maxw : value;
    return (long long)rintf(value);
}

__device__ __forceinline__ long long adc_count(double current, int maxw, double amw, const Physics& P) {
    double value = __dmul_rn(__dmul_rn(current, amw), P.inv_unit);
    if (P.nonlinear != 0) {
        const double slope = P.nonlinear / maxw;
        value = __ddiv_rn(value, __dadd_rn(1.0, fabs(__dmul_rn(slope, value))));
    }
    value = value < 0.0 ? 0.0 : value;
    value = value > (double)maxw ? (double)maxw : value;
    return (long long)rint(value);
}

template <typename T> __device__ __forceinline__ T mul_rn(T a, T b);
template <> __device__ __forceinline__ float mul_rn<float>(float a, float b) { return __fmul_rn(a, b); }
template <> __device__ __forceinline__ double mul_rn<double>(double a, double b) { return __dmul_rn(a, b); }

// ---------------------------------------------------------- physical kernel --
template <typename CodeT, typename CurT, typename OutT, typename ScaleT>
__global__ void __launch_bounds__(THREADS) physical_kernel(Layout L, Physics P, MMArgs a, const CurT* G,
                                                           int group_begin, int group_width, int power,
                                                           long long full) {
    __shared__ CurT sV[PHYS_RCH][PHYS_TV];
    __shared__ CurT sG[PHYS_RCH][PHYS_TC];
    const CodeT* codes = static_cast<const CodeT*>(a.codes);
    const ScaleT* xscale = static_cast<const ScaleT*>(a.xscale);
    const ScaleT* wscale = static_cast<const ScaleT*>(a.wscale);
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    const long long v0 = (long long)blockIdx.x * PHYS_TV;
    const long long col0 = (long long)group_begin * L.C + (long long)blockIdx.y * PHYS_TC;
    const long long col_end = (long long)(group_begin + group_width) * L.C;
    const int MR = a.m * L.reads;
    const long long row_stride = (long long)a.m * L.R;
    const uint64_t read_seed = event_seed(a.seed, a.event);
    const bool output_mode = P.read_mode == 2 && P.read_var != 0;
    const bool pair_mode = P.read_mode == 1 && P.read_var != 0;
    const CurT low = (CurT)P.low;

    Cascade<OutT> acc[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[j].init();

    for (int i = 0; i < MR; ++i) {
        const int arr = i / L.reads, g = i % L.reads;
        const int r0 = g * L.rows;
        const int len = L.rows < L.R - r0 ? L.rows : L.R - r0;
        long long total[4] = {0, 0, 0, 0};
        for (int sa = 0; sa < L.n_in; ++sa) {
            const int amask = L.in_mask[sa];
            for (int sw = 0; sw < L.n_w; ++sw) {
                CurT cur[4] = {0, 0, 0, 0}, mean[4] = {0, 0, 0, 0}, var[4] = {0, 0, 0, 0};
                for (int cb = 0; cb < len; cb += PHYS_RCH) {
                    const int clen = PHYS_RCH < len - cb ? PHYS_RCH : len - cb;
                    __syncthreads();
                    for (int idx = tid; idx < PHYS_TV * PHYS_RCH; idx += THREADS) {
                        const int rr = idx % PHYS_RCH, v = idx / PHYS_RCH;
                        const long long vec = v0 + v;
                        CurT value = 0;
                        if (vec < a.n && rr < clen) {
                            const int r = r0 + cb + rr;
                            const long long code = (long long)codes[vec * row_stride + (long long)arr * L.R + r];
                            const long long d = (code >> L.in_shift[sa]) & amask;
                            if (sizeof(CurT) == 4) {
                                float x = __fmul_rn(__fdiv_rn((float)d, (float)amask), (float)P.voltage);
                                if (P.volt_var != 0) {
                                    const long long address =
                                        (((vec + a.vector_offset) * a.m + arr) * L.n_in + sa) * L.R + r;
                                    float f = __fmul_rn((float)P.volt_var, rng_normal(address, read_seed, 40));
                                    x = __fmul_rn(x, __fadd_rn(1.0f, f));
                                }
                                value = (CurT)x;
                            } else {
                                double x = __dmul_rn(__ddiv_rn((double)d, (double)amask), P.voltage);
                                if (P.volt_var != 0) {
                                    const long long address =
                                        (((vec + a.vector_offset) * a.m + arr) * L.n_in + sa) * L.R + r;
                                    float f = __fmul_rn((float)P.volt_var, rng_normal(address, read_seed, 40));
                                    x = __dmul_rn(x, (double)__fadd_rn(1.0f, f));
                                }
                                value = (CurT)x;
                            }
                        }
                        sV[rr][v] = value;
                    }
                    for (int idx = tid; idx < PHYS_RCH * PHYS_TC; idx += THREADS) {
                        const int c = idx % PHYS_TC, rr = idx / PHYS_TC;
                        const long long col = col0 + c;
                        CurT value = 0;
                        if (col < col_end && rr < clen) {
                            const int r = r0 + cb + rr;
                            const long long t = col / L.C, cc = col % L.C;
                            value = G[((((long long)arr * group_width + (t - group_begin)) * L.n_w + sw) * L.R + r) * L.C + cc];
                            if (pair_mode) {
                                const long long cell = ((((long long)arr * a.p + t) * L.n_w + sw) * L.R + r) * L.C + cc;
                                const float e = expf(__fmul_rn((float)P.read_var,
                                                               rng_normal(cell * L.n_in + sa, read_seed, 20)));
                                value = sizeof(CurT) == 4 ? (CurT)__fmul_rn((float)value, e)
                                                          : (CurT)__dmul_rn((double)value, (double)e);
                            }
                        }
                        sG[rr][c] = value;
                    }
                    __syncthreads();
                    for (int rr = 0; rr < clen; ++rr) {
                        const CurT vr = sV[rr][ty];
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const CurT gv = sG[rr][4 * tx + j];
                            cur[j] = add_rn(cur[j], mul_rn(vr, add_rn(gv, -low)));
                            if (output_mode) {
                                mean[j] = add_rn(mean[j], mul_rn(vr, gv));
                                var[j] = add_rn(var[j], mul_rn(mul_rn(vr, vr), mul_rn(gv, gv)));
                            }
                        }
                    }
                }
                const long long factor = L.in_factor[sa] * L.w_factor[sw];
                const int maxw = L.adc_max[sw];
                const long long vec = v0 + ty;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    CurT current = cur[j];
                    if (output_mode) {
                        const long long col = col0 + 4 * tx + j;
                        const long long t = col / L.C, cc = col % L.C;
                        const long long address =
                            (((((vec + a.vector_offset) * MR + i) * a.p + t) * L.n_in + sa) * L.n_w + sw) * L.C + cc;
                        const float z = rng_normal(address, read_seed, 60);
                        if (sizeof(CurT) == 4) {
                            const float mu = __fmul_rn((float)mean[j], (float)P.mean_factor);
                            const float sig = __fmul_rn((float)var[j], (float)P.var_factor);
                            current = (CurT)__fadd_rn((float)current, __fadd_rn(mu, __fmul_rn(sqrtf(sig), z)));
                        } else {
                            const double mu = __dmul_rn((double)mean[j], P.mean_factor);
                            const double sig = __dmul_rn((double)var[j], P.var_factor);
                            current = (CurT)__dadd_rn((double)current, __dadd_rn(mu, __dmul_rn(sqrt(sig), (double)z)));
                        }
                    }
                    const CurT amw = (CurT)((long long)amask * L.w_mask[sw]);
                    total[j] += adc_count(current, maxw, amw, P) * factor;
                }
            }
        }
        const long long vec = v0 + ty;
        if (vec < a.n) {
            const ScaleT xs = xscale[vec * MR + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const long long col = col0 + 4 * tx + j;
                if (col >= col_end) continue;
                const long long t = col / L.C, cc = col % L.C;
                const ScaleT ws = wscale[((long long)i * a.p + t) * L.C + cc];
                cascade_push(acc[j], scaled_partial<OutT, ScaleT, long long>(total[j], xs, ws), i, power, full);
            }
        }
    }
    OutT* out = static_cast<OutT*>(a.out);
    const ScaleT* bias = static_cast<const ScaleT*>(a.bias);
    const long long vec = v0 + ty;
    if (vec >= a.n) return;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const long long col = col0 + 4 * tx + j;
        if (col >= col_end || col >= a.out_features) continue;
        OutT value = cascade_finish(acc[j]);
        if (bias) value = add_rn(value, (OutT)bias[col]);
        out[vec * a.ldo + col] = value;
    }
}

// ------------------------------------------------- staged physical kernel --
// physical_kernel for reads whose planes fit in shared memory and whose read
// noise does not depend on the slice pair (shared and output read modes): per
// read, the input voltages of every input slice (with their voltage noise) and
// G - LOW of every weight slice are staged once and shared by all slice pairs,
// and each thread accumulates a 2-vector x 4-column block of currents with FMAs
// in ascending row order.
template <typename T> __device__ __forceinline__ T fma_rn(T a, T b, T c);
template <> __device__ __forceinline__ float fma_rn<float>(float a, float b, float c) { return __fmaf_rn(a, b, c); }
template <> __device__ __forceinline__ double fma_rn<double>(double a, double b, double c) { return __fma_rn(a, b, c); }

template <typename CodeT, typename CurT, typename OutT, typename ScaleT, bool OUTPUT_NOISE>
__global__ void __launch_bounds__(THREADS, 2) physical_staged_kernel(Layout L, Physics P, MMArgs a, const CurT* G,
                                                                  int group_begin, int group_width, int power,
                                                                  long long full) {
    extern __shared__ __align__(16) uint8_t staged_raw[];
    CurT* sV = reinterpret_cast<CurT*>(staged_raw);        // [n_in][rows][ST_TV]
    CurT* sG = sV + (size_t)L.n_in * L.rows * ST_TV;         // [n_w][rows][ST_TC], G - LOW
    const CodeT* codes = static_cast<const CodeT*>(a.codes);
    const ScaleT* xscale = static_cast<const ScaleT*>(a.xscale);
    const ScaleT* wscale = static_cast<const ScaleT*>(a.wscale);
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    const long long v0 = (long long)blockIdx.x * ST_TV;
    const long long col0 = (long long)group_begin * L.C + (long long)blockIdx.y * ST_TC;
    const long long col_end = (long long)(group_begin + group_width) * L.C;
    const int MR = a.m * L.reads;
    const long long row_stride = (long long)a.m * L.R;
    const uint64_t read_seed = event_seed(a.seed, a.event);
    constexpr bool output_mode = OUTPUT_NOISE;
    const CurT low = (CurT)P.low;

    Cascade<OutT> acc[2][4];
#pragma unroll
    for (int e = 0; e < 2; ++e)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[e][j].init();

    for (int i = 0; i < MR; ++i) {
        const int arr = i / L.reads, g = i % L.reads;
        const int r0 = g * L.rows;
        const int len = L.rows < L.R - r0 ? L.rows : L.R - r0;
        __syncthreads();
        for (int idx = tid; idx < L.n_in * len * ST_TV; idx += THREADS) {
            const int v = idx % ST_TV, rr = (idx / ST_TV) % len, sa = idx / (ST_TV * len);
            const long long vec = v0 + v;
            CurT value = 0;
            if (vec < a.n) {
                const int r = r0 + rr;
                const int amask = L.in_mask[sa];
                const long long code = (long long)codes[vec * row_stride + (long long)arr * L.R + r];
                const long long d = (code >> L.in_shift[sa]) & amask;
                if (sizeof(CurT) == 4) {
                    float x = __fmul_rn(__fdiv_rn((float)d, (float)amask), (float)P.voltage);
                    if (P.volt_var != 0) {
                        const long long address = (((vec + a.vector_offset) * a.m + arr) * L.n_in + sa) * L.R + r;
                        x = __fmul_rn(x, __fadd_rn(1.0f, __fmul_rn((float)P.volt_var, rng_normal(address, read_seed, 40))));
                    }
                    value = (CurT)x;
                } else {
                    double x = __dmul_rn(__ddiv_rn((double)d, (double)amask), P.voltage);
                    if (P.volt_var != 0) {
                        const long long address = (((vec + a.vector_offset) * a.m + arr) * L.n_in + sa) * L.R + r;
                        const float f = __fmul_rn((float)P.volt_var, rng_normal(address, read_seed, 40));
                        x = __dmul_rn(x, (double)__fadd_rn(1.0f, f));
                    }
                    value = (CurT)x;
                }
            }
            sV[((size_t)sa * L.rows + rr) * ST_TV + v] = value;
        }
        for (int idx = tid; idx < L.n_w * len * ST_TC; idx += THREADS) {
            const int c = idx % ST_TC, rr = (idx / ST_TC) % len, sw = idx / (ST_TC * len);
            const long long col = col0 + c;
            CurT value = 0;
            if (col < col_end) {
                const long long t = col / L.C, cc = col % L.C;
                value = add_rn(G[((((long long)arr * group_width + (t - group_begin)) * L.n_w + sw) * L.R + r0 + rr) *
                                 L.C + cc], -low);
            }
            sG[((size_t)sw * L.rows + rr) * ST_TC + c] = value;
        }
        __syncthreads();
        long long total[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
        for (int sa = 0; sa < L.n_in; ++sa) {
            const int amask = L.in_mask[sa];
            const CurT* pv = sV + (size_t)sa * L.rows * ST_TV;
            for (int sw = 0; sw < L.n_w; ++sw) {
                const CurT* pg = sG + (size_t)sw * L.rows * ST_TC + 4 * tx;
                CurT cur[2][4] = {}, mean[2][4] = {}, var[2][4] = {};
                for (int rr = 0; rr < len; ++rr) {
                    const CurT va = pv[rr * ST_TV + ty], vb = pv[rr * ST_TV + ty + 16];
                    CurT gq[4];
                    if (sizeof(CurT) == 4) {
                        const float4 q4 = *reinterpret_cast<const float4*>(pg + rr * ST_TC);
                        gq[0] = (CurT)q4.x, gq[1] = (CurT)q4.y, gq[2] = (CurT)q4.z, gq[3] = (CurT)q4.w;
                    } else {
#pragma unroll
                        for (int j = 0; j < 4; ++j) gq[j] = pg[rr * ST_TC + j];
                    }
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        cur[0][j] = fma_rn(va, gq[j], cur[0][j]);
                        cur[1][j] = fma_rn(vb, gq[j], cur[1][j]);
                        if (output_mode) {
                            const CurT gv = add_rn(gq[j], low);
                            mean[0][j] = fma_rn(va, gv, mean[0][j]);
                            mean[1][j] = fma_rn(vb, gv, mean[1][j]);
                            var[0][j] = fma_rn(mul_rn(va, va), mul_rn(gv, gv), var[0][j]);
                            var[1][j] = fma_rn(mul_rn(vb, vb), mul_rn(gv, gv), var[1][j]);
                        }
                    }
                }
                const long long factor = L.in_factor[sa] * L.w_factor[sw];
                const int maxw = L.adc_max[sw];
                const CurT amw = (CurT)((long long)amask * L.w_mask[sw]);
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const long long vec = v0 + ty + 16 * e;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        CurT current = cur[e][j];
                        if (output_mode) {
                            const long long col = col0 + 4 * tx + j;
                            const long long t = col / L.C, cc = col % L.C;
                            const long long address =
                                (((((vec + a.vector_offset) * MR + i) * a.p + t) * L.n_in + sa) * L.n_w + sw) * L.C + cc;
                            const float z = rng_normal(address, read_seed, 60);
                            if (sizeof(CurT) == 4) {
                                const float mu = __fmul_rn((float)mean[e][j], (float)P.mean_factor);
                                const float sig = __fmul_rn((float)var[e][j], (float)P.var_factor);
                                current = (CurT)__fadd_rn((float)current, __fadd_rn(mu, __fmul_rn(sqrtf(sig), z)));
                            } else {
                                const double mu = __dmul_rn((double)mean[e][j], P.mean_factor);
                                const double sig = __dmul_rn((double)var[e][j], P.var_factor);
                                current = (CurT)__dadd_rn((double)current, __dadd_rn(mu, __dmul_rn(sqrt(sig), (double)z)));
                            }
                        }
                        total[e][j] += adc_count(current, maxw, amw, P) * factor;
                    }
                }
            }
        }
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const long long vec = v0 + ty + 16 * e;
            if (vec >= a.n) continue;
            const ScaleT xs = xscale[vec * MR + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const long long col = col0 + 4 * tx + j;
                if (col >= col_end) continue;
                const long long t = col / L.C, cc = col % L.C;
                const ScaleT ws = wscale[((long long)i * a.p + t) * L.C + cc];
                cascade_push(acc[e][j], scaled_partial<OutT, ScaleT, long long>(total[e][j], xs, ws), i, power, full);
            }
        }
    }
    OutT* out = static_cast<OutT*>(a.out);
    const ScaleT* bias = static_cast<const ScaleT*>(a.bias);
#pragma unroll
    for (int e = 0; e < 2; ++e) {
        const long long vec = v0 + ty + 16 * e;
        if (vec >= a.n) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const long long col = col0 + 4 * tx + j;
            if (col >= col_end || col >= a.out_features) continue;
            OutT value = cascade_finish(acc[e][j]);
            if (bias) value = add_rn(value, (OutT)bias[col]);
            out[vec * a.ldo + col] = value;
        }
    }
}

// ---------------------------------------------------- tiled physical kernel --
// physical_staged_kernel's computation for FP32 currents without slice-pair or
// output-mode read noise (voltage noise included), with 4 vectors x 4 columns
// per thread: per row, one 128-bit load of four voltages and one of four
// conductances feed 16 FMAs (the staged kernel's 2 x 4 tile needs three loads for
// 8).  The voltages of every input slice are staged once per read, G - LOW one
// weight slice at a time; FMAs run in ascending row order from the same staged
// values, so the currents equal the staged kernel's bit for bit.  Cascade level 1
// lives in shared memory (at most 256 reads per output).
constexpr int TT_V = 64;          // vectors per CTA (4 per thread)
constexpr int TT_C = 64;          // output columns per CTA (4 per thread)

template <typename CodeT>
__global__ void __launch_bounds__(THREADS, 2) physical_tile_kernel(Layout L, Physics P, MMArgs a, const float* G,
                                                                  int group_begin, int group_width, long long full) {
    extern __shared__ __align__(16) uint8_t tile_raw[];
    float* sV = reinterpret_cast<float*>(tile_raw);             // [n_in][rows][TT_V]
    float* sG = sV + (size_t)L.n_in * L.rows * TT_V;           // [rows][TT_C], G - LOW of one weight slice
    float* acc1 = sG + (size_t)L.rows * TT_C;                   // [TT_V][TT_C], cascade level 1
    const CodeT* codes = static_cast<const CodeT*>(a.codes);
    const float* xscale = static_cast<const float*>(a.xscale);
    const float* wscale = static_cast<const float*>(a.wscale);
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    const long long v0 = (long long)blockIdx.x * TT_V;
    const long long col0 = (long long)group_begin * L.C + (long long)blockIdx.y * TT_C;
    const long long col_end = (long long)(group_begin + group_width) * L.C;
    const int MR = a.m * L.reads;
    const long long row_stride = (long long)a.m * L.R;
    const uint64_t read_seed = event_seed(a.seed, a.event);
    const float low = (float)P.low;

    float acc0[4][4];
#pragma unroll
    for (int e = 0; e < 4; ++e)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            acc0[e][j] = 0.0f;
            acc1[(4 * ty + e) * TT_C + 4 * tx + j] = 0.0f;   // each thread owns its 16 cells
        }

    for (int i = 0; i < MR; ++i) {
        const int arr = i / L.reads, g = i % L.reads;
        const int r0 = g * L.rows;
        const int len = L.rows < L.R - r0 ? L.rows : L.R - r0;
        __syncthreads();
        for (int idx = tid; idx < L.n_in * len * TT_V; idx += THREADS) {
            const int v = idx % TT_V, rr = (idx / TT_V) % len, sa = idx / (TT_V * len);
            const long long vec = v0 + v;
            float value = 0.0f;
            if (vec < a.n) {
                const int r = r0 + rr;
                const int amask = L.in_mask[sa];
                const long long code = (long long)codes[vec * row_stride + (long long)arr * L.R + r];
                const long long d = (code >> L.in_shift[sa]) & amask;
                value = __fmul_rn(__fdiv_rn((float)d, (float)amask), (float)P.voltage);
                if (P.volt_var != 0) {
                    const long long address = (((vec + a.vector_offset) * a.m + arr) * L.n_in + sa) * L.R + r;
                    value = __fmul_rn(value, __fadd_rn(1.0f, __fmul_rn((float)P.volt_var,
                                                                      rng_normal(address, read_seed, 40))));
                }
            }
            sV[((size_t)sa * L.rows + rr) * TT_V + v] = value;
        }
        // Totals in wrapping int32 (the host checks |T| < 2^31): the ADC's
        // rint(clamp(value, 0, max_w)) equals the bit pattern of
        // clamp(value + 1.5 * 2^23, ...) minus 0x4B400000 (integer bounds, 0 <= value < 2^22).
        int total[4][4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
#pragma unroll
            for (int j = 0; j < 4; ++j) total[e][j] = 0;
        for (int sw = 0; sw < L.n_w; ++sw) {
            __syncthreads();
            for (int idx = tid; idx < len * TT_C; idx += THREADS) {
                const int c = idx % TT_C, rr = idx / TT_C;
                const long long col = col0 + c;
                float value = 0.0f;
                if (col < col_end) {
                    const long long t = col / L.C, cc = col % L.C;
                    value = __fadd_rn(
                        G[((((long long)arr * group_width + (t - group_begin)) * L.n_w + sw) * L.R + r0 + rr) * L.C +
                          cc],
                        -low);
                }
                sG[rr * TT_C + c] = value;
            }
            __syncthreads();
            const int maxw = L.adc_max[sw];
            for (int sa = 0; sa < L.n_in; ++sa) {
                const float* pv = sV + (size_t)sa * L.rows * TT_V + 4 * ty;
                const float* pg = sG + 4 * tx;
                float cur[4][4];
#pragma unroll
                for (int e = 0; e < 4; ++e)
#pragma unroll
                    for (int j = 0; j < 4; ++j) cur[e][j] = 0.0f;
#pragma unroll 4
                for (int rr = 0; rr < len; ++rr) {
                    const float4 v4 = *reinterpret_cast<const float4*>(pv + rr * TT_V);
                    const float4 g4 = *reinterpret_cast<const float4*>(pg + rr * TT_C);
                    const float vv[4] = {v4.x, v4.y, v4.z, v4.w};
                    const float gg[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e)
#pragma unroll
                        for (int j = 0; j < 4; ++j) cur[e][j] = __fmaf_rn(vv[e], gg[j], cur[e][j]);
                }
                const int factor = (int)(L.in_factor[sa] * L.w_factor[sw]);
                const float amw = (float)((long long)L.in_mask[sa] * L.w_mask[sw]);
                const float inv_unit = (float)P.inv_unit;
                const float slope = (float)(P.nonlinear / maxw);
                constexpr float kMagic = 12582912.0f;   // 1.5 * 2^23
                const float qmax = __fadd_rn((float)maxw, kMagic);
#pragma unroll
                for (int e = 0; e < 4; ++e)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        float value = __fmul_rn(__fmul_rn(cur[e][j], amw), inv_unit);
                        if (P.nonlinear != 0) value = __fdiv_rn(value, __fadd_rn(1.0f, fabsf(__fmul_rn(slope, value))));
                        const float q = fminf(fmaxf(__fadd_rn(value, kMagic), kMagic), qmax);
                        total[e][j] += (__float_as_int(q) - 0x4B400000) * factor;
                    }
            }
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const long long vec = v0 + 4 * ty + e;
            const float xs = vec < a.n ? xscale[vec * MR + i] : 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const long long col = col0 + 4 * tx + j;
                if (col >= col_end) continue;
                const long long t = col / L.C, cc = col % L.C;
                const float ws = wscale[((long long)i * a.p + t) * L.C + cc];
                acc0[e][j] = __fadd_rn(acc0[e][j], scaled_partial<float, float, int>(total[e][j], xs, ws));
            }
        }
        const int done = i + 1;
        if (done <= full && (done & 15) == 0) {
#pragma unroll
            for (int e = 0; e < 4; ++e)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float* slot = acc1 + (4 * ty + e) * TT_C + 4 * tx + j;
                    *slot = __fadd_rn(*slot, acc0[e][j]);
                    acc0[e][j] = 0.0f;
                }
        }
    }
    float* out = static_cast<float*>(a.out);
    const float* bias = static_cast<const float*>(a.bias);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const long long vec = v0 + 4 * ty + e;
        if (vec >= a.n) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const long long col = col0 + 4 * tx + j;
            if (col >= col_end || col >= a.out_features) continue;
            // acc0 + acc1 + acc2 + acc3 (upper levels zero), then the store into zeros.
            float value = __fadd_rn(acc0[e][j], acc1[(4 * ty + e) * TT_C + 4 * tx + j]);
            value = __fadd_rn(value, 0.0f);
            value = __fadd_rn(value, 0.0f);
            value = __fadd_rn(0.0f, value);
            if (bias) value = __fadd_rn(value, bias[col]);
            out[vec * a.ldo + col] = value;
        }
    }
}

size_t staged_smem(const mf_config& c, size_t elem) {
    return ((size_t)c.n_in * c.read_rows * ST_TV + (size_t)c.n_w * c.read_rows * ST_TC) * elem;
}

size_t ideal_smem(const mf_config& c) {
    const size_t r4 = (size_t)(c.read_rows + 3) / 4;
    return ((size_t)c.n_in * IDEAL_TV + (size_t)c.n_w * IDEAL_TC) * r4 * 4;
}


template <typename OutT, typename ScaleT>
mf_status launch_ideal_t(const mf_config& c, const MMArgs& a, cudaStream_t st, TileFilter filter = TileFilter{}) {
    Layout L = make_layout(c);
    const int MR = a.m * c.reads;
    const int power = cascade_power(MR);
    const long long full = (long long)MR - MR % (1LL << power);
    const size_t smem = ideal_smem(c);
    const long long cols = (long long)(a.tile_end - a.tile_begin) * c.cols;
    const int grid_x = (int)((a.n + IDEAL_TV - 1) / IDEAL_TV), grid_y = (int)((cols + IDEAL_TC - 1) / IDEAL_TC);
    // A filtered launch (exact rerun of flagged tiles, usually none) uses at most 4 CTAs
    // per SM stepping over the filter's tiles.
    const long long filter_tiles = (long long)filter.row_tiles * filter.col_tiles;
    dim3 grid = filter.flags ? dim3((unsigned)(filter_tiles < 148 * 4 ? filter_tiles : 148 * 4))
                             : dim3((unsigned)grid_x, (unsigned)grid_y);
    const bool small_totals = reconstruction_bound(c) < 2147483647.0;
#define MF_IDEAL(CODE, TOT)                                                                          \
    do {                                                                                             \
        auto kern = ideal_kernel<CODE, TOT, OutT, ScaleT>;                                           \
        MF_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem), \
                      "ideal kernel smem attribute");                                                \
        kern<<<grid, THREADS, smem, st>>>(L, a, power, full, filter, grid_x, grid_y);                 \
    } while (0)
    if (c.wide_codes) {
        if (small_totals) MF_IDEAL(long long, int); else MF_IDEAL(long long, long long);
    } else {
        if (small_totals) MF_IDEAL(uint8_t, int); else MF_IDEAL(uint8_t, long long);
    }
#undef MF_IDEAL
    MF_LAUNCH_CHECK("ideal_kernel");
    return MF_OK;
}

template <typename CurT, typename OutT, typename ScaleT>
mf_status launch_physical_t(const mf_config& c, const mf_schedule& s, const MMArgs& a, void* ws,
                            size_t ws_bytes, cudaStream_t st) {
    Layout L = make_layout(c);
    Physics P = make_physics(c);
    const int MR = a.m * c.reads;
    const int power = cascade_power(MR);
    const long long full = (long long)MR - MR % (1LL << power);
    const int tiles = a.tile_end - a.tile_begin;
    int width = s.arrays < 1 ? 1 : s.arrays;
    width = width > tiles ? tiles : width;
    const size_t need = physical_workspace_bytes(c, s, a.m, tiles);
    if (ws_bytes < need) {
        set_error("physical workspace too small: %zu < %zu bytes", ws_bytes, need);
        return MF_ERR_RESOURCE;
    }
    CurT* G = static_cast<CurT*>(ws);
    for (int begin = a.tile_begin; begin < a.tile_end; begin += width) {
        const int gw = begin + width <= a.tile_end ? width : a.tile_end - begin;
        const long long cells = (long long)a.m * gw * c.n_w * c.rows * c.cols;
        long long blocks = (cells + 255) / 256;
        if (blocks > 148 * 64) blocks = 148 * 64;
        restore_kernel<CurT><<<(unsigned)blocks, 256, 0, st>>>(L, P, a.packed, c.wide_codes, a.m, a.p, begin, gw,
                                                             a.seed, a.event, G);
        MF_LAUNCH_CHECK("restore_kernel");
        const long long cols = (long long)gw * c.cols;
        const bool pair_noise = c.read_mode == 1 && c.read_var != 0;
        const bool output_noise = c.read_mode == 2 && c.read_var != 0;
        const size_t tsmem = ((size_t)c.n_in * c.read_rows * TT_V + (size_t)c.read_rows * TT_C + TT_V * TT_C) * 4;
        if (sizeof(CurT) == 4 && sizeof(OutT) == 4 && !pair_noise && !output_noise && MR <= 256 &&
            tsmem <= 110 * 1024 && reconstruction_bound(c) < 2147483647.0 && max_adc(c) < (1 << 22)) {
            dim3 grid((unsigned)((a.n + TT_V - 1) / TT_V), (unsigned)((cols + TT_C - 1) / TT_C));
            const long long full16 = (long long)MR - MR % 16;
#define MF_TILED(CODE)                                                                                \
    do {                                                                                              \
        auto kern = physical_tile_kernel<CODE>;                                                       \
        MF_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tsmem), \
                      "tiled smem attribute");                                                         \
        kern<<<grid, THREADS, tsmem, st>>>(L, P, a, reinterpret_cast<const float*>(G), begin, gw, full16); \
    } while (0)
            if (c.wide_codes) MF_TILED(long long); else MF_TILED(uint8_t);
#undef MF_TILED
            MF_LAUNCH_CHECK("physical_tile_kernel");
            continue;
        }
        const size_t smem = staged_smem(c, sizeof(CurT));
        if (!pair_noise && smem <= ST_SMEM_MAX) {
            dim3 grid((unsigned)((a.n + ST_TV - 1) / ST_TV), (unsigned)((cols + ST_TC - 1) / ST_TC));
#define MF_STAGED(CODE, OUTN)                                                                          \
    do {                                                                                               \
        auto kern = physical_staged_kernel<CODE, CurT, OutT, ScaleT, OUTN>;                            \
        MF_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem), \
                      "staged smem attribute");                                                        \
        kern<<<grid, THREADS, smem, st>>>(L, P, a, G, begin, gw, power, full);                         \
    } while (0)
            if (c.wide_codes) {
                if (output_noise) MF_STAGED(long long, true); else MF_STAGED(long long, false);
            } else {
                if (output_noise) MF_STAGED(uint8_t, true); else MF_STAGED(uint8_t, false);
            }
#undef MF_STAGED
            MF_LAUNCH_CHECK("physical_staged_kernel");
            continue;
        }
        dim3 grid((unsigned)((a.n + PHYS_TV - 1) / PHYS_TV), (unsigned)((cols + PHYS_TC - 1) / PHYS_TC));
        if (c.wide_codes)
            physical_kernel<long long, CurT, OutT, ScaleT><<<grid, THREADS, 0, st>>>(L, P, a, G, begin, gw, power, full);
        else
            physical_kernel<uint8_t, CurT, OutT, ScaleT><<<grid, THREADS, 0, st>>>(L, P, a, G, begin, gw, power, full);
        MF_LAUNCH_CHECK("physical_kernel");
    }
    return MF_OK;
}

}  // namespace

Physics make_physics(const mf_config& c) {
    Physics P{};
    P.precise = c.precise_currents;
    P.read_mode = c.read_mode;
    P.high = c.high;
    P.low = c.low;
    P.span = c.high - c.low;
    P.voltage = c.voltage;
    P.inv_unit = 1.0 / c.unit;
    P.write_var = c.write_var;
    P.read_var = c.read_var;
    P.volt_var = c.volt_var;
    P.nonlinear = c.nonlinear;
    P.saf_low = c.saf_low;
    P.saf_cut = c.saf_low + c.saf_high;
    P.drift = c.drift;
    const double s2 = c.read_var * c.read_var;
    P.mean_factor = expm1(0.5 * s2);
    P.var_factor = exp(s2) * expm1(s2);
    return P;
}

int max_adc(const mf_config& c) {
    int m = 0;
    for (int i = 0; i < c.n_w; ++i) m = c.adc_max[i] > m ? c.adc_max[i] : m;
    return m;
}

double reconstruction_bound(const mf_config& c) {
    double in = 0, wt = 0;
    for (int i = 0; i < c.n_in; ++i) in += fabs((double)c.in_factor[i]);
    for (int i = 0; i < c.n_w; ++i) wt += fabs((double)c.w_factor[i]) * c.adc_max[i];
    return in * wt;
}

bool exact_integer_counts(const mf_config& c) {
    int maxadc = 0;
    for (int i = 0; i < c.n_w; ++i) maxadc = c.adc_max[i] > maxadc ? c.adc_max[i] : maxadc;
    const double eps = c.precise_currents ? ldexp(1.0, -52) : ldexp(1.0, -23);
    return (c.read_rows + 16.0) * (maxadc + 1.0) * eps * 4.0 < 0.5;
}

bool generic_ideal_fits(const mf_config& c, const mf_schedule&) {
    for (int i = 0; i < c.n_in; ++i)
        if (c.in_mask[i] > 255) return false;
    for (int i = 0; i < c.n_w; ++i)
        if (c.w_mask[i] > 255) return false;
    return ideal_smem(c) <= 200 * 1024;
}

mf_status generic_ideal(const mf_config& c, const mf_schedule&, const MMArgs& a, cudaStream_t st) {
    if (a.stable) {
        return c.wide ? launch_ideal_t<double, double>(c, a, st) : launch_ideal_t<double, float>(c, a, st);
    }
    return c.wide ? launch_ideal_t<double, double>(c, a, st) : launch_ideal_t<float, float>(c, a, st);
}

mf_status generic_ideal_tiles(const mf_config& c, const MMArgs& a, const unsigned* flags, int rows, int cols,
                              int row_tiles, cudaStream_t st) {
    if (rows % IDEAL_TV || cols % IDEAL_TC) {
        set_error("tile filter %dx%d is not a multiple of the generic tile", rows, cols);
        return MF_ERR_INVALID;
    }
    const long long width = (long long)(a.tile_end - a.tile_begin) * c.cols;
    const TileFilter filter{flags, rows, cols, row_tiles, (int)((width + cols - 1) / cols)};
    return c.wide ? launch_ideal_t<double, double>(c, a, st, filter) : launch_ideal_t<float, float>(c, a, st, filter);
}

size_t physical_workspace_bytes(const mf_config& c, const mf_schedule& s, int32_t m, int32_t tiles) {
    int width = s.arrays < 1 ? 1 : s.arrays;
    width = width > tiles ? tiles : width;
    const size_t elem = c.precise_currents ? 8 : 4;
    return (size_t)m * width * c.n_w * c.rows * c.cols * elem;
}

mf_status physical(const mf_config& c, const mf_schedule& s, const MMArgs& a, void* ws, size_t ws_bytes,
                   cudaStream_t st) {
    const bool dbl_out = c.wide || a.stable;
    if (c.precise_currents) {
        if (!dbl_out) return launch_physical_t<double, float, float>(c, s, a, ws, ws_bytes, st);
        return c.wide ? launch_physical_t<double, double, double>(c, s, a, ws, ws_bytes, st)
                      : launch_physical_t<double, double, float>(c, s, a, ws, ws_bytes, st);
    }
    if (!dbl_out) return launch_physical_t<float, float, float>(c, s, a, ws, ws_bytes, st);
    return c.wide ? launch_physical_t<float, double, double>(c, s, a, ws, ws_bytes, st)
                  : launch_physical_t<float, double, float>(c, s, a, ws, ws_bytes, st);
}

}  // namespace mf

// Group quantisation and bit-slice packing on the device.
//
// Restates memfast/quantization.py for device buffers:
//   grouped_quantize  quantization.py:9-44   (INT: scale = max/upper, clamped to the
//                     smallest subnormal, codes = rint(x/scale) clamped; BFP: shared
//                     power-of-two exponent per group)
//   pack_weight       quantization.py:94-112 (two's-complement mask, [m,p,R,C] tiles,
//                     per-read scale gather with replicate padding)
//   input_tiles       quantization.py:115-137
// Three passes: group |max| (atomic max on the IEEE bit pattern, exact for
// non-negative values), elementwise codes, and the per-read scale gather.
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <float.h>

#include "common.cuh"
#include "kernels.cuh"

namespace mf {

namespace {

template <typename Acc>
__device__ __forceinline__ Acc load_as(const void* base, int dtype, int64_t index);

template <>
__device__ __forceinline__ float load_as<float>(const void* base, int dtype, int64_t index) {
    switch (dtype) {
        case MF_F16: return __half2float(static_cast<const __half*>(base)[index]);
        case MF_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[index]);
        case MF_F64: return __double2float_rn(static_cast<const double*>(base)[index]);
        default: return static_cast<const float*>(base)[index];
    }
}

template <>
__device__ __forceinline__ double load_as<double>(const void* base, int dtype, int64_t index) {
    switch (dtype) {
        case MF_F16: return (double)__half2float(static_cast<const __half*>(base)[index]);
        case MF_BF16: return (double)__bfloat162float(static_cast<const __nv_bfloat16*>(base)[index]);
        case MF_F64: return static_cast<const double*>(base)[index];
        default: return (double)static_cast<const float*>(base)[index];
    }
}

__device__ __forceinline__ void atomic_max_nonneg(float* slot, float value) {
    atomicMax(reinterpret_cast<unsigned int*>(slot), __float_as_uint(value));
}
__device__ __forceinline__ void atomic_max_nonneg(double* slot, double value) {
    atomicMax(reinterpret_cast<unsigned long long*>(slot), (unsigned long long)__double_as_longlong(value));
}

// Logical element (row, col) of the quantised matrix.  Inputs are stored as
// [rows, cols]; weights are quantised as W^T, so logical (k, o) lives at w[o, k].
struct View {
    const void* data;
    int dtype;
    int64_t rows, cols, ld;
    int transposed;
    __device__ __forceinline__ int64_t offset(int64_t r, int64_t c) const {
        return transposed ? c * ld + r : r * ld + c;
    }
};

struct GroupGrid {
    int64_t gr, gc, nc;  // group extents and number of group columns
};

// Each thread scans a run of consecutive stored elements, keeps a running |max|
// while they stay in one group, and publishes it with one atomic per group run.
template <typename Acc>
__global__ void group_amax_kernel(View v, GroupGrid g, Acc* maxima) {
    constexpr int64_t RUN = 8;
    const int64_t inner = v.transposed ? v.rows : v.cols;
    const int64_t total = v.rows * v.cols;
    const int64_t runs = (total + RUN - 1) / RUN;
    for (int64_t run = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; run < runs;
         run += (int64_t)gridDim.x * blockDim.x) {
        int64_t begin = run * RUN, end = begin + RUN < total ? begin + RUN : total;
        int64_t current = -1;
        Acc best = Acc(0);
        for (int64_t i = begin; i < end; ++i) {
            int64_t outer = i / inner, in = i % inner;
            int64_t r = v.transposed ? in : outer;
            int64_t c = v.transposed ? outer : in;
            Acc x = load_as<Acc>(v.data, v.dtype, outer * v.ld + in);
            Acc a = x < Acc(0) ? -x : x;
            int64_t group = (r / g.gr) * g.nc + c / g.gc;
            if (group != current) {
                if (current >= 0) atomic_max_nonneg(&maxima[current], best);
                current = group;
                best = a;
            } else if (a > best) {
                best = a;
            }
        }
        if (current >= 0) atomic_max_nonneg(&maxima[current], best);
    }
}

struct QuantSpec {
    int bits, signed_codes, bfp, bw_e;
    int64_t lower, upper, mask;
};

// Scale of a group from its |max| (quantization.py:27-39).
template <typename Acc>
__device__ __forceinline__ Acc group_scale(Acc maximum, const QuantSpec& s);

template <>
__device__ __forceinline__ float group_scale<float>(float maximum, const QuantSpec& s) {
    float base = maximum > 0.0f ? maximum : 1.0f;
    float scale = __fdiv_rn(base, (float)s.upper);
    const float smallest = 1.40129846e-45f;
    return scale < smallest ? smallest : scale;
}

template <>
__device__ __forceinline__ double group_scale<double>(double maximum, const QuantSpec& s) {
    if (!s.bfp) {
        double base = maximum > 0.0 ? maximum : 1.0;
        double scale = __ddiv_rn(base, (double)s.upper);
        const double smallest = 4.9406564584124654e-324;
        return scale < smallest ? smallest : scale;
    }
    // floor(log2(max(m, DBL_MIN))) is the frexp exponent minus one, exactly.
    int e;
    frexp(maximum > DBL_MIN ? maximum : DBL_MIN, &e);
    int exponent = e - 1;
    int limit = (1 << (s.bw_e - 1)) - 1;
    exponent = exponent < 1 - limit ? 1 - limit : (exponent > limit ? limit : exponent);
    return ldexp(1.0, exponent + 2 - s.bits);
}

template <typename Acc>
__device__ __forceinline__ int64_t quantise(Acc x, Acc scale, const QuantSpec& s) {
    Acc q = rint(x / scale);
    if (q < (Acc)s.lower) q = (Acc)s.lower;
    if (q > (Acc)s.upper) q = (Acc)s.upper;
    return (int64_t)q & s.mask;
}

// FP32 computes codes of at most 8 bits (wider codes and BFP compute in FP64), so the
// clamped value converts through int32 (NaN converts to 0 either way).
template <>
__device__ __forceinline__ int64_t quantise<float>(float x, float scale, const QuantSpec& s) {
    float q = rintf(__fdiv_rn(x, scale));
    if (q < (float)s.lower) q = (float)s.lower;
    if (q > (float)s.upper) q = (float)s.upper;
    return (int64_t)(__float2int_rz(q) & (int)s.mask);
}

// quantise<float> for codes of at most 8 bits without a division per value:
// q = x * fl(1/scale) is within |q| * 2^-23 of x / scale, and its nearest integer
// can differ from the reference's rint(fl(x / scale)) only when q lies within that
// distance of a half-integer (|q| <= 256 here keeps it below 2^-13); those values
// are divided exactly.  q + 1.5 * 2^23 rounds half to even into the low mantissa
// bits, whose low byte is the two's-complement code (NaN gives 0, as in quantise).
__device__ __forceinline__ uint32_t code8(float x, float scale, float inv, const QuantSpec& s) {
    constexpr float kMagic = 12582912.0f;   // 1.5 * 2^23
    float q = __fmul_rn(x, inv);
    const float f = __fsub_rn(q, __fsub_rn(__fadd_rn(q, kMagic), kMagic));
    if (fabsf(__fsub_rn(fabsf(f), 0.5f)) < 1.220703125e-4f) q = __fdiv_rn(x, scale);
    if (q < (float)s.lower) q = (float)s.lower;
    if (q > (float)s.upper) q = (float)s.upper;
    return (uint32_t)__float_as_int(__fadd_rn(q, kMagic)) & (uint32_t)s.mask;
}

// Input codes: [n, m*R] (zero beyond k).
template <typename Acc, typename CodeT>
__global__ void input_code_kernel(View v, GroupGrid g, const Acc* maxima, const Acc* fixed,
                                  QuantSpec s, int64_t padded_cols, CodeT* codes) {
    const int64_t total = v.rows * padded_cols;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t r = i / padded_cols, c = i % padded_cols;
        int64_t code = 0;
        if (c < v.cols) {
            Acc x = load_as<Acc>(v.data, v.dtype, v.offset(r, c));
            Acc scale = fixed ? fixed[c] : group_scale<Acc>(maxima[(r / g.gr) * g.nc + c / g.gc], s);
            code = quantise<Acc>(x, scale, s);
        }
        codes[i] = (CodeT)code;
    }
}

// One pass for per-row input groups of gc = 4 * T consecutive FP32 values (T a
// power of two <= 32): a team of T lanes loads one group with float4 loads, takes
// its |max| with shuffles, quantises and stores four 8-bit codes per lane, and
// publishes the group maximum for the per-read scale gather.  Columns past k
// (up to m * R) get code 0 and do not enter any maximum.
template <int T>
__global__ void input_rowgroup_kernel(const float* x, int64_t n, int64_t k, int64_t ldx, int64_t padded_cols,
                                      int64_t nc, QuantSpec s, float* maxima, uint8_t* codes, float* xscale,
                                      uint32_t* check_flag, uint32_t check_code) {
    constexpr int GC = 4 * T;
    const int64_t groups_per_row = padded_cols / GC;
    const int64_t teams = n * groups_per_row;
    const int lane_in_team = threadIdx.x % T;
    const int64_t stride = ((int64_t)gridDim.x * blockDim.x) / T;
    // Warp-uniform trip count: every lane of a warp takes part in the shuffles.
    for (int64_t team = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / T;
         __any_sync(0xFFFFFFFFu, team < teams); team += stride) {
        const bool active = team < teams;
        int64_t r = 0, j = 0;
        if (active) {
            if (teams <= 0xFFFFFFFFll) {   // 32-bit division where the index fits
                const uint32_t t32 = (uint32_t)team, g32 = (uint32_t)groups_per_row;
                r = t32 / g32;
                j = t32 - (uint32_t)r * g32;
            } else {
                r = team / groups_per_row;
                j = team % groups_per_row;
            }
        }
        const int64_t c = j * GC + 4 * lane_in_team;
        float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const float* row = x + r * ldx;
        if (!active) {
        } else if (c + 3 < k) {
            const float4 q = *reinterpret_cast<const float4*>(row + c);
            v[0] = q.x, v[1] = q.y, v[2] = q.z, v[3] = q.w;
        } else {
#pragma unroll
            for (int e = 0; e < 4; ++e)
                if (c + e < k) v[e] = row[c + e];
        }
        float best = 0.0f;
        bool bad = false;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            best = fmaxf(best, fabsf(v[e]));
            bad |= !(fabsf(v[e]) <= FLT_MAX);   // NaN or infinity (zero padding passes)
        }
        // The operand check of the product, folded into this read of x: the first
        // failing check of the stream keeps its code (mf_check_finite's rule).
        if (bad && check_flag && *(volatile uint32_t*)check_flag == 0u) atomicCAS(check_flag, 0u, check_code);
#pragma unroll
        for (int off = T / 2; off > 0; off >>= 1) best = fmaxf(best, __shfl_xor_sync(0xFFFFFFFFu, best, off, T));
        const float scale = group_scale<float>(best, s);
        const float inv = __frcp_rn(scale);
        uint32_t word = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e)
            if (c + e < k) word |= (code8(v[e], scale, inv, s) & 0xFFu) << (8 * e);
        if (!active) continue;
        *reinterpret_cast<uint32_t*>(codes + r * padded_cols + c) = word;
        if (lane_in_team == 0 && j < nc) {
            maxima[r * nc + j] = best;
            // Groups as wide as a read (xscale non-null): group j is read j's scale, and
            // reads past k take the last group's, as input_scale_kernel gives them.
            if (xscale) {
                xscale[r * groups_per_row + j] = scale;
                if (j == nc - 1)
                    for (int64_t jj = nc; jj < groups_per_row; ++jj) xscale[r * groups_per_row + jj] = scale;
            }
        }
    }
}

// Input per-read scales: xscale[r, i] for read starts i (replicate padding).
template <typename Acc, typename ScaleT>
__global__ void input_scale_kernel(View v, GroupGrid g, const Acc* maxima, const Acc* fixed,
                                   QuantSpec s, int R, int read_rows, int reads, int64_t m,
                                   ScaleT* xscale) {
    const int64_t per_row = m * reads;
    const int64_t total = v.rows * per_row;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t r = i / per_row, idx = i % per_row;
        int64_t start = (idx / reads) * R + (idx % reads) * read_rows;
        int64_t c = start < v.cols ? start : v.cols - 1;
        xscale[i] = (ScaleT)(fixed ? fixed[c] : group_scale<Acc>(maxima[(r / g.gr) * g.nc + c / g.gc], s));
    }
}

// Packed weights [m, p, R, C] from logical W^T[k, o]; a 32x32 tile is staged in
// shared memory so reads (along k in w[o, k]) and writes (along c) both coalesce.
template <typename Acc, typename CodeT>
__global__ void weight_code_kernel(View v, GroupGrid g, const Acc* maxima, QuantSpec s, int R,
                                   int C, int64_t m, int64_t p, CodeT* packed) {
    __shared__ int64_t tile[32][33];
    const int64_t k0 = (int64_t)blockIdx.x * 32, o0 = (int64_t)blockIdx.y * 32;
    const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
    for (int j = ty; j < 32; j += 8) {
        int64_t k = k0 + tx, o = o0 + j;
        int64_t code = 0;
        if (k < v.rows && o < v.cols) {
            Acc x = load_as<Acc>(v.data, v.dtype, v.offset(k, o));
            code = quantise<Acc>(x, group_scale<Acc>(maxima[(k / g.gr) * g.nc + o / g.gc], s), s);
        }
        tile[tx][j] = code;
    }
    __syncthreads();
    for (int j = ty; j < 32; j += 8) {
        int64_t k = k0 + j, o = o0 + tx;
        if (k < m * R && o < p * C) {
            int64_t arr = k / R, r = k % R, t = o / C, c = o % C;
            packed[((arr * p + t) * R + r) * C + c] = (CodeT)tile[j][tx];
        }
    }
}

// One pass for a right-hand FP32 matrix b [K, O] (row-major) with column groups
// of GR rows: a thread owns one (group, column), keeps the GR values in
// registers, takes their |max|, quantises, writes the packed [m, p, R, C] tiles
// (coalesced across the warp's columns) and, when `kmajor` is set, the K-major
// [p*C, m*R] copy the tensor-core kernels read; the group maximum is published
// for the per-read scale gather.  Padding rows and columns are zeroed by the host.
template <int GR>
__global__ void rhs_colgroup_kernel(const float* b, int64_t K, int64_t O, int64_t ldb, QuantSpec s, int R, int C,
                                    int64_t m, int64_t p, float* maxima, uint8_t* packed, uint8_t* kmajor,
                                    float* wscale, uint32_t* check_flag, uint32_t check_code) {
    static_assert(GR % 32 == 0, "K-major stores cover whole 32-row sectors");
    const int64_t groups = (K + GR - 1) / GR;
    const int64_t total = groups * O;
    const int64_t kpad = m * R;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = i / O, o = i % O, k0 = j * GR;
        // Two passes over the group: the maximum, then the codes from a second read
        // of the same lines (still in L1), so that few registers hold values and
        // more warps hide the memory latency.
        const float* col = b + k0 * ldb + o;
        const int rows = K - k0 < GR ? (int)(K - k0) : GR;
        float best = 0.0f;
        bool bad = false;
#pragma unroll 8
        for (int r = 0; r < GR; ++r)
            if (r < rows) {
                const float value = fabsf(__ldg(col + r * ldb));
                best = fmaxf(best, value);
                bad |= !(value <= FLT_MAX);   // NaN or infinity
            }
        // The operand check of the product, folded into this read of b (first failing
        // check of the stream keeps its code).
        if (bad && check_flag && *(volatile uint32_t*)check_flag == 0u) atomicCAS(check_flag, 0u, check_code);
        maxima[j * O + o] = best;
        const float scale = group_scale<float>(best, s);
        const float inv = __frcp_rn(scale);
        if (wscale) {
            // Groups of one read (wscale non-null): wscale[read j, column o]; reads past K
            // and columns past O replicate the last group and column, as
            // weight_scale_kernel's clamped indices give them.
            const int64_t pc = p * C, mr = kpad / GR;
            const int64_t last_read = j == groups - 1 ? mr : j + 1;
            const int64_t last_col = o == O - 1 ? pc : o + 1;
            for (int64_t jr = j; jr < last_read; ++jr)
                for (int64_t oc = o; oc < last_col; ++oc) wscale[jr * pc + oc] = scale;
        }
        const int64_t t = o / C, c = o % C;
        // Array and row of k, stepped along the group (no division or 64-bit product
        // per element): dst points at packed[arr, t, rr, c].
        int64_t arr = k0 / R;
        int rr = (int)(k0 - arr * R);
        uint8_t* dst = packed + ((arr * p + t) * R + rr) * C + c;
        const int64_t next_array = (p - 1) * R * C;   // from row R-1 of one array to row 0 of the next
        // K-major codes leave as whole 32-byte sectors (two 16-byte stores back to back)
        // where the 32 bytes are inside the padded K and aligned, else word by word: a
        // 16-byte store now and its neighbour later cost the memory system two
        // partial-sector writes.
        uint32_t words[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll 16
        for (int r = 0; r < GR; ++r) {
            const int64_t k = k0 + r;
            const uint32_t code = r < rows ? (code8(__ldg(col + r * ldb), scale, inv, s) & 0xFFu) : 0u;
            if (k < kpad) *dst = (uint8_t)code;
            dst += C;
            if (++rr == R) {
                rr = 0;
                dst += next_array;
            }
            words[(r >> 2) & 7] |= code << (8 * (r & 3));
            if ((r & 31) == 31 && kmajor) {
                uint8_t* dst = kmajor + o * kpad + k - 31;
                if (k < kpad && (reinterpret_cast<uintptr_t>(dst) & 31) == 0) {
                    uint4* out = reinterpret_cast<uint4*>(dst);
                    out[0] = make_uint4(words[0], words[1], words[2], words[3]);
                    out[1] = make_uint4(words[4], words[5], words[6], words[7]);
                } else {
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                        if (k - 31 + 4 * q + 3 < kpad) *reinterpret_cast<uint32_t*>(dst + 4 * q) = words[q];
                }
#pragma unroll
                for (int q = 0; q < 8; ++q) words[q] = 0;
            }
        }
    }
}

// Tiled form of rhs_colgroup_kernel for aligned FP32 matrices (row stride a
// multiple of 4, 16-byte-aligned base, R a multiple of GR, C a multiple of 16): a
// CTA stages one GR x 128 tile of b in shared memory with 16-byte coalesced loads
// (one read of every value), a thread per column takes the group maximum and the
// codes from shared memory and writes its K-major run of GR codes as whole
// 32-byte sectors, and the CTA then writes the packed [m, p, R, C] rows of the
// tile as 16-byte chunks.  Same outputs as rhs_colgroup_kernel.
template <int GR>
__global__ void __launch_bounds__(256) rhs_tile_kernel(const float* b, int64_t K, int64_t O, int64_t ldb, QuantSpec s,
                                                       int R, int C, int64_t m, int64_t p, float* maxima,
                                                       uint8_t* packed, uint8_t* kmajor, float* wscale,
                                                       uint32_t* check_flag, uint32_t check_code) {
    constexpr int TC = 128;                         // columns per tile
    constexpr int LD = TC + 4;                      // padded row of the staged tile
    __shared__ __align__(16) float tile[GR][LD];
    __shared__ __align__(16) uint8_t codes[GR][TC];
    const int64_t j = blockIdx.y;                   // column group (GR rows)
    const int64_t k0 = j * GR, o0 = (int64_t)blockIdx.x * TC;
    const int rows = K - k0 < GR ? (int)(K - k0) : GR;
    const int cols = O - o0 < TC ? (int)(O - o0) : TC;
    const int tid = threadIdx.x;
    // Stage: warp w loads rows w, w + 8, ...; lane l the four columns 4l..4l+3.
    bool bad = false;
    {
        const int lane = tid & 31, c4 = 4 * lane;
        for (int r = tid >> 5; r < GR; r += 8) {
            float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (r < rows) {
                const float* src = b + (k0 + r) * ldb + o0 + c4;
                if (c4 + 3 < cols) {
                    v = __ldg(reinterpret_cast<const float4*>(src));
                } else {
                    if (c4 < cols) v.x = __ldg(src);
                    if (c4 + 1 < cols) v.y = __ldg(src + 1);
                    if (c4 + 2 < cols) v.z = __ldg(src + 2);
                }
            }
            bad |= !(fabsf(v.x) <= FLT_MAX) || !(fabsf(v.y) <= FLT_MAX) || !(fabsf(v.z) <= FLT_MAX) ||
                   !(fabsf(v.w) <= FLT_MAX);
            *reinterpret_cast<float4*>(&tile[r][c4]) = v;
        }
    }
    // The operand check of the product, folded into this read of b.
    if (bad && check_flag && *(volatile uint32_t*)check_flag == 0u) atomicCAS(check_flag, 0u, check_code);
    __syncthreads();
    const int64_t kpad = m * R;
    if (tid < TC && tid < cols) {
        const int c = tid;
        const int64_t o = o0 + c;
        float best = 0.0f;
#pragma unroll 8
        for (int r = 0; r < GR; ++r) best = fmaxf(best, fabsf(tile[r][c]));
        maxima[j * O + o] = best;
        const float scale = group_scale<float>(best, s);
        const float inv = __frcp_rn(scale);
        if (wscale) {
            // As rhs_colgroup_kernel: reads past K and columns past O replicate the last
            // group and column.
            const int64_t groups = (K + GR - 1) / GR;
            const int64_t pc = p * C, mr = kpad / GR;
            const int64_t last_read = j == groups - 1 ? mr : j + 1;
            const int64_t last_col = o == O - 1 ? pc : o + 1;
            for (int64_t jr = j; jr < last_read; ++jr)
                for (int64_t oc = o; oc < last_col; ++oc) wscale[jr * pc + oc] = scale;
        }
#pragma unroll
        for (int q = 0; q < GR / 32; ++q) {
            uint32_t words[8];
#pragma unroll
            for (int w = 0; w < 8; ++w) {
                uint32_t word = 0;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int r = 32 * q + 4 * w + e;
                    const uint32_t code = r < rows ? (code8(tile[r][c], scale, inv, s) & 0xFFu) : 0u;
                    codes[r][c] = (uint8_t)code;
                    word |= code << (8 * e);
                }
                words[w] = word;
            }
            if (kmajor) {
                uint4* dst = reinterpret_cast<uint4*>(kmajor + o * kpad + k0 + 32 * q);
                dst[0] = make_uint4(words[0], words[1], words[2], words[3]);
                dst[1] = make_uint4(words[4], words[5], words[6], words[7]);
            }
        }
    }
    __syncthreads();
    // Packed rows: row k0 + r of the tile's columns, 16 columns per chunk (a chunk
    // stays inside one array tile since C is a multiple of 16).
    const int64_t arr = k0 / R;
    const int rr0 = (int)(k0 - arr * R);
    for (int idx = tid; idx < GR * (TC / 16); idx += blockDim.x) {
        const int r = idx / (TC / 16), ch = idx % (TC / 16);
        const int c = 16 * ch;
        if (c >= cols) continue;
        const int64_t o = o0 + c, t = o / C, cc = o % C;
        uint8_t* dst = packed + ((arr * p + t) * R + rr0 + r) * C + cc;
        if (c + 15 < cols) {
            *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(&codes[r][c]);
        } else {
            for (int e = 0; c + e < cols; ++e) dst[e] = codes[r][c + e];
        }
    }
}

// wscale[i, t, c] = scale at (read start row, column) with replicate padding.
template <typename Acc, typename ScaleT>
__global__ void weight_scale_kernel(View v, GroupGrid g, const Acc* maxima, QuantSpec s, int R,
                                    int C, int read_rows, int reads, int64_t m, int64_t p,
                                    ScaleT* wscale) {
    const int64_t total = m * reads * p * C;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t col = i % (p * C), idx = i / (p * C);
        int64_t start = (idx / reads) * R + (idx % reads) * read_rows;
        int64_t k = start < v.rows ? start : v.rows - 1;
        int64_t o = col < v.cols ? col : v.cols - 1;
        wscale[i] = (ScaleT)group_scale<Acc>(maxima[(k / g.gr) * g.nc + o / g.gc], s);
    }
}

// ---- 2-D convolution patches (implicit im2col) --------------------------------
// The patch matrix of one channel group, in F.unfold order
// (memfast/nn/convolution.py:49-55): row v = (b * OH + oh) * OW + ow, column
// k = (c * KH + i) * KW + j for the group's channels c in [0, CG); element
// x[b, C0 + c, oh * SY - PH + i * DH, ow * SX - PW + j * DW], zero outside x.
struct ConvGeom {
    const void* x;
    int dtype;
    int64_t sb, sc, sh, sw;  // element strides of x
    int32_t H, W, C0, KH, KW, SY, SX, PH, PW, DH, DW, OH, OW;
    int64_t rows, cols;      // batch * OH * OW, CG * KH * KW
};

struct PatchRow {
    int64_t base;      // offset of x[b, C0, 0, 0]
    int32_t ih0, iw0;  // input coordinates of the window's top-left tap
};

__device__ __forceinline__ PatchRow patch_row(const ConvGeom& g, int64_t v) {
    const int64_t plane = (int64_t)g.OH * g.OW;
    const int64_t b = v / plane;
    const int32_t l = (int32_t)(v - b * plane);
    const int32_t oh = l / g.OW, ow = l - oh * g.OW;
    return PatchRow{b * g.sb + (int64_t)g.C0 * g.sc, oh * g.SY - g.PH, ow * g.SX - g.PW};
}

// Column k as (channel, kernel row, kernel column); callers then step it.
struct Tap {
    int32_t c, i, j;
    __device__ __forceinline__ void at(const ConvGeom& g, int64_t k) {
        const int32_t taps = g.KH * g.KW;
        c = (int32_t)(k / taps);
        const int32_t rem = (int32_t)(k - (int64_t)c * taps);
        i = rem / g.KW;
        j = rem - i * g.KW;
    }
    __device__ __forceinline__ void next(const ConvGeom& g) {
        if (++j == g.KW) {
            j = 0;
            if (++i == g.KH) {
                i = 0;
                ++c;
            }
        }
    }
};

// Offset of the tap in x, or -1 in the zero padding.
__device__ __forceinline__ int64_t tap_offset(const ConvGeom& g, const PatchRow& r, const Tap& t) {
    const int32_t ih = r.ih0 + t.i * g.DH, iw = r.iw0 + t.j * g.DW;
    if ((unsigned)ih >= (unsigned)g.H || (unsigned)iw >= (unsigned)g.W) return -1;
    return r.base + (int64_t)t.c * g.sc + (int64_t)ih * g.sh + (int64_t)iw * g.sw;
}

__device__ __forceinline__ bool finite_as_stored(const void* base, int dtype, int64_t index) {
    return isfinite(load_as<double>(base, dtype, index));  // exact widening of every stored dtype
}

// Group maxima of the patch matrix.  A warp owns 32 consecutive rows (one per
// lane) and one column group; it walks the group's columns with each load
// coalesced across the lanes' neighbouring output positions and keeps the
// running |max| in registers.  Per-row groups store the maximum; groups spanning
// rows combine with an atomic max (the caller zeroes them).  A non-finite value in
// the compute dtype raises *nonfinite (grouped_quantize's check, quantization.py:14-15).
template <typename Acc>
__global__ void conv_amax_kernel(ConvGeom g, GroupGrid gg, Acc* maxima, unsigned* nonfinite) {
    const int lane = threadIdx.x & 31;
    const int64_t row_blocks = (g.rows + 31) / 32;
    const int64_t items = row_blocks * gg.nc;
    const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t item = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; item < items; item += warps) {
        const int64_t rb = item / gg.nc, group = item - rb * gg.nc;
        const int64_t v = rb * 32 + lane;
        const bool active = v < g.rows;
        const PatchRow r = patch_row(g, active ? v : 0);
        const int64_t k0 = group * gg.gc, k1 = k0 + gg.gc < g.cols ? k0 + gg.gc : g.cols;
        Tap t;
        t.at(g, k0);
        Acc best = Acc(0);
        bool bad = false;
#pragma unroll 4
        for (int64_t k = k0; k < k1; ++k) {
            const int64_t off = active ? tap_offset(g, r, t) : -1;
            const Acc x = off >= 0 ? load_as<Acc>(g.x, g.dtype, off) : Acc(0);
            bad |= !isfinite(x);
            const Acc a = x < Acc(0) ? -x : x;
            best = a > best ? a : best;
            t.next(g);
        }
        if (__any_sync(0xFFFFFFFFu, bad) && lane == 0) atomicOr(nonfinite, 1u);
        if (active) {
            Acc* slot = &maxima[(v / gg.gr) * gg.nc + group];
            if (gg.gr == 1) *slot = best;
            else atomic_max_nonneg(slot, best);
        }
    }
}

// Codes of the patch matrix, [rows, padded] row-major (zero past cols).  A
// 256-thread block owns a tile of 32 rows x 128 columns: each warp quantises 16
// columns for the 32 rows (lanes; loads coalesced along the output positions),
// the codes are staged in shared memory and leave as whole 128-column row
// segments.  With a fixed per-column scale the values are checked finite in their
// stored dtype (input_tiles' check, quantization.py:124-125).
template <typename Acc, typename CodeT>
__global__ void __launch_bounds__(256) conv_code_kernel(ConvGeom g, GroupGrid gg, const Acc* maxima,
                                                        const Acc* fixed, QuantSpec s, int64_t padded,
                                                        CodeT* codes, unsigned* nonfinite) {
    constexpr int TR = 32, TC = 128, PITCH = TC + (sizeof(CodeT) == 1 ? 4 : 1);
    __shared__ __align__(16) CodeT tile[TR][PITCH];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t row_tiles = (g.rows + TR - 1) / TR, col_tiles = (padded + TC - 1) / TC;
    const bool words = sizeof(CodeT) == 1 && (padded & 3) == 0;
    for (int64_t tile_id = blockIdx.x; tile_id < row_tiles * col_tiles; tile_id += gridDim.x) {
        const int64_t rt = tile_id / col_tiles, ct = tile_id - rt * col_tiles;
        const int64_t v = rt * TR + lane;
        const bool active = v < g.rows;
        const PatchRow r = patch_row(g, active ? v : 0);
        const int64_t kb = ct * TC + warp * 16;
        Tap t;
        t.at(g, kb < g.cols ? kb : 0);
        int64_t cached = -1;
        Acc scale = Acc(1);
        bool bad = false;
#pragma unroll 4
        for (int e = 0; e < 16; ++e) {
            const int64_t k = kb + e;
            int64_t code = 0;
            if (active && k < g.cols) {
                const int64_t off = tap_offset(g, r, t);
                const Acc x = off >= 0 ? load_as<Acc>(g.x, g.dtype, off) : Acc(0);
                if (fixed) {
                    scale = fixed[k];
                    bad |= off >= 0 && !finite_as_stored(g.x, g.dtype, off);
                } else {
                    const int64_t group = (v / gg.gr) * gg.nc + k / gg.gc;
                    if (group != cached) {
                        scale = group_scale<Acc>(maxima[group], s);
                        cached = group;
                    }
                }
                code = quantise<Acc>(x, scale, s);
                t.next(g);
            }
            tile[lane][warp * 16 + e] = (CodeT)code;
        }
        if (fixed && __any_sync(0xFFFFFFFFu, bad) && lane == 0) atomicOr(nonfinite, 1u);
        __syncthreads();
        for (int rr = warp; rr < TR; rr += 8) {
            const int64_t row = rt * TR + rr;
            if (row >= g.rows) break;
            CodeT* dst = codes + row * padded + ct * TC;
            const int64_t width = padded - ct * TC < TC ? padded - ct * TC : TC;
            if (words) {
                if (4 * lane < width)
                    reinterpret_cast<uint32_t*>(dst)[lane] = *reinterpret_cast<const uint32_t*>(&tile[rr][4 * lane]);
            } else {
                for (int e = lane; e < width; e += 32) dst[e] = tile[rr][e];
            }
        }
        __syncthreads();
    }
}

// Finiteness of n contiguous values: the first failing check of a stream wins
// the flag word (atomicCAS from 0), so checks launched in the reference's order
// report its first error.  code_own: a non-finite value in its stored dtype;
// code_narrow (FP64 only, 0 = unused): finite in FP64 but not once narrowed to FP32.
__global__ void check_finite_kernel(const void* x, int dtype, int64_t n, uint32_t code_own, uint32_t code_narrow,
                                    uint32_t* flag) {
    uint32_t found = 0;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        if (dtype == MF_F64) {
            const double v = static_cast<const double*>(x)[i];
            if (!isfinite(v)) found = found ? found : code_own;
            else if (code_narrow && !isfinite(__double2float_rn(v))) found = found ? found : code_narrow;
        } else if (!isfinite(load_as<float>(x, dtype, i))) {
            found = code_own;
        }
        if (__any_sync(__activemask(), found != 0)) break;
    }
    // Own-dtype failures outrank narrowing ones within one launch.
    const uint32_t own = __reduce_or_sync(__activemask(), found == code_own && found ? 1u : 0u);
    const uint32_t any = __reduce_or_sync(__activemask(), found ? 1u : 0u);
    if ((threadIdx.x & 31) == 0 && any) atomicCAS(flag, 0u, own ? code_own : code_narrow);
}

// Fast path of the same check (no narrowing test): 16-byte loads, four in flight
// per thread, and an exponent test per element (all-ones exponent = Inf or NaN);
// block 0 also checks the elements after the last whole vector.
__device__ __forceinline__ bool vector_nonfinite(const uint4 v, int dtype) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    bool bad = false;
    if (dtype == MF_F32) {
#pragma unroll
        for (int i = 0; i < 4; ++i) bad |= (w[i] & 0x7F800000u) == 0x7F800000u;
    } else if (dtype == MF_F64) {
        bad = ((w[1] & 0x7FF00000u) == 0x7FF00000u) | ((w[3] & 0x7FF00000u) == 0x7FF00000u);
    } else {
        const uint32_t e = dtype == MF_F16 ? 0x7C00u : 0x7F80u;
#pragma unroll
        for (int i = 0; i < 4; ++i) bad |= ((w[i] & e) == e) | ((w[i] & (e << 16)) == (e << 16));
    }
    return bad;
}

__global__ void check_finite_vector_kernel(const void* x, int dtype, int64_t n, int esize, uint32_t code,
                                           uint32_t* flag) {
    const uint4* vec = static_cast<const uint4*>(x);
    const int64_t nvec = n * esize / 16;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    bool bad = false;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nvec; i += 4 * stride) {
        uint4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) v[u] = i + u * stride < nvec ? __ldg(vec + i + u * stride) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int u = 0; u < 4; ++u) bad |= vector_nonfinite(v[u], dtype);
    }
    if (blockIdx.x == 0) {
        for (int64_t i = nvec * 16 / esize + threadIdx.x; i < n; i += blockDim.x) {
            if (dtype == MF_F64) bad |= !isfinite(static_cast<const double*>(x)[i]);
            else bad |= !isfinite(load_as<float>(x, dtype, i));
        }
    }
    if (__any_sync(0xFFFFFFFFu, bad) && (threadIdx.x & 31) == 0) atomicCAS(flag, 0u, code);
}

int grid_for(int64_t work, int threads) {
    int64_t blocks = (work + threads - 1) / threads;
    if (blocks > 148 * 32) blocks = 148 * 32;
    return blocks < 1 ? 1 : (int)blocks;
}

GroupGrid groups_of(int64_t rows, int64_t cols, int32_t gr, int32_t gc) {
    GroupGrid g;
    g.gr = gr <= 0 ? rows : (gr < rows ? gr : rows);
    g.gc = gc <= 0 ? cols : (gc < cols ? gc : cols);
    if (g.gr < 1) g.gr = 1;
    if (g.gc < 1) g.gc = 1;
    g.nc = (cols + g.gc - 1) / g.gc;
    return g;
}

QuantSpec spec_of(int bits, int signed_codes, int bw_e) {
    QuantSpec s;
    s.bits = bits;
    s.signed_codes = signed_codes;
    s.bfp = bw_e > 0;
    s.bw_e = bw_e;
    s.upper = (int64_t(1) << (bits - (signed_codes ? 1 : 0))) - 1;
    if (s.bfp) {
        s.lower = -(int64_t(1) << (bits - 1));
        s.upper = (int64_t(1) << (bits - 1)) - 1;
    } else {
        s.lower = signed_codes ? -s.upper : 0;
    }
    s.mask = bits >= 63 ? -1 : ((int64_t(1) << bits) - 1);
    return s;
}

bool uses_double(const mf_config& c, int bits) { return bits > 8 || c.bw_e > 0; }

}  // namespace

int64_t conv_output_extent(int64_t size, int32_t kernel, int32_t stride, int32_t pad, int32_t dilation) {
    const int64_t span = (int64_t)dilation * (kernel - 1) + 1;
    const int64_t room = size + 2 * (int64_t)pad - span;
    return room < 0 ? 0 : room / stride + 1;
}

size_t quantize_workspace_bytes(const mf_config& c, bool weight, int64_t rows, int64_t cols) {
    // Logical matrix: inputs [n, k]; weights W^T = [k, o] for w of shape [o, k].
    int64_t lr = weight ? cols : rows, lc = weight ? rows : cols;
    GroupGrid g = weight ? groups_of(lr, lc, c.w_group_rows, c.w_group_cols)
                         : groups_of(lr, lc, c.in_group_rows, c.in_group_cols);
    int64_t nr = (lr + g.gr - 1) / g.gr;
    int bits = weight ? c.weight_bits : c.activation_bits;
    size_t elem = uses_double(c, bits) ? 8 : 4;
    return (size_t)(nr * g.nc) * elem + 256;
}

// The one-pass kernel applies to FP32 rows with 16-byte-aligned rows, dynamic
// per-row groups of 4 * {1,2,...,32} values and 8-bit codes.
static int rowgroup_team(const mf_config& c, const View& v, const GroupGrid& g, const void* fixed) {
    if (fixed || c.wide_codes || v.transposed || v.dtype != MF_F32 || g.gr != 1) return 0;
    if (((uintptr_t)v.data & 15) || (v.ld % 4)) return 0;
    const int64_t padded = ((v.cols + c.rows - 1) / c.rows) * c.rows;
    for (int team = 1; team <= 32; team *= 2)
        if (g.gc == 4 * team && padded % g.gc == 0) return team;
    return 0;
}

template <typename Acc, typename ScaleT>
static mf_status run_input(const mf_config& c, const View& v, const GroupGrid& g, const QuantSpec& s,
                           const void* fixed, void* codes, void* xscale, void* workspace,
                           size_t need, cudaStream_t stream, uint32_t* check_flag = nullptr,
                           uint32_t check_code = 0) {
    const int threads = 256;
    const int64_t n = v.rows, k = v.cols, m = (k + c.rows - 1) / c.rows;
    Acc* maxima = static_cast<Acc*>(workspace);
    const Acc* fx = static_cast<const Acc*>(fixed);
    const int team = sizeof(Acc) == 4 ? rowgroup_team(c, v, g, fixed) : 0;
    if (team) {
        const int64_t padded = m * c.rows;
        const int64_t lanes = n * (padded / g.gc) * team;
        const int blocks = grid_for((lanes + threads - 1) / threads * threads, threads);
        // Per-read scales in the same pass when a group spans exactly one read.
        const bool scales_fused = sizeof(ScaleT) == 4 && g.gc == c.read_rows && c.rows % c.read_rows == 0;
        float* fused_xscale = scales_fused ? reinterpret_cast<float*>(xscale) : nullptr;
#define MF_ROWGROUP(TEAM)                                                                                    \
    input_rowgroup_kernel<TEAM><<<blocks, threads, 0, stream>>>(static_cast<const float*>(v.data), n, k, v.ld, \
                                                                padded, g.nc, s, reinterpret_cast<float*>(maxima), \
                                                                static_cast<uint8_t*>(codes), fused_xscale,     \
                                                                check_flag, check_code)
        switch (team) {
            case 1: MF_ROWGROUP(1); break;
            case 2: MF_ROWGROUP(2); break;
            case 4: MF_ROWGROUP(4); break;
            case 8: MF_ROWGROUP(8); break;
            case 16: MF_ROWGROUP(16); break;
            default: MF_ROWGROUP(32); break;
        }
#undef MF_ROWGROUP
        MF_LAUNCH_CHECK("input_rowgroup_kernel");
        if (scales_fused) return MF_OK;
        input_scale_kernel<Acc, ScaleT><<<grid_for(n * m * c.reads, threads), threads, 0, stream>>>(
            v, g, maxima, fx, s, c.rows, c.read_rows, c.reads, m, static_cast<ScaleT*>(xscale));
        MF_LAUNCH_CHECK("input_scale_kernel");
        return MF_OK;
    }
    if (!fx) {
        MF_CHECK_CUDA(cudaMemsetAsync(maxima, 0, need, stream), "memset group maxima");
        group_amax_kernel<Acc><<<grid_for((n * k + 7) / 8, threads), threads, 0, stream>>>(v, g, maxima);
        MF_LAUNCH_CHECK("group_amax_kernel");
    }
    if (c.wide_codes)
        input_code_kernel<Acc, int64_t><<<grid_for(n * m * c.rows, threads), threads, 0, stream>>>(
            v, g, maxima, fx, s, m * c.rows, static_cast<int64_t*>(codes));
    else
        input_code_kernel<Acc, uint8_t><<<grid_for(n * m * c.rows, threads), threads, 0, stream>>>(
            v, g, maxima, fx, s, m * c.rows, static_cast<uint8_t*>(codes));
    MF_LAUNCH_CHECK("input_code_kernel");
    input_scale_kernel<Acc, ScaleT><<<grid_for(n * m * c.reads, threads), threads, 0, stream>>>(
        v, g, maxima, fx, s, c.rows, c.read_rows, c.reads, m, static_cast<ScaleT*>(xscale));
    MF_LAUNCH_CHECK("input_scale_kernel");
    return MF_OK;
}

mf_status quantize_input(const mf_config& c, const void* x, int dtype, int64_t n, int64_t k,
                         int64_t ldx, const void* fixed, void* codes, void* xscale,
                         void* workspace, size_t ws_bytes, cudaStream_t stream, uint32_t* check_flag,
                         uint32_t check_code) {
    View v{x, dtype, n, k, ldx, 0};
    GroupGrid g = groups_of(n, k, c.in_group_rows, c.in_group_cols);
    QuantSpec s = spec_of(c.activation_bits, 1, c.bw_e);
    size_t need = quantize_workspace_bytes(c, false, n, k) - 256;
    if (!fixed && ws_bytes < need) {
        set_error("quantize workspace too small: %zu < %zu bytes", ws_bytes, need);
        return MF_ERR_RESOURCE;
    }
    // grouped_quantize computes in FP64 iff bits > 8 or BFP; the stored scales are
    // FP64 iff Config.wide (quantization.py:10,131).  A fixed scale arrives in the
    // stored dtype and is applied in it (quantization.py:124-130).
    const bool dbl = uses_double(c, c.activation_bits);
    if (check_flag) {
        // The one-pass kernel checks x as it reads it; every other path gets the
        // separate check first (x must then be contiguous).
        if (dbl || fixed || !rowgroup_team(c, v, g, nullptr)) {
            if (ldx != k) {
                set_error("a folded finiteness check needs contiguous inputs");
                return MF_ERR_INVALID;
            }
            mf_status st = check_finite(x, dtype, n * k, check_code, 0, check_flag, stream);
            if (st) return st;
            check_flag = nullptr;
        }
    }
    if (fixed) {
        return c.wide ? run_input<double, double>(c, v, g, s, fixed, codes, xscale, workspace, need, stream)
                      : run_input<float, float>(c, v, g, s, fixed, codes, xscale, workspace, need, stream);
    }
    if (dbl) return run_input<double, double>(c, v, g, s, nullptr, codes, xscale, workspace, need, stream);
    if (c.wide)
        return run_input<float, double>(c, v, g, s, nullptr, codes, xscale, workspace, need, stream, check_flag,
                                        check_code);
    return run_input<float, float>(c, v, g, s, nullptr, codes, xscale, workspace, need, stream, check_flag,
                                   check_code);
}

mf_status check_finite(const void* x, int dtype, int64_t n, uint32_t code_own, uint32_t code_narrow,
                       uint32_t* flag, cudaStream_t stream) {
    if (n <= 0) return MF_OK;
    const int threads = 256;
    if (!code_narrow && reinterpret_cast<uintptr_t>(x) % 16 == 0) {
        const int esize = dtype == MF_F64 ? 8 : dtype == MF_F32 ? 4 : 2;
        const int64_t nvec = n * esize / 16;
        int64_t blocks = (nvec + 4 * threads - 1) / (4 * threads);
        blocks = blocks < 1 ? 1 : blocks > 148 * 8 ? 148 * 8 : blocks;
        check_finite_vector_kernel<<<(int)blocks, threads, 0, stream>>>(x, dtype, n, esize, code_own, flag);
        MF_LAUNCH_CHECK("check_finite_vector_kernel");
        return MF_OK;
    }
    check_finite_kernel<<<grid_for(n, threads), threads, 0, stream>>>(x, dtype, n, code_own, code_narrow, flag);
    MF_LAUNCH_CHECK("check_finite_kernel");
    return MF_OK;
}

mf_status quantize_conv_input(const mf_config& c, const mf_conv2d& cv, const void* x, int dtype,
                              const void* fixed, void* codes, void* xscale, uint32_t* nonfinite,
                              void* workspace, size_t ws_bytes, cudaStream_t stream) {
    ConvGeom g{};
    g.x = x;
    g.dtype = dtype;
    g.sb = cv.stride_n, g.sc = cv.stride_c, g.sh = cv.stride_h, g.sw = cv.stride_w;
    g.H = (int32_t)cv.height, g.W = (int32_t)cv.width, g.C0 = cv.channel_begin;
    g.KH = cv.kernel_h, g.KW = cv.kernel_w, g.SY = cv.stride_y, g.SX = cv.stride_x;
    g.PH = cv.pad_h, g.PW = cv.pad_w, g.DH = cv.dilation_h, g.DW = cv.dilation_w;
    g.OH = (int32_t)conv_output_extent(cv.height, cv.kernel_h, cv.stride_y, cv.pad_h, cv.dilation_h);
    g.OW = (int32_t)conv_output_extent(cv.width, cv.kernel_w, cv.stride_x, cv.pad_w, cv.dilation_w);
    g.rows = cv.batch * g.OH * g.OW;
    g.cols = (int64_t)cv.group_channels * cv.kernel_h * cv.kernel_w;
    const GroupGrid gg = groups_of(g.rows, g.cols, c.in_group_rows, c.in_group_cols);
    const QuantSpec s = spec_of(c.activation_bits, 1, c.bw_e);
    const size_t need = quantize_workspace_bytes(c, false, g.rows, g.cols) - 256;
    if (!fixed && ws_bytes < need) {
        set_error("conv quantize workspace too small: %zu < %zu bytes", ws_bytes, need);
        return MF_ERR_RESOURCE;
    }
    MF_CHECK_CUDA(cudaMemsetAsync(nonfinite, 0, sizeof(uint32_t), stream), "clear non-finite flag");
    if (g.rows == 0) return MF_OK;
    const int64_t m = (g.cols + c.rows - 1) / c.rows, padded = m * c.rows;
    const int threads = 256;
    const bool dbl = fixed ? c.wide != 0 : uses_double(c, c.activation_bits);
    const View v{x, dtype, g.rows, g.cols, g.cols, 0};
    const int64_t code_tiles = ((g.rows + 31) / 32) * ((padded + 127) / 128);
    const int code_blocks = (int)(code_tiles < 148 * 16 ? code_tiles : 148 * 16);
    auto run = [&](auto acc_tag, auto code_tag, auto scale_tag) -> mf_status {
        using Acc = decltype(acc_tag);
        using CodeT = decltype(code_tag);
        using ScaleT = decltype(scale_tag);
        Acc* maxima = static_cast<Acc*>(workspace);
        const Acc* fx = static_cast<const Acc*>(fixed);
        if (!fx) {
            MF_CHECK_CUDA(cudaMemsetAsync(maxima, 0, need, stream), "memset group maxima");
            const int64_t warps = ((g.rows + 31) / 32) * gg.nc;
            conv_amax_kernel<Acc><<<grid_for(warps * 32, threads), threads, 0, stream>>>(g, gg, maxima, nonfinite);
            MF_LAUNCH_CHECK("conv_amax_kernel");
        }
        conv_code_kernel<Acc, CodeT><<<code_blocks, threads, 0, stream>>>(g, gg, maxima, fx, s, padded,
                                                                          static_cast<CodeT*>(codes), nonfinite);
        MF_LAUNCH_CHECK("conv_code_kernel");
        input_scale_kernel<Acc, ScaleT><<<grid_for(g.rows * m * c.reads, threads), threads, 0, stream>>>(
            v, gg, maxima, fx, s, c.rows, c.read_rows, c.reads, m, static_cast<ScaleT*>(xscale));
        MF_LAUNCH_CHECK("input_scale_kernel");
        return MF_OK;
    };
    if (c.wide_codes) {
        if (dbl) return run(double{}, int64_t{}, double{});
        return c.wide ? run(float{}, int64_t{}, double{}) : run(float{}, int64_t{}, float{});
    }
    if (dbl) return run(double{}, uint8_t{}, double{});
    return c.wide ? run(float{}, uint8_t{}, double{}) : run(float{}, uint8_t{}, float{});
}

template <typename Acc, typename ScaleT>
static mf_status run_weights(const mf_config& c, const View& v, const GroupGrid& g, const QuantSpec& s,
                             void* packed, void* wscale, void* workspace, size_t need,
                             cudaStream_t stream) {
    const int threads = 256;
    const int64_t k = v.rows, o = v.cols;
    const int64_t m = (k + c.rows - 1) / c.rows, p = (o + c.cols - 1) / c.cols;
    Acc* maxima = static_cast<Acc*>(workspace);
    MF_CHECK_CUDA(cudaMemsetAsync(maxima, 0, need, stream), "memset group maxima");
    group_amax_kernel<Acc><<<grid_for((o * k + 7) / 8, threads), threads, 0, stream>>>(v, g, maxima);
    MF_LAUNCH_CHECK("group_amax_kernel");
    dim3 tgrid((unsigned)((m * c.rows + 31) / 32), (unsigned)((p * c.cols + 31) / 32));
    dim3 tblock(32, 8);
    if (c.wide_codes)
        weight_code_kernel<Acc, int64_t><<<tgrid, tblock, 0, stream>>>(
            v, g, maxima, s, c.rows, c.cols, m, p, static_cast<int64_t*>(packed));
    else
        weight_code_kernel<Acc, uint8_t><<<tgrid, tblock, 0, stream>>>(
            v, g, maxima, s, c.rows, c.cols, m, p, static_cast<uint8_t*>(packed));
    MF_LAUNCH_CHECK("weight_code_kernel");
    weight_scale_kernel<Acc, ScaleT><<<grid_for(m * c.reads * p * c.cols, threads), threads, 0, stream>>>(
        v, g, maxima, s, c.rows, c.cols, c.read_rows, c.reads, m, p, static_cast<ScaleT*>(wscale));
    MF_LAUNCH_CHECK("weight_scale_kernel");
    return MF_OK;
}

mf_status program_rhs(const mf_config& c, const void* b, int dtype, int64_t k, int64_t o, int64_t ldb,
                      void* packed, void* wscale, void* kmajor, void* workspace, size_t ws_bytes,
                      cudaStream_t stream, uint32_t* check_flag, uint32_t check_code) {
    View v{b, dtype, k, o, ldb, 0};  // logical [k, o] = b
    GroupGrid g = groups_of(k, o, c.w_group_rows, c.w_group_cols);
    QuantSpec s = spec_of(c.weight_bits, c.weight_signed, c.bw_e);
    size_t need = quantize_workspace_bytes(c, true, o, k) - 256;
    if (ws_bytes < need) {
        set_error("weight workspace too small: %zu < %zu bytes", ws_bytes, need);
        return MF_ERR_RESOURCE;
    }
    const int64_t m = (k + c.rows - 1) / c.rows, p = (o + c.cols - 1) / c.cols;
    const bool dbl = uses_double(c, c.weight_bits);
    // The fused pass stores the K-major copy as 32-bit words: rows of m*R bytes
    // must keep them aligned.
    const bool words_aligned = !kmajor || ((m * c.rows) % 4 == 0 && (reinterpret_cast<uintptr_t>(kmajor) & 3) == 0);
    const bool fused = !dbl && !c.wide && !c.wide_codes && dtype == MF_F32 && g.gc == 1 &&
                       (g.gr == 32 || g.gr == 64) && words_aligned;
    if (check_flag && !fused) {
        // Only the one-pass kernel checks b as it reads it: the others get the
        // separate check first (b must then be contiguous).
        if (ldb != o) {
            set_error("a folded finiteness check needs a contiguous right-hand matrix");
            return MF_ERR_INVALID;
        }
        mf_status st = check_finite(b, dtype, k * o, check_code, 0, check_flag, stream);
        if (st) return st;
        check_flag = nullptr;
    }
    if (fused) {
        const size_t packed_bytes = (size_t)m * p * c.rows * c.cols;
        if (k < m * c.rows || o < p * c.cols) {
            MF_CHECK_CUDA(cudaMemsetAsync(packed, 0, packed_bytes, stream), "zero packed padding");
            if (kmajor) MF_CHECK_CUDA(cudaMemsetAsync(kmajor, 0, packed_bytes, stream), "zero K-major padding");
        }
        const int threads = 256;
        const int64_t work = ((k + g.gr - 1) / g.gr) * o;
        float* maxima = static_cast<float*>(workspace);
        // Per-read weight scales in the same pass when a group spans exactly one read.
        const bool scales_fused = g.gr == c.read_rows && c.rows % c.read_rows == 0;
        float* fused_wscale = scales_fused ? static_cast<float*>(wscale) : nullptr;
        // The tiled kernel wherever b's rows and the tiles allow 16-byte loads and chunks.
        const int64_t tile_rows = (k + g.gr - 1) / g.gr;
        const bool tiled = c.rows % g.gr == 0 && c.cols % 16 == 0 && ldb % 4 == 0 &&
                           (reinterpret_cast<uintptr_t>(b) & 15) == 0 && tile_rows <= 65535 &&
                           (!kmajor || (reinterpret_cast<uintptr_t>(kmajor) & 15) == 0);
        if (tiled) {
            const dim3 grid((unsigned)((o + 127) / 128), (unsigned)tile_rows);
            if (g.gr == 32)
                rhs_tile_kernel<32><<<grid, 256, 0, stream>>>(
                    static_cast<const float*>(b), k, o, ldb, s, c.rows, c.cols, m, p, maxima,
                    static_cast<uint8_t*>(packed), static_cast<uint8_t*>(kmajor), fused_wscale, check_flag, check_code);
            else
                rhs_tile_kernel<64><<<grid, 256, 0, stream>>>(
                    static_cast<const float*>(b), k, o, ldb, s, c.rows, c.cols, m, p, maxima,
                    static_cast<uint8_t*>(packed), static_cast<uint8_t*>(kmajor), fused_wscale, check_flag, check_code);
            MF_LAUNCH_CHECK("rhs_tile_kernel");
        } else {
            if (g.gr == 32)
                rhs_colgroup_kernel<32><<<grid_for(work, threads), threads, 0, stream>>>(
                    static_cast<const float*>(b), k, o, ldb, s, c.rows, c.cols, m, p, maxima,
                    static_cast<uint8_t*>(packed), static_cast<uint8_t*>(kmajor), fused_wscale, check_flag,
                    check_code);
            else
                rhs_colgroup_kernel<64><<<grid_for(work, threads), threads, 0, stream>>>(
                    static_cast<const float*>(b), k, o, ldb, s, c.rows, c.cols, m, p, maxima,
                    static_cast<uint8_t*>(packed), static_cast<uint8_t*>(kmajor), fused_wscale, check_flag,
                    check_code);
            MF_LAUNCH_CHECK("rhs_colgroup_kernel");
        }
        if (scales_fused) return MF_OK;
        weight_scale_kernel<float, float><<<grid_for(m * c.reads * p * c.cols, threads), threads, 0, stream>>>(
            v, g, maxima, s, c.rows, c.cols, c.read_rows, c.reads, m, p, static_cast<float*>(wscale));
        MF_LAUNCH_CHECK("weight_scale_kernel");
        return MF_OK;
    }
    mf_status st;
    if (dbl) st = run_weights<double, double>(c, v, g, s, packed, wscale, workspace, need, stream);
    else if (c.wide) st = run_weights<float, double>(c, v, g, s, packed, wscale, workspace, need, stream);
    else st = run_weights<float, float>(c, v, g, s, packed, wscale, workspace, need, stream);
    if (st || !kmajor) return st;
    if (c.wide_codes) {
        set_error("a K-major copy needs 8-bit codes");
        return MF_ERR_UNSUPPORTED;
    }
    return tc_weights_kmajor(packed, static_cast<uint8_t*>(kmajor), (int)m, (int)p, c.rows, c.cols, stream);
}

mf_status program_weights(const mf_config& c, const void* w, int dtype, int64_t o, int64_t k,
                          int64_t ldw, void* packed, void* wscale, void* workspace,
                          size_t ws_bytes, cudaStream_t stream) {
    View v{w, dtype, k, o, ldw, 1};  // logical [k, o] = w^T
    GroupGrid g = groups_of(k, o, c.w_group_rows, c.w_group_cols);
    QuantSpec s = spec_of(c.weight_bits, c.weight_signed, c.bw_e);
    size_t need = quantize_workspace_bytes(c, true, o, k) - 256;
    if (ws_bytes < need) {
        set_error("weight workspace too small: %zu < %zu bytes", ws_bytes, need);
        return MF_ERR_RESOURCE;
    }
    const bool dbl = uses_double(c, c.weight_bits);
    if (dbl) return run_weights<double, double>(c, v, g, s, packed, wscale, workspace, need, stream);
    if (c.wide) return run_weights<float, double>(c, v, g, s, packed, wscale, workspace, need, stream);
    return run_weights<float, float>(c, v, g, s, packed, wscale, workspace, need, stream);
}

}  // namespace mf

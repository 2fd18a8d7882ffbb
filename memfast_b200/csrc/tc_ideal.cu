// tcgen05 / TMEM fast path for the ideal-device sliced product (sm_100a).
//
// The reference computes, for every read of rows_per_read rows and every
// (input slice a, weight slice w) pair, an ADC count min(D_aw, m_w) with
// D_aw = sum_r d_a(r) d_w(r), and reconstructs T = sum_aw s_a s_w count
// (memfast/reference.py:81-115, kernels.cu:108-169).  Because
// min(D, m) = D - relu(D - m) and sum_aw s_a s_w D_aw = x . w (the signed codes),
//
//     T = x . w  -  sum over clip-capable pairs of s_a s_w relu(D_aw - m_w).
//
// A pair is clip-capable when rows * Ma * Mw > m_w.  The kernel therefore runs
// one kind::i8 MMA of the raw codes per read plus one kind::f8f6f4 MMA per
// clip-capable pair group, all accumulating into TMEM.  Digits d <= 7 are fed
// to the tensor core as raw bytes, which read as E4M3 subnormals d * 2^-9, so
// every D arrives exactly as D * 2^-18 in FP32.  "Conditional" pairs (whose
// threshold is rarely reached) are only issued for (read, column block) jobs
// where a digit-sum bound, max_n Mw*S_a(n) and max_o Ma*S_w(o), admits a clip.
//
// The epilogue (FFMA.SAT relu, f32x2 FMAs) rebuilds T exactly in FP32
// (|T| < 2^24), applies fl(fl(T*xs)*ws) and accumulates the reads in PyTorch's
// CPU cascade order in registers (simulator.py:578-585), so no partial ever
// reaches HBM.
//
// Warp roles (128 + 32 * EPI_WARPS threads, 1 CTA per SM, 128 rows x 128 columns per CTA):
//   warp 0      TMA producer: code tiles of x [128 x 32] and w [128 x 32] per read
//   warp 1      TMEM owner and MMA issuer (one elected thread)
//   warps 2-3   transform: digit planes in shared memory (elementwise on the
//               swizzled tiles), conditional-pair flags, per-read scale rings
//   warps 4..   epilogue: EPI_WARPS / 4 warps per TMEM lane quadrant, EC columns
//               of every 32-column job each; cascade level 0 in registers,
//               level 1 in shared memory
// Every mbarrier wait is bounded; on timeout the CTA records an error code,
// waits (bounded) for its own TMA loads and MMAs, frees its TMEM and exits.
#include <cuda.h>
#include <cuda_runtime.h>
#include <string.h>

#include "common.cuh"
#include "kernels.cuh"
#include "tcgen05.cuh"

namespace mf {
namespace tc {

constexpr int BM = 128;          // vectors per CTA (TMEM lanes)
constexpr int BN = 128;          // output columns per CTA
constexpr int SUB = 32;          // columns per MMA job
constexpr int NSUB = BN / SUB;   // jobs per read; job j runs on TMEM half j & 1
constexpr int KR = 32;           // rows per read (MMA K for 8-bit operands)
constexpr int STAGES = 4;
constexpr int RING = 8;          // per-read flag ring
constexpr int SCB = 4;           // reads per scale block
constexpr int SCRING = 4;        // scale blocks in flight
constexpr int MAXPA = 3;         // max clip-capable input-slice planes
constexpr int MAXPB = 4;         // max clip-capable weight-slice planes
constexpr int EPI_WARPS = 16;    // epilogue warps: EPI_WARPS / 4 per TMEM lane quadrant
constexpr int EC = SUB / (EPI_WARPS / 4);   // columns of a job per epilogue thread
constexpr int THREADS = 128 + 32 * EPI_WARPS;
constexpr int TILE = BM * KR;    // 4096 bytes: one [128 x 32] 8-bit tile
constexpr int HALF_COLS = 256;   // TMEM columns per half
// Register split between warpgroup 0 (producer, MMA, transform) and the two
// epilogue warpgroups.  setmaxnreg.inc draws on the registers the block was
// launched with, so 128 * REG_LOW + 32 * EPI_WARPS * REG_HIGH must not exceed
// THREADS * (registers per thread at launch); the host checks this before
// every launch (launch_tc), because an increase that cannot be met never returns.
constexpr int LAUNCH_REGS = (65536 / THREADS) / 8 * 8;
constexpr int REG_LOW = EPI_WARPS == 16 ? 56 : 88;
constexpr int REG_HIGH = EPI_WARPS == 16 ? 104 : 208;
static_assert(128 * REG_LOW + 32 * EPI_WARPS * REG_HIGH <= THREADS * LAUNCH_REGS,
              "register split exceeds the launch pool");

// Shared memory plan (1024-aligned tiles first).
struct Smem {
    uint8_t x[STAGES][TILE];                        // TMA: activation codes [128 rows][32 B]
    uint8_t w[STAGES][TILE];                        // TMA: weight codes, K-major [128 cols][32 B]
    uint8_t ap[STAGES][MAXPA][TILE];                // A digit planes
    uint8_t bp[STAGES][NSUB][MAXPB][SUB * KR];      // B digit planes [job][plane][32 rows][32 B]
    float acc1[BN][BM];                             // cascade level 1, [column][row]
    float xs[SCRING][BM][SCB];                      // TMA: input scales [row][read]
    float ws[SCRING][SCB][BN];                      // TMA: weight scales [read][column]
    uint32_t flags[RING][2];                        // one word per transform warp
    uint32_t pbits[RING][2];                        // always-plane clip bounds (see transform)
    uint64_t full[STAGES], ready[STAGES], empty[STAGES];
    uint64_t flag_full[RING], flag_empty[RING];
    uint64_t sc_full[SCRING], sc_empty[SCRING];
    uint64_t unit_full[2], unit_empty[2];
    uint64_t drained;
    uint32_t tmem_base;
    int abort;
};
static_assert(sizeof(Smem) + 1024 <= 232448, "tcgen05 kernel exceeds the 227 KB shared-memory limit");

struct Plan {
    int na, nwa, nwc;                  // A planes, always-W planes, conditional-W planes
    int a_shift[MAXPA], a_mask[MAXPA];
    int w_shift[MAXPB], w_mask[MAXPB]; // always planes first, then conditional
    float coef[MAXPA][MAXPB];          // -(s_a s_w) * 2^k_w
    float dscale[MAXPB];               // 2^(18 - k_w)
    float offset[MAXPB];               // -m_w * 2^-k_w
    float thresh[MAXPB];               // m_w * 2^-18: D * 2^-18 above it clips
    int row_limit;                     // conditional: flag a row when S_a(n) > row_limit
    int col_limit[MAXPB];              // plane q can clip in column o only if S_wq(o) > col_limit[q]
    int prow_limit[MAXPB];             // plane q can clip in row n only if max_a S_a(n) > prow_limit[q]
    int b_signed;                      // weight codes signed (s8) or unsigned (u8)
};

struct Args {
    Plan plan;
    const float* bias;      // [out_features] or null
    float* out;
    long long n, ldo;
    int out_features, MR;
    long long full;         // reads in complete 16-read cascade blocks
    int col_begin;          // first output column of this call (tile_begin * C)
    int col_end;            // one past the last column (tile_end * C)
    unsigned* error;        // device error word
    int raster;             // 0: blockIdx.x walks vector blocks; 1: blockIdx.x walks column blocks
};

using namespace tg;

__device__ __forceinline__ float fma_sat(float a, float b, float c) {
    float d;
    asm("fma.rn.sat.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}


__device__ __forceinline__ bool job_flagged(int nwc, uint32_t f0, uint32_t f1, int j) {
    const uint32_t f = f0 | f1;
    return nwc > 0 && (f & 1u) && (f & (2u << j));
}

// T is kept as packed FP32 pairs (b64) so the f32x2 instructions need no moves.
// T from the x.w accumulator: |x.w| < 2^22, so 1.5*2^23 + x.w holds the integer
// exactly in its mantissa and subtracting 1.5*2^23 recovers it.
template <int E>
__device__ __forceinline__ void base_to_float(const uint32_t (&v)[E], uint64_t (&T)[E / 2]) {
    const uint64_t magic = 0xCB400000CB400000ull;    // (-1.5*2^23, -1.5*2^23)
#pragma unroll
    for (int e = 0; e < E / 2; ++e)
        asm("{\n\t.reg .b32 a, b;\n\t.reg .b64 p;\n\t"
            "add.s32 a, %1, 0x4B400000;\n\t"
            "add.s32 b, %2, 0x4B400000;\n\t"
            "mov.b64 p, {a, b};\n\t"
            "add.rn.f32x2 %0, p, %3;\n\t}"
            : "=l"(T[e])
            : "r"(v[2 * e]), "r"(v[2 * e + 1]), "l"(magic));
}

// T -= s_a s_w relu(D - m) for one pair plane; D arrives as D * 2^-18, and
// fma.sat gives relu(D - m) * 2^-k exactly (k chosen on the host).
template <int E>
__device__ __forceinline__ void relu_correct(const uint32_t (&v)[E], uint64_t (&T)[E / 2], float ds, float off,
                                             float cf) {
    uint64_t c2;
    asm("mov.b64 %0, {%1, %1};" : "=l"(c2) : "f"(cf));
#pragma unroll
    for (int e = 0; e < E / 2; ++e)
        asm("{\n\t.reg .f32 y0, y1;\n\t.reg .b64 y;\n\t"
            "fma.rn.sat.f32 y0, %1, %3, %4;\n\t"
            "fma.rn.sat.f32 y1, %2, %3, %4;\n\t"
            "mov.b64 y, {y0, y1};\n\t"
            "fma.rn.f32x2 %0, y, %5, %0;\n\t}"
            : "+l"(T[e])
            : "f"(__uint_as_float(v[2 * e])), "f"(__uint_as_float(v[2 * e + 1])), "f"(ds), "f"(off), "l"(c2));
}

__device__ __forceinline__ float2 unpack(uint64_t t) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(t));
    return r;
}

__device__ __forceinline__ float max3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// Largest D * 2^-18 over this thread's E columns of NA input-slice planes (all
// values are non-negative and exact, so comparing it with m * 2^-18 tells
// exactly whether any of them clips).
template <int NA, int E>
__device__ __forceinline__ float planes_max(const uint32_t (&v)[NA > 0 ? NA : 1][E]) {
    float m[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
        if (NA >= 3) {
            m[e] = max3(__uint_as_float(v[0][e]), __uint_as_float(v[1][e]), __uint_as_float(v[2][e]));
#pragma unroll
            for (int a = 3; a < NA; ++a) m[e] = fmaxf(m[e], __uint_as_float(v[a][e]));
        } else {
            m[e] = __uint_as_float(v[0][e]);
#pragma unroll
            for (int a = 1; a < NA; ++a) m[e] = fmaxf(m[e], __uint_as_float(v[a][e]));
        }
    }
    if (E == 16) {
        const float t0 = max3(m[0], m[1], m[2]), t1 = max3(m[3], m[4], m[5]), t2 = max3(m[6], m[7], m[8]);
        const float t3 = max3(m[9], m[10], m[11]), t4 = max3(m[12], m[13], m[14]);
        return fmaxf(max3(t0, t1, t2), max3(t3, t4, m[E - 1]));
    }
    const float t0 = max3(m[0], m[1], m[2]), t1 = max3(m[3], m[4], m[5]);
    return max3(t0, t1, fmaxf(m[6], m[7]));
}

// ------------------------------------------------------------------- kernel
// NA / NWA / NWC: plan sizes (clip-capable input planes, always and conditional
// weight planes).  A job's TMEM unit on its half: base x.w at column 0 (32 cols),
// always group a at 32 + 64a (NWA x 32 cols); a conditional unit (flagged jobs
// only) reuses the half with group a at 64a.
template <int NA, int NWA, int NWC>
__global__ void __launch_bounds__(THREADS, 1)
    tc_ideal_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                    const __grid_constant__ CUtensorMap map_xs, const __grid_constant__ CUtensorMap map_ws,
                    const Args args) {
    static_assert(NA <= MAXPA && NWA + NWC <= MAXPB, "plan exceeds shared-memory planes");
    static_assert(32 + NA * NWA * SUB <= HALF_COLS && NA * NWC * SUB <= HALF_COLS, "unit exceeds a TMEM half");
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    Smem& s = *reinterpret_cast<Smem*>(smem_align1024(smem_raw));
    const Plan& P = args.plan;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long n0 = (long long)raster_vector_block(args.raster) * BM;
    const int c0 = args.col_begin + raster_column_block(args.raster) * BN;   // first output column of this CTA
    const int MR = args.MR;
    unsigned* err = args.error;

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.ready[i], 2);
            mbar_init(&s.empty[i], 1);
        }
        for (int i = 0; i < RING; ++i) {
            mbar_init(&s.flag_full[i], 2);
            mbar_init(&s.flag_empty[i], EPI_WARPS);
        }
        for (int i = 0; i < SCRING; ++i) {
            mbar_init(&s.sc_full[i], 1);
            mbar_init(&s.sc_empty[i], EPI_WARPS);
        }
        for (int h = 0; h < 2; ++h) {
            mbar_init(&s.unit_full[h], 1);
            mbar_init(&s.unit_empty[h], EPI_WARPS);
        }
        mbar_init(&s.drained, 1);
        s.abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int idx = threadIdx.x; idx < BN * BM; idx += THREADS) (&s.acc1[0][0])[idx] = 0.0f;
    if (warp == 0 && lane == 0) {
        prefetch_map(&map_x);
        prefetch_map(&map_w);
        prefetch_map(&map_xs);
        prefetch_map(&map_ws);
    }
    if (warp == 1) {
        tmem_alloc(&s.tmem_base, 512);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s.tmem_base;

    if (warp < 4) {
        set_maxnreg_dec<REG_LOW>();
        if (warp == 0) {
            // -------------------------------------------------------- producer
            if (lane == 0) {
                int issued = 0, scissued = 0;
                for (int i = 0; i < MR; ++i) {
                    if (i % SCB == 0) {
                        const int b = i / SCB, sb = b % SCRING;
                        if (!mbar_wait(&s.sc_empty[sb], ((b / SCRING) & 1) ^ 1, &s.abort, err, 12)) break;
                        mbar_expect_tx(&s.sc_full[sb], (BM + BN) * SCB * 4);
                        tma_load_2d(s.xs[sb], &map_xs, i, (int)n0, &s.sc_full[sb]);
                        tma_load_2d(s.ws[sb], &map_ws, c0, i, &s.sc_full[sb]);
                        scissued = b + 1;
                    }
                    const int st = i % STAGES;
                    if (!mbar_wait(&s.empty[st], ((i / STAGES) & 1) ^ 1, &s.abort, err, 1)) break;
                    mbar_expect_tx(&s.full[st], 2 * TILE);
                    tma_load_2d(s.x[st], &map_x, i * KR, (int)n0, &s.full[st]);
                    tma_load_2d(s.w[st], &map_w, i * KR, c0, &s.full[st]);
                    issued = i + 1;
                }
                // Every issued load lands before the CTA may exit.
                for (int i = issued - STAGES > 0 ? issued - STAGES : 0; i < issued; ++i)
                    mbar_drain(&s.full[i % STAGES], (i / STAGES) & 1);
                for (int b = scissued - SCRING > 0 ? scissued - SCRING : 0; b < scissued; ++b)
                    mbar_drain(&s.sc_full[b % SCRING], (b / SCRING) & 1);
            }
        } else if (warp == 1) {
            // -------------------------------------------------------- MMA issuer
            if (lane == 0) {
                const uint32_t id_base = idesc_i8(BM, SUB, true, P.b_signed != 0);
                const uint32_t id_always = idesc_e4m3(BM, SUB * (NWA > 0 ? NWA : 1));
                const uint32_t id_cond = idesc_e4m3(BM, SUB * (NWC > 0 ? NWC : 1));
                uint32_t units = 0;   // units issued; unit u uses buffer u & 1
                bool ok = true;
                for (int i = 0; i < MR && ok; ++i) {
                    const int st = i % STAGES;
                    if (!mbar_wait(&s.ready[st], (i / STAGES) & 1, &s.abort, err, 2)) break;
                    tc_fence_after();
                    const uint32_t f0 = *(volatile uint32_t*)&s.flags[i % RING][0];
                    const uint32_t f1 = *(volatile uint32_t*)&s.flags[i % RING][1];
                    const uint64_t dx = desc_sw32(s.x[st]);
#pragma unroll
                    for (int j = 0; j < NSUB; ++j) {
                        uint32_t b = units & 1;
                        if (!mbar_wait(&s.unit_empty[b], ((units >> 1) & 1) ^ 1, &s.abort, err, 3)) { ok = false; break; }
                        tc_fence_after();
                        uint32_t buf = tmem + b * HALF_COLS;
                        mma_i8(buf, dx, desc_sw32(s.w[st] + j * SUB * KR), id_base, 0);
#pragma unroll
                        for (int a = 0; a < NA; ++a)
                            mma_f8(buf + 32 + a * NWA * SUB, desc_sw32(s.ap[st][a]), desc_sw32(s.bp[st][j][0]),
                                   id_always, 0);
                        mma_commit(&s.unit_full[b]);
                        ++units;
                        if (NWC > 0 && job_flagged(NWC, f0, f1, j)) {
                            b = units & 1;
                            if (!mbar_wait(&s.unit_empty[b], ((units >> 1) & 1) ^ 1, &s.abort, err, 4)) { ok = false; break; }
                            tc_fence_after();
                            buf = tmem + b * HALF_COLS;
#pragma unroll
                            for (int a = 0; a < NA; ++a)
                                mma_f8(buf + a * NWC * SUB, desc_sw32(s.ap[st][a]), desc_sw32(s.bp[st][j][NWA]),
                                       id_cond, 0);
                            mma_commit(&s.unit_full[b]);
                            ++units;
                        }
                    }
                    if (ok) mma_commit(&s.empty[st]);
                }
                // All issued MMAs complete before TMEM is released.
                mma_commit(&s.drained);
                mbar_drain(&s.drained, 0);
            }
        } else {
            // -------------------------------------------------------- transform
            const int tw = warp - 2;              // 0 or 1
            for (int i = 0; i < MR; ++i) {
                const int st = i % STAGES, rs = i % RING;
                bool ok = mbar_wait(&s.full[st], (i / STAGES) & 1, &s.abort, err, 5);
                ok = ok && mbar_wait(&s.flag_empty[rs], ((i / RING) & 1) ^ 1, &s.abort, err, 6);
                if (!__all_sync(0xFFFFFFFFu, ok)) break;
                uint32_t word = 0, bits = 0;
#pragma unroll 1
                for (int hh = 0; hh < 2; ++hh) {
                    const int t = tw * 32 + lane + 64 * hh;   // A row t and B column t (0..127)
                    // Row t of a [128 x 32] SW32 tile keeps both 16-byte chunks inside the
                    // row, so an elementwise transform written at the same offsets stays swizzled.
                    const uint4* xrow = reinterpret_cast<const uint4*>(s.x[st] + t * KR);
                    const uint4 xa = xrow[0], xb = xrow[1];
                    const uint32_t xw[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
                    uint32_t rowmax = 0;   // max over clip-capable A slices of the read's digit sum
#pragma unroll
                    for (int a = 0; a < NA; ++a) {
                        const uint32_t m4 = (uint32_t)P.a_mask[a] * 0x01010101u;
                        uint32_t d[8], sum = 0;
#pragma unroll
                        for (int k = 0; k < 8; ++k) {
                            d[k] = (xw[k] >> P.a_shift[a]) & m4;
                            sum = __dp4a(d[k], 0x01010101u, sum);
                        }
                        uint4* dst = reinterpret_cast<uint4*>(s.ap[st][a] + t * KR);
                        dst[0] = make_uint4(d[0], d[1], d[2], d[3]);
                        dst[1] = make_uint4(d[4], d[5], d[6], d[7]);
                        rowmax = sum > rowmax ? sum : rowmax;
                    }
                    if (n0 + t >= args.n) rowmax = 0;
                    const uint4* wrow = reinterpret_cast<const uint4*>(s.w[st] + t * KR);
                    const uint4 wa = wrow[0], wb = wrow[1];
                    const uint32_t ww[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
                    bool colflag = false;
                    const int job = t >> 5, quad = t >> 5;   // this warp's rows form quadrant t>>5
#pragma unroll
                    for (int q = 0; q < NWA + NWC; ++q) {
                        const uint32_t m4 = (uint32_t)P.w_mask[q] * 0x01010101u;
                        uint32_t d[8], sum = 0;
#pragma unroll
                        for (int k = 0; k < 8; ++k) {
                            d[k] = (ww[k] >> P.w_shift[q]) & m4;
                            sum = __dp4a(d[k], 0x01010101u, sum);
                        }
                        uint4* dst = reinterpret_cast<uint4*>(s.bp[st][job][q] + (t & 31) * KR);
                        dst[0] = make_uint4(d[0], d[1], d[2], d[3]);
                        dst[1] = make_uint4(d[4], d[5], d[6], d[7]);
                        const bool cbig = (int)sum > P.col_limit[q];
                        if (q >= NWA) {
                            colflag |= cbig;
                        } else {
                            // Plane q can clip in this (row quadrant, column job) only if some row
                            // and some column both exceed their digit-sum limits.
                            if (__any_sync(0xFFFFFFFFu, cbig)) bits |= 1u << (16 + job * 4 + q);
                            if (__any_sync(0xFFFFFFFFu, (int)rowmax > P.prow_limit[q])) bits |= 1u << (quad * 4 + q);
                        }
                    }
                    const bool rowflag = NWC > 0 && (int)rowmax > P.row_limit;
                    if (__any_sync(0xFFFFFFFFu, rowflag)) word |= 1u;
                    if (__any_sync(0xFFFFFFFFu, colflag)) word |= 2u << job;
                }
                if (lane == 0) {
                    s.flags[rs][tw] = word;
                    s.pbits[rs][tw] = bits;
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&s.ready[st]);
                    mbar_arrive(&s.flag_full[rs]);
                }
            }
        }
    } else {
        set_maxnreg_inc<REG_HIGH>();
        // ------------------------------------------------------------ epilogue
        // Every epilogue warp consumes every unit: warp w reads TMEM lane quadrant w & 3
        // and the EC-column slice hc of each 32-column job.  Two TMEM buffers alternate,
        // so the MMA fills one while the epilogue drains the other.
        const int quad = warp & 3;
        const int hc = (warp - 4) >> 2;             // which EC-column slice of every job
        const int r = quad * 32 + lane;             // CTA row = TMEM lane
        const long long row = n0 + r;
        const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16) + hc * EC;
        float acc0[NSUB][EC];
#pragma unroll
        for (int j = 0; j < NSUB; ++j)
#pragma unroll
            for (int e = 0; e < EC; ++e) acc0[j][e] = 0.0f;
        uint32_t units = 0;
        bool ok = true;
        for (int i = 0; i < MR && ok; ++i) {
            const int rs = i % RING, b = i / SCB, sb = b % SCRING;
            if (i % SCB == 0) {
                ok = __all_sync(0xFFFFFFFFu, mbar_wait(&s.sc_full[sb], (b / SCRING) & 1, &s.abort, err, 13));
                if (!ok) break;
            }
            ok = __all_sync(0xFFFFFFFFu, mbar_wait(&s.flag_full[rs], (i / RING) & 1, &s.abort, err, 7));
            if (!ok) break;
            const float xs = s.xs[sb][r][i % SCB];
            const uint32_t f0 = *(volatile uint32_t*)&s.flags[rs][0];
            const uint32_t f1 = *(volatile uint32_t*)&s.flags[rs][1];
            const uint32_t pb = *(volatile uint32_t*)&s.pbits[rs][0] | *(volatile uint32_t*)&s.pbits[rs][1];
            // Jobs share one copy of the TMEM/correction code (a runtime loop keeps the hot
            // code small enough for the instruction cache); only the register-resident
            // scale-and-accumulate step is specialised per job.
#pragma unroll 1
            for (int j = 0; j < NSUB; ++j) {
                const bool flagged = NWC > 0 && job_flagged(NWC, f0, f1, j);
                uint32_t bsel = units & 1;
                ok = __all_sync(0xFFFFFFFFu, mbar_wait(&s.unit_full[bsel], (units >> 1) & 1, &s.abort, err, 9));
                if (!ok) break;
                tc_fence_after();
                uint32_t buf = lane_base + bsel * HALF_COLS;
                uint64_t T[EC / 2];
                {
                    // Base x.w and the first always plane of every input slice in one batch.
                    uint32_t vt[EC], v0[NA > 0 ? NA : 1][EC];
                    tmem_ld(buf, vt);
#pragma unroll
                    for (int a = 0; a < NA; ++a) tmem_ld(buf + 32 + a * NWA * SUB, v0[a]);
                    tmem_wait(vt);
#pragma unroll
                    for (int a = 0; a < NA; ++a) tmem_wait(v0[a]);
                    base_to_float(vt, T);
                    // Corrections only where some D of the warp exceeds m (the relu is zero
                    // elsewhere, so skipping it there changes nothing).
                    if (NWA > 0 && ((pb >> (quad * 4)) & 1u) && ((pb >> (16 + j * 4)) & 1u) &&
                        __any_sync(0xFFFFFFFFu, planes_max<NA, EC>(v0) > P.thresh[0])) {
#pragma unroll
                        for (int a = 0; a < NA; ++a) relu_correct(v0[a], T, P.dscale[0], P.offset[0], P.coef[a][0]);
                    }
                }
#pragma unroll
                for (int q = 1; q < NWA; ++q) {
                    // Further always planes: skipped when no row of this quadrant and no column of
                    // this job can exceed the plane's ADC limit.
                    if (((pb >> (quad * 4 + q)) & 1u) && ((pb >> (16 + j * 4 + q)) & 1u)) {
                        uint32_t v1[NA > 0 ? NA : 1][EC];
#pragma unroll
                        for (int a = 0; a < NA; ++a) tmem_ld(buf + 32 + (a * NWA + q) * SUB, v1[a]);
#pragma unroll
                        for (int a = 0; a < NA; ++a) tmem_wait(v1[a]);
                        if (__any_sync(0xFFFFFFFFu, planes_max<NA, EC>(v1) > P.thresh[q])) {
#pragma unroll
                            for (int a = 0; a < NA; ++a)
                                relu_correct(v1[a], T, P.dscale[q], P.offset[q], P.coef[a][q]);
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&s.unit_empty[bsel]);
                ++units;
                if (flagged) {
                    bsel = units & 1;
                    ok = __all_sync(0xFFFFFFFFu, mbar_wait(&s.unit_full[bsel], (units >> 1) & 1, &s.abort, err, 10));
                    if (!ok) break;
                    tc_fence_after();
                    buf = lane_base + bsel * HALF_COLS;
#pragma unroll
                    for (int q = 0; q < NWC; ++q) {
                        uint32_t v1[NA > 0 ? NA : 1][EC];
#pragma unroll
                        for (int a = 0; a < NA; ++a) tmem_ld(buf + (a * NWC + q) * SUB, v1[a]);
#pragma unroll
                        for (int a = 0; a < NA; ++a) tmem_wait(v1[a]);
#pragma unroll
                        for (int a = 0; a < NA; ++a)
                            relu_correct(v1[a], T, P.dscale[NWA + q], P.offset[NWA + q], P.coef[a][NWA + q]);
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&s.unit_empty[bsel]);
                    ++units;
                }
                // fl(fl(T * xs) * ws) pushed into cascade level 0 for read i: packed
                // round-to-nearest multiplies, then SCALAR adds (a packed multiply
                // followed by a packed add was observed to round once, as an FMA,
                // which the reference does not).
                const float2* wsr = reinterpret_cast<const float2*>(&s.ws[sb][i % SCB][j * SUB + hc * EC]);
                float v[EC];
#pragma unroll
                for (int e = 0; e < EC / 2; ++e) {
                    const float2 w2 = wsr[e];
                    const float2 t2 = unpack(T[e]);
                    const float2 pr = __fmul2_rn(__fmul2_rn(t2, make_float2(xs, xs)), w2);
                    v[2 * e] = pr.x;
                    v[2 * e + 1] = pr.y;
                }
                switch (j) {
#define MF_ACC(J)                                                         \
    case J:                                                               \
        _Pragma("unroll") for (int e = 0; e < EC; ++e) acc0[J][e] = __fadd_rn(acc0[J][e], v[e]); \
        break;
                    MF_ACC(0)
                    MF_ACC(1)
                    MF_ACC(2)
                    MF_ACC(3)
#undef MF_ACC
                }
            }
            if (!ok) break;
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&s.flag_empty[rs]);
                if (i % SCB == SCB - 1 || i == MR - 1) mbar_arrive(&s.sc_empty[sb]);
            }
            // Block boundary of the 16-read cascade: level 1 += level 0 (MR <= 256 keeps two levels).
            const int done = i + 1;
            if (done <= args.full && (done & 15) == 0) {
#pragma unroll
                for (int j = 0; j < NSUB; ++j)
#pragma unroll
                    for (int e = 0; e < EC; ++e) {
                        const int cl = j * SUB + hc * EC + e;
                        s.acc1[cl][r] = __fadd_rn(s.acc1[cl][r], acc0[j][e]);
                        acc0[j][e] = 0.0f;
                    }
            }
        }
        if (ok && row < args.n) {
#pragma unroll
            for (int j = 0; j < NSUB; ++j)
#pragma unroll
                for (int e = 0; e < EC; ++e) {
                    const int cl = j * SUB + hc * EC + e;
                    const int col = c0 + cl;
                    if (col >= args.col_end || col >= args.out_features) continue;
                    // acc0 + acc1 + acc2 + acc3 (upper levels zero), then the reference's
                    // store into a zero-filled output.
                    float value = __fadd_rn(acc0[j][e], s.acc1[cl][r]);
                    value = __fadd_rn(value, 0.0f);
                    value = __fadd_rn(value, 0.0f);
                    value = __fadd_rn(0.0f, value);
                    if (args.bias) value = __fadd_rn(value, args.bias[col]);
                    args.out[row * args.ldo + col] = value;
                }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

}  // namespace tc

// =================================================================== host side
// Host-side plan: which slice pairs can clip and how the epilogue undoes them.
bool tc_plan(const mf_config& c, tc::Plan& P) {
    memset(&P, 0, sizeof(P));
    const int rows = c.read_rows;
    int amask = -1;
    int clip_a[MF_MAX_SLICES], na = 0;
    bool pair_clip[MF_MAX_SLICES][MF_MAX_SLICES];
    for (int a = 0; a < c.n_in; ++a)
        for (int w = 0; w < c.n_w; ++w)
            pair_clip[a][w] = (long long)rows * c.in_mask[a] * c.w_mask[w] > c.adc_max[w];
    for (int a = 0; a < c.n_in; ++a) {
        bool any = false;
        for (int w = 0; w < c.n_w; ++w) any |= pair_clip[a][w];
        if (!any) continue;
        if (amask >= 0 && c.in_mask[a] != amask) return false;  // product set needs one A digit width
        amask = c.in_mask[a];
        clip_a[na++] = a;
    }
    if (na > tc::MAXPA) return false;
    // Every clip-capable A slice must pair with the same W set.
    int always[MF_MAX_SLICES], cond[MF_MAX_SLICES], nwa = 0, nwc = 0;
    for (int w = 0; w < c.n_w; ++w) {
        bool first = na ? pair_clip[clip_a[0]][w] : false;
        for (int i = 1; i < na; ++i)
            if (pair_clip[clip_a[i]][w] != first) return false;
        if (!first) continue;
        const long long dmax = (long long)rows * amask * c.w_mask[w];
        if (c.adc_max[w] * 4 >= dmax * 3) cond[nwc++] = w;
        else always[nwa++] = w;
    }
    for (int a = 0; a < c.n_in; ++a) {
        bool listed = false;
        for (int i = 0; i < na; ++i) listed |= clip_a[i] == a;
        for (int w = 0; w < c.n_w; ++w)
            if (pair_clip[a][w] && !listed) return false;
    }
    if (na == 0) nwa = nwc = 0;
    if (nwa + nwc > tc::MAXPB || (na > 0 && nwa == 0 && nwc == 0)) return false;
    if (na > 0 && nwa == 0) return false;   // keep at least one always group (simplifies the slot walk)
    P.na = na;
    P.nwa = nwa;
    P.nwc = nwc;
    for (int i = 0; i < na; ++i) {
        P.a_shift[i] = c.in_shift[clip_a[i]];
        P.a_mask[i] = c.in_mask[clip_a[i]];
    }
    int order[tc::MAXPB];
    for (int i = 0; i < nwa; ++i) order[i] = always[i];
    for (int i = 0; i < nwc; ++i) order[nwa + i] = cond[i];
    P.row_limit = 1 << 30;
    for (int q = 0; q < nwa + nwc; ++q) {
        const int w = order[q];
        P.w_shift[q] = c.w_shift[w];
        P.w_mask[q] = c.w_mask[w];
        const long long dmax = (long long)rows * amask * c.w_mask[w];
        const long long span = dmax - c.adc_max[w];
        int k = 0;
        while ((1LL << k) < span) ++k;
        P.dscale[q] = ldexpf(1.0f, 18 - k);
        P.offset[q] = -ldexpf((float)c.adc_max[w], -k);
        P.thresh[q] = ldexpf((float)c.adc_max[w], -18);
        for (int i = 0; i < na; ++i)
            P.coef[i][q] = -(float)(c.in_factor[clip_a[i]] * c.w_factor[w]) * ldexpf(1.0f, k);
        // D <= Mw * S_a(n) and D <= Ma * S_w(o): below these limits plane q cannot clip.
        P.prow_limit[q] = c.adc_max[w] / c.w_mask[w];
        P.col_limit[q] = c.adc_max[w] / amask;
        if (q >= nwa) P.row_limit = P.prow_limit[q] < P.row_limit ? P.prow_limit[q] : P.row_limit;
    }
    return true;
}

// Plan shapes with a compiled kernel: (NA, NWA, NWC).
static bool tc_shape_supported(int na, int nwa, int nwc) {
    return (na == 3 && nwa == 2 && nwc == 2) ||
           (na == 3 && nwa == 2 && nwc == 0) || (na == 3 && nwa == 1 && nwc == 0) ||
           (na == 3 && nwa == 1 && nwc == 2) || (na == 0 && nwa == 0 && nwc == 0);
}

bool tc_eligible(const mf_config& c, int32_t m) {
    if (!c.ideal || !exact_integer_counts(c) || c.wide || c.wide_codes) return false;
    if (c.activation_bits != 8 || c.weight_bits != 8) return false;
    if (c.read_rows != tc::KR || c.rows % tc::KR) return false;
    for (int i = 0; i < c.n_in; ++i)
        if (c.in_mask[i] > 7) return false;
    for (int i = 0; i < c.n_w; ++i)
        if (c.w_mask[i] > 7) return false;
    const long long MR = (long long)m * c.reads;
    if (MR > 256 || MR % tc::SCB) return false;
    if (reconstruction_bound(c) >= 16777216.0) return false;
    tc::Plan P;
    if (!tc_plan(c, P)) return false;
    return tc_shape_supported(P.na, P.nwa, P.nwc);
}

int tc_block_threads() { return tc::THREADS; }

size_t tc_workspace_bytes(const mf_config& c, int32_t m, int32_t p) {
    return (size_t)p * c.cols * m * c.rows + 256;
}

template <int NA, int NWA, int NWC>
static mf_status launch_tc(const CUtensorMap& mx, const CUtensorMap& mw, const CUtensorMap& mxs,
                           const CUtensorMap& mws, const tc::Args& args, dim3 grid, cudaStream_t st) {
    const size_t smem = sizeof(tc::Smem) + 1024;
    auto kern = tc::tc_ideal_kernel<NA, NWA, NWC>;
    int regs = 0;
    {
        const mf_status r = kernel_setup(reinterpret_cast<const void*>(kern), smem, &regs);
        if (r) return r;
    }
    // Registers are allocated per thread in multiples of 8.
    const long long pool = (long long)((regs + 7) / 8 * 8) * tc::THREADS;
    const long long split = 128LL * tc::REG_LOW + 32LL * tc::EPI_WARPS * tc::REG_HIGH;
    if (split > pool) {
        set_error("tcgen05 kernel launched with %d registers/thread cannot host the %d/%d register split",
                  regs, tc::REG_LOW, tc::REG_HIGH);
        return MF_ERR_RESOURCE;
    }
    kern<<<grid, tc::THREADS, smem, st>>>(mx, mw, mxs, mws, args);
    MF_LAUNCH_CHECK("tc_ideal_kernel");
    return MF_OK;
}

mf_status tc_sliced_mm(const mf_config& c, const MMArgs& a, void* workspace, size_t ws_bytes, cudaStream_t st) {
    int dev = 0;
    MF_CHECK_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
    int major = 0;
    MF_CHECK_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev), "capability");
    if (major != 10) {
        set_error("tcgen05 path needs an sm_100 device");
        return MF_ERR_UNSUPPORTED;
    }
    const size_t need = tc_workspace_bytes(c, a.m, a.p);
    if (ws_bytes < need || !workspace) {
        set_error("tcgen05 workspace too small: %zu < %zu bytes", ws_bytes, need);
        return MF_ERR_RESOURCE;
    }
    tc::Args args{};
    if (!tc_plan(c, args.plan) || !tc_shape_supported(args.plan.na, args.plan.nwa, args.plan.nwc)) {
        set_error("configuration outside the tcgen05 plan");
        return MF_ERR_UNSUPPORTED;
    }
    args.plan.b_signed = c.weight_signed;
    const long long K = (long long)a.m * c.rows;
    const long long O = (long long)a.p * c.cols;
    const int MR = a.m * c.reads;
    uint8_t* wk = static_cast<uint8_t*>(workspace);
    mf_status r = a.kmajor_ready ? MF_OK : tc_weights_kmajor(a.packed, wk, a.m, a.p, c.rows, c.cols, st);
    if (r) return r;
    CUtensorMap mx, mw, mxs, mws;
    r = tc_make_map(&mx, a.codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)K, (uint64_t)a.n, (uint64_t)K,
                           tc::KR, tc::BM, CU_TENSOR_MAP_SWIZZLE_32B);
    if (!r) r = tc_make_map(&mw, wk, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)K, (uint64_t)O, (uint64_t)K, tc::KR,
                         tc::BN, CU_TENSOR_MAP_SWIZZLE_32B);
    // Scales: xscale [n, MR] -> boxes [128 rows][4 reads]; wscale [MR, O] -> [4 reads][128 cols].
    if (!r) r = tc_make_map(&mxs, a.xscale, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)MR, (uint64_t)a.n,
                         (uint64_t)MR, tc::SCB, tc::BM, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (!r) r = tc_make_map(&mws, a.wscale, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)O, (uint64_t)MR, (uint64_t)O,
                         tc::BN, tc::SCB, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (r) return r;
    unsigned* err = nullptr;
    r = tc_error_word(&err);
    if (r) return r;
    args.bias = static_cast<const float*>(a.bias);
    args.out = static_cast<float*>(a.out);
    args.n = a.n;
    args.ldo = a.ldo;
    args.out_features = a.out_features;
    args.MR = MR;
    args.full = (long long)MR - MR % 16;
    args.col_begin = a.tile_begin * c.cols;
    args.col_end = a.tile_end * c.cols;
    args.error = err;
    args.raster = a.raster;
    const long long cols = (long long)(a.tile_end - a.tile_begin) * c.cols;
    const dim3 grid = raster_grid((a.n + tc::BM - 1) / tc::BM, (cols + tc::BN - 1) / tc::BN, a.raster);
    const tc::Plan& P = args.plan;
#define MF_TC(NA_, NWA_, NWC_) \
    if (P.na == NA_ && P.nwa == NWA_ && P.nwc == NWC_) return launch_tc<NA_, NWA_, NWC_>(mx, mw, mxs, mws, args, grid, st)
    MF_TC(3, 2, 2);
    MF_TC(3, 2, 0);
    MF_TC(3, 1, 0);
    MF_TC(3, 1, 2);
    MF_TC(0, 0, 0);
#undef MF_TC
    set_error("no compiled tcgen05 kernel for plan (%d, %d, %d)", P.na, P.nwa, P.nwc);
    return MF_ERR_UNSUPPORTED;
}


}  // namespace mf

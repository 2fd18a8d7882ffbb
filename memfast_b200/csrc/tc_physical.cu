// tcgen05 path for nonideal devices (sm_100a): the FP32 currents of every
// (input slice, weight slice) pair of every read on the tensor cores.
//
// The reference computes, per read of rows_per_read rows, the current
//     I_aw = sum_r V_a(r) (G_w(r) - LOW),    V_a = voltage * d_a / M_a
// of every slice pair, converts it with the (optionally S-shaped) ADC and
// reconstructs T = sum_aw s_a s_w count_aw (memfast/reference.py:63-117).  Here
//     I_aw = (voltage / M_a) * sum_r d_a(r) * G'_w(r),    G' = G - LOW,
// with the digit d_a exact in FP16.  G' is carried as a 22-bit fixed-point
// integer X = rint(G' * 2^s) = 2048 H + L with 11-bit halves H and L (FP16
// integers), whose products with the digits are summed in separate FP32
// accumulators: every partial sum is an integer below 2^24, so the tensor core
// accumulates both exactly, whatever its internal rounding, and the epilogue
// joins them with one round-to-nearest FMA, 2048 S_H + S_L.  (A single FP32
// accumulator of floating parts would truncate at every MMA and bias the
// currents low.)  The 1-bit configuration, whose small counts showed no flips
// either way, keeps one accumulator of two floating FP16 parts, which leaves
// room for twice the columns.  The currents then differ from the reference's
// FP32 bmm by rounding only; the ADC scales, rounds half to even and clamps as
// the reference does.
//
// Ideal devices whose counts the packed and FP8 kernels do not take (64-row
// reads, Config's 1-bit defaults, the 256 x 256 format configurations) use the
// same kernel with the weight digits as the B operand (one FP16 part): every
// product and partial sum is then a small integer, so the accumulator holds the
// exact digit dot D and the epilogue's count is min(D, m), bit-exact wherever
// exact_integer_counts holds.
//
// Scope: FP32 currents and epilogue (not Config.wide / precise_currents), input
// digits of at most 3 bits, 32- or 64-row reads, at most 256 reads per output.
// Read noise of the shared mode is folded into G' per read event by
// b_operand_kernel; in the slice-pair mode (32-row reads, no voltage noise) it
// writes one G' operand per input slice (PAIRB instantiations), whose draws are
// keyed by cell * A + a (reference.py:88-91).  Everything else (the output read
// mode among it) runs on the SIMT kernels in generic.cu.
//
// Per CTA: 128 vectors x BC = NJB * BN output columns.  Per read:
//   warp 0      TMA: the read's activation codes [128 x KR] and, for every job,
//               the FP16 tile of G' (both halves) per 16-row MMA step
//   warp 1      TMEM owner and MMA issuer: per job and input slice a, FP32
//               accumulators of NP = BN x NW columns (output-column major) per
//               half; jobs alternate between TMEM units so that the MMAs of one
//               job run while the epilogue drains another
//   warps 2-3   transform: FP16 digit planes of every input slice (byte lookup)
//   warps 4-19  epilogue: ADC of every pair, signed reconstruction,
//               fl(fl(T * xs) * ws) and PyTorch's CPU cascade over the reads
//               (simulator.py:575-586)
// Every mbarrier wait is bounded; on timeout the CTA records an error code,
// drains its own asynchronous work, frees its TMEM and exits.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <string.h>

#include <type_traits>

#include "common.cuh"
#include "kernels.cuh"
#include "tcgen05.cuh"

namespace mf {
namespace tcp {

using namespace tg;

constexpr int BM = 128;          // vectors per CTA (TMEM lanes)
constexpr int PARTS = 2;         // FP16 parts of G'
constexpr int STAGES = 2;        // TMA stages (codes + G' tiles)
constexpr int EPI_WARPS = 16;
constexpr int THREADS = 128 + 32 * EPI_WARPS;
constexpr int LAUNCH_REGS = (65536 / THREADS) / 8 * 8;
constexpr int REG_LOW = 56;
constexpr int REG_HIGH = 104;
static_assert(128 * REG_LOW + 32 * EPI_WARPS * REG_HIGH <= THREADS * LAUNCH_REGS,
              "register split exceeds the launch pool");
constexpr int MAXS = 8;          // slices per operand in the tables below

// Shared-memory and TMEM geometry of one instantiation.  A job is one input
// slice a of one BN-column block: one accumulator set of NT columns, fed by
// KS (split halves stacked along N) or 2 KS MMAs; jobs rotate over U units.
//
// VOLT (voltage noise): the A operand is no longer a digit but the noisy voltage
// d * (1 + sigma z) of every (vector, row, input slice), precomputed by
// a_operand_kernel as two FP16 parts (hi = fp16(v), lo = fp16(v - hi)) in the
// MMA's tile layout.  A stage then holds those tiles instead of the code tile,
// no digit planes are built, and each job issues the MMAs of both parts into the
// same accumulators.
// PAIRB (slice-pair read noise): G' differs per input slice, so a stage holds the
// B tiles of every input slice (NIN sets) and job (a, block) reads set a.
//
// WIDE (16-bit BFP and other configurations with more than 8 bits, Config.wide):
// the codes are int64 and the digits reach 4 bits, so digit_operand_kernel writes
// the FP16 digits of every input slice in the MMA's tile layout once per call and
// a stage loads them as VOLT loads its voltage tiles (one part); totals are int64,
// scaled by restore_scales in FP64 and summed in FP64 (simulator.py:57-66,575-586).
//
// OUTM (output-mode read noise, reference.py:107-114): a job also needs the digit
// sum S_d = sum_r d(r) of its input slice and Q = sum_r d(r)^2 G(r)^2.  The B tile
// gets a row of ones after the two halves of G' (its MMA column of the current
// accumulators is S_d) and two floating FP16 parts of G^2, which the digit-square
// planes multiply into one more accumulator of NP columns.
template <int NIN, int NW, int BN, int NJB, int KR, bool SPLIT, int NPART, bool VOLT = false, bool PAIRB = false,
          bool WIDE = false, bool OUTM = false>
struct Geo {
    static constexpr bool AOP = VOLT || WIDE;              // A tiles loaded from a precomputed operand
    static constexpr int APARTS = VOLT ? 2 : 1;            // FP16 parts of that operand
    static constexpr int ACCB = WIDE ? 8 : 4;              // bytes of a cascade value
    static constexpr int KS = KR / 16;                     // MMA K steps per read
    static constexpr int EC = BN / 4;                      // columns per epilogue thread per block
    static constexpr int NP = NW * BN;                     // accumulator columns of one half (jj * NW + w)
    static constexpr int NT = SPLIT ? (NPART * NP + 15) / 16 * 16 : (NP + 15) / 16 * 16;   // MMA N
    static constexpr int PSTRIDE = SPLIT ? NP : NT;        // B rows between the halves of a tile
    static constexpr int NTC = OUTM ? NT + 16 : NT;        // N of the current MMA (OUTM: + the ones row)
    static constexpr int NPV = OUTM ? (NP + 15) / 16 * 16 : 0;   // OUTM: columns of the Q accumulator
    static constexpr int G2ROW = NTC;                      // OUTM: first B row of the G^2 parts
    static constexpr int BROWS = OUTM ? (NTC + 2 * NP + 7) / 8 * 8
                                      : ((NPART * PSTRIDE > NT ? NPART * PSTRIDE : NT) + 7) / 8 * 8;   // B tile rows
    static constexpr int ACCS = SPLIT ? NPART : 1;         // accumulators per slice pair
    static constexpr int UNIT = NTC + NPV;                 // TMEM columns of a job
    static constexpr int U = 512 / UNIT < NJB * NIN ? 512 / UNIT : NJB * NIN;   // TMEM units
    static constexpr int BC = NJB * BN;                    // output columns per CTA
    static constexpr int VALS = NW * EC;                   // TMEM columns a thread reads per accumulator
    static constexpr int AT = BM * 32;                     // one [128 x 16] FP16 tile
    static constexpr int XB = AOP ? NIN * APARTS * KS * AT : BM * KR;   // operand tiles, or the code tile
    static constexpr int BT = BROWS * 32;                  // one [BROWS x 16] FP16 tile (both halves)
    // A TMA box has at most 256 rows: taller B tiles load as two boxes of BBOX rows.
    static constexpr int BLOADS = BROWS > 256 ? 2 : 1;
    static constexpr int BBOX = BROWS / BLOADS;
    static constexpr int BSETS = PAIRB ? NIN : 1;           // B tile sets per stage
    static constexpr int BB = BSETS * NJB * KS * BT;
    static constexpr int STAGE = (XB + BB + 1023) / 1024 * 1024;
    static constexpr int AB = AOP ? 0 : (OUTM ? 2 : 1) * NIN * KS * AT;   // digit (and OUTM square) planes
    // Digit planes double-buffered (transform of read i+1 overlaps the MMAs of read i) when they fit.
    static constexpr int ABUF = AOP ? 0 : STAGES * STAGE + 2 * AB + BC * BM * ACCB + 1024 <= 227 * 1024 ? 2 : 1;
    static constexpr int ABUF1 = ABUF > 0 ? ABUF : 1;      // divisor for the buffer rotation
    static constexpr int OFF_A = STAGES * STAGE;
    static constexpr int OFF_ACC1 = OFF_A + ABUF * AB;
    static constexpr int OFF_BAR = OFF_ACC1 + BC * BM * ACCB;
    static constexpr int NBAR = 2 * STAGES + 2 * ABUF + 2 * U + 1;
    static constexpr int BYTES = OFF_BAR + NBAR * 8 + 16;
    static constexpr int TMEM_COLS = U * UNIT <= 256 ? 256 : 512;
    static_assert(U >= 1 && U * UNIT <= 512 && NTC <= 256, "accumulators exceed TMEM or the MMA's N");
    static_assert(!OUTM || (SPLIT && NPART == 2 && !VOLT && !PAIRB && !WIDE && NP % 16 == 0),
                  "output-mode noise: split halves of G', NP a multiple of 16, no other operand variant");
    static_assert(BN % 4 == 0 && KR % 16 == 0 && NIN <= MAXS && NW <= MAXS, "unsupported shape");
    static_assert(!VOLT || SPLIT, "voltage tiles pair with split conductance halves");
    static_assert(!PAIRB || (SPLIT && !VOLT), "per-slice conductance tiles: split halves, no voltage tiles");
    static_assert(!WIDE || (SPLIT && !VOLT && !PAIRB), "wide configurations: split halves, digits as tiles");
    static_assert(VALS % 2 == 0, "TMEM loads start on even columns");
    static_assert(BBOX * BLOADS == BROWS && BBOX % 8 == 0 && BBOX <= 256,
                  "B tile boxes: at most 256 rows, whole 8-row swizzle atoms");
    static_assert(BYTES + 1024 <= 232448, "exceeds the 227 KB shared-memory limit");
};

struct Args {
    const float* bias;       // [out_features] or null
    const float* xscale;     // [n, MR]
    const float* wscale;     // [MR, ldw]
    float* out;
    long long n, ldo, ldw;
    int out_features, MR;
    long long full;          // reads in complete 16-read cascade blocks
    int col_begin, col_end;  // output columns of this call
    unsigned* error;
    int a_shift[MAXS];
    uint32_t a_mask4[MAXS];  // digit mask replicated in every byte
    uint32_t lut_lo, lut_hi; // FP16 high bytes of the digits 0..7 (low bytes are 0)
    float cw[MAXS];          // voltage * M_w / unit * 2^-s: FP16-part sum -> ADC input
    float slope[MAXS];       // S-curve: nonlinear / max_w
    float cws[MAXS];         // cw / max_w: the ADC input as a fraction of full scale
    float inv_maxw[MAXS];    // 1 / max_w
    float maxw[MAXS];
    int factor[MAXS][MAXS];  // s_a * s_w
    int offset;              // -0x4B400000 * sum of factor over the slice pairs (mod 2^32)
    long long offset64;      // the same mod 2^64 (int64 totals of wide configurations)
    float ffactor[MAXS][MAXS];  // s_a * s_w as FP32 (float totals of the digit mode)
    int raster;              // 0: blockIdx.x walks vector blocks; 1: blockIdx.x walks column blocks
    int n_pad;               // VOLT: rows of one (slice, part) plane of the voltage operand
    int gblocks;             // PAIRB: column blocks of one input slice's G' operand
    // OUTM: current x (FP16-part units) -> noisy x = x + mf (x + l2s S_d) + z sqrt(vf2 Q),
    // z the normal of stream 60 at (((((v + vector_offset) MR + i) p + tile) A + a) W + w) C + c.
    float out_mf, out_vf2, out_l2s;
    long long vector_offset;
    int p_total, cols_c;
    unsigned long long read_seed;
    uint32_t sq_lo_lo, sq_lo_hi, sq_hi_lo, sq_hi_hi;   // FP16 low / high bytes of d^2, d = 0..7
};

__device__ __forceinline__ float mul_sat(float a, float b) {
    float d;
    asm("mul.rn.sat.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
    return d;
}

template <int N>
__device__ __forceinline__ void tmem_load_cols(uint32_t addr, uint32_t* v) {
    if constexpr (N >= 8) {
        tmem_ld(addr, *reinterpret_cast<uint32_t(*)[8]>(v));
        tmem_load_cols<N - 8>(addr + 8, v + 8);
    } else if constexpr (N >= 4) {
        tmem_ld(addr, *reinterpret_cast<uint32_t(*)[4]>(v));
        tmem_load_cols<N - 4>(addr + 4, v + 4);
    } else if constexpr (N >= 2) {
        tmem_ld(addr, *reinterpret_cast<uint32_t(*)[2]>(v));
        tmem_load_cols<N - 2>(addr + 2, v + 2);
    } else if constexpr (N == 1) {
        tmem_ld(addr, *reinterpret_cast<uint32_t(*)[1]>(v));
    }
}

// After tcgen05.wait::ld: route every loaded register through an asm statement
// ordered after the wait, so that no use is scheduled ahead of it.
template <int N>
__device__ __forceinline__ void tmem_loaded(uint32_t* v) {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int k = 0; k < N; ++k) asm volatile("" : "+r"(v[k]));
}

// FSUM (digit mode, reconstruction bound below 2^24): the count min(D, max_w) and
// the total are FP32 integers, summed exactly with one FMNMX and one FFMA per event.
template <int NIN, int NW, int BN, int NJB, int KR, bool SPLIT, int NPART, bool NONLINEAR, bool FSUM = false,
          bool VOLT = false, bool PAIRB = false, bool WIDE = false, bool OUTM = false>
__global__ void __launch_bounds__(THREADS, 1)
    tc_physical_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_g,
                       const __grid_constant__ Args args) {
    using G = Geo<NIN, NW, BN, NJB, KR, SPLIT, NPART, VOLT, PAIRB, WIDE, OUTM>;
    // Cascade values, scales and outputs: FP64 for wide configurations (Config.wide).
    using Real = typename std::conditional<WIDE, double, float>::type;
    static_assert(!WIDE || !FSUM, "the digit mode's FP32 totals are not wide");
    // The digit mode sums counts in FP32, exact only while every accumulator read from
    // TMEM is the integer digit dot itself: one FP16 part, no split halves.
    static_assert(!FSUM || (!SPLIT && NPART == 1), "FSUM needs exact integer digit dots (one FP16 part)");
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* base = smem_align1024(smem_raw);
    uint8_t* a_planes = base + G::OFF_A;
    Real* acc1 = reinterpret_cast<Real*>(base + G::OFF_ACC1);               // [BC][BM]
    uint64_t* bars = reinterpret_cast<uint64_t*>(base + G::OFF_BAR);
    uint64_t* full = bars;                      // [STAGES] codes and G' tiles landed
    uint64_t* empty = bars + STAGES;            // [STAGES] the read's MMAs are done with them
    uint64_t* a_ready = bars + 2 * STAGES;      // [ABUF] digit planes written
    uint64_t* a_free = a_ready + G::ABUF;       // [ABUF] the read's MMAs are done with them
    uint64_t* unit_full = a_free + G::ABUF;     // [U] a job's accumulators complete
    uint64_t* unit_empty = unit_full + G::U;    // [U] ... and read out by every epilogue warp
    uint64_t* drained = unit_empty + G::U;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + G::NBAR);
    int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const unsigned vblk = raster_vector_block(args.raster), cb_cta = raster_column_block(args.raster);
    const long long n0 = (long long)vblk * BM;
    const int c0 = args.col_begin + cb_cta * G::BC;   // first output column of this CTA
    const int MR = args.MR;
    unsigned* err = args.error;

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int b = 0; b < G::ABUF; ++b) {
            mbar_init(&a_ready[b], 2);
            mbar_init(&a_free[b], 1);
        }
        for (int u = 0; u < G::U; ++u) {
            mbar_init(&unit_full[u], 1);
            mbar_init(&unit_empty[u], EPI_WARPS);
        }
        mbar_init(drained, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int idx = threadIdx.x; idx < G::BC * BM; idx += THREADS) acc1[idx] = Real(0);
    if (warp == 0 && lane == 0) {
        prefetch_map(&map_x);
        prefetch_map(&map_g);
    }
    if (warp == 1) tmem_alloc(tmem_slot, G::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp < 4) {
        set_maxnreg_dec<REG_LOW>();
        if (warp == 0) {
            // ------------------------------------------------------------ producer
            if (lane == 0) {
                const int cb0 = cb_cta * NJB;              // first BN-column block of this CTA
                int issued = 0;
                for (int i = 0; i < MR; ++i) {
                    const int st = i % STAGES;
                    if (!mbar_wait(&empty[st], ((i / STAGES) & 1) ^ 1, abort_flag, err, 41)) break;
                    uint8_t* stage = base + st * G::STAGE;
                    mbar_expect_tx(&full[st], G::XB + G::BB);
                    if (G::AOP) {
                        // Tile (a, part, ks): rows (a * APARTS + part) * n_pad + n0 of the operand.
#pragma unroll 1
                        for (int t = 0; t < NIN * G::APARTS; ++t)
#pragma unroll
                            for (int ks = 0; ks < G::KS; ++ks)
                                tma_load_2d(stage + (t * G::KS + ks) * G::AT, &map_x, i * KR + ks * 16,
                                            (int)(t * args.n_pad + n0), &full[st]);
                    } else {
                        tma_load_2d(stage, &map_x, i * KR, (int)n0, &full[st]);
                    }
#pragma unroll 1
                    for (int set = 0; set < G::BSETS; ++set)
#pragma unroll 1
                        for (int cb = 0; cb < NJB; ++cb)
#pragma unroll
                            for (int ks = 0; ks < G::KS; ++ks)
#pragma unroll
                                for (int h = 0; h < G::BLOADS; ++h)
                                    tma_load_2d(stage + G::XB + ((set * NJB + cb) * G::KS + ks) * G::BT +
                                                    h * G::BBOX * 32,
                                                &map_g, i * KR + ks * 16,
                                                (set * args.gblocks + cb0 + cb) * G::BROWS + h * G::BBOX, &full[st]);
                    issued = i + 1;
                }
                // Every issued load lands before the CTA may exit.
                for (int i = issued - STAGES > 0 ? issued - STAGES : 0; i < issued; ++i)
                    mbar_drain(&full[i % STAGES], (i / STAGES) & 1);
            }
        } else if (warp == 1) {
            // ------------------------------------------------------------ MMA issuer
            if (lane == 0) {
                // SPLIT: both halves in one MMA (N = NT) into adjacent accumulators;
                // otherwise one MMA per half into the same accumulator.
                const uint32_t idesc = idesc_f16(BM, G::NTC);
                const uint32_t idesc_q = idesc_f16(BM, OUTM ? G::NPV : 16);   // OUTM: the Q accumulator
                bool ok = true;
                int job = 0;                               // job sequence number: unit job % U
                for (int i = 0; i < MR && ok; ++i) {
                    const int st = i % STAGES;
                    if (!mbar_wait(&full[st], (i / STAGES) & 1, abort_flag, err, 42)) break;
                    const int ab = i % G::ABUF1;
                    if (!G::AOP && !mbar_wait(&a_ready[ab], (i / G::ABUF1) & 1, abort_flag, err, 43)) break;
                    tc_fence_after();
                    const uint8_t* btiles = base + st * G::STAGE + G::XB;
                    // VOLT / WIDE: the stage's operand tiles (a, part, ks); otherwise the digit planes (a, ks).
                    const uint8_t* planes = G::AOP ? base + st * G::STAGE : a_planes + ab * G::AB;
#pragma unroll 1
                    for (int cb = 0; cb < NJB && ok; ++cb) {
#pragma unroll 1
                        for (int a = 0; a < NIN; ++a, ++job) {
                            // Descriptors advance by (byte offset >> 4) in their address field.
                            const uint64_t db = desc_sw32(btiles + ((PAIRB ? a * NJB : 0) + cb) * G::KS * G::BT);
                            const int unit = job % G::U;
                            if (!mbar_wait(&unit_empty[unit], (uint32_t)((job / G::U) & 1) ^ 1u, abort_flag, err,
                                           44)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            const uint32_t d = tmem + unit * G::UNIT;
                            if (G::AOP) {
                                // Every part into the same accumulators (B halves stacked along N).
                                const uint64_t da = desc_sw32(planes + a * G::APARTS * G::KS * G::AT);
#pragma unroll
                                for (int vp = 0; vp < G::APARTS; ++vp)
#pragma unroll
                                    for (int ks = 0; ks < G::KS; ++ks)
                                        mma_f16(d, da + (uint64_t)(((vp * G::KS + ks) * G::AT) >> 4),
                                                db + (uint64_t)((ks * G::BT) >> 4), idesc, (vp | ks) != 0);
                            } else {
                                const uint64_t da = desc_sw32(planes + a * G::KS * G::AT);
#pragma unroll
                                for (int part = 0; part < (SPLIT ? 1 : NPART); ++part)
#pragma unroll
                                    for (int ks = 0; ks < G::KS; ++ks)
                                        mma_f16(d, da + (uint64_t)((ks * G::AT) >> 4),
                                                db + (uint64_t)((ks * G::BT + part * G::PSTRIDE * 32) >> 4), idesc,
                                                (part | ks) != 0);
                                if constexpr (OUTM) {
                                    // Q = sum d^2 G^2: digit-square planes against both floating
                                    // parts of G^2, into one accumulator after the current's.
                                    const uint64_t dq = desc_sw32(planes + (NIN + a) * G::KS * G::AT);
#pragma unroll
                                    for (int ks = 0; ks < G::KS; ++ks)
#pragma unroll
                                        for (int part = 0; part < 2; ++part)
                                            mma_f16(d + G::NTC, dq + (uint64_t)((ks * G::AT) >> 4),
                                                    db + (uint64_t)((ks * G::BT + (G::G2ROW + part * G::NP) * 32) >> 4),
                                                    idesc_q, (ks | part) != 0);
                                }
                            }
                            mma_commit(&unit_full[unit]);
                        }
                    }
                    if (!ok) break;
                    if (!G::AOP) mma_commit(&a_free[ab]);
                    mma_commit(&empty[st]);
                }
                // All issued MMAs complete before TMEM is released.
                mma_commit(drained);
                mbar_drain(drained, 0);
            }
        } else {
            // ------------------------------------------------------------ transform
            // Row t of the code tile holds the read's KR codes (no swizzle); each
            // 16-code step becomes one [128 x 16] FP16 plane per input slice in the
            // 32-byte-swizzled K-major layout (16-byte halves swapped in rows with bit 2 set).
            const int tw = warp - 2;
            for (int i = 0; i < (G::AOP ? 0 : MR); ++i) {
                const int st = i % STAGES;
                const int ab = i % G::ABUF1;
                bool ok = mbar_wait(&full[st], (i / STAGES) & 1, abort_flag, err, 45);
                ok = ok && mbar_wait(&a_free[ab], ((i / G::ABUF1) & 1) ^ 1, abort_flag, err, 46);
                if (!__all_sync(0xFFFFFFFFu, ok)) break;
                const uint8_t* codes = base + st * G::STAGE;
                uint8_t* planes = a_planes + ab * G::AB;
#pragma unroll 1
                for (int hh = 0; hh < 2; ++hh) {
                    const int t = tw * 32 + lane + 64 * hh;
                    const uint32_t flip = ((uint32_t)t >> 2) & 1u;
#pragma unroll 1
                    for (int ks = 0; ks < G::KS; ++ks) {
                        const uint4 c16 = *reinterpret_cast<const uint4*>(codes + t * KR + ks * 16);
                        const uint32_t w4[4] = {c16.x, c16.y, c16.z, c16.w};
#pragma unroll
                        for (int a = 0; a < NIN; ++a) {
                            uint32_t o[8];
#pragma unroll
                            for (int k = 0; k < 4; ++k) {
                                const uint32_t d = (w4[k] >> args.a_shift[a]) & args.a_mask4[a];
                                // Output bytes [0, hi(d0), 0, hi(d1)] and [0, hi(d2), 0, hi(d3)].
                                o[2 * k] = __byte_perm(args.lut_lo, args.lut_hi, (d << 4) & 0xF0F0u);
                                o[2 * k + 1] = __byte_perm(args.lut_lo, args.lut_hi, (d >> 12) & 0xF0F0u);
                            }
                            uint8_t* row = planes + (a * G::KS + ks) * G::AT + t * 32;
                            *reinterpret_cast<uint4*>(row + (flip << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
                            *reinterpret_cast<uint4*>(row + ((flip ^ 1u) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
                            if constexpr (OUTM) {
                                // FP16 d^2: low bytes at positions 0 and 2, high bytes at 1 and 3.
#pragma unroll
                                for (int k = 0; k < 4; ++k) {
                                    const uint32_t d = (w4[k] >> args.a_shift[a]) & args.a_mask4[a];
                                    o[2 * k] = __byte_perm(args.sq_lo_lo, args.sq_lo_hi, d & 0x0F0Fu) |
                                               __byte_perm(args.sq_hi_lo, args.sq_hi_hi, (d << 4) & 0xF0F0u);
                                    o[2 * k + 1] = __byte_perm(args.sq_lo_lo, args.sq_lo_hi, (d >> 16) & 0x0F0Fu) |
                                                   __byte_perm(args.sq_hi_lo, args.sq_hi_hi, (d >> 12) & 0xF0F0u);
                                }
                                uint8_t* sq = planes + ((NIN + a) * G::KS + ks) * G::AT + t * 32;
                                *reinterpret_cast<uint4*>(sq + (flip << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
                                *reinterpret_cast<uint4*>(sq + ((flip ^ 1u) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
                            }
                        }
                    }
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(&a_ready[ab]);
            }
        }
    } else {
        set_maxnreg_inc<REG_HIGH>();
        // ---------------------------------------------------------------- epilogue
        // Warp w reads TMEM lane quadrant w & 3 (rows) and the EC-column slice hc of
        // every block; in a job's accumulators (input slice a of one block), output
        // column jj and weight slice w of half acc sit at column acc * NP + jj * NW + w.
        const int quad = warp & 3;
        const int hc = (warp - 4) >> 2;
        const int r = quad * 32 + lane;
        const long long row = n0 + r;
        const bool live = row < args.n;
        const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16) + hc * G::VALS;
        Real acc0[NJB][G::EC];
#pragma unroll
        for (int cb = 0; cb < NJB; ++cb)
#pragma unroll
            for (int e = 0; e < G::EC; ++e) acc0[cb][e] = Real(0);
        // FP32 or FP64 (wide) per-read scales.
        const Real* xscale = reinterpret_cast<const Real*>(args.xscale);
        const Real* wscale = reinterpret_cast<const Real*>(args.wscale);
        // Per-read scales are loaded one read ahead so their latency hides behind a read's work.
        const int colbase = c0 + hc * G::EC;
        Real xs_next = live ? __ldg(xscale + row * MR) : Real(0);
        Real ws_next[NJB][G::EC];
#pragma unroll
        for (int cb = 0; cb < NJB; ++cb)
#pragma unroll
            for (int e = 0; e < G::EC; ++e)
                ws_next[cb][e] = colbase + cb * BN + e < args.col_end ? __ldg(wscale + colbase + cb * BN + e)
                                                                      : Real(0);
        // OUTM: the hash address of an ADC event,
        // (((((row + vector_offset) MR + i) p + tile) A + a) W + w) C + cc, is
        // ev_row + i * ev_read + (a W + w) C + e: this thread's columns colbase + e lie in
        // one tile (NJB = 1 and BN divides C).  The hash's stream keys and its fold of
        // the address's high word are kept across events (the word rarely changes).
        long long ev_row = 0, ev_read = 0;
        uint32_t key0 = 0, key1 = 0, fold0 = 0, fold1 = 0, fold_high = 0;
        if constexpr (OUTM) {
            const int tile = colbase / args.cols_c;
            ev_read = (long long)args.p_total * NIN * NW * args.cols_c;
            ev_row = (row + args.vector_offset) * MR * ev_read + (long long)tile * NIN * NW * args.cols_c +
                     (colbase - tile * args.cols_c);
            key0 = rng_key(args.read_seed, 60);
            key1 = rng_key(args.read_seed, 61);
            fold_high = (uint32_t)((uint64_t)ev_row >> 32);
            fold0 = rng_fold(fold_high, args.read_seed, key0);
            fold1 = rng_fold(fold_high, args.read_seed, key1);
        }
        bool ok = true;
        int job = 0;
        for (int i = 0; i < MR && ok; ++i) {
            const Real xs = xs_next;
            Real ws_now[NJB][G::EC];
#pragma unroll
            for (int cb = 0; cb < NJB; ++cb)
#pragma unroll
                for (int e = 0; e < G::EC; ++e) ws_now[cb][e] = ws_next[cb][e];
            if (i + 1 < MR) {
                xs_next = live ? __ldg(xscale + row * MR + i + 1) : Real(0);
#pragma unroll
                for (int cb = 0; cb < NJB; ++cb)
#pragma unroll
                    for (int e = 0; e < G::EC; ++e) {
                        const int col = colbase + cb * BN + e;
                        ws_next[cb][e] =
                            col < args.col_end ? __ldg(wscale + (long long)(i + 1) * args.ldw + col) : Real(0);
                    }
            }
            // Unrolled: acc0 and the scales stay in registers (a dynamic block index would
            // put them in local memory).
#pragma unroll
            for (int cb = 0; cb < NJB; ++cb) {
                // ADC: the saturating multiply clamps z / max_w to [0, 1], and
                // q = (z / max_w) * max_w + 1.5 * 2^23 rounds the clamped z half to even into
                // the low mantissa bits (max_w < 2^22); the bit pattern of q is
                // 0x4B400000 + count, so the total accumulates bits * factor in wrapping int32
                // and the constant part is removed once.
                // Wide configurations: 64-bit totals (the reference's int64 totals,
                // reference.py:115), accumulated modulo 2^64 like the 32-bit ones.
                using Tot = typename std::conditional<WIDE, unsigned long long, int>::type;
                Tot total[G::EC];
                float ftotal[G::EC];
#pragma unroll
                for (int e = 0; e < G::EC; ++e) {
                    total[e] = WIDE ? (Tot)args.offset64 : (Tot)args.offset;
                    ftotal[e] = 0.0f;
                }
#pragma unroll 1
                for (int a = 0; a < NIN; ++a, ++job) {
                    const int unit = job % G::U;
                    ok = __all_sync(0xFFFFFFFFu,
                                    mbar_wait(&unit_full[unit], (uint32_t)(job / G::U) & 1u, abort_flag, err, 47));
                    if (!ok) break;
                    tc_fence_after();
                    uint32_t v[G::ACCS + (OUTM ? 1 : 0)][G::VALS];
                    uint32_t sd[1] = {0u};
#pragma unroll
                    for (int acc = 0; acc < G::ACCS; ++acc)
                        tmem_load_cols<G::VALS>(lane_base + unit * G::UNIT + acc * G::NP, v[acc]);
                    if constexpr (OUTM) {
                        // Q of this thread's columns, and the row's digit sum (the ones column).
                        tmem_load_cols<G::VALS>(lane_base + unit * G::UNIT + G::NTC, v[G::ACCS]);
                        tmem_ld(tmem + ((uint32_t)(quad * 32) << 16) + unit * G::UNIT + G::NT, sd);
                    }
                    tmem_loaded<(G::ACCS + (OUTM ? 1 : 0)) * G::VALS>(&v[0][0]);
                    if constexpr (OUTM) tmem_loaded<1>(sd);
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&unit_empty[unit]);
                    constexpr float kMagic = 12582912.0f;   // 1.5 * 2^23
                    if constexpr (SPLIT && !OUTM && !FSUM) {
                        // The ADC two events at a time (flattened index k = e * NW + w):
                        // packed FMAs round each lane once, as the scalar ones below do.
#pragma unroll
                        for (int k = 0; k < G::VALS; k += 2) {
                            const int e0 = k / NW, w0 = k % NW, e1 = (k + 1) / NW, w1 = (k + 1) % NW;
                            const float2 x2 = __ffma2_rn(
                                make_float2(__uint_as_float(v[0][k]), __uint_as_float(v[0][k + 1])),
                                make_float2(2048.0f, 2048.0f),
                                make_float2(__uint_as_float(v[1][k]), __uint_as_float(v[1][k + 1])));
                            float2 s2;
                            if constexpr (NONLINEAR) {
                                // S-curve per lane: z = x c / (1 + |slope z|), clamped to [0, 1] of max_w.
                                float z0 = __fmul_rn(x2.x, args.cw[w0]), z1 = __fmul_rn(x2.y, args.cw[w1]);
                                z0 = __fdiv_rn(z0, __fadd_rn(1.0f, fabsf(__fmul_rn(args.slope[w0], z0))));
                                z1 = __fdiv_rn(z1, __fadd_rn(1.0f, fabsf(__fmul_rn(args.slope[w1], z1))));
                                s2 = make_float2(mul_sat(z0, args.inv_maxw[w0]), mul_sat(z1, args.inv_maxw[w1]));
                            } else {
                                s2 = make_float2(mul_sat(x2.x, args.cws[w0]), mul_sat(x2.y, args.cws[w1]));
                            }
                            const float2 q2 =
                                __ffma2_rn(s2, make_float2(args.maxw[w0], args.maxw[w1]), make_float2(kMagic, kMagic));
                            if constexpr (WIDE) {
                                total[e0] += (Tot)(long long)__float_as_int(q2.x) * (Tot)(long long)args.factor[a][w0];
                                total[e1] += (Tot)(long long)__float_as_int(q2.y) * (Tot)(long long)args.factor[a][w1];
                            } else {
                                total[e0] += __float_as_int(q2.x) * args.factor[a][w0];
                                total[e1] += __float_as_int(q2.y) * args.factor[a][w1];
                            }
                        }
                    } else
#pragma unroll
                    for (int e = 0; e < G::EC; ++e)
#pragma unroll
                        for (int w = 0; w < NW; ++w) {
                            // SPLIT: 2048 S_H + S_L, both exact integers, rounded once.
                            float x = SPLIT ? __fmaf_rn(__uint_as_float(v[0][e * NW + w]), 2048.0f,
                                                        __uint_as_float(v[SPLIT ? 1 : 0][e * NW + w]))
                                            : __uint_as_float(v[0][e * NW + w]);
                            if constexpr (OUTM) {
                                // Output-mode read noise (reference.py:107-114) in the units of x:
                                // mean = mf (x + LOW 2^s S_d), deviation sqrt(vf2 Q) z, z the
                                // normal of stream 60 at the event's address.
                                const long long address =
                                    ev_row + i * ev_read + (long long)((a * NW + w) * args.cols_c + e);
                                const uint32_t high = (uint32_t)((uint64_t)address >> 32);
                                if (high != fold_high) {
                                    fold_high = high;
                                    fold0 = rng_fold(high, args.read_seed, key0);
                                    fold1 = rng_fold(high, args.read_seed, key1);
                                }
                                const float z = box_muller(rng_unit((uint32_t)address, fold0, key0),
                                                           rng_unit((uint32_t)address, fold1, key1));
                                const float q = __uint_as_float(v[G::ACCS][e * NW + w]);
                                const float mean = __fmul_rn(args.out_mf, __fmaf_rn(args.out_l2s, __uint_as_float(sd[0]), x));
                                x = __fadd_rn(x, __fadd_rn(mean, __fmul_rn(sqrtf(__fmul_rn(args.out_vf2, q)), z)));
                            }
                            if (FSUM) {
                                ftotal[e] = __fmaf_rn(fminf(x, args.maxw[w]), args.ffactor[a][w], ftotal[e]);
                                continue;
                            }
                            float s;
                            if (NONLINEAR) {
                                float z = __fmul_rn(x, args.cw[w]);
                                z = __fdiv_rn(z, __fadd_rn(1.0f, fabsf(__fmul_rn(args.slope[w], z))));
                                s = mul_sat(z, args.inv_maxw[w]);
                            } else {
                                s = mul_sat(x, args.cws[w]);
                            }
                            const float q = __fmaf_rn(s, args.maxw[w], kMagic);
                            if constexpr (WIDE)
                                total[e] += (Tot)(long long)__float_as_int(q) * (Tot)(long long)args.factor[a][w];
                            else
                                total[e] += __float_as_int(q) * args.factor[a][w];
                        }
                }
                if (!ok) break;
#pragma unroll
                for (int e = 0; e < G::EC; ++e) {
                    if constexpr (WIDE) {
                        // restore_scales in FP64 (simulator.py:57-66).
                        acc0[cb][e] = __dadd_rn(acc0[cb][e], restore_scales(__ll2double_rn((long long)total[e]), xs,
                                                                           ws_now[cb][e]));
                    } else {
                        acc0[cb][e] = __fadd_rn(
                            acc0[cb][e],
                            __fmul_rn(__fmul_rn(FSUM ? ftotal[e] : __int2float_rn(total[e]), xs), ws_now[cb][e]));
                    }
                }
            }
            if (!ok) break;
            // Block boundary of the 16-read cascade: level 1 += level 0 (MR <= 256 keeps two levels).
            const int done = i + 1;
            if (done <= args.full && (done & 15) == 0) {
#pragma unroll
                for (int cb = 0; cb < NJB; ++cb)
#pragma unroll
                    for (int e = 0; e < G::EC; ++e) {
                        Real* slot = acc1 + (cb * BN + hc * G::EC + e) * BM + r;
                        *slot = add_rn<Real>(*slot, acc0[cb][e]);
                        acc0[cb][e] = Real(0);
                    }
            }
        }
        if (ok && live) {
#pragma unroll
            for (int cb = 0; cb < NJB; ++cb)
#pragma unroll
                for (int e = 0; e < G::EC; ++e) {
                    const int cl = cb * BN + hc * G::EC + e;
                    const int col = c0 + cl;
                    if (col >= args.col_end || col >= args.out_features) continue;
                    // acc0 + acc1 + acc2 + acc3 (upper levels zero), then the reference's
                    // store into a zero-filled output.
                    Real value = add_rn<Real>(acc0[cb][e], acc1[cl * BM + r]);
                    value = add_rn<Real>(value, Real(0));
                    value = add_rn<Real>(value, Real(0));
                    value = add_rn<Real>(Real(0), value);
                    if (args.bias) value = add_rn<Real>(value, reinterpret_cast<const Real*>(args.bias)[col]);
                    reinterpret_cast<Real*>(args.out)[row * args.ldo + col] = value;
                }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, G::TMEM_COLS);
    }
}

// The B operand of one column block: rows (block * brows + part * pstride +
// jj * nwp + w) for output column col_begin + block * BN + jj and weight slice w
// (other rows zero), K contiguous.  One CTA per (column block, KC-row chunk of
// K): the chunk's codes are staged in shared memory (a block lies inside one
// tile and a chunk inside one array), so no element needs an index division.
//   parts == 1 (ideal devices): the weight digit, an exact FP16 integer.
//   parts == 2: G' = G - LOW, computed once per (row, column, slice) and written
//   as two FP16 parts.  fixed: X = rint(G' * scale) (|X| < 2^22) as the integers
//   H = rint(X / 2048) and L = X - 2048 H; otherwise x = G' * scale (< 2^14) as
//   hi = fp16(x), lo = fp16(x - hi).  The conductance is the SIMT path's
//   (restored_conductance_f32).
constexpr int KC = 64;           // K rows per CTA of the operand builder
constexpr int MAXBN = 32;        // columns per block, at most

//   pair_slices > 0 (slice-pair read noise): one operand per input slice a, set a
//   starting at row a * blocks * brows, its G scaled by exp(sigma_r z) with z the
//   normal of stream 20 at cell * pair_slices + a (reference.py:88-91).
template <typename CodeT>
__global__ void __launch_bounds__(256) b_operand_kernel(Layout L, Physics P, const CodeT* packed, int p,
                                                        int col_begin, int blocks, int bn, int nwp, int brows,
                                                        int pstride, int parts, int kc, long long kpad, uint32_t seed,
                                                        uint64_t event, float scale, int fixed, int pair_slices,
                                                        int ones_row, int g2row, float scale2, __half* gs) {
    __shared__ uint16_t codes[KC][MAXBN];   // weight codes have at most 16 bits
    for (int block = blockIdx.y; block < blocks; block += gridDim.y) {
        const long long k0 = (long long)blockIdx.x * kc;
        const long long o0 = (long long)col_begin + (long long)block * bn;
        const long long tile = o0 / L.C;
        const int c0 = (int)(o0 - tile * L.C);
        const long long arr = k0 / L.R;
        const int r0 = (int)(k0 - arr * L.R);
        const long long tile_base = (arr * p + tile) * L.R;
        for (int idx = threadIdx.x; idx < kc * bn; idx += blockDim.x) {
            const int kk = idx / bn, jj = idx - kk * bn;
            codes[kk][jj] = (uint16_t)packed[(tile_base + r0 + kk) * L.C + c0 + jj];
        }
        __syncthreads();
        const uint64_t read_seed = event_seed(seed, event);
        const float low = (float)P.low;
        const int np = nwp * bn;
        const int sets = pair_slices > 0 ? pair_slices : 1;
        const long long set_stride = (long long)blocks * brows * kpad;   // elements of one input slice's operand
        __half* out = gs + (long long)block * brows * kpad + k0;
        for (int idx = threadIdx.x; idx < pstride * kc; idx += blockDim.x) {
            const int prow = idx / kc, kk = idx - prow * kc;
            const int jj = prow / nwp, w = prow - jj * nwp;
            const bool cell = prow < np && w < L.n_w;
            const long long state = cell ? ((long long)codes[kk][jj] >> L.w_shift[w]) & L.w_mask[w] : 0;
            const long long address = (((arr * p + tile) * L.n_w + w) * L.R + r0 + kk) * L.C + c0 + jj;
            const float g = cell && parts != 1 ? restored_conductance_f32(P, state, L.w_mask[w], address, seed,
                                                                          read_seed)
                                               : 0.0f;
            for (int set = 0; set < sets; ++set) {
                __half hi = __float2half_rn(0.0f), lo = hi;
                if (cell) {
                    if (parts == 1) {
                        hi = __float2half_rn((float)state);
                    } else {
                        float gs_a = g;
                        if (pair_slices > 0)
                            gs_a = __fmul_rn(g, expf(__fmul_rn((float)P.read_var,
                                                               rng_normal(address * pair_slices + set, read_seed, 20))));
                        const float x = __fmul_rn(__fadd_rn(gs_a, -low), scale);
                        if (fixed) {
                            const float X = rintf(x);
                            const float H = rintf(__fmul_rn(X, 1.0f / 2048.0f));
                            hi = __float2half_rn(H);
                            lo = __float2half_rn(__fsub_rn(X, __fmul_rn(H, 2048.0f)));
                        } else {
                            hi = __float2half_rn(x);
                            lo = __float2half_rn(__fsub_rn(x, __half2float(hi)));
                        }
                    }
                }
                __half* dst = out + set * set_stride;
                dst[(long long)prow * kpad + kk] = hi;
                if (parts == 2) dst[(long long)(pstride + prow) * kpad + kk] = lo;
                if (g2row >= 0) {
                    // Output-mode noise: G^2 (not G - LOW) as two floating FP16 parts.
                    __half hi2 = __float2half_rn(0.0f), lo2 = hi2;
                    if (cell) {
                        const float x2 = __fmul_rn(__fmul_rn(g, g), scale2);
                        hi2 = __float2half_rn(x2);
                        lo2 = __float2half_rn(__fsub_rn(x2, __half2float(hi2)));
                    }
                    dst[(long long)(g2row + prow) * kpad + kk] = hi2;
                    dst[(long long)(g2row + pstride + prow) * kpad + kk] = lo2;
                }
            }
        }
        // Rows past the parts (MMA padding) are zero, except the row of ones that
        // gives the output mode its digit sums; the G^2 rows were written above.
        for (int set = 0; set < sets; ++set)
            for (int idx = parts * pstride * kc + threadIdx.x; idx < brows * kc; idx += blockDim.x) {
                const int row = idx / kc, kk = idx - row * kc;
                if (g2row >= 0 && row >= g2row && row < g2row + 2 * pstride) continue;
                out[set * set_stride + (long long)row * kpad + kk] = __float2half_rn(row == ones_row ? 1.0f : 0.0f);
            }
        __syncthreads();   // the next block's codes overwrite the staging tile
    }
}

// The A operand of the voltage-noise path.  For vector v (global index
// vector_offset + v), reduction index k (array k / R, row k % R) and input slice
// a, the voltage factor of the reference, d * (1 + sigma * z) with d the slice's
// digit and z the normal of stream 40 at address ((v * m + array) * NIN + a) * R
// + row under the read event's seed (memfast/reference.py:83-86), written as two
// FP16 parts hi = fp16(x), lo = fp16(x - hi) (x to about 22 bits).  Planes
// [a][part][n_pad][kpad], K contiguous, so that one TMA box of 16 K x 128 rows is
// an MMA A tile; rows at or beyond n are zero.  One thread per (row, k) draws the
// noise of every input slice.
__global__ void __launch_bounds__(256) a_operand_kernel(Layout L, float volt_var, const uint8_t* codes, long long n,
                                                        long long n_pad, int m, long long kpad,
                                                        long long vector_offset, uint64_t read_seed, __half* va) {
    const long long k = (long long)blockIdx.x * 256 + threadIdx.x;
    if (k >= kpad) return;
    const long long arr = k / L.R;
    const int row = (int)(k - arr * L.R);
    for (long long v = blockIdx.y; v < n_pad; v += gridDim.y) {
        const long long code = v < n ? (long long)codes[v * kpad + k] : 0;
        for (int a = 0; a < L.n_in; ++a) {
            __half hi = __float2half_rn(0.0f), lo = hi;
            const long long d = (code >> L.in_shift[a]) & L.in_mask[a];
            if (d != 0) {
                const long long address = (((vector_offset + v) * m + arr) * L.n_in + a) * L.R + row;
                const float f = __fadd_rn(1.0f, __fmul_rn(volt_var, rng_normal(address, read_seed, 40)));
                const float x = __fmul_rn((float)d, f);
                hi = __float2half_rn(x);
                lo = __float2half_rn(__fsub_rn(x, __half2float(hi)));
            }
            va[((long long)(a * 2) * n_pad + v) * kpad + k] = hi;
            va[((long long)(a * 2 + 1) * n_pad + v) * kpad + k] = lo;
        }
    }
}

// Digit operand of a wide configuration: the FP16 digit of every input slice a of
// every (vector, row of K) at row a * n_pad + v, K contiguous (the layout of the
// voltage operand with one part); rows past n are zero.  The current kernel loads
// its [128 x 16] tiles with TMA as the A operand.
template <typename CodeT>
__global__ void __launch_bounds__(256) digit_operand_kernel(Layout L, const CodeT* codes, long long n,
                                                            long long n_pad, long long kpad, __half* out) {
    const long long k = (long long)blockIdx.x * 256 + threadIdx.x;
    if (k >= kpad) return;
    for (long long v = blockIdx.y; v < n_pad; v += gridDim.y) {
        const long long code = v < n ? (long long)codes[v * kpad + k] : 0;
        for (int a = 0; a < L.n_in; ++a) {
            const long long d = (code >> L.in_shift[a]) & L.in_mask[a];
            out[((long long)a * n_pad + v) * kpad + k] = __float2half_rn((float)d);
        }
    }
}

// Instantiations: (input slices, weight slices) -> columns per block, blocks per
// CTA, split accumulators.  Each MMA is as wide as TMEM and the 256-column limit of
// N allow (the tensor core's cost here is per instruction rather than per column).
struct Shape {
    int nin, nw, bn, njb, split;
};
constexpr Shape kShapes[] = {{5, 5, 16, 2, 1}, {3, 3, 32, 1, 1}, {8, 8, 16, 1, 0}, {4, 4, 16, 2, 1}};
// Ideal devices: one FP16 part (the digits), so a block can hold twice the columns.
constexpr Shape kDigitShapes[] = {{5, 5, 32, 1, 0}, {3, 3, 32, 2, 0}, {8, 8, 16, 1, 0}, {4, 4, 32, 1, 0}};

// Slice-pair read noise: one G' operand per input slice (PAIRB instantiations).
bool pair_mode(const mf_config& c) { return !c.ideal && c.read_var != 0 && c.read_mode == 1; }

// Output-mode read noise: digit sums and second moments per job (OUTM instantiations).
bool output_mode(const mf_config& c) { return !c.ideal && c.read_var != 0 && c.read_mode == 2; }

bool shape_of(const mf_config& c, Shape& s) {
    for (const Shape& k : c.ideal ? kDigitShapes : kShapes)
        if (k.nin == c.n_in && k.nw == c.n_w) {
            s = k;
            // A stage holds every input slice's tiles (slice-pair noise) or the digit
            // tiles of a wide configuration: one column block per CTA.
            if (pair_mode(c) || output_mode(c) || (!c.ideal && (c.wide || c.wide_codes))) s.njb = 1;
            return true;
        }
    return false;
}

int parts_of(const mf_config& c) { return c.ideal ? 1 : PARTS; }

// B tile rows per column block (rounded to 8) and the row offset of the second half,
// as Geo computes them; with outm also the row of ones (after the current's MMA
// rows) and the first row of the G^2 parts.
void rows_of(const Shape& s, int npart, int& brows8, int& pstride, bool outm, int* ones_row, int* g2row) {
    const int np = s.nw * s.bn;
    const int nt = s.split ? (npart * np + 15) / 16 * 16 : (np + 15) / 16 * 16;
    pstride = s.split ? np : nt;
    int brows = npart * pstride > nt ? npart * pstride : nt;
    if (ones_row) *ones_row = outm ? nt : -1;
    if (g2row) *g2row = outm ? nt + 16 : -1;
    if (outm) brows = nt + 16 + 2 * np;
    brows8 = (brows + 7) / 8 * 8;
}

// Rows of one TMA box of a B tile (Geo::BBOX): tiles over 256 rows load as two boxes.
int box_rows(int brows8) { return brows8 > 256 ? brows8 / 2 : brows8; }

// Scale 2^u of G^2 as two floating FP16 parts (largest value below 2^14).
float square_scale(const mf_config& c) {
    const double gmax = fmax(fabs(c.high), fabs(c.low)) * fmax(c.drift, 1e-30) * exp(8.0 * (c.write_var + c.read_var));
    const int u = (int)floor(log2(16384.0 / (gmax * gmax)));
    return (float)ldexp(1.0, u);
}

// Scale 2^s of G': the largest |G'| (nominal level, drift, an 8-sigma write and
// read variation) stays below 2^22 (fixed-point halves) or 2^14 (floating parts).
float split_scale(const mf_config& c, bool fixed) {
    const double gmax = fmax(fabs(c.high), fabs(c.low)) * fmax(c.drift, 1e-30) * exp(8.0 * (c.write_var + c.read_var));
    const int s = (int)floor(log2((fixed ? 4194303.0 : 16384.0) / gmax));
    return (float)ldexp(1.0, s);
}

}  // namespace tcp

// =================================================================== host side
// Ideal devices: the accumulator holds the exact digit dot D (FP16 digits, every
// partial sum an integer below 2^24) and the epilogue's count is min(D, max_w), the
// reference's count wherever exact_integer_counts holds; the int32 totals are exact
// below 2^31.
static bool digits_eligible(const mf_config& c, int32_t m) {
    if (!exact_integer_counts(c) || c.wide || c.wide_codes || c.precise_currents) return false;
    if (c.read_rows != 32 && c.read_rows != 64) return false;
    tcp::Shape s;
    if (!tcp::shape_of(c, s)) return false;
    if (c.rows % c.read_rows || c.cols % s.bn) return false;
    for (int i = 0; i < c.n_in; ++i)
        if (c.in_mask[i] > 7) return false;
    for (int i = 0; i < c.n_w; ++i)
        if (c.w_mask[i] > 2047 || c.adc_max[i] < 1 || c.adc_max[i] >= (1 << 22)) return false;
    const long long MR = (long long)m * c.reads;
    return MR <= 256 && reconstruction_bound(c) < 2147483647.0;
}

bool tc_physical_eligible(const mf_config& c, int32_t m) {
    if (c.ideal) return digits_eligible(c, m);
    if (c.precise_currents) return false;
    // Wide configurations (16-bit BFP): five-slice operands, digits as FP16 tiles, int64 totals.
    const bool wide = c.wide || c.wide_codes;
    if (wide && (c.n_in != 5 || c.n_w != 5 || c.volt_var != 0 || tcp::pair_mode(c))) return false;
    if (c.write_var + c.read_var > 1.0) return false;
    if (c.read_rows != 32 && c.read_rows != 64) return false;
    tcp::Shape s;
    if (!tcp::shape_of(c, s)) return false;
    // Voltage noise: the voltage tiles of a stage fit shared memory for 32-row reads of
    // the split-halves shapes.
    if (c.volt_var != 0 && (c.read_rows != 32 || !s.split)) return false;
    // Slice-pair read noise: every input slice's G' tiles in a stage, which fits for
    // 32-row reads of the split-halves shapes without voltage tiles.
    if (tcp::pair_mode(c) && (c.read_rows != 32 || !s.split || c.volt_var != 0)) return false;
    // Output-mode read noise: 32-row reads of the split-halves shapes, no voltage noise.
    if (tcp::output_mode(c) && (c.read_rows != 32 || !s.split || c.volt_var != 0 || wide ||
                                (s.nw * s.bn) % 16 != 0))
        return false;
    if (c.rows % c.read_rows || c.cols % s.bn) return false;
    // Digit planes are built by byte lookup for digits up to 7; wide configurations
    // take their digits as FP16 tiles (exact up to 2048).
    for (int i = 0; i < c.n_in; ++i)
        if (c.in_mask[i] > (wide ? 2047 : 7)) return false;
    for (int i = 0; i < c.n_w; ++i)
        if (c.adc_max[i] < 1 || c.adc_max[i] >= (1 << 22)) return false;
    const long long MR = (long long)m * c.reads;
    // Totals are exact in FP32 below 2^24 (int64 and FP64 below 2^53 when wide), and
    // adc_max < 2^22 keeps the rounding trick exact.
    return MR <= 256 && c.high > 0 && c.drift > 0 &&
           reconstruction_bound(c) < (wide ? 9007199254740992.0 : 16777216.0);
}

int tc_physical_threads() { return tcp::THREADS; }

// Bytes of the conductance operand, rounded to 256.
static size_t b_operand_bytes(const mf_config& c, const tcp::Shape& s, int32_t m, int32_t tiles) {
    const long long blocks = (long long)tiles * c.cols / s.bn;
    int brows = 0, pstride = 0;
    tcp::rows_of(s, tcp::parts_of(c), brows, pstride, tcp::output_mode(c), nullptr, nullptr);
    const size_t sets = tcp::pair_mode(c) ? (size_t)c.n_in : 1;
    return (sets * blocks * brows * (size_t)m * c.rows * sizeof(__half) + 255) / 256 * 256;
}

// Rows of one (slice, part) plane of the voltage operand.
static long long voltage_rows(int64_t n) { return (n + tcp::BM - 1) / tcp::BM * tcp::BM; }

size_t tc_physical_workspace_bytes(const mf_config& c, int64_t n, int32_t m, int32_t tiles) {
    tcp::Shape s;
    if (!tcp::shape_of(c, s)) return 256;
    size_t bytes = b_operand_bytes(c, s, m, tiles) + 256;
    if (!c.ideal && c.volt_var != 0)
        bytes += (size_t)c.n_in * 2 * voltage_rows(n) * (size_t)m * c.rows * sizeof(__half);
    else if (!c.ideal && (c.wide || c.wide_codes))
        bytes += (size_t)c.n_in * voltage_rows(n) * (size_t)m * c.rows * sizeof(__half);
    return bytes;
}

template <int NIN, int NW, int BN, int NJB, bool SPLIT, int NPART, int KR, bool NL, bool FSUM = false,
          bool VOLT = false, bool PAIRB = false, bool WIDE = false, bool OUTM = false>
static mf_status launch_tcp(const CUtensorMap& mx, const CUtensorMap& mg, const tcp::Args& args, dim3 grid,
                            cudaStream_t st) {
    using G = tcp::Geo<NIN, NW, BN, NJB, KR, SPLIT, NPART, VOLT, PAIRB, WIDE, OUTM>;
    const size_t smem = G::BYTES + 1024;
    auto kern = tcp::tc_physical_kernel<NIN, NW, BN, NJB, KR, SPLIT, NPART, NL, FSUM, VOLT, PAIRB, WIDE, OUTM>;
    int regs = 0;
    {
        const mf_status r = kernel_setup(reinterpret_cast<const void*>(kern), smem, &regs);
        if (r) return r;
    }
    const long long pool = (long long)((regs + 7) / 8 * 8) * tcp::THREADS;
    const long long split = 128LL * tcp::REG_LOW + 32LL * tcp::EPI_WARPS * tcp::REG_HIGH;
    if (split > pool) {
        set_error("tcgen05 physical kernel launched with %d registers/thread cannot host the %d/%d split",
                  regs, tcp::REG_LOW, tcp::REG_HIGH);
        return MF_ERR_RESOURCE;
    }
    kern<<<grid, tcp::THREADS, smem, st>>>(mx, mg, args);
    MF_LAUNCH_CHECK("tc_physical_kernel");
    return MF_OK;
}

template <int NIN, int NW, int BN, int NJB, bool SPLIT>
static mf_status dispatch_tcp(const mf_config& c, const CUtensorMap& mx, const CUtensorMap& mg,
                              const tcp::Args& args, dim3 grid, cudaStream_t st) {
    const bool nl = c.nonlinear != 0;
    if constexpr (SPLIT && NIN == 5 && NW == 5) {
        // Wide configurations (tc_physical_eligible): the digits as FP16 tiles, one column
        // block per CTA, int64 totals and the FP64 epilogue.
        if (c.wide || c.wide_codes) {
            if (c.read_rows == 32)
                return nl ? launch_tcp<5, 5, BN, 1, true, tcp::PARTS, 32, true, false, false, false, true>(
                                mx, mg, args, grid, st)
                          : launch_tcp<5, 5, BN, 1, true, tcp::PARTS, 32, false, false, false, false, true>(
                                mx, mg, args, grid, st);
            return nl ? launch_tcp<5, 5, BN, 1, true, tcp::PARTS, 64, true, false, false, false, true>(mx, mg, args,
                                                                                                       grid, st)
                      : launch_tcp<5, 5, BN, 1, true, tcp::PARTS, 64, false, false, false, false, true>(mx, mg, args,
                                                                                                        grid, st);
        }
    }
    if constexpr (SPLIT) {
        // Output-mode read noise (32-row reads, no voltage noise, tc_physical_eligible):
        // digit sums and second moments per job, the normal draw per ADC event.
        if (tcp::output_mode(c))
            return nl ? launch_tcp<NIN, NW, BN, 1, true, tcp::PARTS, 32, true, false, false, false, false, true>(
                            mx, mg, args, grid, st)
                      : launch_tcp<NIN, NW, BN, 1, true, tcp::PARTS, 32, false, false, false, false, false, true>(
                            mx, mg, args, grid, st);
        // Slice-pair read noise (32-row reads, no voltage noise, tc_physical_eligible): one
        // column block per CTA, every input slice's G' tiles per stage.
        if (tcp::pair_mode(c))
            return nl ? launch_tcp<NIN, NW, BN, 1, true, tcp::PARTS, 32, true, false, false, true>(mx, mg, args, grid,
                                                                                                   st)
                      : launch_tcp<NIN, NW, BN, 1, true, tcp::PARTS, 32, false, false, false, true>(mx, mg, args,
                                                                                                    grid, st);
        // Voltage noise (32-row reads only, tc_physical_eligible): voltage tiles as the A operand.
        if (c.volt_var != 0)
            return nl ? launch_tcp<NIN, NW, BN, NJB, true, tcp::PARTS, 32, true, false, true>(mx, mg, args, grid, st)
                      : launch_tcp<NIN, NW, BN, NJB, true, tcp::PARTS, 32, false, false, true>(mx, mg, args, grid, st);
    }
    if (c.read_rows == 32)
        return nl ? launch_tcp<NIN, NW, BN, NJB, SPLIT, tcp::PARTS, 32, true>(mx, mg, args, grid, st)
                  : launch_tcp<NIN, NW, BN, NJB, SPLIT, tcp::PARTS, 32, false>(mx, mg, args, grid, st);
    return nl ? launch_tcp<NIN, NW, BN, NJB, SPLIT, tcp::PARTS, 64, true>(mx, mg, args, grid, st)
              : launch_tcp<NIN, NW, BN, NJB, SPLIT, tcp::PARTS, 64, false>(mx, mg, args, grid, st);
}

// Ideal devices: one part (the digits), linear ADC.
template <int NIN, int NW, int BN, int NJB>
static mf_status dispatch_digits(const mf_config& c, const CUtensorMap& mx, const CUtensorMap& mg,
                                 const tcp::Args& args, dim3 grid, cudaStream_t st) {
    // Integer totals below 2^24 are exact in FP32.
    if (reconstruction_bound(c) < 16777216.0) {
        if (c.read_rows == 32) return launch_tcp<NIN, NW, BN, NJB, false, 1, 32, false, true>(mx, mg, args, grid, st);
        return launch_tcp<NIN, NW, BN, NJB, false, 1, 64, false, true>(mx, mg, args, grid, st);
    }
    if (c.read_rows == 32) return launch_tcp<NIN, NW, BN, NJB, false, 1, 32, false>(mx, mg, args, grid, st);
    return launch_tcp<NIN, NW, BN, NJB, false, 1, 64, false>(mx, mg, args, grid, st);
}

mf_status tc_physical_sliced_mm(const mf_config& c, const MMArgs& a, void* workspace, size_t ws_bytes,
                                cudaStream_t st) {
    int dev = 0, major = 0;
    MF_CHECK_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
    MF_CHECK_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev), "capability");
    if (major != 10) {
        set_error("tcgen05 path needs an sm_100 device");
        return MF_ERR_UNSUPPORTED;
    }
    tcp::Shape shape;
    if (!tc_physical_eligible(c, a.m) || !tcp::shape_of(c, shape)) {
        set_error("configuration outside the tcgen05 physical plan");
        return MF_ERR_UNSUPPORTED;
    }
    const int tiles = a.tile_end - a.tile_begin;
    const size_t need = tc_physical_workspace_bytes(c, a.n, a.m, tiles);
    if (!workspace || ws_bytes < need) {
        set_error("tcgen05 physical workspace too small: %zu < %zu bytes", ws_bytes, need);
        return MF_ERR_RESOURCE;
    }
    const long long K = (long long)a.m * c.rows;
    const int cols = tiles * c.cols;
    const int blocks = cols / shape.bn;
    int brows = 0, pstride = 0, ones_row = -1, g2row = -1;
    const bool outm = tcp::output_mode(c);
    tcp::rows_of(shape, tcp::parts_of(c), brows, pstride, outm, &ones_row, &g2row);
    const float scale = c.ideal ? 1.0f : tcp::split_scale(c, shape.split != 0);
    const float scale2 = outm ? tcp::square_scale(c) : 1.0f;
    __half* gs = static_cast<__half*>(workspace);
    {
        const int kc = c.rows % tcp::KC == 0 ? tcp::KC : 32;
        const dim3 grid((unsigned)(K / kc), (unsigned)(blocks < 65535 ? blocks : 65535));
        const int pair = tcp::pair_mode(c) ? c.n_in : 0;
        if (c.wide_codes)
            tcp::b_operand_kernel<long long><<<grid, 256, 0, st>>>(
                make_layout(c), make_physics(c), static_cast<const long long*>(a.packed), a.p, a.tile_begin * c.cols,
                blocks, shape.bn, shape.nw, brows, pstride, tcp::parts_of(c), kc, K, a.seed, a.event, scale,
                shape.split, pair, ones_row, g2row, scale2, gs);
        else
            tcp::b_operand_kernel<uint8_t><<<grid, 256, 0, st>>>(
                make_layout(c), make_physics(c), static_cast<const uint8_t*>(a.packed), a.p, a.tile_begin * c.cols,
                blocks, shape.bn, shape.nw, brows, pstride, tcp::parts_of(c), kc, K, a.seed, a.event, scale,
                shape.split, pair, ones_row, g2row, scale2, gs);
        MF_LAUNCH_CHECK("b_operand_kernel");
    }
    CUtensorMap mx, mg;
    const bool volt = !c.ideal && c.volt_var != 0;
    const bool wide = !c.ideal && (c.wide || c.wide_codes);
    const long long n_pad = voltage_rows(a.n);
    mf_status r = MF_OK;
    if (volt && (long long)c.n_in * 2 * n_pad > 2147483647LL) {
        set_error("voltage operand of %lld rows exceeds the TMA row coordinate", (long long)c.n_in * 2 * n_pad);
        return MF_ERR_RESOURCE;
    }
    if (volt) {
        // The voltage operand follows the conductance operand in the workspace.
        __half* va = reinterpret_cast<__half*>(static_cast<uint8_t*>(workspace) + b_operand_bytes(c, shape, a.m, tiles));
        const dim3 grid((unsigned)((K + 255) / 256), (unsigned)(n_pad < 65535 ? n_pad : 65535));
        tcp::a_operand_kernel<<<grid, 256, 0, st>>>(make_layout(c), (float)c.volt_var,
                                                   static_cast<const uint8_t*>(a.codes), a.n, n_pad, a.m, K,
                                                   a.vector_offset, event_seed(a.seed, a.event), va);
        MF_LAUNCH_CHECK("a_operand_kernel");
        r = tc_make_map(&mx, va, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)K, (uint64_t)c.n_in * 2 * n_pad,
                        (uint64_t)K, 16, tcp::BM, CU_TENSOR_MAP_SWIZZLE_32B);
    } else if (wide) {
        // The digit operand follows the conductance operand in the workspace.
        if ((long long)c.n_in * n_pad > 2147483647LL) {
            set_error("digit operand of %lld rows exceeds the TMA row coordinate", (long long)c.n_in * n_pad);
            return MF_ERR_RESOURCE;
        }
        __half* da = reinterpret_cast<__half*>(static_cast<uint8_t*>(workspace) + b_operand_bytes(c, shape, a.m, tiles));
        const dim3 grid((unsigned)((K + 255) / 256), (unsigned)(n_pad < 65535 ? n_pad : 65535));
        if (c.wide_codes)
            tcp::digit_operand_kernel<long long><<<grid, 256, 0, st>>>(
                make_layout(c), static_cast<const long long*>(a.codes), a.n, n_pad, K, da);
        else
            tcp::digit_operand_kernel<uint8_t><<<grid, 256, 0, st>>>(
                make_layout(c), static_cast<const uint8_t*>(a.codes), a.n, n_pad, K, da);
        MF_LAUNCH_CHECK("digit_operand_kernel");
        r = tc_make_map(&mx, da, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)K, (uint64_t)c.n_in * n_pad,
                        (uint64_t)K, 16, tcp::BM, CU_TENSOR_MAP_SWIZZLE_32B);
    } else {
        r = tc_make_map(&mx, a.codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)K, (uint64_t)a.n,
                        (uint64_t)K, (uint32_t)c.read_rows, tcp::BM, CU_TENSOR_MAP_SWIZZLE_NONE);
    }
    const long long sets = tcp::pair_mode(c) ? c.n_in : 1;
    if (!r) r = tc_make_map(&mg, gs, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)K,
                            (uint64_t)(sets * blocks * brows), (uint64_t)K, 16, (uint32_t)tcp::box_rows(brows),
                            CU_TENSOR_MAP_SWIZZLE_32B);
    if (r) return r;
    tcp::Args args{};
    r = tc_error_word(&args.error);
    if (r) return r;
    args.bias = static_cast<const float*>(a.bias);
    args.xscale = static_cast<const float*>(a.xscale);
    args.wscale = static_cast<const float*>(a.wscale);
    args.out = static_cast<float*>(a.out);
    args.n = a.n;
    args.ldo = a.ldo;
    args.ldw = (long long)a.p * c.cols;
    args.out_features = a.out_features;
    args.MR = a.m * c.reads;
    args.full = (long long)args.MR - args.MR % 16;
    args.col_begin = a.tile_begin * c.cols;
    args.col_end = a.tile_end * c.cols;
    args.n_pad = (int)n_pad;
    args.gblocks = blocks;
    if (outm) {
        // Output-mode noise in the units of x (FP16-part sums of d * G' * 2^s):
        // mean factor expm1(s^2/2), variance factor exp(s^2) expm1(s^2) (reference.py:107-114)
        // carried from (2^u G^2) to x^2 units by 2^(2s) / 2^u, and LOW * 2^s for the digit sums.
        const double v2 = c.read_var * c.read_var;
        args.out_mf = (float)expm1(0.5 * v2);
        args.out_vf2 = (float)(exp(v2) * expm1(v2) * (double)scale * (double)scale / (double)scale2);
        args.out_l2s = (float)(c.low * (double)scale);
        args.vector_offset = a.vector_offset;
        args.p_total = a.p;
        args.cols_c = c.cols;
        args.read_seed = event_seed(a.seed, a.event);
        // FP16 bit patterns of d^2 for d = 0..7: 0, 1, 4, 9, 16, 25, 36, 49.
        const uint16_t sq[8] = {0x0000, 0x3C00, 0x4400, 0x4880, 0x4C00, 0x4E40, 0x5080, 0x5220};
        uint8_t lo[8], hi[8];
        for (int d = 0; d < 8; ++d) {
            lo[d] = (uint8_t)(sq[d] & 0xFF);
            hi[d] = (uint8_t)(sq[d] >> 8);
        }
        args.sq_lo_lo = lo[0] | lo[1] << 8 | lo[2] << 16 | (uint32_t)lo[3] << 24;
        args.sq_lo_hi = lo[4] | lo[5] << 8 | lo[6] << 16 | (uint32_t)lo[7] << 24;
        args.sq_hi_lo = hi[0] | hi[1] << 8 | hi[2] << 16 | (uint32_t)hi[3] << 24;
        args.sq_hi_hi = hi[4] | hi[5] << 8 | hi[6] << 16 | (uint32_t)hi[7] << 24;
    }
    // FP16 high bytes of the digits 0..7 (1.0 = 0x3C00, 2.0 = 0x4000, 3.0 = 0x4200, ...).
    const uint8_t hi[8] = {0x00, 0x3C, 0x40, 0x42, 0x44, 0x45, 0x46, 0x47};
    args.lut_lo = hi[0] | hi[1] << 8 | hi[2] << 16 | (uint32_t)hi[3] << 24;
    args.lut_hi = hi[4] | hi[5] << 8 | hi[6] << 16 | (uint32_t)hi[7] << 24;
    for (int i = 0; i < c.n_in; ++i) {
        args.a_shift[i] = c.in_shift[i];
        args.a_mask4[i] = (uint32_t)c.in_mask[i] * 0x01010101u;
    }
    const double inv_unit = 1.0 / c.unit;
    uint32_t sum = 0;
    for (int w = 0; w < c.n_w; ++w) {
        args.cw[w] = (float)(c.voltage * c.w_mask[w] * inv_unit / scale);
        args.slope[w] = (float)(c.nonlinear / c.adc_max[w]);
        // Ideal devices: the accumulator is the digit dot D and the count min(D, max_w).
        args.cws[w] = c.ideal ? (float)(1.0 / c.adc_max[w])
                              : (float)(c.voltage * c.w_mask[w] * inv_unit / scale / c.adc_max[w]);
        args.inv_maxw[w] = (float)(1.0 / c.adc_max[w]);
        args.maxw[w] = (float)c.adc_max[w];
        for (int i = 0; i < c.n_in; ++i) {
            args.factor[i][w] = (int)(c.in_factor[i] * c.w_factor[w]);
            args.ffactor[i][w] = (float)args.factor[i][w];
            sum += (uint32_t)args.factor[i][w];
        }
    }
    args.offset = (int)(0u - 0x4B400000u * sum);
    {
        // The same constant modulo 2^64 for the int64 totals of wide configurations.
        uint64_t sum64 = 0;
        for (int w = 0; w < c.n_w; ++w)
            for (int i = 0; i < c.n_in; ++i) sum64 += (uint64_t)(int64_t)(c.in_factor[i] * c.w_factor[w]);
        args.offset64 = (long long)(0ull - 0x4B400000ull * sum64);
    }
    const int bc = shape.bn * shape.njb;
    args.raster = a.raster;
    const dim3 grid = raster_grid((a.n + tcp::BM - 1) / tcp::BM, (cols + bc - 1) / bc, a.raster);
    if (c.ideal) {
        if (shape.nin == 5) return dispatch_digits<5, 5, 32, 1>(c, mx, mg, args, grid, st);
        if (shape.nin == 3) return dispatch_digits<3, 3, 32, 2>(c, mx, mg, args, grid, st);
        if (shape.nin == 8) return dispatch_digits<8, 8, 16, 1>(c, mx, mg, args, grid, st);
        return dispatch_digits<4, 4, 32, 1>(c, mx, mg, args, grid, st);
    }
    if (shape.nin == 5) return dispatch_tcp<5, 5, 16, 2, true>(c, mx, mg, args, grid, st);
    if (shape.nin == 3) return dispatch_tcp<3, 3, 32, 1, true>(c, mx, mg, args, grid, st);
    if (shape.nin == 8) return dispatch_tcp<8, 8, 16, 1, false>(c, mx, mg, args, grid, st);
    return dispatch_tcp<4, 4, 16, 2, true>(c, mx, mg, args, grid, st);
}

}  // namespace mf

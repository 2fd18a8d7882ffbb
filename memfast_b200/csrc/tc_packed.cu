// tcgen05 / TMEM kernel for the ideal-device sliced product with packed
// integer counts (sm_100a).
//
// The reference's count for input slice a, weight slice w and one read of
// rows_per_read rows is min(D_aw, m_w), D_aw = sum_r d_a(r) d_w(r)
// (memfast/reference.py:81-115, kernels.cu:108-169), and the read's total is
// T = sum_aw s_a s_w count.  With min(D, m) = D - relu(D - m):
//
//     T = x . w  +  sum over clip-capable (a, w) of (-s_a s_w) relu(D_aw - m_w)
//
// x . w comes from one kind::i8 MMA of the raw codes.  The clip-capable pairs
// whose threshold is within reach of ordinary data ("always" pairs) are counted
// by further kind::i8 MMAs of unsigned digit planes.  Several D_aw share one
// 32-bit TMEM accumulator: plane bytes are pre-scaled by powers of two,
// (d_a << ka) * (d_w << kb), so D_aw lands at bit ka + kb of the count column
// and the exact s32 accumulation keeps the fields apart.  Because m_w + 1 is a
// power of two, "some D of this warp clips" is one OR over the loaded columns
// and a mask; the relu corrections run only for the fields that fire.
//
// The remaining clip-capable pairs have thresholds near their maximum (for
// example m = 255 for two 2-bit digits over 32 rows, at most 288).  They are
// not counted: a column whose digit sum bounds D_aw <= m_w for every read is
// exact without them.  Otherwise the CTA raises its tile flag and
// tc_packed_sliced_mm reruns that 128 x 128 tile with the generic kernel.
//
// Tensor-core instructions on these shapes cost about the same whatever their
// N, so the MMAs are made as wide as TMEM allows: a job is 64 output columns,
// a TMEM unit holds its base x . w block and up to three 64-column count
// blocks, and MMAs that share an input plane are merged across adjacent count
// blocks (N up to 192) with their weight planes laid out contiguously.  The
// host chooses the block order, the weight-plane slot layout and the MMA order.
//
// Roles (THREADS threads, 1 CTA per SM, 128 rows x 128 columns per CTA):
//   warp 0            TMA producer: code tiles of x and w per read, scale blocks
//   warp 1            TMEM owner and MMA issuer (one elected thread)
//   warps 2-3         idle after set-up
//   warps 4 .. 4+E-1  epilogue: E / 4 warps per TMEM lane quadrant, 16 columns
//                     of every 64-column job each
//   last warpgroup    transform: input digit planes and weight digit-plane slots
//                     in shared memory, rare-pair column bounds
// Two TMEM units alternate, so one job's MMAs overlap the other job's epilogue.
// The finished 128 x 128 tile is staged in shared memory and stored coalesced.
// Every mbarrier wait is bounded; on timeout the CTA records an error code,
// waits (bounded) for its own TMA loads and MMAs, frees TMEM and exits, and its
// tile takes the generic rerun.
#include <cuda.h>
#include <cuda_runtime.h>
#include <string.h>

#include "common.cuh"
#include "kernels.cuh"
#include "tcgen05.cuh"

namespace mf {
namespace tp {

using namespace tg;

constexpr int BM = 128;          // vectors per CTA (TMEM lanes)
constexpr int BN = 128;          // output columns per CTA
constexpr int JOBN = 64;         // output columns per job (base MMA N)
constexpr int NJOB = BN / JOBN;  // jobs per read
constexpr int KR = 32;           // rows per read (MMA K for 8-bit operands)
constexpr int STAGES = 3;
constexpr int SCB = 4;           // reads per scale block
constexpr int SCRING = 4;        // scale blocks in flight
constexpr int MAXA = 3;          // scaled input digit planes
constexpr int MAXB = 5;          // scaled weight digit planes
constexpr int MAXSLOT = 6;       // weight-plane slots per job (a plane may fill several)
constexpr int MAXCOL = 3;        // packed count blocks per job
constexpr int MAXFIELD = 3;      // counts per count block
constexpr int MAXMMA = 6;        // plane MMAs per job
constexpr int MAXRARE = 8;       // weight slices of rare pairs (column bounds), 64-row reads
constexpr int MAXRARE_32 = 4;    // the same for 32-row reads (keeps the transform's registers)
constexpr int UNITS = 512 / (JOBN * (1 + MAXCOL));
constexpr int UNIT_COLS = JOBN * (1 + MAXCOL);
constexpr int EPI_WARPS = 16;
constexpr int EC = JOBN / (EPI_WARPS / 4);   // columns of a job per epilogue thread
constexpr int EH = 8;                        // columns loaded from TMEM at a time
constexpr int XF_WARPS = 4;
constexpr int EPI_WARP0 = 4;
constexpr int XF_WARP0 = EPI_WARP0 + EPI_WARPS;
constexpr int THREADS = 32 * (XF_WARP0 + XF_WARPS);
constexpr int TILE = BM * KR;    // one [128 x 32] 8-bit tile
constexpr int SLOT = JOBN * KR;  // one [JOBN x 32] 8-bit weight-plane slot
constexpr int EPI_BARRIER = 1;   // named barrier of the epilogue warps

// Register split.  setmaxnreg draws on the registers the block was launched
// with, so the three warpgroup shares must fit THREADS * LAUNCH_REGS; the host
// checks the launched register count before every launch.
constexpr int LAUNCH_REGS = (65536 / THREADS) / 8 * 8;
constexpr int REG_CTRL = 56;
constexpr int REG_XF = 40;
constexpr int REG_EPI = ((THREADS * LAUNCH_REGS - 128 * REG_CTRL - 32 * XF_WARPS * REG_XF) / (32 * EPI_WARPS)) / 8 * 8;
static_assert(REG_EPI >= 64 && REG_EPI <= 256, "epilogue register share out of range");
static_assert(128 * REG_CTRL + 32 * XF_WARPS * REG_XF + 32 * EPI_WARPS * REG_EPI <= THREADS * LAUNCH_REGS,
              "register split exceeds the launch pool");
static_assert(UNITS * UNIT_COLS <= 512, "TMEM holds 512 columns");
static_assert(EC % EH == 0 && EH >= 4 && EH % 2 == 0, "epilogue slices");

struct Smem {
    uint8_t x[STAGES][TILE];                        // TMA: activation codes [128 rows][32 B]
    uint8_t w[STAGES][TILE];                        // TMA: weight codes, K-major [128 cols][32 B]
    uint8_t ap[STAGES][MAXA][TILE];                 // scaled input digit planes
    uint8_t bp[STAGES][NJOB][MAXSLOT][SLOT];        // weight digit-plane slots per job
    float acc1[BN][BM + 1];                         // cascade level 1 / output staging, [column][row]
    float xs[SCRING][BM][SCB];                      // TMA: input scales [row][read]
    float ws[SCRING][SCB][BN];                      // TMA: weight scales [read][column]
    uint64_t full[STAGES], ready[STAGES], empty[STAGES];
    uint64_t sc_full[SCRING], sc_empty[SCRING];
    uint64_t unit_full[UNITS], unit_empty[UNITS];
    uint64_t drained;
    uint32_t tmem_base;
    int abort;
    unsigned rare;
    int4 field[MAXCOL * MAXFIELD];                  // (shift, width mask, m, coef) of every count
    uint8_t fieldbit[MAXCOL][32];                   // field of count block c holding bit b
};
static_assert(sizeof(Smem) + 1024 <= 232448, "packed kernel exceeds the 227 KB shared-memory limit");

// One packed count: D = (column >> shift) & width_mask; the read's total gains
// coef * max(D - m, 0).  `clip` holds the field's bits at or above log2(m + 1).
struct Field {
    int shift;
    int width_mask;
    int m;
    int coef;
    uint32_t clip;
};

// One plane MMA of a job: input plane `a` times weight slots [slot, slot + n)
// into count blocks [block, block + n); `acc` = 0 overwrites them.
struct Mma {
    int a, slot, n, block, acc;
};

struct Plan {
    int na, nb, nslot, ncol, nmma, nrare;
    int a_src[MAXA], a_mask[MAXA], a_scale[MAXA];   // plane byte = ((code >> src) & mask) << scale
    int b_src[MAXB], b_mask[MAXB], b_scale[MAXB];
    int slot_plane[MAXSLOT];                        // weight plane held by each slot
    Mma mma[MAXMMA];
    int nfield[MAXCOL];
    Field field[MAXCOL][MAXFIELD];                  // fields of count block c
    uint32_t colclip[MAXCOL];                       // union of the block's field clip bits
    int r_src[MAXRARE], r_mask[MAXRARE], r_limit[MAXRARE];   // rare: flag if digit sum > limit
    int b_signed;
};

struct Args {
    Plan plan;
    const float* bias;      // [out_features] or null
    float* out;
    long long n, ldo;
    int out_features, MR;
    long long full;         // reads in complete 16-read cascade blocks
    int col_begin, col_end;
    unsigned* error;        // device error word
    unsigned* tile_flags;   // [column blocks][vector blocks]: 1 = tile needs the generic rerun
    int raster;             // 0: blockIdx.x walks vector blocks; 1: blockIdx.x walks column blocks
    int stop_stage;         // test hook (mf_debug_stall_next_launch): the producer issues no
                            // load from this pipeline stage on; -1 = off
    long long wait_cycles;  // budget of every bounded wait of the launch
    float* peer_out[MF_MAX_PEERS];   // other GPUs' output buffers (same offsets as out), or none
    int n_peers;
};

__device__ __forceinline__ uint32_t or3(uint32_t a, uint32_t b, uint32_t c) { return a | b | c; }

__device__ __forceinline__ void epilogue_barrier() {
    asm volatile("bar.sync %0, %1;" ::"n"(EPI_BARRIER), "n"(32 * EPI_WARPS) : "memory");
}

// H: 32-row stages per read (1 for 32-row reads, 2 for 64-row reads: both
// stages' MMAs accumulate into the read's TMEM unit before the epilogue sees it).
template <int NCOL, int H>
__global__ void __launch_bounds__(THREADS, 1)
    packed_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                  const __grid_constant__ CUtensorMap map_xs, const __grid_constant__ CUtensorMap map_ws,
                  const __grid_constant__ Args args) {
    static_assert(NCOL <= MAXCOL, "too many count blocks");
    static_assert(H == 1 || H == 2, "reads of 32 or 64 rows");
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    Smem& s = *reinterpret_cast<Smem*>(smem_align1024(smem_raw));
    const Plan& P = args.plan;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const unsigned vblk = raster_vector_block(args.raster), cblk = raster_column_block(args.raster);
    const long long n0 = (long long)vblk * BM;
    const int c0 = args.col_begin + cblk * BN;
    const int MR = args.MR;
    unsigned* err = args.error;
    const long long budget = args.wait_cycles;

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.ready[i], XF_WARPS);
            mbar_init(&s.empty[i], 1);
        }
        for (int i = 0; i < SCRING; ++i) {
            mbar_init(&s.sc_full[i], 1);
            mbar_init(&s.sc_empty[i], EPI_WARPS);
        }
        for (int u = 0; u < UNITS; ++u) {
            mbar_init(&s.unit_full[u], 1);
            mbar_init(&s.unit_empty[u], EPI_WARPS);
        }
        mbar_init(&s.drained, 1);
        s.abort = 0;
        s.rare = 0;
        for (int c = 0; c < MAXCOL; ++c)
            for (int f = 0; f < MAXFIELD; ++f) {
                const Field F = P.field[c][f];
                s.field[c * MAXFIELD + f] = make_int4(F.shift, F.width_mask, F.m, F.coef);
            }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int idx = threadIdx.x; idx < BN * (BM + 1); idx += THREADS) (&s.acc1[0][0])[idx] = 0.0f;
    if (threadIdx.x < MAXCOL * 32) {
        const int c = threadIdx.x / 32, b = threadIdx.x % 32;
        uint8_t holder = 0;
        for (int f = 0; f < P.nfield[c]; ++f) {
            const Field F = P.field[c][f];
            if (b >= F.shift && b < F.shift + __popc((unsigned)F.width_mask)) holder = (uint8_t)f;
        }
        s.fieldbit[c][b] = holder;
    }
    if (warp == 0 && lane == 0) {
        prefetch_map(&map_x);
        prefetch_map(&map_w);
        prefetch_map(&map_xs);
        prefetch_map(&map_ws);
    }
    if (warp == 1) tmem_alloc(&s.tmem_base, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s.tmem_base;

    if (warp < EPI_WARP0) {
        set_maxnreg_dec<REG_CTRL>();
        if (warp == 0 && lane == 0) {
            // ------------------------------------------------------------ producer
            int issued = 0, scissued = 0;
            for (int stage = 0; stage < MR * H; ++stage) {
                // Test hook: stop issuing here; the consumers' waits on this stage then
                // run out of budget and the CTA takes its error exit.
                if (stage == args.stop_stage) break;
                const int i = stage / H;
                if (stage % H == 0 && i % SCB == 0) {
                    const int b = i / SCB, sb = b % SCRING;
                    if (!mbar_wait(&s.sc_empty[sb], ((b / SCRING) & 1) ^ 1, &s.abort, err, 21, budget)) break;
                    mbar_expect_tx(&s.sc_full[sb], (BM + BN) * SCB * 4);
                    tma_load_2d(s.xs[sb], &map_xs, i, (int)n0, &s.sc_full[sb]);
                    tma_load_2d(s.ws[sb], &map_ws, c0, i, &s.sc_full[sb]);
                    scissued = b + 1;
                }
                const int st = stage % STAGES;
                if (!mbar_wait(&s.empty[st], ((stage / STAGES) & 1) ^ 1, &s.abort, err, 22, budget)) break;
                mbar_expect_tx(&s.full[st], 2 * TILE);
                tma_load_2d(s.x[st], &map_x, stage * KR, (int)n0, &s.full[st]);
                tma_load_2d(s.w[st], &map_w, stage * KR, c0, &s.full[st]);
                issued = stage + 1;
            }
            // Every issued load lands before the CTA may exit.
            for (int i = issued - STAGES > 0 ? issued - STAGES : 0; i < issued; ++i)
                mbar_drain(&s.full[i % STAGES], (i / STAGES) & 1);
            for (int b = scissued - SCRING > 0 ? scissued - SCRING : 0; b < scissued; ++b)
                mbar_drain(&s.sc_full[b % SCRING], (b / SCRING) & 1);
        } else if (warp == 1 && lane == 0) {
            // ------------------------------------------------------------ MMA issuer
            // One thread issues every MMA, so the loop body is kept to a few integer
            // adds per MMA: descriptors are built once for stage 0 / job 0 and moved by
            // adding the 16-byte-unit offset of the stage, job, plane and slot to their
            // start-address field (all shared-memory offsets stay below 256 KB, so the
            // 14-bit field never carries).
            const uint32_t id_base = idesc_i8(BM, JOBN, true, P.b_signed != 0);
            const uint64_t dx0 = desc_sw32(s.x[0]), dw0 = desc_sw32(s.w[0]);
            const uint64_t da0 = desc_sw32(s.ap[0][0]), db0 = desc_sw32(s.bp[0][0][0]);
            constexpr uint32_t kStageX = sizeof(s.x[0]) >> 4, kStageA = sizeof(s.ap[0]) >> 4;
            constexpr uint32_t kStageB = sizeof(s.bp[0]) >> 4, kJobB = sizeof(s.bp[0][0]) >> 4;
            constexpr uint32_t kJobW = (JOBN * KR) >> 4;
            const int nmma = P.nmma;
            uint32_t a_off[MAXMMA], b_off[MAXMMA], t_off[MAXMMA], idesc[MAXMMA], acc[MAXMMA];
#pragma unroll
            for (int k = 0; k < MAXMMA; ++k) {
                const Mma M = P.mma[k];
                a_off[k] = (uint32_t)M.a * (TILE >> 4);
                b_off[k] = (uint32_t)M.slot * (SLOT >> 4);
                t_off[k] = (uint32_t)(1 + M.block) * JOBN;
                idesc[k] = idesc_i8(BM, JOBN * (M.n > 0 ? M.n : 1), false, false);
                acc[k] = (uint32_t)M.acc;
            }
            uint32_t u = 0, uphase = 0;
            bool ok = true;
            for (int stage = 0; stage < MR * H && ok; ++stage) {
                const int st = stage % STAGES;
                // Stage hh of a read: the first takes the read's units (waiting for the
                // epilogue to free them) and overwrites them; later stages accumulate,
                // and the last one hands the units to the epilogue.
                const uint32_t hh = (uint32_t)(stage % H);
                if (!mbar_wait(&s.ready[st], (stage / STAGES) & 1, &s.abort, err, 23, budget)) break;
                tc_fence_after();
                const uint64_t dx = dx0 + st * kStageX, dw = dw0 + st * kStageX;
                const uint64_t da = da0 + st * kStageA, dbs = db0 + st * kStageB;
                uint32_t uj = u, ph = uphase;
#pragma unroll
                for (int j = 0; j < NJOB; ++j) {
                    if (hh == 0 && !mbar_wait(&s.unit_empty[uj], ph ^ 1, &s.abort, err, 24, budget)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t buf = tmem + uj * UNIT_COLS;
                    mma_i8(buf, dx, dw + j * kJobW, id_base, hh != 0);
                    const uint64_t db = dbs + j * kJobB;
#pragma unroll
                    for (int k = 0; k < MAXMMA; ++k)
                        if (k < nmma)
                            mma_i8(buf + t_off[k], da + a_off[k], db + b_off[k], idesc[k], acc[k] | (hh != 0));
                    if (hh == H - 1) mma_commit(&s.unit_full[uj]);
                    if (++uj == UNITS) {
                        uj = 0;
                        ph ^= 1;
                    }
                }
                if (hh == H - 1) {
                    u = uj;
                    uphase = ph;
                }
                if (ok) mma_commit(&s.empty[st]);
            }
            // All issued MMAs complete before TMEM is released.
            mma_commit(&s.drained);
            mbar_drain(&s.drained, 0);
        }
    } else if (warp >= XF_WARP0) {
        set_maxnreg_dec<REG_XF>();
        // ---------------------------------------------------------------- transform
        // Thread t builds row t of every input plane and column t of every weight
        // slot.  Row t of a [rows x 32] SW32 tile keeps its two 16-byte chunks inside
        // the row and its swizzle phase depends on t mod 8 only, so an elementwise
        // transform written at the same offsets stays swizzled, also inside a
        // 64-row slot.
        const int t = threadIdx.x - 32 * XF_WARP0;
        const int job = t / JOBN;
        const int jrow = t % JOBN;
        // ((x >> src) & m) << sc per byte of a word as one rotate and one mask:
        // rotating right by src - sc (mod 32) moves each byte's digit to bit sc of
        // the same byte, and the bits that cross a byte boundary land outside the
        // mask (src + width <= 8), also in the rotate's wrap-around.
        uint32_t a_rot[MAXA], a_m4[MAXA];
        uint32_t s_rot[MAXSLOT], s_m4[MAXSLOT];
        constexpr int NRARE = H > 1 ? MAXRARE : MAXRARE_32;
        uint32_t r_src[NRARE], r_m4[NRARE];
        int r_lim[NRARE];
        // Rare-pair digit sums run over a whole read (both stages of a 64-row read).
        uint32_t rsum[H > 1 ? NRARE : 1];
        const int na = P.na, nslot = P.nslot, nr = P.nrare;
#pragma unroll
        for (int a = 0; a < MAXA; ++a) {
            a_rot[a] = (uint32_t)(P.a_src[a] - P.a_scale[a]) & 31u;
            a_m4[a] = ((uint32_t)P.a_mask[a] << P.a_scale[a]) * 0x01010101u;
        }
#pragma unroll
        for (int q = 0; q < MAXSLOT; ++q) {
            const int b = P.slot_plane[q];
            s_rot[q] = (uint32_t)(P.b_src[b] - P.b_scale[b]) & 31u;
            s_m4[q] = ((uint32_t)P.b_mask[b] << P.b_scale[b]) * 0x01010101u;
        }
#pragma unroll
        for (int q = 0; q < NRARE; ++q) {
            r_src[q] = P.r_src[q];
            r_m4[q] = (uint32_t)P.r_mask[q] * 0x01010101u;
            r_lim[q] = P.r_limit[q];
        }
#pragma unroll
        for (int q = 0; q < (H > 1 ? NRARE : 1); ++q) rsum[q] = 0;
        bool rare = false;
        for (int stage = 0; stage < MR * H; ++stage) {
            const int st = stage % STAGES;
            const int hh = stage % H;
            if (!__all_sync(0xFFFFFFFFu, mbar_wait(&s.full[st], (stage / STAGES) & 1, &s.abort, err, 25, budget))) break;
            const uint4* xrow = reinterpret_cast<const uint4*>(s.x[st] + t * KR);
            const uint4 xa = xrow[0], xb = xrow[1];
            const uint32_t xw[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
            for (int a = 0; a < MAXA; ++a) {
                if (a >= na) break;
                uint32_t d[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) d[k] = __funnelshift_r(xw[k], xw[k], a_rot[a]) & a_m4[a];
                uint4* dst = reinterpret_cast<uint4*>(s.ap[st][a] + t * KR);
                dst[0] = make_uint4(d[0], d[1], d[2], d[3]);
                dst[1] = make_uint4(d[4], d[5], d[6], d[7]);
            }
            const uint4* wrow = reinterpret_cast<const uint4*>(s.w[st] + t * KR);
            const uint4 wa = wrow[0], wb = wrow[1];
            const uint32_t ww[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
            for (int q = 0; q < MAXSLOT; ++q) {
                if (q >= nslot) break;
                uint32_t d[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) d[k] = __funnelshift_r(ww[k], ww[k], s_rot[q]) & s_m4[q];
                uint4* dst = reinterpret_cast<uint4*>(s.bp[st][job][q] + jrow * KR);
                dst[0] = make_uint4(d[0], d[1], d[2], d[3]);
                dst[1] = make_uint4(d[4], d[5], d[6], d[7]);
            }
#pragma unroll
            for (int q = 0; q < NRARE; ++q) {
                if (q >= nr) break;
                uint32_t sum = (H == 1 || hh == 0) ? 0u : rsum[H > 1 ? q : 0];
#pragma unroll
                for (int k = 0; k < 8; ++k) sum = __dp4a((ww[k] >> r_src[q]) & r_m4[q], 0x01010101u, sum);
                if (hh == H - 1) rare |= (int)sum > r_lim[q];
                else rsum[H > 1 ? q : 0] = sum;
            }
            // Plane writes (generic proxy) must be visible to the tensor core (async proxy).
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.ready[st]);
        }
        if (__any_sync(0xFFFFFFFFu, rare) && lane == 0) atomicOr(&s.rare, 1u);
    } else {
        set_maxnreg_inc<REG_EPI>();
        // ---------------------------------------------------------------- epilogue
        // Warp w reads TMEM lane quadrant w & 3 and the EC-column slice hc of each
        // job, EH columns at a time.  A unit is handed back to the MMA as soon as
        // its last columns are in registers.
        const int quad = warp & 3;
        const int hc = (warp - EPI_WARP0) >> 2;
        const int r = quad * 32 + lane;             // CTA row = TMEM lane
        const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16) + hc * EC;
        float acc0[NJOB][EC];
#pragma unroll
        for (int j = 0; j < NJOB; ++j)
#pragma unroll
            for (int e = 0; e < EC; ++e) acc0[j][e] = 0.0f;
        uint32_t u = 0, uphase = 0;
        bool ok = true;
        for (int i = 0; i < MR && ok; ++i) {
            const int b = i / SCB, sb = b % SCRING;
            if (i % SCB == 0) {
                ok = __all_sync(0xFFFFFFFFu, mbar_wait(&s.sc_full[sb], (b / SCRING) & 1, &s.abort, err, 26, budget));
                if (!ok) break;
            }
            const float xs = s.xs[sb][r][i % SCB];
#pragma unroll
            for (int j = 0; j < NJOB; ++j) {
                ok = __all_sync(0xFFFFFFFFu, mbar_wait(&s.unit_full[u], uphase, &s.abort, err, 27, budget));
                if (!ok) break;
                tc_fence_after();
                const uint32_t buf = lane_base + u * UNIT_COLS;
#pragma unroll
                for (int h = 0; h < EC / EH; ++h) {
                    uint32_t vb[EH], vc[NCOL > 0 ? NCOL : 1][EH];
                    tmem_ld(buf + h * EH, vb);
#pragma unroll
                    for (int c = 0; c < NCOL; ++c) tmem_ld(buf + (1 + c) * JOBN + h * EH, vc[c]);
                    tmem_wait(vb);
#pragma unroll
                    for (int c = 0; c < NCOL; ++c) tmem_wait(vc[c]);
                    if (h == EC / EH - 1) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&s.unit_empty[u]);
                    }
                    int T[EH];
#pragma unroll
                    for (int e = 0; e < EH; ++e) T[e] = (int)vb[e];
                    if (NCOL > 0) {
                        // Exact clip test: some D of the warp exceeds its m iff a clip bit is set.
                        // o[c]: OR of block c's columns; hit = OR of (o[c] & clip bits), one
                        // three-input logic operation per block.
                        uint32_t o[NCOL > 0 ? NCOL : 1];
                        uint32_t hit = 0;
#pragma unroll
                        for (int c = 0; c < NCOL; ++c) {
                            uint32_t acc = or3(vc[c][0], vc[c][1], vc[c][2]);
#pragma unroll
                            for (int e = 3; e + 1 < EH; e += 2) acc = or3(acc, vc[c][e], vc[c][e + 1]);
                            acc |= vc[c][EH - 1];
                            o[c] = acc;
                            hit = (acc & P.colclip[c]) | hit;
                        }
                        if (hit != 0) {
                            // Only the lanes whose own counts clip (usually one lane of a
                            // chunk, when any): per count block, the clip bits set in this
                            // lane's columns name the counts that clip, and
                            // T += -s_a s_w * max(D - m, 0) for those only.  (A warp-wide
                            // vote and reduction of the clip bits measured 3% slower.)
#pragma unroll
                            for (int c = 0; c < NCOL; ++c) {
                                uint32_t fired = o[c] & P.colclip[c];
                                while (fired) {
                                    const int4 F = s.field[c * MAXFIELD + s.fieldbit[c][__ffs(fired) - 1]];
                                    fired &= ~((uint32_t)F.y << F.x);
#pragma unroll
                                    for (int e = 0; e < EH; ++e) {
                                        const int d = (int)((vc[c][e] >> F.x) & (uint32_t)F.y);
                                        T[e] += F.w * __viaddmax_s32(d, -F.z, 0);
                                    }
                                }
                            }
                        }
                    }
                    // fl(fl(T * xs) * ws) pushed into cascade level 0 for read i (|T| < 2^22:
                    // float(T) is exact).  Packed round-to-nearest multiplies, then SCALAR
                    // adds (a packed multiply followed by a packed add was observed to round
                    // once, as an FMA, which the reference does not).
                    const float2* wsr =
                        reinterpret_cast<const float2*>(&s.ws[sb][i % SCB][j * JOBN + hc * EC + h * EH]);
#pragma unroll
                    for (int e = 0; e < EH / 2; ++e) {
                        const float2 tf = make_float2(__int2float_rn(T[2 * e]), __int2float_rn(T[2 * e + 1]));
                        const float2 pr = __fmul2_rn(__fmul2_rn(tf, make_float2(xs, xs)), wsr[e]);
                        acc0[j][h * EH + 2 * e] = __fadd_rn(acc0[j][h * EH + 2 * e], pr.x);
                        acc0[j][h * EH + 2 * e + 1] = __fadd_rn(acc0[j][h * EH + 2 * e + 1], pr.y);
                    }
                }
                if (++u == UNITS) {
                    u = 0;
                    uphase ^= 1;
                }
            }
            if (!ok) break;
            __syncwarp();
            if (lane == 0 && (i % SCB == SCB - 1 || i == MR - 1)) mbar_arrive(&s.sc_empty[sb]);
            // Block boundary of the 16-read cascade: level 1 += level 0 (MR <= 256 keeps two levels).
            const int done = i + 1;
            if (done <= args.full && (done & 15) == 0) {
#pragma unroll
                for (int j = 0; j < NJOB; ++j)
#pragma unroll
                    for (int e = 0; e < EC; ++e) {
                        const int cl = j * JOBN + hc * EC + e;
                        s.acc1[cl][r] = __fadd_rn(s.acc1[cl][r], acc0[j][e]);
                        acc0[j][e] = 0.0f;
                    }
            }
        }
        // Finish in place: acc0 + acc1 + acc2 + acc3 (upper levels zero), the
        // reference's store into a zero-filled output, then the bias.
#pragma unroll
        for (int j = 0; j < NJOB; ++j)
#pragma unroll
            for (int e = 0; e < EC; ++e) {
                const int cl = j * JOBN + hc * EC + e;
                const int col = c0 + cl;
                float value = __fadd_rn(acc0[j][e], s.acc1[cl][r]);
                value = __fadd_rn(value, 0.0f);
                value = __fadd_rn(value, 0.0f);
                value = __fadd_rn(0.0f, value);
                if (args.bias && col < args.col_end && col < args.out_features) value = __fadd_rn(value, args.bias[col]);
                s.acc1[cl][r] = value;
            }
        epilogue_barrier();
        const int q = threadIdx.x - 32 * EPI_WARP0;
        const int cl = q % BN;
        const int col = c0 + cl;
        if (ok && col < args.col_end && col < args.out_features) {
            // Coalesced store: each warp writes 32 consecutive columns of one row.
            for (int rr = q / BN; rr < BM; rr += (32 * EPI_WARPS) / BN) {
                const long long row = n0 + rr;
                if (row >= args.n) continue;
                const float value = s.acc1[cl][rr];
                args.out[row * args.ldo + col] = value;
                // Row-sharded products: the same output into every peer's buffer over
                // NVLink (plain stores), in place of an all-gather after the kernel.
                for (int g = 0; g < args.n_peers; ++g) args.peer_out[g][row * args.ldo + col] = value;
            }
            // The peer stores are performed before anything this GPU does after the kernel.
            if (args.n_peers) __threadfence_system();
        }
    }
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0)
        args.tile_flags[(size_t)cblk * raster_vector_blocks(args.raster) + vblk] = (s.rare || s.abort) ? 1u : 0u;
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

}  // namespace tp

// =================================================================== host side
namespace {

int bitlen(long long v) {
    int b = 0;
    while ((1LL << b) <= v) ++b;
    return b;
}

// Largest k with mask << k still an unsigned byte.
int max_scale(int mask) {
    int k = 0;
    while ((mask << (k + 1)) <= 255) ++k;
    return k;
}

struct Count {
    int a, w;        // input / weight slice
    int width;       // bits that hold the largest D
    int clipbit;     // log2(m + 1)
    int m, coef;
};

// Depth-first assignment of the always-pair counts to count blocks, shifts and
// scaled digit planes within the kernel's budgets.
struct Packer {
    const mf_config& c;
    Count f[64];
    int nf = 0;
    int ncol = 0, top[tp::MAXCOL] = {}, nfc[tp::MAXCOL] = {};
    int col[64], ka[64], kb[64], shift[64];
    int a_idx[tp::MAXA], a_k[tp::MAXA], na = 0;
    int b_idx[tp::MAXB], b_k[tp::MAXB], nb = 0;
    long nodes = 0;

    explicit Packer(const mf_config& cfg) : c(cfg) {}

    int find_a(int a, int k) const {
        for (int i = 0; i < na; ++i)
            if (a_idx[i] == a && a_k[i] == k) return i;
        return -1;
    }
    int find_b(int w, int k) const {
        for (int i = 0; i < nb; ++i)
            if (b_idx[i] == w && b_k[i] == k) return i;
        return -1;
    }

    bool place(int i) {
        if (i == nf) return true;
        if (++nodes > 200000) return false;
        const Count& q = f[i];
        const int mka = max_scale(c.in_mask[q.a]), mkb = max_scale(c.w_mask[q.w]);
        for (int cc = 0; cc <= ncol && cc < tp::MAXCOL; ++cc) {
            const bool fresh = cc == ncol;
            const int sh = fresh ? 0 : top[cc];
            if (!fresh && nfc[cc] >= tp::MAXFIELD) continue;
            if (sh + q.width > 31) continue;
            // Splits that reuse existing planes first.
            for (int pass = 0; pass < 3; ++pass) {
                for (int k1 = 0; k1 <= mka; ++k1) {
                    const int k2 = sh - k1;
                    if (k2 < 0 || k2 > mkb) continue;
                    const int ea = find_a(q.a, k1), eb = find_b(q.w, k2);
                    const int reuse = (ea >= 0) + (eb >= 0);
                    if (reuse != 2 - pass) continue;
                    const bool new_a = ea < 0, new_b = eb < 0;
                    if (new_a && na >= tp::MAXA) continue;
                    if (new_b && nb >= tp::MAXB) continue;
                    if (new_a) { a_idx[na] = q.a; a_k[na] = k1; ++na; }
                    if (new_b) { b_idx[nb] = q.w; b_k[nb] = k2; ++nb; }
                    const int saved_top = fresh ? 0 : top[cc];
                    if (fresh) { ++ncol; top[cc] = 0; nfc[cc] = 0; }
                    col[i] = cc; ka[i] = k1; kb[i] = k2; shift[i] = sh;
                    top[cc] = sh + q.width;
                    ++nfc[cc];
                    if (place(i + 1)) return true;
                    --nfc[cc];
                    top[cc] = saved_top;
                    if (fresh) --ncol;
                    if (new_b) --nb;
                    if (new_a) --na;
                }
            }
        }
        return false;
    }
};

// A run of fields sharing one input plane over consecutive count blocks: one MMA.
struct Run {
    int a, pos, n;               // input plane, first block position, blocks
    int plane[tp::MAXCOL];       // weight plane of each block
};

bool next_permutation(int* v, int n) {
    int k = n - 2;
    while (k >= 0 && v[k] >= v[k + 1]) --k;
    if (k < 0) return false;
    int l = n - 1;
    while (v[l] <= v[k]) --l;
    int tmp = v[k];
    v[k] = v[l];
    v[l] = tmp;
    for (int a = k + 1, b = n - 1; a < b; ++a, --b) {
        tmp = v[a];
        v[a] = v[b];
        v[b] = tmp;
    }
    return true;
}

bool contains(const int* lay, int len, const int* seq, int n, int* at) {
    for (int st = 0; st + n <= len; ++st) {
        bool eq = true;
        for (int q = 0; q < n && eq; ++q) eq = lay[st + q] == seq[q];
        if (eq) {
            if (at) *at = st;
            return true;
        }
    }
    return false;
}

// Shortest weight-slot layout in which every run's planes are contiguous: every
// order of the multi-block runs, each appended with the largest overlap.
bool slot_layout(const Run* runs, int nrun, int nb, int* slots, int* nslot, int* run_slot) {
    int multi[64], nmulti = 0;
    for (int i = 0; i < nrun; ++i)
        if (runs[i].n > 1) multi[nmulti++] = i;
    if (nmulti > 6) return false;
    int perm[6];
    for (int i = 0; i < nmulti; ++i) perm[i] = i;
    int best = 1 << 30;
    do {
        int lay[64], len = 0;
        for (int pi = 0; pi < nmulti; ++pi) {
            const Run& R = runs[multi[perm[pi]]];
            if (contains(lay, len, R.plane, R.n, nullptr)) continue;
            int ov = 0;
            for (int k = (R.n < len ? R.n : len); k > 0 && !ov; --k) {
                bool eq = true;
                for (int q = 0; q < k && eq; ++q) eq = lay[len - k + q] == R.plane[q];
                if (eq) ov = k;
            }
            for (int q = ov; q < R.n; ++q) lay[len++] = R.plane[q];
        }
        for (int b = 0; b < nb; ++b)
            if (!contains(lay, len, &b, 1, nullptr)) lay[len++] = b;
        if (len < best && len <= tp::MAXSLOT) {
            best = len;
            *nslot = len;
            for (int q = 0; q < len; ++q) slots[q] = lay[q];
        }
    } while (next_permutation(perm, nmulti));
    if (best == (1 << 30)) return false;
    for (int i = 0; i < nrun; ++i)
        if (!contains(slots, *nslot, runs[i].plane, runs[i].n, &run_slot[i])) return false;
    return true;
}

bool base_eligible(const mf_config& c, int32_t m) {
    if (!c.ideal || !exact_integer_counts(c) || c.wide || c.wide_codes) return false;
    if (c.activation_bits != 8 || c.weight_bits != 8) return false;
    // 32-row reads, or 64-row reads as two 32-row stages per read.
    if ((c.read_rows != tp::KR && c.read_rows != 2 * tp::KR) || c.rows % c.read_rows) return false;
    const long long MR = (long long)m * c.reads;
    if (MR > 256 || MR % tp::SCB) return false;
    // |T| < 2^22 keeps the integer-to-float step exact.
    return reconstruction_bound(c) < 4194304.0;
}

// Block order, slot layout and MMA list with the fewest MMAs for the packed
// fields (field i: block pk.col[i], input plane fa[i], weight plane fb[i]).
bool merge_mmas(const Packer& pk, const int* fa, const int* fb, tp::Plan& P, int* pos_of_col) {
    const int ncol = pk.ncol;
    if (ncol == 0) {
        P.nslot = 0;
        P.nmma = 0;
        return true;
    }
    int perm[tp::MAXCOL];
    for (int i = 0; i < ncol; ++i) perm[i] = i;
    int best_mma = 1 << 30;
    do {
        int pos[tp::MAXCOL];
        for (int p = 0; p < ncol; ++p) pos[perm[p]] = p;
        // Runs: per input plane, fields by block position, cut where the position
        // does not advance by one.
        Run runs[128];
        int nrun = 0;
        bool used[64] = {};
        for (int a = 0; a < pk.na; ++a) {
            while (true) {
                int first = -1;
                for (int i = 0; i < pk.nf; ++i)
                    if (!used[i] && fa[i] == a && (first < 0 || pos[pk.col[i]] < pos[pk.col[first]])) first = i;
                if (first < 0) break;
                Run R{};
                R.a = a;
                R.pos = pos[pk.col[first]];
                R.n = 1;
                R.plane[0] = fb[first];
                used[first] = true;
                while (R.pos + R.n < ncol) {
                    int next = -1;
                    for (int i = 0; i < pk.nf && next < 0; ++i)
                        if (!used[i] && fa[i] == a && pos[pk.col[i]] == R.pos + R.n) next = i;
                    if (next < 0) break;
                    R.plane[R.n++] = fb[next];
                    used[next] = true;
                }
                runs[nrun++] = R;
            }
        }
        // Issue order: a run initialises its blocks when none was written yet and
        // accumulates when all were; a run over mixed blocks is split into singles.
        Run list[128];
        int acc_flag[128], nlist = 0, remaining = nrun;
        bool done[128] = {}, init[tp::MAXCOL] = {};
        while (remaining > 0) {
            int pick = -1, mode = 0;
            for (int i = 0; i < nrun && pick < 0; ++i) {
                if (done[i]) continue;
                bool all_new = true, all_old = true;
                for (int q = 0; q < runs[i].n; ++q) {
                    all_new &= !init[runs[i].pos + q];
                    all_old &= init[runs[i].pos + q];
                }
                if (all_new || all_old) {
                    pick = i;
                    mode = all_old ? 1 : 0;
                }
            }
            if (pick < 0) {
                int split = -1;
                for (int i = 0; i < nrun && split < 0; ++i)
                    if (!done[i] && runs[i].n > 1) split = i;
                if (split < 0 || nrun + tp::MAXCOL > 128) break;
                for (int q = 1; q < runs[split].n; ++q) {
                    Run R{};
                    R.a = runs[split].a;
                    R.pos = runs[split].pos + q;
                    R.n = 1;
                    R.plane[0] = runs[split].plane[q];
                    runs[nrun++] = R;
                    ++remaining;
                }
                runs[split].n = 1;
                continue;
            }
            done[pick] = true;
            --remaining;
            for (int q = 0; q < runs[pick].n; ++q) init[runs[pick].pos + q] = true;
            acc_flag[nlist] = mode;
            list[nlist++] = runs[pick];
        }
        if (remaining == 0 && nlist <= tp::MAXMMA && nlist < best_mma) {
            int slots[tp::MAXSLOT], nslot = 0, run_slot[128];
            if (slot_layout(list, nlist, pk.nb, slots, &nslot, run_slot)) {
                best_mma = nlist;
                P.nslot = nslot;
                for (int q = 0; q < tp::MAXSLOT; ++q) P.slot_plane[q] = q < nslot ? slots[q] : 0;
                P.nmma = nlist;
                for (int k = 0; k < nlist; ++k) {
                    P.mma[k].a = list[k].a;
                    P.mma[k].slot = run_slot[k];
                    P.mma[k].n = list[k].n;
                    P.mma[k].block = list[k].pos;
                    P.mma[k].acc = acc_flag[k];
                }
                for (int cc = 0; cc < ncol; ++cc) pos_of_col[cc] = pos[cc];
            }
        }
    } while (next_permutation(perm, ncol));
    return best_mma != (1 << 30);
}

}  // namespace

bool tc_packed_plan(const mf_config& c, tp::Plan& P) {
    memset(&P, 0, sizeof(P));
    const int rows = c.read_rows;
    Packer pk(c);
    int rare_w[MF_MAX_SLICES] = {};
    int rare_amask[MF_MAX_SLICES] = {};
    for (int w = 0; w < c.n_w; ++w) {
        if (c.w_mask[w] > 255 || c.w_shift[w] > 7) return false;
        const int m = c.adc_max[w];
        for (int a = 0; a < c.n_in; ++a) {
            const long long dmax = (long long)rows * c.in_mask[a] * c.w_mask[w];
            if (dmax <= m) continue;                       // never clips
            if ((long long)m * 4 >= dmax * 3) {            // threshold near the maximum: rare
                rare_w[w] = 1;
                rare_amask[w] = c.in_mask[a] > rare_amask[w] ? c.in_mask[a] : rare_amask[w];
                continue;
            }
            if (((m + 1) & m) != 0) return false;          // clip test needs m + 1 = 2^b
            if (pk.nf >= 64) return false;
            Count& q = pk.f[pk.nf++];
            q.a = a;
            q.w = w;
            q.width = bitlen(dmax);
            q.clipbit = bitlen(m);
            q.m = m;
            const long long coef = -(long long)c.in_factor[a] * c.w_factor[w];
            if (coef > 2147483647LL || coef < -2147483647LL) return false;
            q.coef = (int)coef;
        }
    }
    // Widest counts first: they constrain the packing most.
    for (int i = 1; i < pk.nf; ++i)
        for (int j = i; j > 0 && pk.f[j].width > pk.f[j - 1].width; --j) {
            Count tmp = pk.f[j];
            pk.f[j] = pk.f[j - 1];
            pk.f[j - 1] = tmp;
        }
    if (!pk.place(0)) return false;
    P.na = pk.na;
    P.nb = pk.nb;
    P.ncol = pk.ncol;
    for (int i = 0; i < pk.na; ++i) {
        P.a_src[i] = c.in_shift[pk.a_idx[i]];
        P.a_mask[i] = c.in_mask[pk.a_idx[i]];
        P.a_scale[i] = pk.a_k[i];
    }
    for (int i = 0; i < pk.nb; ++i) {
        P.b_src[i] = c.w_shift[pk.b_idx[i]];
        P.b_mask[i] = c.w_mask[pk.b_idx[i]];
        P.b_scale[i] = pk.b_k[i];
    }
    int fa[64], fb[64], pos_of_col[tp::MAXCOL] = {};
    for (int i = 0; i < pk.nf; ++i) {
        fa[i] = pk.find_a(pk.f[i].a, pk.ka[i]);
        fb[i] = pk.find_b(pk.f[i].w, pk.kb[i]);
    }
    if (!merge_mmas(pk, fa, fb, P, pos_of_col)) return false;
    for (int i = 0; i < pk.nf; ++i) {
        const Count& q = pk.f[i];
        const int blk = pos_of_col[pk.col[i]];
        tp::Field& F = P.field[blk][P.nfield[blk]++];
        F.shift = pk.shift[i];
        F.width_mask = (int)((1LL << q.width) - 1);
        F.m = q.m;
        F.coef = q.coef;
        F.clip = (uint32_t)(((1LL << q.width) - 1) & ~((1LL << q.clipbit) - 1)) << F.shift;
        P.colclip[blk] |= F.clip;
    }
    // Rare pairs of weight slice w: D <= Ma * S_w(o), so a column is exact when
    // its digit sum stays at or below m_w / Ma (Ma = widest input digit paired).
    for (int w = 0; w < c.n_w; ++w) {
        if (!rare_w[w]) continue;
        if (P.nrare >= (rows > tp::KR ? tp::MAXRARE : tp::MAXRARE_32)) return false;
        P.r_src[P.nrare] = c.w_shift[w];
        P.r_mask[P.nrare] = c.w_mask[w];
        P.r_limit[P.nrare] = c.adc_max[w] / rare_amask[w];
        ++P.nrare;
    }
    return true;
}

bool tc_packed_eligible(const mf_config& c, int32_t m) {
    if (!base_eligible(c, m)) return false;
    tp::Plan P;
    return tc_packed_plan(c, P);
}

int tc_packed_threads() { return tp::THREADS; }

size_t tc_packed_workspace_bytes(const mf_config& c, int64_t n, int32_t m, int32_t p, int32_t tiles) {
    const size_t kmajor = ((size_t)p * c.cols * m * c.rows + 255) / 256 * 256;
    const size_t cols = (size_t)tiles * c.cols;
    const size_t ctas = (size_t)((n + tp::BM - 1) / tp::BM) * ((cols + tp::BN - 1) / tp::BN);
    return kmajor + ctas * sizeof(unsigned) + 256;
}

template <int NCOL, int H>
static mf_status launch_packed(const CUtensorMap& mx, const CUtensorMap& mw, const CUtensorMap& mxs,
                               const CUtensorMap& mws, const tp::Args& args, dim3 grid, cudaStream_t st) {
    const size_t smem = sizeof(tp::Smem) + 1024;
    auto kern = tp::packed_kernel<NCOL, H>;
    int regs = 0;
    {
        const mf_status r = kernel_setup(reinterpret_cast<const void*>(kern), smem, &regs);
        if (r) return r;
    }
    // Registers are allocated per thread in multiples of 8.
    const long long pool = (long long)((regs + 7) / 8 * 8) * tp::THREADS;
    const long long split =
        128LL * tp::REG_CTRL + 32LL * tp::XF_WARPS * tp::REG_XF + 32LL * tp::EPI_WARPS * tp::REG_EPI;
    if (split > pool) {
        set_error("packed kernel launched with %d registers/thread cannot host its register split", regs);
        return MF_ERR_RESOURCE;
    }
    kern<<<grid, tp::THREADS, smem, st>>>(mx, mw, mxs, mws, args);
    MF_LAUNCH_CHECK("packed_kernel");
    return MF_OK;
}

mf_status tc_packed_sliced_mm(const mf_config& c, const MMArgs& a, void* workspace, size_t ws_bytes,
                              cudaStream_t st) {
    int dev = 0;
    MF_CHECK_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
    int major = 0;
    MF_CHECK_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev), "capability");
    if (major != 10) {
        set_error("tcgen05 path needs an sm_100 device");
        return MF_ERR_UNSUPPORTED;
    }
    const int tiles = a.tile_end - a.tile_begin;
    const size_t need = tc_packed_workspace_bytes(c, a.n, a.m, a.p, tiles);
    if (ws_bytes < need || !workspace) {
        set_error("packed tcgen05 workspace too small: %zu < %zu bytes", ws_bytes, need);
        return MF_ERR_RESOURCE;
    }
    tp::Args args{};
    if (!base_eligible(c, a.m) || !tc_packed_plan(c, args.plan)) {
        set_error("configuration outside the packed tcgen05 plan");
        return MF_ERR_UNSUPPORTED;
    }
    args.plan.b_signed = c.weight_signed;
    const long long K = (long long)a.m * c.rows;
    const long long O = (long long)a.p * c.cols;
    const int MR = a.m * c.reads;
    uint8_t* wk = static_cast<uint8_t*>(workspace);
    const size_t kmajor = ((size_t)O * K + 255) / 256 * 256;
    unsigned* flags = reinterpret_cast<unsigned*>(wk + kmajor);
    mf_status r = a.kmajor_ready ? MF_OK : tc_weights_kmajor(a.packed, wk, a.m, a.p, c.rows, c.cols, st);
    if (r) return r;
    CUtensorMap mx, mw, mxs, mws;
    r = tc_make_map(&mx, a.codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)K, (uint64_t)a.n, (uint64_t)K, tp::KR,
                    tp::BM, CU_TENSOR_MAP_SWIZZLE_32B);
    if (!r) r = tc_make_map(&mw, wk, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)K, (uint64_t)O, (uint64_t)K, tp::KR,
                            tp::BN, CU_TENSOR_MAP_SWIZZLE_32B);
    // Scales: xscale [n, MR] -> boxes [128 rows][4 reads]; wscale [MR, O] -> [4 reads][128 cols].
    if (!r) r = tc_make_map(&mxs, a.xscale, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)MR, (uint64_t)a.n,
                            (uint64_t)MR, tp::SCB, tp::BM, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (!r) r = tc_make_map(&mws, a.wscale, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)O, (uint64_t)MR,
                            (uint64_t)O, tp::BN, tp::SCB, CU_TENSOR_MAP_SWIZZLE_NONE);
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
    args.tile_flags = flags;
    args.raster = a.raster;
    args.stop_stage = a.stall_stage;
    args.wait_cycles = a.stall_stage >= 0 ? a.stall_cycles : tg::kWaitCycles;
    args.n_peers = a.n_peers;
    for (int i = 0; i < a.n_peers; ++i) args.peer_out[i] = static_cast<float*>(a.peer_out[i]);
    const long long cols = (long long)tiles * c.cols;
    const long long vblocks = (a.n + tp::BM - 1) / tp::BM;
    const dim3 grid = raster_grid(vblocks, (cols + tp::BN - 1) / tp::BN, a.raster);
    const bool two = c.read_rows == 2 * tp::KR;
    switch (args.plan.ncol) {
        case 0: r = two ? launch_packed<0, 2>(mx, mw, mxs, mws, args, grid, st)
                        : launch_packed<0, 1>(mx, mw, mxs, mws, args, grid, st); break;
        case 1: r = two ? launch_packed<1, 2>(mx, mw, mxs, mws, args, grid, st)
                        : launch_packed<1, 1>(mx, mw, mxs, mws, args, grid, st); break;
        case 2: r = two ? launch_packed<2, 2>(mx, mw, mxs, mws, args, grid, st)
                        : launch_packed<2, 1>(mx, mw, mxs, mws, args, grid, st); break;
        default: r = two ? launch_packed<3, 2>(mx, mw, mxs, mws, args, grid, st)
                         : launch_packed<3, 1>(mx, mw, mxs, mws, args, grid, st); break;
    }
    if (r) return r;
    // Tiles whose rare pairs could clip are recomputed exactly by the generic kernel.
    return generic_ideal_tiles(c, a, flags, tp::BM, tp::BN, (int)vblocks, st);
}

}  // namespace mf

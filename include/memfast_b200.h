/*
 * memfast_b200 -- C ABI of the B200 engine for MemFast's sliced matrix product.
 *
 * The reference (HUST-ISMD-Odyssey/MemFast v0.3.0) crosses into device code in
 * memfast/cuda.py: it JIT-compiles memfast/kernels.cu with NVRTC (cuda.py:130-220)
 * and launches two kernels through ctypes cuLaunchKernel (cuda.py:275-310) from
 * ``partial(q, packed, config, schedule, seed, event, begin, end)``
 * (cuda.py:322-373), after which AnalogMatrix._execute scales and sums the
 * partials in PyTorch (simulator.py:561-616).  This library replaces that whole
 * boundary with prebuilt sm_100a kernels: partials never reach HBM, and the
 * quantisation (memfast/quantization.py:9-137) also runs on the device.
 *
 * Conventions
 *   - Plain pointers and sizes only.  Every pointer argument is DEVICE memory
 *     unless its comment says "host"; the caller owns every buffer, including
 *     workspaces (query their size first).  The library never allocates device
 *     memory on these paths.
 *   - All work is enqueued asynchronously on `stream` (a cudaStream_t, passed as
 *     void*; NULL is the legacy default stream).
 *   - Return value: MF_OK, or an error code; mf_last_error() gives the message of
 *     the calling thread's last failure.  No exception crosses the ABI.
 *   - Thread safety: calls are reentrant; per-device one-time set-up runs under
 *     a mutex.
 *   - Slice tables are least-significant-slice first, as in
 *     memfast/config.py:193-209 (Config.input_layout / weight_layout).
 */
#ifndef MEMFAST_B200_H
#define MEMFAST_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MF_ABI_VERSION 3
#define MF_MAX_SLICES 32

typedef enum {
    MF_OK = 0,
    MF_ERR_INVALID = 1,   /* bad argument or configuration  (reference: ValueError)    */
    MF_ERR_RESOURCE = 2,  /* workspace/grid/shared-memory limit (reference: ResourceError, cuda.py:15) */
    MF_ERR_CUDA = 3,      /* CUDA runtime failure          (reference: RuntimeError, cuda.py:19-21) */
    MF_ERR_UNSUPPORTED = 4
} mf_status;

typedef enum { MF_F32 = 0, MF_F16 = 1, MF_BF16 = 2, MF_F64 = 3 } mf_dtype;

/* POD mirror of Config + Nonidealities (memfast/config.py:21-224); every
 * derived quantity is precomputed on the host exactly as the reference derives it
 * (drift factor as in cuda.py:74). */
typedef struct {
    int32_t abi_version;             /* MF_ABI_VERSION */
    int32_t activation_bits, weight_bits, weight_signed, bw_e;   /* bw_e 0 = INT */
    int32_t n_in, n_w;               /* physical input / weight slices */
    int32_t in_shift[MF_MAX_SLICES], in_mask[MF_MAX_SLICES];
    int64_t in_factor[MF_MAX_SLICES];
    int32_t w_shift[MF_MAX_SLICES], w_mask[MF_MAX_SLICES];
    int64_t w_factor[MF_MAX_SLICES];
    int32_t adc_max[MF_MAX_SLICES];  /* per weight slice */
    int32_t rows, cols;              /* array_size */
    int32_t read_rows, reads;        /* rows per ADC read, reads per array */
    int32_t in_group_rows, in_group_cols;   /* input_quant_gran, 0 = whole extent */
    int32_t w_group_rows, w_group_cols;     /* weight_quant_gran over [K,O], 0 = whole */
    int32_t wide;                    /* FP64 scales and reconstruction (Config.wide) */
    int32_t wide_codes;              /* int64 codes instead of uint8 */
    int32_t precise_currents;        /* FP64 currents (Config.precise_currents) */
    int32_t read_mode;               /* 0 shared, 1 slice_pair, 2 output */
    int32_t ideal;                   /* no effect perturbs a current */
    double high, low, voltage, unit;
    double write_var, read_var, volt_var, nonlinear, saf_low, saf_high, drift;
} mf_config;

/* Execution schedule (the reference's tuned-mode grid, simulator.py:27-45,
 * re-declared over this engine's tile shapes).  For ideal devices every
 * schedule gives bit-identical output.  For nonideal devices kernel 1 (SIMT)
 * and the tensor-core currents (0 / 2) sum each read's FP32 currents in
 * different orders, so a few ADC roundings differ between them (the tuned mode's
 * bitwise check then keeps the default's kernel). */
typedef struct {
    int32_t kernel;     /* 0 auto, 1 generic SIMT, 2 tcgen05 (ideal: packed integer counts when
                           the configuration fits (32- or 64-row reads), else FP8 digit planes
                           (32-row reads), else FP16 digit dots; nonideal: FP16 digit x
                           conductance currents when the configuration fits), 3 tcgen05 FP8
                           digit planes (ideal) */
    int32_t tile_n;     /* reserved: no kernel reads it (the SIMT kernels size their CTAs */
    int32_t tile_o;     /* from the configuration) */
    int32_t arrays;     /* tiles restored per group in physical mode (>=1) */
    int32_t kmajor_ready; /* 1: the workspace starts with the K-major weight copy that
                             mf_program_rhs wrote for these packed weights (tensor-core
                             kernels then skip rebuilding it); 0: rebuilt per call */
    int32_t raster;     /* tensor-core kernels, order in which CTAs (128 vectors x one column
                           block each) are launched: 0 = vector blocks first (the CTAs in
                           flight share weight tiles in L2), 1 = column blocks first (they
                           share input-code tiles); the output is the same either way */
} mf_schedule;

typedef struct {
    size_t workspace_bytes;
    int32_t threads, shared_bytes, registers, local_bytes, blocks_per_sm;
    size_t kmajor_bytes;  /* > 0: the chosen kernel reads a K-major weight copy of this many
                             bytes at the start of its workspace (see kmajor_ready) */
    int32_t path;         /* kernel family the schedule resolves to: an mf_path value, below */
} mf_resources;

/* One channel group of a 2-D convolution over an NCHW input (AnalogConv2d,
 * memfast/nn/convolution.py:10-62, which lowers it to F.unfold patches times one
 * programmed matrix per group). */
typedef struct {
    int64_t batch, channels, height, width;          /* x: [batch, channels, height, width] */
    int64_t stride_n, stride_c, stride_h, stride_w;  /* element strides of x (any layout) */
    int32_t kernel_h, kernel_w;
    int32_t stride_y, stride_x;                      /* Conv2d.stride */
    int32_t pad_h, pad_w;                            /* zero padding (Conv2d.padding) */
    int32_t dilation_h, dilation_w;
    int32_t channel_begin, group_channels;           /* the group's input channels */
} mf_conv2d;

int32_t mf_abi_version(void);

/* Message of this thread's last failure ("" if none).  Returns its length. */
int32_t mf_last_error(char* buffer, size_t capacity);

/* Kernels this library has launched in this process (all devices, all entry points). */
uint64_t mf_launch_count(void);

/* Number of visible devices and whether device `index` is an sm_100 part. */
mf_status mf_device_check(int32_t index, int32_t* is_sm100);

/* Replaces memfast/quantization.py input_tiles (:115-137) with grouped_quantize
 * (:9-44).  x: [n, k] row stride ldx elements, dtype x_dtype.  fixed_scale:
 * NULL for dynamic groups, else [k] FP32 (FP64 when cfg->wide) per-column scales
 * (AnalogMatrix.set_input_scale, simulator.py:432-450).  codes: [n, m*rows]
 * uint8 (int64 when cfg->wide_codes), m = ceil(k/rows).  xscale: [n, m*reads]
 * FP32 (FP64 when cfg->wide).  workspace: mf_quantize_workspace() bytes. */
mf_status mf_quantize_input(const mf_config* cfg, const void* x, int32_t x_dtype, int64_t n,
                            int64_t k, int64_t ldx, const void* fixed_scale, void* codes,
                            void* xscale, void* workspace, size_t workspace_bytes, void* stream);

/* Replaces quantization.py weight_tiles (:82-91) + pack_weight (:94-112).
 * w: PyTorch-layout [o, k] weights, row stride ldw.  packed: [m, p, rows, cols]
 * uint8 (int64 when cfg->wide_codes); wscale: [m*reads, p, cols] FP32/FP64. */
mf_status mf_program_weights(const mf_config* cfg, const void* w, int32_t w_dtype, int64_t o,
                             int64_t k, int64_t ldw, void* packed, void* wscale,
                             void* workspace, size_t workspace_bytes, void* stream);

/* Programs the right-hand matrix of a product, b [k, o] with row stride ldb (the
 * reference programs it as weight_tiles(b.T), quantization.py:82-112 via
 * simulator.py:121-171), without materialising the transpose.  packed / wscale as
 * mf_program_weights.  kmajor: NULL, or [ceil(o/cols)*cols, ceil(k/rows)*rows]
 * bytes receiving the K-major copy of the 8-bit codes that the tensor-core kernels
 * read; pass it as the start of mf_sliced_mm's workspace with kmajor_ready = 1.
 * workspace: mf_quantize_workspace(cfg, 1, o, k) bytes. */
mf_status mf_program_rhs(const mf_config* cfg, const void* b, int32_t b_dtype, int64_t k, int64_t o,
                         int64_t ldb, void* packed, void* wscale, void* kmajor, void* workspace,
                         size_t workspace_bytes, void* stream);

/* Capacity of the library's own scratch for mf_quantize_input_static: 4 MiB,
 * i.e. 1,048,576 FP32 (or 524,288 FP64) group maxima. */
#define MF_STATIC_QUANTIZE_SCRATCH_BYTES (4u << 20)

/* mf_quantize_input without a caller workspace (no counterpart in the
 * reference, which always allocates its temporaries through torch).  Same
 * arguments, results and errors as mf_quantize_input; the group maxima live in
 * a fixed device array inside the library instead of `workspace`.
 *   - For callers that cannot hand out device memory: a plain C host that owns
 *     only its input and output buffers, or one that must not call cudaMalloc
 *     between launches because cudaMalloc can wait for the whole device.
 *   - Neither it nor its set-up allocates device memory.  The first call on
 *     each device resolves the array's address (cudaGetSymbolAddress); a caller
 *     that wants no set-up work inside a later phase (for example a stream
 *     capture) makes one call on that device before the phase begins.
 *   - Limit: when dynamic scales need more than
 *     MF_STATIC_QUANTIZE_SCRATCH_BYTES of group maxima (mf_quantize_workspace()
 *     minus its 256-byte pad), the call fails with MF_ERR_RESOURCE and enqueues
 *     nothing; use mf_quantize_input with a workspace instead.
 *   - One array per device: calls that can overlap on a device (other streams,
 *     other host threads without ordering between them) race on it and give
 *     wrong codes.  Keep such calls on one stream.
 *   - The array's address is looked up once per device and kept for the life of
 *     the process.  cudaDeviceReset unloads the module, so that address does not
 *     survive it: do not call this entry point on a device after resetting it. */
mf_status mf_quantize_input_static(const mf_config* cfg, const void* x, int32_t x_dtype, int64_t n,
                                   int64_t k, int64_t ldx, const void* fixed_scale, void* codes,
                                   void* xscale, void* stream);

/* Bytes of scratch mf_quantize_input (is_weight=0, shape [n,k]) or
 * mf_program_weights (is_weight=1, shape [o,k]) needs. */
mf_status mf_quantize_workspace(const mf_config* cfg, int32_t is_weight, int64_t rows,
                                int64_t cols, size_t* bytes);

/* mf_quantize_input on the patch matrix of one convolution group without
 * building it (replaces F.unfold + transpose + input_tiles,
 * memfast/nn/convolution.py:49-55 with quantization.py:115-137).  The patch
 * matrix has rows v = (b*OH + oh)*OW + ow (mf_conv_output gives OH, OW) and
 * columns k = (c*kernel_h + i)*kernel_w + j for c < group_channels, holding
 * x[b, channel_begin + c, oh*stride_y - pad_h + i*dilation_h,
 *   ow*stride_x - pad_w + j*dilation_w] (0 outside x).  codes / xscale /
 * fixed_scale as mf_quantize_input for that [rows, cols] matrix.  nonfinite: a
 * device uint32 set to 1 when a quantised value is not finite (the reference
 * raises ValueError then; results are invalid), else 0.
 * workspace: mf_quantize_workspace(cfg, 0, rows, cols) bytes. */
mf_status mf_quantize_conv_input(const mf_config* cfg, const mf_conv2d* conv, const void* x, int32_t x_dtype,
                                 const void* fixed_scale, void* codes, void* xscale, uint32_t* nonfinite,
                                 void* workspace, size_t workspace_bytes, void* stream);

/* Finiteness check on the device without a host synchronisation (the checks of
 * memfast/functional.py:50-53 and quantization.py:12-15, read later together with
 * other flags): over n contiguous values of dtype x_dtype, sets the device word
 * *flag to `code` if it is still 0 and a value is not finite, or to narrow_code
 * (non-zero: FP64 input only) if a value is finite in FP64 but not in FP32.
 * Checks enqueued on one stream report the first failing one. */
mf_status mf_check_finite(const void* x, int32_t x_dtype, int64_t n, uint32_t code, uint32_t narrow_code,
                          uint32_t* flag, void* stream);

/* The operand checks of one product in one call (memfast/functional.py:50-53 with
 * quantization.py:12-15): clears flags[0..flag_words) on `stream`, then checks A
 * (code 1), B (code 2, or b_narrow_code when B's FP64 values overflow FP32) and,
 * when a_narrow_code is non-zero, A again in FP32, each as mf_check_finite into
 * flags[0]; the first failure in that order wins. */
mf_status mf_check_operands(const void* a, int32_t a_dtype, int64_t a_count, uint32_t a_narrow_code,
                            const void* b, int32_t b_dtype, int64_t b_count, uint32_t b_narrow_code,
                            uint32_t* flags, int32_t flag_words, void* stream);

/* Output height and width of a convolution group; MF_ERR_INVALID for a bad geometry. */
mf_status mf_conv_output(const mf_conv2d* conv, int64_t* out_height, int64_t* out_width);

/* The analog product for output tiles [tile_begin, tile_end): replaces
 * cuda.partial (cuda.py:322-373) and the scale/sum epilogue of
 * AnalogMatrix._execute (simulator.py:561-586), plus the bias add (:612-613).
 *   codes/xscale: from mf_quantize_input ([n, m*rows], [n, m*reads]).
 *   packed/wscale: from mf_program_weights ([m, p, rows, cols], [m*reads, p, cols]).
 *   bias: NULL or [out_features] FP32 (FP64 when wide or stable).
 *   out: FP32 (FP64 when cfg->wide or stable); output column `col` of vector
 *        `v` goes to out[v*ldo + col] for the written columns
 *        [tile_begin*cols, min(tile_end*cols, out_features)).  ldo is at least
 *        the written width: out_features for a full [n, out_features] buffer, or
 *        the shard's width for a buffer holding only the shard's columns (then
 *        `out` is that buffer's address minus tile_begin*cols elements; nothing
 *        below the written columns is touched).
 *   seed: AnalogMatrix.seed; event: read-event counter (simulator.py:427-429,633).
 *   vector_offset: global index of row 0 (noise addresses stay global when rows
 *        are sharded across calls or GPUs).
 *   stable: 1 = FP64 restore_scales epilogue (simulator.py:57-66, the non-finite
 *        rerun at :614-615).
 *   workspace: mf_sliced_mm_workspace() bytes. */
mf_status mf_sliced_mm(const mf_config* cfg, const mf_schedule* schedule, const void* codes,
                       const void* xscale, const void* packed, const void* wscale,
                       const void* bias, void* out, int64_t n, int32_t m, int32_t p,
                       int32_t out_features, int64_t ldo, int32_t tile_begin, int32_t tile_end,
                       uint32_t seed, uint64_t event, int64_t vector_offset, int32_t stable,
                       void* workspace, size_t workspace_bytes, void* stream);

mf_status mf_sliced_mm_workspace(const mf_config* cfg, const mf_schedule* schedule, int64_t n,
                                 int32_t m, int32_t p, int32_t tile_begin, int32_t tile_end,
                                 size_t* bytes);

/* Most peer output buffers of one mf_mm call (eight GPUs of a node). */
#define MF_MAX_PEERS 7

/* Caller-owned device buffers of one mf_mm call. */
typedef struct {
    void* codes;                 /* [n, m*rows] input codes, as mf_quantize_input writes them */
    void* xscale;                /* [n, m*reads] per-read input scales */
    void* packed;                /* [m, p, rows, cols] program of b, rewritten by the call */
    void* wscale;                /* [m*reads, p, cols] */
    void* out;                   /* [n, o] contiguous, FP32 (FP64 when cfg->wide) */
    uint32_t* flags;             /* 2 device words: [operand check, output check] */
    void* quantize_workspace;    /* mf_quantize_workspace(cfg, 0, n, k) bytes */
    size_t quantize_workspace_bytes;
    void* program_workspace;     /* mf_quantize_workspace(cfg, 1, o, k) bytes */
    size_t program_workspace_bytes;
    void* mm_workspace;          /* mf_sliced_mm_workspace(cfg, schedule, n, m, p, 0, p) bytes */
    size_t mm_workspace_bytes;
    /* Row-sharded products on one node: n_peers (at most MF_MAX_PEERS) addresses of
     * other GPUs' output buffers mapped into this process (CUDA IPC), each at the
     * element that corresponds to out[0].  The product stores every output into
     * `out` and into each of them from the kernel's epilogue, which takes the place
     * of an all-gather of the rows; the kernel ends with a system-scope fence, so
     * the stores are visible to a peer once it has synchronised with this GPU after
     * the call (for example through a collective enqueued after it).  Only the
     * packed tcgen05 path stores to peers: MF_ERR_UNSUPPORTED otherwise, with
     * nothing enqueued.  n_peers = 0: no peers. */
    void* peer_out[MF_MAX_PEERS];
    int32_t n_peers;
} mf_mm_buffers;

/* One default-mode product out = A @ B with B programmed by the call, enqueued on
 * `stream` with no host synchronisation: the sequence that memfast.mm /
 * Simulator.mm runs per call (functional.py:50-53, simulator.py:121-171 and
 * 561-616 of the reference), in one crossing of this ABI instead of one per step.
 *   a: [n, k] and b: [k, o], contiguous, both of dtype `dtype`.
 *   Checks (flags cleared first): flags[0] becomes 1 if A is not finite, else 2
 *   if B is not finite (or b_narrow_code when B's FP64 values overflow FP32),
 *   else a_narrow_code when that is non-zero and A's FP64 values overflow FP32,
 *   as mf_check_operands gives them; flags[1] becomes 1 if an output is not
 *   finite.  For FP32 operands of the one-pass quantisers the operand checks
 *   ride on the quantisers' reads instead of separate passes.
 *   Then A is quantised (mf_quantize_input), b programmed into packed/wscale
 *   (mf_program_rhs) with the K-major copy written at the start of
 *   mm_workspace when the schedule's kernel reads one, and the fused product
 *   of all p tiles runs (mf_sliced_mm: seed, event, vector_offset as there).
 *   error_word: NULL, or pinned host memory receiving the device error word
 *   (mf_stage_device_error) after the product.
 * The results equal those of the separate calls bit for bit. */
mf_status mf_mm(const mf_config* cfg, const mf_schedule* schedule, const void* a, const void* b, int32_t dtype,
                int64_t n, int64_t k, int64_t o, uint32_t a_narrow_code, uint32_t b_narrow_code,
                const mf_mm_buffers* buffers, uint32_t seed, uint64_t event, int64_t vector_offset,
                uint32_t* error_word, void* stream);

/* Lets kernels on the current device read and write memory of device
 * `peer_device` (cudaDeviceEnablePeerAccess; already enabled counts as success).
 * The peer-store path of mf_mm needs it for every peer buffer's device: a buffer
 * mapped from another process lives in that device's context.  MF_ERR_UNSUPPORTED
 * when the two devices cannot reach each other. */
mf_status mf_enable_peer_access(int32_t peer_device);

/* The CUDA IPC handle (handle_bytes = sizeof(cudaIpcMemHandle_t), 64) of the
 * device allocation that contains `ptr`, and ptr's byte offset in it, for another
 * process to map with mf_ipc_open. */
mf_status mf_ipc_export(const void* ptr, void* handle, size_t handle_bytes, size_t* offset);

/* Maps a device buffer of another process into the current device's address
 * space (cudaIpcOpenMemHandle with lazy peer access): `handle` holds the
 * handle_bytes bytes of that process's cudaIpcMemHandle_t for the buffer's
 * allocation, *base receives the allocation's address here.  Kernels on the
 * current device may then read and write it (the peer outputs of mf_mm).
 * MF_ERR_INVALID when handle_bytes is not the size of a CUDA IPC handle. */
mf_status mf_ipc_open(const void* handle, size_t handle_bytes, void** base);

/* Unmaps an allocation mapped by mf_ipc_open. */
mf_status mf_ipc_close(void* base);

/* Kernel families behind mf_sliced_mm.  The reference has one pair of SIMT
 * kernels (memfast/kernels.cu:43-202); this engine picks among these per
 * configuration and schedule. */
typedef enum {
    MF_PATH_NONE = 0,
    MF_PATH_GENERIC_IDEAL = 1,   /* ideal devices, dp4a digit dots (SIMT) */
    MF_PATH_PACKED = 2,          /* ideal devices, tcgen05 kind::i8 packed counts */
    MF_PATH_FP8_PLANES = 3,      /* ideal devices, tcgen05 kind::f8f6f4 digit planes */
    MF_PATH_TC_CURRENTS = 4,     /* tcgen05 kind::f16 digit x conductance (or digit) currents */
    MF_PATH_SIMT_CURRENTS = 5    /* restored conductances, FP32/FP64 SIMT currents */
} mf_path;

/* The mf_path of this thread's last successful mf_sliced_mm call (MF_PATH_NONE
 * before one).  Tests and tuned-mode reports use it to see which kernel ran. */
int32_t mf_last_path(void);

/* Test hook for the failure-detection path (no counterpart in the reference,
 * which has no device-side waits).  Arms a one-shot stall consumed by the next
 * mf_sliced_mm call in this process: if that call runs the packed tcgen05
 * kernel, its load producer issues nothing from pipeline stage `stop_stage` on
 * (a 32-row stage; reads of 64 rows take two), so every wait on a later stage
 * runs out after `wait_cycles` SM clock cycles instead of about two seconds.
 * Each CTA then records the wait's code in the device error word, drains its
 * own loads and MMAs, frees its TMEM and exits, and mf_take_device_error reports
 * MF_ERR_CUDA; the library stays usable.  Other paths ignore the stall.
 * MF_ERR_INVALID unless stop_stage >= 0 and 1000 <= wait_cycles <= 4e9. */
mf_status mf_debug_stall_next_launch(int32_t stop_stage, int64_t wait_cycles);

/* Reads and clears the library's device error word (a synchronising call).  A
 * non-zero code means a bounded device-side wait gave up inside a kernel: the
 * launch recorded the failure, released its resources and returned without
 * finishing its outputs.  Returns MF_ERR_CUDA in that case, MF_OK otherwise. */
mf_status mf_take_device_error(uint32_t* code);

/* Enqueues on `stream` a copy of the device error word into `host_word` (pinned
 * host memory), without clearing it: after the stream's next synchronisation a
 * non-zero word means mf_take_device_error will report a failure.  Lets a caller
 * test for device-side failures in the synchronisation it makes anyway. */
mf_status mf_stage_device_error(uint32_t* host_word, void* stream);

/* Resource admission for a schedule (replaces Simulator._admit, simulator.py:216-237,
 * and Program.resources, cuda.py:239-273).  MF_ERR_RESOURCE if it cannot run. */
mf_status mf_query(const mf_config* cfg, const mf_schedule* schedule, int64_t n, int32_t m,
                   int32_t p, mf_resources* out);

#ifdef __cplusplus
}
#endif

#endif /* MEMFAST_B200_H */

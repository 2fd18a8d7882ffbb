// Internal host-side entry points shared by the C ABI and the kernel files.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace mf {

size_t quantize_workspace_bytes(const mf_config& c, bool weight, int64_t rows, int64_t cols);

// check_flag (optional): the finiteness check of x folded into the pass (the
// device word becomes check_code if still 0 and a value of x is not finite).
mf_status quantize_input(const mf_config& c, const void* x, int dtype, int64_t n, int64_t k,
                         int64_t ldx, const void* fixed, void* codes, void* xscale,
                         void* workspace, size_t ws_bytes, cudaStream_t stream, uint32_t* check_flag = nullptr,
                         uint32_t check_code = 0);

mf_status program_weights(const mf_config& c, const void* w, int dtype, int64_t o, int64_t k,
                          int64_t ldw, void* packed, void* wscale, void* workspace,
                          size_t ws_bytes, cudaStream_t stream);

// Physical constants of a configuration for device code (reference.py, config.py).
Physics make_physics(const mf_config& c);

// Sets *flag (if still 0) to code_own when a value is not finite in its dtype, or to
// code_narrow when an FP64 value is finite but overflows FP32.
mf_status check_finite(const void* x, int dtype, int64_t n, uint32_t code_own, uint32_t code_narrow,
                       uint32_t* flag, cudaStream_t stream);

// Output extent of a convolution along one axis (0 when the window does not fit).
int64_t conv_output_extent(int64_t size, int32_t kernel, int32_t stride, int32_t pad, int32_t dilation);

// Quantise the patch matrix of one channel group of a 2-D convolution straight
// from the NCHW input (no unfold); same buffers as quantize_input on the patches.
mf_status quantize_conv_input(const mf_config& c, const mf_conv2d& cv, const void* x, int dtype,
                              const void* fixed, void* codes, void* xscale, uint32_t* nonfinite,
                              void* workspace, size_t ws_bytes, cudaStream_t stream);

// Program a right-hand [k, o] matrix b (row stride ldb); optionally also write the
// K-major [p*C, m*R] copy of the packed codes the tensor-core kernels read.
// check_flag as quantize_input's, for b.
mf_status program_rhs(const mf_config& c, const void* b, int dtype, int64_t k, int64_t o, int64_t ldb,
                      void* packed, void* wscale, void* kmajor, void* workspace, size_t ws_bytes,
                      cudaStream_t stream, uint32_t* check_flag = nullptr, uint32_t check_code = 0);

// Everything one sliced product needs, validated by the ABI layer.
struct MMArgs {
    const void* codes;
    const void* xscale;
    const void* packed;
    const void* wscale;
    const void* bias;
    void* out;
    int64_t n;
    int32_t m, p, out_features;
    int64_t ldo;
    int32_t tile_begin, tile_end;
    uint32_t seed;
    uint64_t event;
    int64_t vector_offset;
    int32_t stable;
    int32_t kmajor_ready;   // the workspace already starts with the K-major weight copy
    int32_t raster;         // tensor-core kernels: 0 = vector blocks first, 1 = column blocks first
    int32_t stall_stage;    // mf_debug_stall_next_launch: packed kernel stops its loads here (-1 off)
    int64_t stall_cycles;   // ... and its waits give up after this many SM cycles
    // Peer outputs (mf_mm_buffers.peer_out): every finished output is also stored at
    // the same offset from each of these addresses, other GPUs' buffers mapped into
    // this process (packed kernel and its exact rerun only).
    void* peer_out[MF_MAX_PEERS];
    int32_t n_peers;
};

// Grid of a tensor-core launch over nb vector blocks x cb column blocks in the
// schedule's raster order, and a CTA's (vector block, column block) in it.
inline dim3 raster_grid(long long nb, long long cb, int raster) {
    return raster ? dim3((unsigned)cb, (unsigned)nb) : dim3((unsigned)nb, (unsigned)cb);
}

// Largest |signed reconstruction| of one read, as in config.py:114-122.
double reconstruction_bound(const mf_config& c);
int max_adc(const mf_config& c);

// True when ideal ADC counts equal exact integer digit dots for this config: the
// reference's FP32 (or FP64) current error stays below half a count.
bool exact_integer_counts(const mf_config& c);

#ifdef __CUDACC__
__device__ __forceinline__ unsigned raster_vector_block(int raster) { return raster ? blockIdx.y : blockIdx.x; }
__device__ __forceinline__ unsigned raster_column_block(int raster) { return raster ? blockIdx.x : blockIdx.y; }
__device__ __forceinline__ unsigned raster_vector_blocks(int raster) { return raster ? gridDim.y : gridDim.x; }
#endif

// Generic SIMT engine (all configurations).
bool generic_ideal_fits(const mf_config& c, const mf_schedule& s);
mf_status generic_ideal(const mf_config& c, const mf_schedule& s, const MMArgs& a, cudaStream_t st);
// The same product restricted to the rows x cols output tiles whose flag is set
// (flags[col_tile * row_tiles + row_tile], device memory).
mf_status generic_ideal_tiles(const mf_config& c, const MMArgs& a, const unsigned* flags, int rows, int cols,
                              int row_tiles, cudaStream_t st);
size_t physical_workspace_bytes(const mf_config& c, const mf_schedule& s, int32_t m, int32_t tiles);
mf_status physical(const mf_config& c, const mf_schedule& s, const MMArgs& a, void* workspace,
                   size_t ws_bytes, cudaStream_t st);

// Shared by the tensor-core kernels (tc_common.cu).
mf_status tc_weights_kmajor(const void* packed, uint8_t* out, int m, int p, int R, int C, cudaStream_t st);
mf_status tc_make_map(CUtensorMap* map, const void* base, CUtensorMapDataType type, int bytes, uint64_t inner,
                      uint64_t outer, uint64_t stride, uint32_t box_inner, uint32_t box_outer,
                      CUtensorMapSwizzle swizzle);
mf_status tc_error_word(unsigned** word);
mf_status tc_take_error(unsigned* code);
mf_status tc_stage_error(unsigned* host_word, cudaStream_t st);
// Registers per thread of `kernel` as launched, with its dynamic shared memory
// raised to `smem` bytes (queried and set once per kernel and device).
mf_status kernel_setup(const void* kernel, size_t smem, int* regs);

// tcgen05 / TMEM fast path with FP8 digit planes (ideal INT8 configurations, tc_ideal.cu).
bool tc_eligible(const mf_config& c, int32_t m);
size_t tc_workspace_bytes(const mf_config& c, int32_t m, int32_t p);
int tc_block_threads();
mf_status tc_sliced_mm(const mf_config& c, const MMArgs& a, void* workspace, size_t ws_bytes, cudaStream_t st);

// Nonideal tensor-core path (tc_physical.cu).
bool tc_physical_eligible(const mf_config& c, int32_t m);
size_t tc_physical_workspace_bytes(const mf_config& c, int64_t n, int32_t m, int32_t tiles);
int tc_physical_threads();
mf_status tc_physical_sliced_mm(const mf_config& c, const MMArgs& a, void* workspace, size_t ws_bytes,
                                cudaStream_t st);

// tcgen05 / TMEM fast path with packed integer counts (tc_packed.cu).
bool tc_packed_eligible(const mf_config& c, int32_t m);
size_t tc_packed_workspace_bytes(const mf_config& c, int64_t n, int32_t m, int32_t p, int32_t tiles);
int tc_packed_threads();
mf_status tc_packed_sliced_mm(const mf_config& c, const MMArgs& a, void* workspace, size_t ws_bytes,
                              cudaStream_t st);

}  // namespace mf

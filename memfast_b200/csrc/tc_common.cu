// Host-side pieces shared by the tensor-core kernels: the K-major weight copy
// that TMA reads, tensor-map encoding, and the device error word that bounded
// waits write when they give up.
#include <cuda.h>
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"
#include "kernels.cuh"

namespace mf {
namespace {

// Weight codes [m, p, R, C] -> K-major [p*C, m*R] (8-bit, same bytes).
__global__ void weights_kmajor_kernel(const uint8_t* packed, uint8_t* out, int m, int p, int R, int C) {
    __shared__ uint8_t tile[32][33];
    const long long k0 = (long long)blockIdx.x * 32, o0 = (long long)blockIdx.y * 32;
    const long long K = (long long)m * R, O = (long long)p * C;
    // Array/row of k0 and tile/column of this thread's o, once per thread; rows step
    // from there (no division per element).
    const long long arr0 = k0 / R;
    const int r0 = (int)(k0 - arr0 * R);
    const long long o = o0 + threadIdx.x;
    const long long t = o / C;
    const int c = (int)(o - t * C);
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const long long k = k0 + j;
        uint8_t v = 0;
        if (k < K && o < O) {
            long long arr = arr0;
            int r = r0 + j;
            while (r >= R) {
                r -= R;
                ++arr;
            }
            v = packed[((arr * p + t) * R + r) * C + c];
        }
        tile[j][threadIdx.x] = v;
    }
    __syncthreads();
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const long long ot = o0 + j, k = k0 + threadIdx.x;
        if (k < K && ot < O) out[ot * K + k] = tile[threadIdx.x][j];
    }
}

typedef CUresult (*EncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
    static EncodeTiled fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    }
    return fn;
}

__device__ unsigned g_tc_error = 0;

}  // namespace

mf_status tc_weights_kmajor(const void* packed, uint8_t* out, int m, int p, int R, int C, cudaStream_t st) {
    const long long K = (long long)m * R, O = (long long)p * C;
    dim3 grid((unsigned)((K + 31) / 32), (unsigned)((O + 31) / 32));
    weights_kmajor_kernel<<<grid, dim3(32, 8), 0, st>>>(static_cast<const uint8_t*>(packed), out, m, p, R, C);
    MF_LAUNCH_CHECK("weights_kmajor_kernel");
    return MF_OK;
}

mf_status tc_make_map(CUtensorMap* map, const void* base, CUtensorMapDataType type, int bytes, uint64_t inner,
                      uint64_t outer, uint64_t stride, uint32_t box_inner, uint32_t box_outer,
                      CUtensorMapSwizzle swizzle) {
    EncodeTiled fn = encoder();
    if (!fn) {
        set_error("cuTensorMapEncodeTiled unavailable");
        return MF_ERR_CUDA;
    }
    if (((uintptr_t)base & 15) || (stride * bytes) % 16) {
        set_error("tensor map needs 16-byte aligned base and row stride");
        return MF_ERR_INVALID;
    }
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {stride * bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t elem[2] = {1, 1};
    CUresult r = fn(map, type, 2, const_cast<void*>(base), dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
        return MF_ERR_CUDA;
    }
    return MF_OK;
}

mf_status tc_error_word(unsigned** word) {
    // The symbol's address per device, looked up once.
    static unsigned* cached[64] = {};
    int dev = 0;
    MF_CHECK_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev < 0 || dev >= 64) {
        MF_CHECK_CUDA(cudaGetSymbolAddress((void**)word, g_tc_error), "error symbol");
        return MF_OK;
    }
    if (!cached[dev]) MF_CHECK_CUDA(cudaGetSymbolAddress((void**)&cached[dev], g_tc_error), "error symbol");
    *word = cached[dev];
    return MF_OK;
}

mf_status kernel_setup(const void* kernel, size_t smem, int* regs) {
    // (kernel, device) -> (registers at launch, dynamic shared memory opted in): the
    // attribute calls cost microseconds of host time, so each is made once.
    static std::mutex lock;
    static std::map<std::pair<const void*, int>, std::pair<int, size_t>> known;
    int dev = 0;
    MF_CHECK_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
    const auto key = std::make_pair(kernel, dev);
    {
        std::lock_guard<std::mutex> guard(lock);
        auto it = known.find(key);
        if (it != known.end() && it->second.second >= smem) {
            *regs = it->second.first;
            return MF_OK;
        }
    }
    cudaFuncAttributes attr;
    MF_CHECK_CUDA(cudaFuncGetAttributes(&attr, kernel), "kernel attributes");
    MF_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                  "kernel shared-memory attribute");
    std::lock_guard<std::mutex> guard(lock);
    known[key] = std::make_pair(attr.numRegs, smem);
    *regs = attr.numRegs;
    return MF_OK;
}

mf_status tc_stage_error(unsigned* host_word, cudaStream_t st) {
    unsigned* word = nullptr;
    mf_status r = tc_error_word(&word);
    if (r) return r;
    MF_CHECK_CUDA(cudaMemcpyAsync(host_word, word, sizeof(unsigned), cudaMemcpyDeviceToHost, st),
                  "stage device error");
    return MF_OK;
}

mf_status tc_take_error(unsigned* code) {
    unsigned value = 0, zero = 0;
    MF_CHECK_CUDA(cudaMemcpyFromSymbol(&value, g_tc_error, sizeof(value)), "read device error");
    if (value) MF_CHECK_CUDA(cudaMemcpyToSymbol(g_tc_error, &zero, sizeof(zero)), "clear device error");
    *code = value;
    return MF_OK;
}

}  // namespace mf

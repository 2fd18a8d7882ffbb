// C ABI of libmemfast_b200 (declared in include/memfast_b200.h).
//
// Validation mirrors the argument checks the reference performs before it
// launches (cuda.py:322-373, simulator.py:216-237); failures return a status
// and leave a message for mf_last_error() instead of raising.
#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include <cuda.h>

#include "common.cuh"
#include "kernels.cuh"

namespace mf {

static thread_local std::string g_last_error;
static thread_local int32_t g_last_path = MF_PATH_NONE;
// mf_debug_stall_next_launch: armed by the test hook, consumed by the next mf_sliced_mm.
static std::atomic<int32_t> g_stall_stage{-1};
static std::atomic<int64_t> g_stall_cycles{0};
static std::atomic<unsigned long long> g_launches{0};

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

void set_error(const char* fmt, ...) {
    char buffer[512];
    va_list args;
    va_start(args, fmt);
    vsnprintf(buffer, sizeof(buffer), fmt, args);
    va_end(args);
    g_last_error = buffer;
}

mf_status cuda_status(cudaError_t err, const char* what) {
    set_error("%s: %s (%s)", what, cudaGetErrorString(err), cudaGetErrorName(err));
    return MF_ERR_CUDA;
}

static mf_status check_config(const mf_config* c) {
    if (!c) {
        set_error("config is NULL");
        return MF_ERR_INVALID;
    }
    if (c->abi_version != MF_ABI_VERSION) {
        set_error("config ABI version %d, library expects %d", c->abi_version, MF_ABI_VERSION);
        return MF_ERR_INVALID;
    }
    if (c->n_in < 1 || c->n_in > MF_MAX_SLICES || c->n_w < 1 || c->n_w > MF_MAX_SLICES) {
        set_error("slice counts must be in [1, %d]", MF_MAX_SLICES);
        return MF_ERR_INVALID;
    }
    if (c->rows < 1 || c->cols < 4 || c->cols % 4 || c->read_rows < 1 || c->read_rows > c->rows ||
        c->reads != (c->rows + c->read_rows - 1) / c->read_rows) {
        set_error("invalid array geometry (rows %d, cols %d, read_rows %d, reads %d)", c->rows, c->cols,
                  c->read_rows, c->reads);
        return MF_ERR_INVALID;
    }
    for (int i = 0; i < c->n_w; ++i)
        if (c->adc_max[i] < 1 || c->adc_max[i] > 65535) {
            set_error("adc maximum %d out of range", c->adc_max[i]);
            return MF_ERR_INVALID;
        }
    if (c->read_mode < 0 || c->read_mode > 2) {
        set_error("read_mode must be 0 (shared), 1 (slice_pair) or 2 (output)");
        return MF_ERR_INVALID;
    }
    return MF_OK;
}

}  // namespace mf

using namespace mf;

extern "C" {

int32_t mf_abi_version(void) { return MF_ABI_VERSION; }

uint64_t mf_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int32_t mf_last_error(char* buffer, size_t capacity) {
    const std::string& e = g_last_error;
    if (buffer && capacity) {
        size_t n = e.size() < capacity - 1 ? e.size() : capacity - 1;
        memcpy(buffer, e.data(), n);
        buffer[n] = 0;
    }
    return (int32_t)e.size();
}

mf_status mf_device_check(int32_t index, int32_t* is_sm100) {
    int count = 0;
    MF_CHECK_CUDA(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
    if (index < 0 || index >= count) {
        set_error("device %d not present (%d visible)", index, count);
        return MF_ERR_INVALID;
    }
    int major = 0, minor = 0;
    MF_CHECK_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, index), "capability");
    MF_CHECK_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, index), "capability");
    if (is_sm100) *is_sm100 = (major == 10 && minor == 0);
    return MF_OK;
}

mf_status mf_quantize_workspace(const mf_config* cfg, int32_t is_weight, int64_t rows, int64_t cols,
                                size_t* bytes) {
    mf_status st = check_config(cfg);
    if (st) return st;
    if (!bytes || rows < 1 || cols < 1) {
        set_error("quantize workspace query needs positive shape and an output pointer");
        return MF_ERR_INVALID;
    }
    *bytes = quantize_workspace_bytes(*cfg, is_weight != 0, rows, cols);
    return MF_OK;
}

mf_status mf_quantize_input(const mf_config* cfg, const void* x, int32_t x_dtype, int64_t n, int64_t k,
                            int64_t ldx, const void* fixed_scale, void* codes, void* xscale,
                            void* workspace, size_t workspace_bytes, void* stream) {
    mf_status st = check_config(cfg);
    if (st) return st;
    if (!x || !codes || !xscale || n < 1 || k < 1 || ldx < k || x_dtype < MF_F32 || x_dtype > MF_F64) {
        set_error("mf_quantize_input: invalid operands (n=%lld k=%lld ldx=%lld dtype=%d)", (long long)n,
                  (long long)k, (long long)ldx, x_dtype);
        return MF_ERR_INVALID;
    }
    if (!fixed_scale && !workspace) {
        set_error("mf_quantize_input: dynamic scales need a workspace");
        return MF_ERR_INVALID;
    }
    return quantize_input(*cfg, x, x_dtype, n, k, ldx, fixed_scale, codes, xscale, workspace,
                          workspace_bytes, (cudaStream_t)stream);
}

mf_status mf_check_finite(const void* x, int32_t x_dtype, int64_t n, uint32_t code, uint32_t narrow_code,
                          uint32_t* flag, void* stream) {
    if ((!x && n > 0) || !flag || n < 0 || x_dtype < MF_F32 || x_dtype > MF_F64 || !code) {
        set_error("mf_check_finite: invalid operands");
        return MF_ERR_INVALID;
    }
    return check_finite(x, x_dtype, n, code, narrow_code, flag, (cudaStream_t)stream);
}

mf_status mf_check_operands(const void* a, int32_t a_dtype, int64_t a_count, uint32_t a_narrow_code,
                            const void* b, int32_t b_dtype, int64_t b_count, uint32_t b_narrow_code,
                            uint32_t* flags, int32_t flag_words, void* stream) {
    if (!flags || flag_words < 1 || (!a && a_count > 0) || (!b && b_count > 0) || a_count < 0 || b_count < 0 ||
        a_dtype < MF_F32 || a_dtype > MF_F64 || b_dtype < MF_F32 || b_dtype > MF_F64) {
        set_error("mf_check_operands: invalid operands");
        return MF_ERR_INVALID;
    }
    const cudaStream_t st = (cudaStream_t)stream;
    MF_CHECK_CUDA(cudaMemsetAsync(flags, 0, sizeof(uint32_t) * (size_t)flag_words, st), "clear operand flags");
    mf_status r = check_finite(a, a_dtype, a_count, 1, 0, flags, st);
    if (!r) r = check_finite(b, b_dtype, b_count, 2, b_narrow_code, flags, st);
    if (!r && a_narrow_code) r = check_finite(a, a_dtype, a_count, 1, a_narrow_code, flags, st);
    return r;
}

static bool conv_geometry(const mf_conv2d* cv, int64_t* oh, int64_t* ow) {
    if (!cv || cv->batch < 0 || cv->channels < 1 || cv->height < 1 || cv->width < 1 || cv->kernel_h < 1 ||
        cv->kernel_w < 1 || cv->stride_y < 1 || cv->stride_x < 1 || cv->pad_h < 0 || cv->pad_w < 0 ||
        cv->dilation_h < 1 || cv->dilation_w < 1 || cv->channel_begin < 0 || cv->group_channels < 1 ||
        (int64_t)cv->channel_begin + cv->group_channels > cv->channels || cv->height > INT32_MAX / 2 ||
        cv->width > INT32_MAX / 2 || cv->stride_n < 0 || cv->stride_c < 0 || cv->stride_h < 0 || cv->stride_w < 0) {
        set_error("invalid convolution geometry");
        return false;
    }
    *oh = conv_output_extent(cv->height, cv->kernel_h, cv->stride_y, cv->pad_h, cv->dilation_h);
    *ow = conv_output_extent(cv->width, cv->kernel_w, cv->stride_x, cv->pad_w, cv->dilation_w);
    if (*oh < 1 || *ow < 1) {
        set_error("convolution window larger than the padded input");
        return false;
    }
    return true;
}

mf_status mf_conv_output(const mf_conv2d* conv, int64_t* out_height, int64_t* out_width) {
    int64_t oh = 0, ow = 0;
    if (!out_height || !out_width || !conv_geometry(conv, &oh, &ow)) {
        if (!out_height || !out_width) set_error("mf_conv_output: NULL output");
        return MF_ERR_INVALID;
    }
    *out_height = oh;
    *out_width = ow;
    return MF_OK;
}

mf_status mf_quantize_conv_input(const mf_config* cfg, const mf_conv2d* conv, const void* x, int32_t x_dtype,
                                 const void* fixed_scale, void* codes, void* xscale, uint32_t* nonfinite,
                                 void* workspace, size_t workspace_bytes, void* stream) {
    mf_status st = check_config(cfg);
    if (st) return st;
    int64_t oh = 0, ow = 0;
    if (!conv_geometry(conv, &oh, &ow)) return MF_ERR_INVALID;
    if (!x || !codes || !xscale || !nonfinite || x_dtype < MF_F32 || x_dtype > MF_F64) {
        set_error("mf_quantize_conv_input: invalid operands (dtype=%d)", x_dtype);
        return MF_ERR_INVALID;
    }
    if (!fixed_scale && !workspace) {
        set_error("mf_quantize_conv_input: dynamic scales need a workspace");
        return MF_ERR_INVALID;
    }
    return quantize_conv_input(*cfg, *conv, x, x_dtype, fixed_scale, codes, xscale, nonfinite, workspace,
                               workspace_bytes, (cudaStream_t)stream);
}

}  // extern "C"

// Group-maxima scratch of mf_quantize_input_static.  It is a module global so
// that hosts which own no spare device memory (plain C callers holding only
// their operands, or loops that must not call cudaMalloc because it can stall
// the whole device) can still quantise with dynamic scales.  One copy exists
// per device; its address is looked up once per device and cached.
namespace {
constexpr int kStaticDevices = 64;
__device__ __align__(256) unsigned char g_static_quantize_scratch[MF_STATIC_QUANTIZE_SCRATCH_BYTES];
std::mutex g_static_mutex;
void* g_static_scratch[kStaticDevices] = {};

mf_status static_scratch(void** out) {
    int dev = 0;
    MF_CHECK_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev < 0 || dev >= kStaticDevices) {
        set_error("device %d beyond the %d devices the static scratch table covers", dev, kStaticDevices);
        return MF_ERR_RESOURCE;
    }
    std::lock_guard<std::mutex> lock(g_static_mutex);
    if (!g_static_scratch[dev]) {
        void* p = nullptr;
        MF_CHECK_CUDA(cudaGetSymbolAddress(&p, g_static_quantize_scratch), "static quantize scratch address");
        g_static_scratch[dev] = p;
    }
    *out = g_static_scratch[dev];
    return MF_OK;
}
}  // namespace

extern "C" {

mf_status mf_quantize_input_static(const mf_config* cfg, const void* x, int32_t x_dtype, int64_t n, int64_t k,
                                   int64_t ldx, const void* fixed_scale, void* codes, void* xscale, void* stream) {
    mf_status st = check_config(cfg);
    if (st) return st;
    if (!x || !codes || !xscale || n < 1 || k < 1 || ldx < k || x_dtype < MF_F32 || x_dtype > MF_F64) {
        set_error("mf_quantize_input_static: invalid operands (n=%lld k=%lld ldx=%lld dtype=%d)", (long long)n,
                  (long long)k, (long long)ldx, x_dtype);
        return MF_ERR_INVALID;
    }
    // quantize_workspace_bytes pads by 256 bytes; the maxima themselves need the rest.
    const size_t need = quantize_workspace_bytes(*cfg, false, n, k) - 256;
    if (!fixed_scale && need > MF_STATIC_QUANTIZE_SCRATCH_BYTES) {
        set_error("mf_quantize_input_static: %zu bytes of group maxima exceed the %u-byte static scratch; "
                  "use mf_quantize_input with a workspace", need, MF_STATIC_QUANTIZE_SCRATCH_BYTES);
        return MF_ERR_RESOURCE;
    }
    void* scratch = nullptr;
    st = static_scratch(&scratch);
    if (st) return st;
    // Nothing from an earlier call leaks into this one: each path of the shared
    // quantiser either clears the maxima before its atomic max pass
    // (cudaMemsetAsync) or, in the one-pass row-group kernel, writes every maximum
    // it later reads; a fixed scale reads none.
    return quantize_input(*cfg, x, x_dtype, n, k, ldx, fixed_scale, codes, xscale, scratch,
                          MF_STATIC_QUANTIZE_SCRATCH_BYTES, (cudaStream_t)stream);
}

mf_status mf_program_rhs(const mf_config* cfg, const void* b, int32_t b_dtype, int64_t k, int64_t o, int64_t ldb,
                         void* packed, void* wscale, void* kmajor, void* workspace, size_t workspace_bytes,
                         void* stream) {
    mf_status st = check_config(cfg);
    if (st) return st;
    if (!b || !packed || !wscale || !workspace || o < 1 || k < 1 || ldb < o || b_dtype < MF_F32 ||
        b_dtype > MF_F64) {
        set_error("mf_program_rhs: invalid operands (k=%lld o=%lld ldb=%lld dtype=%d)", (long long)k, (long long)o,
                  (long long)ldb, b_dtype);
        return MF_ERR_INVALID;
    }
    return program_rhs(*cfg, b, b_dtype, k, o, ldb, packed, wscale, kmajor, workspace, workspace_bytes,
                       (cudaStream_t)stream);
}

mf_status mf_program_weights(const mf_config* cfg, const void* w, int32_t w_dtype, int64_t o, int64_t k,
                             int64_t ldw, void* packed, void* wscale, void* workspace,
                             size_t workspace_bytes, void* stream) {
    mf_status st = check_config(cfg);
    if (st) return st;
    if (!w || !packed || !wscale || !workspace || o < 1 || k < 1 || ldw < k || w_dtype < MF_F32 ||
        w_dtype > MF_F64) {
        set_error("mf_program_weights: invalid operands (o=%lld k=%lld ldw=%lld dtype=%d)", (long long)o,
                  (long long)k, (long long)ldw, w_dtype);
        return MF_ERR_INVALID;
    }
    return program_weights(*cfg, w, w_dtype, o, k, ldw, packed, wscale, workspace, workspace_bytes,
                           (cudaStream_t)stream);
}

static bool use_ideal(const mf_config& c, const mf_schedule& s) {
    if (!c.ideal || !exact_integer_counts(c)) return false;
    return generic_ideal_fits(c, s);
}

// Tensor-core kernels: 2 = packed integer counts when the configuration fits its
// plan, else FP8 digit planes; 3 = FP8 digit planes; 0 (automatic) = as 2.
static bool use_packed(const mf_config& c, const mf_schedule& s, int32_t m, int32_t stable) {
    return (s.kernel == 0 || s.kernel == 2) && !stable && tc_packed_eligible(c, m);
}

// Nonideal tensor-core currents (tc_physical.cu): automatic choice and schedule
// kernel 2 when the configuration fits its plan; kernel 1 keeps the SIMT kernels.
static bool use_tc_physical(const mf_config& c, const mf_schedule& s, int32_t m, int32_t stable) {
    return (s.kernel == 0 || s.kernel == 2) && !stable && tc_physical_eligible(c, m);
}

static bool use_tc(const mf_config& c, const mf_schedule& s, int32_t m, int32_t stable) {
    return (s.kernel == 0 || s.kernel == 2 || s.kernel == 3) && !stable && tc_eligible(c, m);
}

static mf_schedule schedule_or_default(const mf_schedule* s) {
    mf_schedule d{0, 32, 64, 2, 0, 0};
    return s ? *s : d;
}

mf_status mf_sliced_mm_workspace(const mf_config* cfg, const mf_schedule* schedule, int64_t n, int32_t m,
                                 int32_t p, int32_t tile_begin, int32_t tile_end, size_t* bytes) {
    mf_status st = check_config(cfg);
    if (st) return st;
    if (!bytes || n < 0 || m < 1 || p < 1 || tile_begin < 0 || tile_end > p || tile_begin >= tile_end) {
        set_error("mf_sliced_mm_workspace: invalid shape");
        return MF_ERR_INVALID;
    }
    mf_schedule s = schedule_or_default(schedule);
    if (use_packed(*cfg, s, m, 0)) *bytes = tc_packed_workspace_bytes(*cfg, n, m, p, tile_end - tile_begin);
    else if (use_tc(*cfg, s, m, 0)) *bytes = tc_workspace_bytes(*cfg, m, p);
    else if (use_tc_physical(*cfg, s, m, 0)) *bytes = tc_physical_workspace_bytes(*cfg, n, m, tile_end - tile_begin);
    else *bytes = use_ideal(*cfg, s) ? 0 : physical_workspace_bytes(*cfg, s, m, tile_end - tile_begin);
    return MF_OK;
}

}  // extern "C"

// mf_sliced_mm with optional peer outputs (mf_mm_buffers.peer_out): the packed
// path only, checked by the caller before anything is enqueued.
static mf_status sliced_mm(const mf_config* cfg, const mf_schedule* schedule, const void* codes,
                           const void* xscale, const void* packed, const void* wscale, const void* bias,
                           void* out, int64_t n, int32_t m, int32_t p, int32_t out_features, int64_t ldo,
                           int32_t tile_begin, int32_t tile_end, uint32_t seed, uint64_t event,
                           int64_t vector_offset, int32_t stable, void* workspace, size_t workspace_bytes,
                           void* stream, void* const* peers, int32_t n_peers) {
    mf_status st = check_config(cfg);
    if (st) return st;
    if (!codes || !xscale || !packed || !wscale || !out || n < 0 || m < 1 || p < 1 || out_features < 1 ||
        out_features > (int64_t)p * cfg->cols || tile_begin < 0 || tile_end > p ||
        ldo < std::min((int64_t)tile_end * cfg->cols, (int64_t)out_features) - (int64_t)tile_begin * cfg->cols ||
        tile_begin >= tile_end || vector_offset < 0) {
        set_error("mf_sliced_mm: invalid operands (n=%lld m=%d p=%d out=%d ldo=%lld tiles=[%d,%d))",
                  (long long)n, m, p, out_features, (long long)ldo, tile_begin, tile_end);
        return MF_ERR_INVALID;
    }
    if (n == 0) return MF_OK;
    if ((long long)(n + 31) / 32 > 2147483647LL) {
        set_error("mf_sliced_mm: too many vectors for one launch");
        return MF_ERR_RESOURCE;
    }
    mf_schedule s = schedule_or_default(schedule);
    if (s.raster < 0 || s.raster > 1) {
        set_error("mf_sliced_mm: raster must be 0 or 1");
        return MF_ERR_INVALID;
    }
    // A stall armed by mf_debug_stall_next_launch applies to this call only, whatever path it takes.
    const int32_t stall_stage = g_stall_stage.exchange(-1);
    MMArgs a{codes, xscale, packed, wscale, bias, out, n, m, p, out_features, ldo, tile_begin, tile_end,
             seed, event, vector_offset, stable, s.kmajor_ready != 0, s.raster, stall_stage,
             g_stall_cycles.load()};
    for (int32_t i = 0; i < n_peers; ++i) a.peer_out[i] = peers[i];
    a.n_peers = n_peers;
    if (n_peers && !use_packed(*cfg, s, m, stable)) {
        set_error("peer outputs need the packed tcgen05 path");
        return MF_ERR_UNSUPPORTED;
    }
    int32_t path;
    mf_status r;
    if (use_packed(*cfg, s, m, stable)) {
        path = MF_PATH_PACKED;
        r = tc_packed_sliced_mm(*cfg, a, workspace, workspace_bytes, (cudaStream_t)stream);
    } else if (use_tc(*cfg, s, m, stable)) {
        path = MF_PATH_FP8_PLANES;
        r = tc_sliced_mm(*cfg, a, workspace, workspace_bytes, (cudaStream_t)stream);
    } else if (use_tc_physical(*cfg, s, m, stable)) {
        path = MF_PATH_TC_CURRENTS;
        r = tc_physical_sliced_mm(*cfg, a, workspace, workspace_bytes, (cudaStream_t)stream);
    } else if (use_ideal(*cfg, s)) {
        path = MF_PATH_GENERIC_IDEAL;
        r = generic_ideal(*cfg, s, a, (cudaStream_t)stream);
    } else {
        path = MF_PATH_SIMT_CURRENTS;
        r = physical(*cfg, s, a, workspace, workspace_bytes, (cudaStream_t)stream);
    }
    if (r == MF_OK) g_last_path = path;
    return r;
}

extern "C" {

mf_status mf_sliced_mm(const mf_config* cfg, const mf_schedule* schedule, const void* codes,
                       const void* xscale, const void* packed, const void* wscale, const void* bias,
                       void* out, int64_t n, int32_t m, int32_t p, int32_t out_features, int64_t ldo,
                       int32_t tile_begin, int32_t tile_end, uint32_t seed, uint64_t event,
                       int64_t vector_offset, int32_t stable, void* workspace, size_t workspace_bytes,
                       void* stream) {
    return sliced_mm(cfg, schedule, codes, xscale, packed, wscale, bias, out, n, m, p, out_features, ldo, tile_begin,
                     tile_end, seed, event, vector_offset, stable, workspace, workspace_bytes, stream, nullptr, 0);
}

mf_status mf_mm(const mf_config* cfg, const mf_schedule* schedule, const void* a, const void* b, int32_t dtype,
                int64_t n, int64_t k, int64_t o, uint32_t a_narrow_code, uint32_t b_narrow_code,
                const mf_mm_buffers* buffers, uint32_t seed, uint64_t event, int64_t vector_offset,
                uint32_t* error_word, void* stream) {
    mf_status st = check_config(cfg);
    if (st) return st;
    const mf_mm_buffers* B = buffers;
    if (!a || !b || !B || !B->codes || !B->xscale || !B->packed || !B->wscale || !B->out || !B->flags ||
        !B->program_workspace || n < 1 || k < 1 || o < 1 || vector_offset < 0 ||
        dtype < MF_F32 || dtype > MF_F64) {
        set_error("mf_mm: invalid operands (n=%lld k=%lld o=%lld dtype=%d)", (long long)n, (long long)k,
                  (long long)o, dtype);
        return MF_ERR_INVALID;
    }
    const mf_config& c = *cfg;
    const int64_t m64 = (k + c.rows - 1) / c.rows, p64 = (o + c.cols - 1) / c.cols;
    if (m64 > INT32_MAX || p64 > INT32_MAX || o > INT32_MAX) {
        set_error("mf_mm: matrix too large for one product");
        return MF_ERR_RESOURCE;
    }
    const int32_t m = (int32_t)m64, p = (int32_t)p64;
    const mf_schedule s = schedule_or_default(schedule);
    if (B->n_peers < 0 || B->n_peers > MF_MAX_PEERS) {
        set_error("mf_mm: n_peers %d outside [0, %d]", B->n_peers, MF_MAX_PEERS);
        return MF_ERR_INVALID;
    }
    for (int32_t i = 0; i < B->n_peers; ++i)
        if (!B->peer_out[i]) {
            set_error("mf_mm: peer output %d is NULL", i);
            return MF_ERR_INVALID;
        }
    if (B->n_peers && !use_packed(c, s, m, 0)) {
        set_error("mf_mm: peer outputs need the packed tcgen05 path");
        return MF_ERR_UNSUPPORTED;
    }
    const size_t quantize_need = quantize_workspace_bytes(c, false, n, k);
    const size_t program_need = quantize_workspace_bytes(c, true, o, k);
    size_t mm_need = 0;
    st = mf_sliced_mm_workspace(cfg, &s, n, m, p, 0, p, &mm_need);
    if (st) return st;
    if (B->quantize_workspace_bytes < quantize_need || !B->quantize_workspace ||
        B->program_workspace_bytes < program_need || B->mm_workspace_bytes < mm_need ||
        (mm_need && !B->mm_workspace)) {
        set_error("mf_mm: workspaces too small (%zu/%zu, %zu/%zu, %zu/%zu bytes)", B->quantize_workspace_bytes,
                  quantize_need, B->program_workspace_bytes, program_need, B->mm_workspace_bytes, mm_need);
        return MF_ERR_RESOURCE;
    }
    const cudaStream_t stream_ = (cudaStream_t)stream;
    uint32_t* flags = B->flags;
    MF_CHECK_CUDA(cudaMemsetAsync(flags, 0, 2 * sizeof(uint32_t), stream_), "clear mf_mm flags");
    // Operand checks in the reference's order (A, then B, then the quantisers' FP32
    // narrowing): folded into the quantiser passes when nothing narrows, else run
    // first as mf_check_operands runs them.
    uint32_t* fold = flags;
    if (a_narrow_code || b_narrow_code) {
        st = check_finite(a, dtype, n * k, 1, 0, flags, stream_);
        if (!st) st = check_finite(b, dtype, k * o, 2, b_narrow_code, flags, stream_);
        if (!st && a_narrow_code) st = check_finite(a, dtype, n * k, 1, a_narrow_code, flags, stream_);
        if (st) return st;
        fold = nullptr;
    }
    st = quantize_input(c, a, dtype, n, k, k, nullptr, B->codes, B->xscale, B->quantize_workspace,
                        B->quantize_workspace_bytes, stream_, fold, 1);
    if (st) return st;
    // The tensor-core kernels read a K-major copy of the codes at the start of their
    // workspace; programming writes it in the same pass.
    const bool kmajor = !c.wide_codes && (use_packed(c, s, m, 0) || use_tc(c, s, m, 0));
    st = program_rhs(c, b, dtype, k, o, o, B->packed, B->wscale, kmajor ? B->mm_workspace : nullptr,
                     B->program_workspace, B->program_workspace_bytes, stream_, fold, 2);
    if (st) return st;
    mf_schedule run = s;
    run.kmajor_ready = kmajor ? 1 : 0;
    st = sliced_mm(cfg, &run, B->codes, B->xscale, B->packed, B->wscale, nullptr, B->out, n, m, p, (int32_t)o, o, 0,
                   p, seed, event, vector_offset, 0, B->mm_workspace, B->mm_workspace_bytes, stream, B->peer_out,
                   B->n_peers);
    if (st) return st;
    st = check_finite(B->out, c.wide ? MF_F64 : MF_F32, n * o, 1, 0, flags + 1, stream_);
    if (st) return st;
    return error_word ? tc_stage_error(error_word, stream_) : MF_OK;
}

mf_status mf_enable_peer_access(int32_t peer_device) {
    int device = 0, count = 0, can = 0;
    MF_CHECK_CUDA(cudaGetDevice(&device), "cudaGetDevice");
    MF_CHECK_CUDA(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
    if (peer_device < 0 || peer_device >= count) {
        set_error("peer device %d not present (%d visible)", peer_device, count);
        return MF_ERR_INVALID;
    }
    if (peer_device == device) return MF_OK;
    MF_CHECK_CUDA(cudaDeviceCanAccessPeer(&can, device, peer_device), "cudaDeviceCanAccessPeer");
    if (!can) {
        set_error("device %d cannot access device %d", device, peer_device);
        return MF_ERR_UNSUPPORTED;
    }
    const cudaError_t err = cudaDeviceEnablePeerAccess(peer_device, 0);
    if (err == cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError();   // clear the sticky-free status this call leaves
        return MF_OK;
    }
    MF_CHECK_CUDA(err, "cudaDeviceEnablePeerAccess");
    return MF_OK;
}

mf_status mf_ipc_export(const void* ptr, void* handle, size_t handle_bytes, size_t* offset) {
    if (!ptr || !handle || !offset || handle_bytes != sizeof(cudaIpcMemHandle_t)) {
        set_error("mf_ipc_export: a pointer, a %zu-byte handle buffer and an offset output are required",
                  sizeof(cudaIpcMemHandle_t));
        return MF_ERR_INVALID;
    }
    // The allocation's base (an IPC handle names a whole allocation), from the driver.
    typedef CUresult (*AddressRange)(CUdeviceptr*, size_t*, CUdeviceptr);
    static AddressRange range = nullptr;
    if (!range) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            range = reinterpret_cast<AddressRange>(p);
    }
    if (!range) {
        set_error("cuMemGetAddressRange unavailable");
        return MF_ERR_CUDA;
    }
    CUdeviceptr base = 0;
    size_t size = 0;
    const CUresult r = range(&base, &size, (CUdeviceptr)(uintptr_t)ptr);
    if (r != CUDA_SUCCESS || !base) {
        set_error("cuMemGetAddressRange failed (%d)", (int)r);
        return MF_ERR_CUDA;
    }
    cudaIpcMemHandle_t h;
    MF_CHECK_CUDA(cudaIpcGetMemHandle(&h, (void*)(uintptr_t)base), "cudaIpcGetMemHandle");
    memcpy(handle, &h, sizeof(h));
    *offset = (size_t)((uintptr_t)ptr - (uintptr_t)base);
    return MF_OK;
}

mf_status mf_ipc_open(const void* handle, size_t handle_bytes, void** base) {
    if (!handle || !base || handle_bytes != sizeof(cudaIpcMemHandle_t)) {
        set_error("mf_ipc_open: a %zu-byte CUDA IPC handle and an output are required", sizeof(cudaIpcMemHandle_t));
        return MF_ERR_INVALID;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    *base = nullptr;
    MF_CHECK_CUDA(cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
    return MF_OK;
}

mf_status mf_ipc_close(void* base) {
    if (!base) {
        set_error("mf_ipc_close: NULL address");
        return MF_ERR_INVALID;
    }
    MF_CHECK_CUDA(cudaIpcCloseMemHandle(base), "cudaIpcCloseMemHandle");
    return MF_OK;
}

int32_t mf_last_path(void) { return g_last_path; }

mf_status mf_debug_stall_next_launch(int32_t stop_stage, int64_t wait_cycles) {
    if (stop_stage < 0 || wait_cycles < 1000 || wait_cycles > 4000000000LL) {
        set_error("mf_debug_stall_next_launch: stop_stage >= 0 and wait_cycles in [1000, 4e9] required");
        return MF_ERR_INVALID;
    }
    g_stall_cycles.store(wait_cycles);
    g_stall_stage.store(stop_stage);
    return MF_OK;
}

mf_status mf_query(const mf_config* cfg, const mf_schedule* schedule, int64_t n, int32_t m, int32_t p,
                   mf_resources* out) {
    mf_status st = check_config(cfg);
    if (st) return st;
    if (!out || m < 1 || p < 1 || n < 0) {
        set_error("mf_query: invalid shape");
        return MF_ERR_INVALID;
    }
    mf_schedule s = schedule_or_default(schedule);
    memset(out, 0, sizeof(*out));
    if (s.raster < 0 || s.raster > 1) {
        set_error("mf_query: raster must be 0 or 1");
        return MF_ERR_INVALID;
    }
    if (use_packed(*cfg, s, m, 0)) {
        out->workspace_bytes = tc_packed_workspace_bytes(*cfg, n, m, p, p);
        out->threads = tc_packed_threads();
        out->kmajor_bytes = (size_t)p * cfg->cols * m * cfg->rows;
        out->path = MF_PATH_PACKED;
    } else if (use_tc(*cfg, s, m, 0)) {
        out->workspace_bytes = tc_workspace_bytes(*cfg, m, p);
        out->threads = tc_block_threads();
        out->path = MF_PATH_FP8_PLANES;
    } else if (use_tc_physical(*cfg, s, m, 0)) {
        // The conductance (or digit) operand is built from the packed codes each call:
        // no K-major copy.
        out->workspace_bytes = tc_physical_workspace_bytes(*cfg, n, m, p);
        out->threads = tc_physical_threads();
        out->path = MF_PATH_TC_CURRENTS;
    } else {
        const bool ideal = use_ideal(*cfg, s);
        out->workspace_bytes = ideal ? 0 : physical_workspace_bytes(*cfg, s, m, p);
        out->threads = 256;
        out->path = ideal ? MF_PATH_GENERIC_IDEAL : MF_PATH_SIMT_CURRENTS;
    }
    return MF_OK;
}

mf_status mf_stage_device_error(uint32_t* host_word, void* stream) {
    if (!host_word) {
        set_error("mf_stage_device_error: NULL output");
        return MF_ERR_INVALID;
    }
    return tc_stage_error(host_word, (cudaStream_t)stream);
}

mf_status mf_take_device_error(uint32_t* code) {
    if (!code) {
        set_error("mf_take_device_error: NULL output");
        return MF_ERR_INVALID;
    }
    unsigned value = 0;
    mf_status st = tc_take_error(&value);
    *code = value;
    if (st) return st;
    if (value) {
        set_error("a device-side wait timed out (code %u); results of the affected launch are invalid", value);
        return MF_ERR_CUDA;
    }
    return MF_OK;
}

}  // extern "C"

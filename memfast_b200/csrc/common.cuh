// Shared device helpers for the memfast_b200 kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "memfast_b200.h"

namespace mf {

// ------------------------------------------------------------------ errors --
void set_error(const char* fmt, ...);
mf_status cuda_status(cudaError_t err, const char* what);

#define MF_CHECK_CUDA(expr, what)                               \
    do {                                                        \
        cudaError_t mf_err__ = (expr);                          \
        if (mf_err__ != cudaSuccess) return mf::cuda_status(mf_err__, what); \
    } while (0)

// Every kernel launch is followed by MF_LAUNCH_CHECK, which also counts it.
void count_launch();
#define MF_LAUNCH_CHECK(what)                                   \
    do {                                                        \
        mf::count_launch();                                     \
        MF_CHECK_CUDA(cudaGetLastError(), what);                \
    } while (0)

// ------------------------------------------------------------------ config --
// Kernel-parameter copy of mf_config restricted to what device code reads.
struct Layout {
    int n_in, n_w;
    int in_shift[MF_MAX_SLICES], in_mask[MF_MAX_SLICES];
    long long in_factor[MF_MAX_SLICES];
    int w_shift[MF_MAX_SLICES], w_mask[MF_MAX_SLICES];
    long long w_factor[MF_MAX_SLICES];
    int adc_max[MF_MAX_SLICES];
    int R, C, rows, reads;
};

inline Layout make_layout(const mf_config& c) {
    Layout L{};
    L.n_in = c.n_in;
    L.n_w = c.n_w;
    for (int i = 0; i < MF_MAX_SLICES; ++i) {
        L.in_shift[i] = c.in_shift[i];
        L.in_mask[i] = c.in_mask[i];
        L.in_factor[i] = c.in_factor[i];
        L.w_shift[i] = c.w_shift[i];
        L.w_mask[i] = c.w_mask[i];
        L.w_factor[i] = c.w_factor[i];
        L.adc_max[i] = c.adc_max[i];
    }
    L.R = c.rows;
    L.C = c.cols;
    L.rows = c.read_rows;
    L.reads = c.reads;
    return L;
}

// Physical constants of one array read, precomputed on the host in the dtype
// the reference computes them in (memfast/reference.py, memfast/config.py).
struct Physics {
    int precise;        // FP64 currents
    int read_mode;      // 0 shared, 1 slice_pair, 2 output
    double high, low, span, voltage, inv_unit;
    double write_var, read_var, volt_var, nonlinear, saf_low, saf_cut, drift;
    double mean_factor, var_factor;   // output read mode: expm1(s^2/2), exp(s^2)expm1(s^2)
};

// ------------------------------------------------------------------ RNG -----
// Counter-based address hash of memfast/random.py:8-33.  Same bit operations,
// same FP32 conversion; every sample is a pure function of (address, seed, stream).
__device__ __forceinline__ uint32_t rng_mix(uint32_t v) {
    v = (v ^ (v >> 16)) * 0x7FEB352Du;
    v = (v ^ (v >> 15)) * 0x846CA68Bu;
    return v ^ (v >> 16);
}

// The hash in three parts, so that a loop over many addresses can keep the parts
// that depend only on the stream (rng_key) and on the address's high word (rng_fold).
__device__ __forceinline__ uint32_t rng_key(uint64_t seed, uint32_t stream) {
    return rng_mix((uint32_t)seed ^ (stream * 0x9E3779B9u));
}

__device__ __forceinline__ uint32_t rng_fold(uint32_t high, uint64_t seed, uint32_t key) {
    uint32_t folded = rng_mix(high ^ rng_mix((uint32_t)(seed >> 32)));
    if (high != 0) folded ^= rng_mix(high ^ key);
    return folded;
}

// (hashed >> 8 + 0.5) / 2^24: the quotient is exact, so it is a product by 2^-24.
__device__ __forceinline__ float rng_unit(uint32_t low, uint32_t folded, uint32_t key) {
    const uint32_t hashed = rng_mix(low ^ folded ^ key);
    return __fmul_rn(__fadd_rn((float)(hashed >> 8), 0.5f), 5.9604644775390625e-8f);
}

__device__ __forceinline__ float rng_uniform(int64_t address, uint64_t seed, uint32_t stream) {
    const uint32_t key = rng_key(seed, stream);
    return rng_unit((uint32_t)address, rng_fold((uint32_t)((uint64_t)address >> 32), seed, key), key);
}

__host__ __device__ __forceinline__ uint64_t event_seed(uint64_t seed, uint64_t event) {
    auto mix = [](uint32_t v) {
        v = (v ^ (v >> 16)) * 0x7FEB352Du;
        v = (v ^ (v >> 15)) * 0x846CA68Bu;
        return v ^ (v >> 16);
    };
    return (seed ^ (uint64_t)mix((uint32_t)event)) | ((uint64_t)mix((uint32_t)(event >> 32)) << 32);
}

// Box-Muller of streams s and s+1 (random.py:29-33), in FP32.
__device__ __forceinline__ float box_muller(float first, float second) {
    const float radius = sqrtf(__fmul_rn(-2.0f, logf(first)));
    return __fmul_rn(radius, cosf(__fmul_rn(6.283185307179586f, second)));
}

__device__ __forceinline__ float rng_normal(int64_t address, uint64_t seed, uint32_t stream) {
    return box_muller(rng_uniform(address, seed, stream), rng_uniform(address, seed, stream + 1));
}

// ------------------------------------------------- restored conductance --
// FP32 conductance of one cell (reference.py:10-51): nominal level of the weight
// digit, write variation (stream 10), drift, stuck-at faults (stream 30) and,
// in shared read mode, the read event's variation (stream 20).  `address` is the
// global cell address (((array * p + tile) * W + w) * R + row) * C + col.
__device__ __forceinline__ float restored_conductance_f32(const Physics& P, long long state, int mask,
                                                          long long address, uint64_t seed, uint64_t read_seed) {
    const float high = (float)P.high, low = (float)P.low, span = (float)P.span;
    float f;
    if (mask == 1) f = state ? high : low;
    else f = __fadd_rn(low, __fmul_rn(span, __fdiv_rn((float)state, (float)mask)));
    if (P.write_var != 0) f = __fmul_rn(f, expf(__fmul_rn((float)P.write_var, rng_normal(address, seed, 10))));
    f = __fmul_rn(f, (float)P.drift);
    if (P.saf_cut != 0) {
        const float u = rng_uniform(address, seed, 30);
        const float lo = (float)P.saf_low, hi = (float)P.saf_cut;
        if (u < lo) f = low;
        if (u >= lo && u < hi) f = high;
    }
    if (P.read_mode == 0 && P.read_var != 0)
        f = __fmul_rn(f, expf(__fmul_rn((float)P.read_var, rng_normal(address, read_seed, 20))));
    return f;
}

// ------------------------------------------------------------- cascade sum --
// PyTorch's CPU reduction over a non-innermost dimension (SumKernel.cpp
// multi_row_sum): values are summed from +0.0 in blocks of 2^power; at every
// block boundary the block sum moves up one level, and higher levels fold in
// when their counters wrap.  `index` is the number of values already pushed.
template <typename T>
struct Cascade {
    T acc[4];
    __device__ __forceinline__ void init() { acc[0] = acc[1] = acc[2] = acc[3] = T(0); }
};

template <typename T>
__device__ __forceinline__ T add_rn(T a, T b);
template <>
__device__ __forceinline__ float add_rn<float>(float a, float b) { return __fadd_rn(a, b); }
template <>
__device__ __forceinline__ double add_rn<double>(double a, double b) { return __dadd_rn(a, b); }

// Push value number `index` (0-based) of a reduction of `size` values whose
// full blocks end at `full` = size - size % step.
template <typename T>
__device__ __forceinline__ void cascade_push(Cascade<T>& c, T value, int64_t index, int power,
                                             int64_t full) {
    c.acc[0] = add_rn(c.acc[0], value);
    int64_t done = index + 1;
    if (done <= full && (done & ((int64_t(1) << power) - 1)) == 0) {
        const int64_t mask = (int64_t(1) << power) - 1;
#pragma unroll
        for (int j = 1; j < 4; ++j) {
            c.acc[j] = add_rn(c.acc[j], c.acc[j - 1]);
            c.acc[j - 1] = T(0);
            if ((done & (mask << (j * power))) != 0) break;
        }
    }
}

template <typename T>
__device__ __forceinline__ T cascade_finish(const Cascade<T>& c) {
    T s = c.acc[0];
    s = add_rn(s, c.acc[1]);
    s = add_rn(s, c.acc[2]);
    s = add_rn(s, c.acc[3]);
    return add_rn(T(0), s);
}

// ------------------------------------------------------- scale restoration --
// simulator.py:57-66 restore_scales: frexp each factor, multiply mantissas,
// add exponents, ldexp in two steps.  torch.ldexp multiplies by
// torch.pow(2.0, int32 exponent), which PyTorch evaluates in FP32.
__device__ __forceinline__ double pow2_as_f32(int e) { return (double)ldexpf(1.0f, e); }

__device__ __forceinline__ double restore_scales(double value, double xs, double ws) {
    int ve, xe, we;
    double vm = frexp(value, &ve);
    double xm = frexp(xs, &xe);
    double wm = frexp(ws, &we);
    double mantissa = __dmul_rn(__dmul_rn(vm, xm), wm);
    int exponent = ve + xe + we;
    int first = exponent < -1022 ? -1022 : (exponent > 1023 ? 1023 : exponent);
    double restored = __dmul_rn(mantissa, pow2_as_f32(first));
    restored = __dmul_rn(restored, pow2_as_f32(exponent - first));
    return mantissa == 0.0 ? 0.0 : restored;
}

__host__ __device__ inline int ceil_log2_i64(int64_t x) {
    int bits = 0;
    while ((int64_t(1) << bits) < x) ++bits;
    return bits;
}

// Level width of the cascade for a reduction of `size` values.
__host__ __device__ inline int cascade_power(int64_t size) {
    int p = ceil_log2_i64(size) / 4;
    return p < 4 ? 4 : p;
}

}  // namespace mf

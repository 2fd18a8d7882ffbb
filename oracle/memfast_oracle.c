/*
 * TEST INFRASTRUCTURE ONLY -- CPU oracle for the memfast_b200 parity tests.
 *
 * Plain-C restatement of the reference MemFast CPU path for the sliced matrix
 * product (HUST-ISMD-Odyssey/MemFast v0.3.0).  Only tests/, the smoke check
 * and bench.py's CPU-baseline leg load this library; the product never does.
 *
 *   rng_*          memfast/random.py:8-33          (mix, uniform, event_seed, normal)
 *   orc_restore    memfast/reference.py:10-51      (conductance restore per cell)
 *   orc_partial    memfast/reference.py:63-117     (per-read slice-pair currents,
 *                                                   ADC, signed reconstruction)
 *   orc_adc_count  memfast/reference.py:54-60
 *   orc_epilogue_* memfast/simulator.py:561-586    (scale products, sum over reads)
 *   cascade_*      PyTorch CPU sum over a non-innermost dimension
 *                  (aten/src/ATen/native/cpu/SumKernel.cpp multi_row_sum: 16-row
 *                  blocks summed from +0.0, block sums accumulated level by level)
 *
 * All floating-point statements are written one IEEE operation at a time and the
 * file is compiled with -ffp-contract=off, so every product and sum rounds exactly
 * where the reference's elementwise PyTorch expressions round.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    int n_in, n_w;                 /* physical input / weight slices            */
    int in_shift[32], in_mask[32];
    long long in_factor[32];
    int w_shift[32], w_mask[32];
    long long w_factor[32];
    int adc_max[32];               /* per weight slice, least significant first */
    int R, C, rows, reads;         /* array rows, columns, rows per read, reads */
    int precise;                   /* FP64 currents (Config.precise_currents)   */
    int read_mode;                 /* 0 shared, 1 slice_pair, 2 output          */
    double high, low, voltage, unit;
    double write_var, read_var, volt_var, nonlinear, saf_low, saf_high, drift;
} orc_cfg;

/* ------------------------------------------------------------------ RNG -- */
static inline uint32_t rng_mix(uint32_t v) {
    v = (v ^ (v >> 16)) * 0x7FEB352Du;
    v = (v ^ (v >> 15)) * 0x846CA68Bu;
    return v ^ (v >> 16);
}

float rng_uniform(int64_t address, uint64_t seed, uint32_t stream) {
    uint32_t key = rng_mix((uint32_t)seed ^ (stream * 0x9E3779B9u));
    uint32_t high = (uint32_t)((uint64_t)address >> 32);
    uint32_t folded = rng_mix(high ^ rng_mix((uint32_t)(seed >> 32)));
    if (high != 0) folded ^= rng_mix(high ^ key);
    uint32_t hashed = rng_mix((uint32_t)address ^ folded ^ key);
    float f = (float)(hashed >> 8);
    f = f + 0.5f;
    return f / 16777216.0f;
}

uint64_t rng_event_seed(uint64_t seed, uint64_t event) {
    return (seed ^ (uint64_t)rng_mix((uint32_t)event)) |
           ((uint64_t)rng_mix((uint32_t)(event >> 32)) << 32);
}

float rng_normal(int64_t address, uint64_t seed, uint32_t stream) {
    float first = rng_uniform(address, seed, stream);
    float second = rng_uniform(address, seed, stream + 1);
    float radius = sqrtf(-2.0f * logf(first));
    float angle = 6.283185307179586f * second;
    return radius * cosf(angle);
}

/* ------------------------------------------------------------- restore -- */
/* Conductance of every cell of tiles [begin,end): g[m][width][W][R][C].
 * packed: [m][p][R][C] weight codes.  Same element order as reference.py:10-51. */
static void restore_f32(const orc_cfg* k, const int64_t* packed, int m, int p, int begin,
                        int end, uint32_t seed, uint64_t event, float* g) {
    const int W = k->n_w, R = k->R, C = k->C, width = end - begin;
    const float high = (float)k->high, low = (float)k->low, span = (float)(k->high - k->low);
    const float drift = (float)k->drift, wv = (float)k->write_var, rv = (float)k->read_var;
    const float saf_lo = (float)k->saf_low, saf_hi = (float)(k->saf_low + k->saf_high);
    const uint64_t read_seed = rng_event_seed(seed, event);
#pragma omp parallel for collapse(2) schedule(static)
    for (int arr = 0; arr < m; ++arr)
        for (int t = 0; t < width; ++t)
            for (int w = 0; w < W; ++w)
                for (int r = 0; r < R; ++r)
                    for (int c = 0; c < C; ++c) {
                        int tile = begin + t;
                        int64_t address = ((((int64_t)arr * p + tile) * W + w) * R + r) * C + c;
                        int64_t code = packed[(((int64_t)arr * p + tile) * R + r) * C + c];
                        int64_t state = (code >> k->w_shift[w]) & k->w_mask[w];
                        float raw;
                        if (k->w_mask[w] == 1) {
                            raw = state ? high : low;
                        } else {
                            float frac = (float)state / (float)k->w_mask[w];
                            float scaled = span * frac;
                            raw = low + scaled;
                        }
                        if (k->write_var != 0) {
                            float z = rng_normal(address, seed, 10);
                            float e = wv * z;
                            raw = raw * expf(e);
                        }
                        raw = raw * drift;
                        if (k->saf_low + k->saf_high != 0) {
                            float u = rng_uniform(address, seed, 30);
                            if (u < saf_lo) raw = low;
                            if (u >= saf_lo && u < saf_hi) raw = high;
                        }
                        if (k->read_mode == 0 && k->read_var != 0) {
                            float z = rng_normal(address, read_seed, 20);
                            float e = rv * z;
                            raw = raw * expf(e);
                        }
                        g[((((int64_t)arr * width + t) * W + w) * R + r) * C + c] = raw;
                    }
}

static void restore_f64(const orc_cfg* k, const int64_t* packed, int m, int p, int begin,
                        int end, uint32_t seed, uint64_t event, double* g) {
    const int W = k->n_w, R = k->R, C = k->C, width = end - begin;
    const double high = k->high, low = k->low, span = k->high - k->low;
    const uint64_t read_seed = rng_event_seed(seed, event);
#pragma omp parallel for collapse(2) schedule(static)
    for (int arr = 0; arr < m; ++arr)
        for (int t = 0; t < width; ++t)
            for (int w = 0; w < W; ++w)
                for (int r = 0; r < R; ++r)
                    for (int c = 0; c < C; ++c) {
                        int tile = begin + t;
                        int64_t address = ((((int64_t)arr * p + tile) * W + w) * R + r) * C + c;
                        int64_t code = packed[(((int64_t)arr * p + tile) * R + r) * C + c];
                        int64_t state = (code >> k->w_shift[w]) & k->w_mask[w];
                        double raw;
                        if (k->w_mask[w] == 1) {
                            raw = state ? high : low;
                        } else {
                            double frac = (double)state / (double)k->w_mask[w];
                            raw = low + span * frac;
                        }
                        /* The reference multiplies the FP64 raw by FP32 noise factors. */
                        if (k->write_var != 0) {
                            float z = rng_normal(address, seed, 10);
                            float e = (float)k->write_var * z;
                            raw = raw * (double)expf(e);
                        }
                        raw = raw * k->drift;
                        if (k->saf_low + k->saf_high != 0) {
                            float u = rng_uniform(address, seed, 30);
                            /* PyTorch compares the FP32 sample with FP32-cast probabilities. */
                            const float lo = (float)k->saf_low, hi = (float)(k->saf_low + k->saf_high);
                            if (u < lo) raw = low;
                            if (u >= lo && u < hi) raw = high;
                        }
                        if (k->read_mode == 0 && k->read_var != 0) {
                            float z = rng_normal(address, read_seed, 20);
                            float e = (float)k->read_var * z;
                            raw = raw * (double)expf(e);
                        }
                        g[((((int64_t)arr * width + t) * W + w) * R + r) * C + c] = raw;
                    }
}

void orc_restore_f32(const orc_cfg* k, const int64_t* packed, int m, int p, int begin, int end,
                     uint32_t seed, uint64_t event, float* g) {
    restore_f32(k, packed, m, p, begin, end, seed, event, g);
}

/* ------------------------------------------------------------------ ADC -- */
static inline double adc_count_f32(const orc_cfg* k, float current, int w) {
    int maximum = k->adc_max[w];
    float value = current * (float)(1.0 / k->unit);
    if (k->nonlinear != 0) {
        float slope = (float)(k->nonlinear / maximum);
        float bend = fabsf(slope * value);
        value = value / (1.0f + bend);
    }
    if (value < 0.0f) value = 0.0f;
    if (value > (float)maximum) value = (float)maximum;
    return (double)rintf(value);
}

static inline double adc_count_f64(const orc_cfg* k, double current, int w) {
    int maximum = k->adc_max[w];
    double value = current * (1.0 / k->unit);
    if (k->nonlinear != 0) {
        double slope = k->nonlinear / maximum;
        value = value / (1.0 + fabs(slope * value));
    }
    if (value < 0.0) value = 0.0;
    if (value > (double)maximum) value = (double)maximum;
    return rint(value);
}

double orc_adc_count(const orc_cfg* k, double current, int w) {
    return k->precise ? adc_count_f64(k, current, w) : adc_count_f32(k, (float)current, w);
}

/* ------------------------------------------------------ ideal partials -- */
/* Exact-integer ideal device: count = min(sum_r d_a d_w, adc_max[w]).  This is
 * what reference.py:63-117 computes whenever its FP32/FP64 current error stays
 * below half a count (every configuration the parity tests use).
 * q: [n][m][R] activation codes; packed: [m][p][R][C]; totals: [n][m*reads][width][C]. */
void orc_partial_ideal(const orc_cfg* k, const int64_t* q, const int64_t* packed, int n, int m,
                       int p, int begin, int end, int64_t* totals) {
    const int R = k->R, C = k->C, reads = k->reads, width = end - begin;
#pragma omp parallel for collapse(2) schedule(static)
    for (int v = 0; v < n; ++v)
        for (int arr = 0; arr < m; ++arr)
            for (int g = 0; g < reads; ++g)
                for (int t = 0; t < width; ++t)
                    for (int c = 0; c < C; ++c) {
                        int r0 = g * k->rows, r1 = r0 + k->rows < R ? r0 + k->rows : R;
                        int64_t total = 0;
                        for (int a = 0; a < k->n_in; ++a)
                            for (int w = 0; w < k->n_w; ++w) {
                                int64_t dot = 0;
                                for (int r = r0; r < r1; ++r) {
                                    int64_t da = (q[((int64_t)v * m + arr) * R + r] >> k->in_shift[a]) & k->in_mask[a];
                                    int64_t code = packed[(((int64_t)arr * p + begin + t) * R + r) * C + c];
                                    int64_t dw = (code >> k->w_shift[w]) & k->w_mask[w];
                                    dot += da * dw;
                                }
                                if (dot > k->adc_max[w]) dot = k->adc_max[w];
                                total += dot * k->in_factor[a] * k->w_factor[w];
                            }
                        totals[((((int64_t)v * m + arr) * reads + g) * width + t) * C + c] = total;
                    }
}

/* --------------------------------------------------- physical partials -- */
/* Mirror of reference.py:63-117 with explicit currents (FP32, or FP64 when
 * k->precise), all noise streams and the three read-variation modes.  The dot
 * over rows runs in ascending row order without FMA contraction. */
void orc_partial_physical(const orc_cfg* k, const int64_t* q, const int64_t* packed, int n,
                          int m, int p, int begin, int end, uint32_t seed, uint64_t event,
                          int64_t* totals) {
    const int R = k->R, C = k->C, reads = k->reads, W = k->n_w, A = k->n_in;
    const int width = end - begin;
    const uint64_t read_seed = rng_event_seed(seed, event);
    size_t cells = (size_t)m * width * W * R * C;
    float* g32 = NULL;
    double* g64 = NULL;
    if (k->precise) {
        g64 = (double*)malloc(cells * sizeof(double));
        restore_f64(k, packed, m, p, begin, end, seed, event, g64);
    } else {
        g32 = (float*)malloc(cells * sizeof(float));
        restore_f32(k, packed, m, p, begin, end, seed, event, g32);
    }
    memset(totals, 0, sizeof(int64_t) * (size_t)n * m * reads * width * C);
    const float low32 = (float)k->low, volt32 = (float)k->voltage, vv32 = (float)k->volt_var;
    const float rv32 = (float)k->read_var;
    const double s2 = k->read_var * k->read_var;
    const float mean_f = (float)expm1(0.5 * s2), var_f = (float)(exp(s2) * expm1(s2));
#pragma omp parallel for collapse(2) schedule(static)
    for (int v = 0; v < n; ++v)
        for (int arr = 0; arr < m; ++arr) {
            double* volt = (double*)malloc(sizeof(double) * R);
            for (int a = 0; a < A; ++a) {
                int amask = k->in_mask[a];
                for (int r = 0; r < R; ++r) {
                    int64_t d = (q[((int64_t)v * m + arr) * R + r] >> k->in_shift[a]) & amask;
                    if (k->precise) {
                        double x = (double)d / (double)amask * k->voltage;
                        if (k->volt_var != 0) {
                            int64_t address = (((int64_t)v * m + arr) * A + a) * R + r;
                            float z = rng_normal(address, read_seed, 40);
                            float f = vv32 * z;
                            f = 1.0f + f;
                            x = x * (double)f;
                        }
                        volt[r] = x;
                    } else {
                        float x = (float)d / (float)amask;
                        x = x * volt32;
                        if (k->volt_var != 0) {
                            int64_t address = (((int64_t)v * m + arr) * A + a) * R + r;
                            float z = rng_normal(address, read_seed, 40);
                            float f = vv32 * z;
                            f = 1.0f + f;
                            x = x * f;
                        }
                        volt[r] = x;
                    }
                }
                for (int w = 0; w < W; ++w) {
                    int wmask = k->w_mask[w];
                    for (int grp = 0; grp < reads; ++grp) {
                        int r0 = grp * k->rows, r1 = r0 + k->rows < R ? r0 + k->rows : R;
                        int read_part = arr * reads + grp;
                        for (int t = 0; t < width; ++t)
                            for (int c = 0; c < C; ++c) {
                                double current_d = 0.0, mean_d = 0.0, var_d = 0.0;
                                float current = 0.0f, mean = 0.0f, var = 0.0f;
                                for (int r = r0; r < r1; ++r) {
                                    size_t gi = ((((size_t)arr * width + t) * W + w) * R + r) * C + c;
                                    int64_t cell = ((((int64_t)arr * p + begin + t) * W + w) * R + r) * C + c;
                                    if (k->precise) {
                                        double gval = g64[gi];
                                        if (k->read_mode == 1 && k->read_var != 0) {
                                            float z = rng_normal(cell * A + a, read_seed, 20);
                                            gval = gval * (double)expf(rv32 * z);
                                        }
                                        double prod = volt[r] * (gval - k->low);
                                        current_d = current_d + prod;
                                        if (k->read_mode == 2 && k->read_var != 0) {
                                            mean_d = mean_d + volt[r] * gval;
                                            var_d = var_d + (volt[r] * volt[r]) * (gval * gval);
                                        }
                                    } else {
                                        float gval = g32[gi];
                                        if (k->read_mode == 1 && k->read_var != 0) {
                                            float z = rng_normal(cell * A + a, read_seed, 20);
                                            float e = rv32 * z;
                                            gval = gval * expf(e);
                                        }
                                        float vr = (float)volt[r];
                                        float eff = gval - low32;
                                        float prod = vr * eff;
                                        current = current + prod;
                                        if (k->read_mode == 2 && k->read_var != 0) {
                                            float pm = vr * gval;
                                            mean = mean + pm;
                                            float vsq = vr * vr, gsq = gval * gval;
                                            float pv = vsq * gsq;
                                            var = var + pv;
                                        }
                                    }
                                }
                                int64_t address = (((((int64_t)v * m * reads + read_part) * p + begin + t) * A + a) * W + w) * C + c;
                                double count;
                                if (k->precise) {
                                    if (k->read_mode == 2 && k->read_var != 0) {
                                        double mu = mean_d * expm1(0.5 * s2);
                                        double sig = var_d * (exp(s2) * expm1(s2));
                                        float z = rng_normal(address, read_seed, 60);
                                        current_d = current_d + (mu + sqrt(sig) * (double)z);
                                    }
                                    count = adc_count_f64(k, current_d * (double)((int64_t)amask * wmask), w);
                                } else {
                                    if (k->read_mode == 2 && k->read_var != 0) {
                                        float mu = mean * mean_f;
                                        float sig = var * var_f;
                                        float z = rng_normal(address, read_seed, 60);
                                        float noise = sqrtf(sig) * z;
                                        float shift = mu + noise;
                                        current = current + shift;
                                    }
                                    float scaled = current * (float)((int64_t)amask * wmask);
                                    count = adc_count_f32(k, scaled, w);
                                }
                                size_t ti = ((((size_t)v * m + arr) * reads + grp) * width + t) * C + c;
                                totals[ti] += (int64_t)count * (k->in_factor[a] * k->w_factor[w]);
                            }
                    }
                }
            }
            free(volt);
        }
    free(g32);
    free(g64);
}

/* --------------------------------------------------------- epilogues -- */
static int ceil_log2(int64_t x) {
    int bits = 0;
    while (((int64_t)1 << bits) < x) ++bits;
    return bits;
}

/* PyTorch CPU multi_row_sum over `size` values x[i*stride], float accumulators. */
static float cascade_f32(const float* x, int64_t size, int64_t stride) {
    const int levels = 4;
    int power = ceil_log2(size) / levels;
    if (power < 4) power = 4;
    const int64_t step = (int64_t)1 << power, mask = step - 1;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    int64_t i = 0;
    while (i + step <= size) {
        for (int64_t j = 0; j < step; ++j, ++i) acc[0] = acc[0] + x[i * stride];
        for (int j = 1; j < levels; ++j) {
            acc[j] = acc[j] + acc[j - 1];
            acc[j - 1] = 0.0f;
            if ((i & (mask << (j * power))) != 0) break;
        }
    }
    for (; i < size; ++i) acc[0] = acc[0] + x[i * stride];
    for (int j = 1; j < levels; ++j) acc[0] = acc[0] + acc[j];
    return acc[0];
}

static double cascade_f64(const double* x, int64_t size, int64_t stride) {
    const int levels = 4;
    int power = ceil_log2(size) / levels;
    if (power < 4) power = 4;
    const int64_t step = (int64_t)1 << power, mask = step - 1;
    double acc[4] = {0.0, 0.0, 0.0, 0.0};
    int64_t i = 0;
    while (i + step <= size) {
        for (int64_t j = 0; j < step; ++j, ++i) acc[0] = acc[0] + x[i * stride];
        for (int j = 1; j < levels; ++j) {
            acc[j] = acc[j] + acc[j - 1];
            acc[j - 1] = 0.0;
            if ((i & (mask << (j * power))) != 0) break;
        }
    }
    for (; i < size; ++i) acc[0] = acc[0] + x[i * stride];
    for (int j = 1; j < levels; ++j) acc[0] = acc[0] + acc[j];
    return acc[0];
}

float orc_cascade_f32(const float* x, int64_t size, int64_t stride) { return cascade_f32(x, size, stride); }
double orc_cascade_f64(const double* x, int64_t size, int64_t stride) { return cascade_f64(x, size, stride); }

/* simulator.py:578-585 (narrow formats): out[v][t*C+c] = sum_i fl(fl(T*xs)*ws).
 * totals: [n][MR][width][C] int64; xscale [n][MR] f32; wscale [MR][p][C] f32;
 * out: [n][width*C] f32 (the tile-group slice of the [n, p*C] output). */
void orc_epilogue_f32(const int64_t* totals, const float* xscale, const float* wscale, int n,
                      int MR, int p, int C, int begin, int end, float* out, int64_t out_stride) {
    const int width = end - begin;
#pragma omp parallel for schedule(static)
    for (int v = 0; v < n; ++v) {
        float* column = (float*)malloc(sizeof(float) * MR);
        for (int t = 0; t < width; ++t)
            for (int c = 0; c < C; ++c) {
                for (int i = 0; i < MR; ++i) {
                    float value = (float)totals[(((int64_t)v * MR + i) * width + t) * C + c];
                    value = value * xscale[(int64_t)v * MR + i];
                    value = value * wscale[((int64_t)i * p + begin + t) * C + c];
                    column[i] = value;
                }
                float s = cascade_f32(column, MR, 1);
                out[(int64_t)v * out_stride + t * C + c] = 0.0f + s;
            }
        free(column);
    }
}

/* torch.ldexp(x, e) multiplies by torch.pow(2.0, e) with an int32 exponent,
 * which PyTorch evaluates in the default FP32 dtype before the FP64 product. */
static inline double pow2_as_f32(int e) { return (double)ldexpf(1.0f, e); }

/* simulator.py:57-66 restore_scales followed by the FP64 sum over reads. */
void orc_epilogue_f64(const int64_t* totals, const double* xscale, const double* wscale, int n,
                      int MR, int p, int C, int begin, int end, double* out, int64_t out_stride) {
    const int width = end - begin;
#pragma omp parallel for schedule(static)
    for (int v = 0; v < n; ++v) {
        double* column = (double*)malloc(sizeof(double) * MR);
        for (int t = 0; t < width; ++t)
            for (int c = 0; c < C; ++c) {
                for (int i = 0; i < MR; ++i) {
                    double value = (double)totals[(((int64_t)v * MR + i) * width + t) * C + c];
                    int ve, xe, we;
                    double vm = frexp(value, &ve);
                    double xm = frexp(xscale[(int64_t)v * MR + i], &xe);
                    double wm = frexp(wscale[((int64_t)i * p + begin + t) * C + c], &we);
                    double mantissa = vm * xm;
                    mantissa = mantissa * wm;
                    int exponent = ve + xe + we;
                    int first = exponent < -1022 ? -1022 : (exponent > 1023 ? 1023 : exponent);
                    double restored = mantissa * pow2_as_f32(first);
                    restored = restored * pow2_as_f32(exponent - first);
                    column[i] = mantissa == 0.0 ? 0.0 : restored;
                }
                double s = cascade_f64(column, MR, 1);
                out[(int64_t)v * out_stride + t * C + c] = 0.0 + s;
            }
        free(column);
    }
}

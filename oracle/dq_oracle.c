/*
 * dq_oracle.c -- CPU restatement of dyn-quant's fused dynamic-precision GEMV.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the oracle: the parity tests, the
 * smoke check and the CPU-baseline leg of the benchmark call it to check or to
 * time against.  The product (the sm_100a kernels behind include/dq_abi.h)
 * never links, loads or calls it.
 *
 * Every function restates one piece of the reference, citing the file:line it
 * follows (paths inside the dyn-quant project):
 *
 *   dqo_quantize          src/quant_format.cuh:48-53, 58-97   (bit-exact)
 *   dqo_detect            src/outlier_detect.cuh:18-49, 104-205
 *   dqo_split_gemv        src/split_gemv.cu:75-158
 *   dqo_int4_gemv         src/int4_gemv.cu:30-78
 *   dqo_reference_gemv    src/reference_gemv.cu:9-57 (kernel), :59-78 (launcher)
 *   dqo_dense_gemv_f64    (no counterpart: FP32/FP64 dense accuracy yardstick)
 *
 * Arithmetic is IEEE-754 binary32 in the reference's order of operations.
 * Build with -ffp-contract=off and without -ffast-math so that no FMA
 * contraction or reassociation changes the rounding.  The reference's GPU
 * build uses -use_fast_math (approximate divide and square root), so the
 * detector threshold here can differ from the reference GPU's in the last
 * bits; the parity rule for the outlier mask allows channels within 1e-5
 * relative of the threshold to differ.
 *
 * Two deliberate readings of the reference, both where its source does not
 * compile or does not do what its comments say:
 *   (1) src/split_gemv.cu:63 passes a float* where src/outlier_detect.cuh:108
 *       declares int*.  The comment on both lines says float*; the float
 *       reading is used (mean kept as float, not truncated to int).
 *   (2) src/split_gemv.cu:85-93 stages packed bytes only for rows 0..1 of
 *       each 4-row block (128 threads, r = tid/64), so warps 2..3 read shared
 *       memory that is never written.  The intended semantics -- every row
 *       uses its own packed bytes -- are restated here.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <float.h>
#include <limits.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define DQO_GROUP 128          /* src/quant_format.cuh:10 */
#define DQO_BLOCK 128          /* src/split_gemv.cu:9 (4 warps) */
#define DQO_WARPS 4
#define DQO_MAX_OUTLIER_FRAC_INV 4  /* src/split_gemv.cu:11 */

/* ------------------------------------------------------------------------ */
/* IEEE binary16 <-> binary32 (own implementation from the IEEE definition)  */
/* ------------------------------------------------------------------------ */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* Exact widening of a binary16 bit pattern. */
float dqo_h2f(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    if (exp == 0x1Fu) return u2f(sign | 0x7F800000u | (man << 13));   /* inf / nan */
    if (exp == 0) {
        if (man == 0) return u2f(sign);
        /* subnormal: value = man * 2^-24, exact in binary32 */
        float v = (float)man * 0x1p-24f;
        return sign ? -v : v;
    }
    return u2f(sign | ((exp + 112u) << 23) | (man << 13));
}

/* Round-to-nearest-even narrowing to binary16.  NaN becomes 0x7FFF, the
 * canonical NaN that CUDA's conversions produce. */
uint16_t dqo_f2h(float f) {
    uint32_t u = f2u(f);
    uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    uint32_t a = u & 0x7FFFFFFFu;
    if (a > 0x7F800000u) return 0x7FFFu;
    if (a == 0x7F800000u) return sign | 0x7C00u;
    int e = (int)(a >> 23) - 127;          /* unbiased exponent */
    uint32_t m = (a & 0x7FFFFFu) | 0x800000u;  /* 24-bit significand */
    if (a < 0x00800000u) return sign;       /* binary32 subnormal -> 0 */
    if (e > 15) return sign | 0x7C00u;
    int shift;                              /* bits to drop from the 24-bit significand */
    uint32_t base;
    if (e >= -14) { shift = 13; base = (uint32_t)(e + 15) << 10; m &= 0x7FFFFFu; m |= 0x800000u; }
    else { shift = 13 + (-14 - e); base = 0; }
    if (shift > 24) return sign;            /* below half of the smallest subnormal */
    uint32_t keep = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1);
    uint32_t out;
    if (e >= -14) out = base + (keep & 0x3FFu);  /* implicit bit dropped, exponent in base */
    else out = keep;                              /* subnormal: no implicit bit */
    if (rem > half || (rem == half && (out & 1u))) out += 1u;  /* carry may bump the exponent: correct */
    return sign | (uint16_t)out;
}

void dqo_h2f_array(const uint16_t* h, float* f, int64_t n) {
    for (int64_t i = 0; i < n; ++i) f[i] = dqo_h2f(h[i]);
}

void dqo_f2h_array(const float* f, uint16_t* h, int64_t n) {
    for (int64_t i = 0; i < n; ++i) h[i] = dqo_f2h(f[i]);
}

/* ------------------------------------------------------------------------ */
/* Quantizer: src/quant_format.cuh:48-53 and :58-97                         */
/* ------------------------------------------------------------------------ */

/* (int)t with the x86-64 cvttss2si result for NaN and out-of-range input
 * (INT_MIN), which is what the reference's host build computes. */
static inline int trunc_to_int_x86(float t) {
    if (!(t >= -2147483648.0f && t < 2147483648.0f)) return INT_MIN;
    return (int)t;
}

/* src/quant_format.cuh:48-53 */
static inline int quantize_val(float val, float min_val, float inv_scale) {
    float d = val - min_val;
    float p = d * inv_scale;
    float s = p + 0.5f;
    int code = trunc_to_int_x86(s);
    if (code < 0) code = 0;
    if (code > 15) code = 15;
    return code;
}

/* src/quant_format.cuh:58-97 -- the packing loop (the cudaMalloc / H2D tail,
 * :99-115, is the caller's business).  w: row-major [d_out][d_in] binary16. */
int dqo_quantize(const uint16_t* w, int d_out, int d_in,
                 uint8_t* packed, uint16_t* scales, uint16_t* zeros) {
    if (d_out < 0 || d_in <= 0 || d_in % DQO_GROUP) return 1;
    const int G = d_in / DQO_GROUP;
    #pragma omp parallel for schedule(static)
    for (int row = 0; row < d_out; ++row) {
        const uint16_t* src = w + (size_t)row * d_in;
        for (int g = 0; g < G; ++g) {
            int c0 = g * DQO_GROUP;
            float gmin = FLT_MAX, gmax = -FLT_MAX;
            for (int i = 0; i < DQO_GROUP; ++i) {
                float v = dqo_h2f(src[c0 + i]);
                if (v < gmin) gmin = v;
                if (v > gmax) gmax = v;
            }
            float range = gmax - gmin;
            float scale_f = (range < 1e-8f) ? 1.0f : range / 15.0f;
            float inv_scale = 1.0f / scale_f;
            float zero_f = -gmin * inv_scale;
            scales[(size_t)row * G + g] = dqo_f2h(scale_f);
            zeros[(size_t)row * G + g] = dqo_f2h(zero_f);
            for (int i = 0; i < DQO_GROUP; i += 2) {
                int lo = quantize_val(dqo_h2f(src[c0 + i]), gmin, inv_scale);
                int hi = quantize_val(dqo_h2f(src[c0 + i + 1]), gmin, inv_scale);
                packed[(size_t)row * (d_in / 2) + (c0 + i) / 2] =
                    (uint8_t)((lo & 0xF) | ((hi & 0xF) << 4));
            }
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Outlier detector: src/outlier_detect.cuh:18-49 and :104-205              */
/* ------------------------------------------------------------------------ */

typedef struct { float mean; float M2; int count; } welford_t;

/* src/outlier_detect.cuh:18-23 */
static inline void welford_update(welford_t* s, float x) {
    s->count += 1;
    float delta = x - s->mean;
    float q = delta / (float)s->count;
    s->mean = s->mean + q;
    float d2 = x - s->mean;
    float p = delta * d2;
    s->M2 = s->M2 + p;
}

/* src/outlier_detect.cuh:26-37 -- note the order: ((delta*nb)/n) and
 * (((delta*delta)*(na*nb))/n), then left-to-right additions. */
static inline welford_t welford_merge(welford_t a, welford_t b) {
    if (a.count == 0) return b;
    if (b.count == 0) return a;
    welford_t o;
    o.count = a.count + b.count;
    float delta = b.mean - a.mean;
    float t = delta * (float)b.count;
    t = t / (float)o.count;
    o.mean = a.mean + t;
    float dd = delta * delta;
    float nn = (float)a.count * (float)b.count;
    float u = dd * nn;
    u = u / (float)o.count;
    float m = a.M2 + b.M2;
    o.M2 = m + u;
    return o;
}

/* src/outlier_detect.cuh:40-49: xor butterfly; every lane merges (own, partner)
 * with all lanes stepping together. */
static void warp_reduce_welford(welford_t lanes[32]) {
    for (int off = 16; off >= 1; off >>= 1) {
        welford_t prev[32];
        memcpy(prev, lanes, sizeof(prev));
        for (int l = 0; l < 32; ++l) lanes[l] = welford_merge(prev[l], prev[l ^ off]);
    }
}

/*
 * dqo_detect -- the block-cooperative scan of src/outlier_detect.cuh:104-205
 * as launched by src/split_gemv.cu:61-64 (128 threads, capacity d_in/4).
 *
 * Outputs (any may be NULL):
 *   mask[d_in]     1 where the channel is kept as an outlier, else 0
 *   indices[cap]   the kept indices in the reference's list order
 *                  (warp 0's stripe ascending, then warp 1's, ...)
 *   stats[4]       mean, thresh, var, M2 (binary32)
 * Returns the kept count (<= d_in/4), or -1 on bad arguments.
 */
int dqo_detect(const uint16_t* x, int n, float k,
               uint8_t* mask, int32_t* indices, float* stats) {
    if (n <= 0) return -1;
    const int capacity = n / DQO_MAX_OUTLIER_FRAC_INV;   /* src/split_gemv.cu:172 */
    const int warp_cap = capacity / DQO_WARPS;            /* src/outlier_detect.cuh:160 */

    /* Phase 1: per-thread Welford over i = tid, tid+128, ... (:124-125) */
    welford_t th[DQO_BLOCK];
    for (int t = 0; t < DQO_BLOCK; ++t) {
        th[t].mean = 0.f; th[t].M2 = 0.f; th[t].count = 0;
        for (int i = t; i < n; i += DQO_BLOCK) welford_update(&th[t], dqo_h2f(x[i]));
    }
    /* warp butterflies (:127), lane 0 publishes (:128-132) */
    welford_t warp_state[DQO_WARPS];
    for (int w = 0; w < DQO_WARPS; ++w) {
        welford_t lanes[32];
        memcpy(lanes, &th[w * 32], sizeof(lanes));
        warp_reduce_welford(lanes);
        warp_state[w] = lanes[0];
    }
    /* thread 0 merges serially from an empty state (:135-147) */
    welford_t g = {0.f, 0.f, 0};
    for (int w = 0; w < DQO_WARPS; ++w) g = welford_merge(g, warp_state[w]);

    float mean = g.mean;
    float var = (g.count > 1) ? g.M2 / (float)(g.count - 1) : 0.f;   /* :151-153 */
    float thresh = k * sqrtf(fmaxf(var, 1e-8f));                     /* :154 */
    if (stats) { stats[0] = mean; stats[1] = thresh; stats[2] = var; stats[3] = g.M2; }

    if (mask) memset(mask, 0, (size_t)n);
    /* Phase 2: each warp walks its stripe base = w*32 + j*128, ballot-compacts
     * ascending indices, keeps the first warp_cap (:160-178). Phase 3 concatenates
     * warp lists in warp order (:181-204). */
    int total = 0;
    for (int w = 0; w < DQO_WARPS; ++w) {
        int warp_out = 0;
        for (int base = w * 32; base < n; base += DQO_WARPS * 32) {
            for (int lane = 0; lane < 32; ++lane) {
                int idx = base + lane;
                if (idx >= n) continue;
                float val = dqo_h2f(x[idx]);
                if (fabsf(val - mean) > thresh) {
                    if (warp_out < warp_cap) {
                        if (mask) mask[idx] = 1;
                        if (indices) indices[total] = idx;
                        ++total;
                    }
                    ++warp_out;
                }
            }
        }
    }
    return total;
}

/* ------------------------------------------------------------------------ */
/* GEMVs                                                                      */
/* ------------------------------------------------------------------------ */

/* The 32-lane __shfl_down_sync tree of src/split_gemv.cu:144-148 (same in
 * int4_gemv.cu:61-65 and reference_gemv.cu:43-47); returns lane 0's value. */
static float shfl_down_tree(float acc[32]) {
    float a[32];
    memcpy(a, acc, sizeof(a));
    for (int off = 16; off >= 1; off >>= 1) {
        float b[32];
        for (int l = 0; l < 32; ++l) b[l] = a[l] + ((l + off < 32) ? a[l + off] : a[l]);
        memcpy(a, b, sizeof(a));
    }
    return a[0];
}

/*
 * src/split_gemv.cu:75-158 for rows [0, d_out): outlier columns (mask[c] != 0)
 * take the FP16 weight, the rest sf*(code - zf); per lane two column pairs per
 * 128-column tile, acc += w0*x0 + w1*x1; then the shuffle tree; y16 = RN(y32).
 * fp16_w: row-major [d_out][d_in].  mask: from dqo_detect.
 */
void dqo_split_gemv_masked(const uint8_t* packed, const uint16_t* scales, const uint16_t* zeros,
                           const uint16_t* fp16_w, const uint16_t* x, const uint8_t* mask,
                           int d_out, int d_in, float* y32, uint16_t* y16) {
    const int T = d_in / DQO_GROUP;
    float* xf = (float*)malloc(sizeof(float) * (size_t)d_in);
    for (int c = 0; c < d_in; ++c) xf[c] = dqo_h2f(x[c]);
    #pragma omp parallel for schedule(static)
    for (int row = 0; row < d_out; ++row) {
        float acc[32];
        for (int l = 0; l < 32; ++l) acc[l] = 0.f;
        const uint8_t* prow = packed + (size_t)row * (d_in / 2);
        const uint16_t* wrow = fp16_w ? fp16_w + (size_t)row * d_in : NULL;
        for (int t = 0; t < T; ++t) {
            int cs = t * DQO_GROUP;
            float sf = dqo_h2f(scales[(size_t)row * T + t]);
            float zf = dqo_h2f(zeros[(size_t)row * T + t]);
            for (int lane = 0; lane < 32; ++lane) {
                for (int i = 0; i < 2; ++i) {
                    int c0 = lane * 4 + i * 2, c1 = c0 + 1;
                    int g0 = cs + c0, g1 = cs + c1;
                    float x0 = xf[g0], x1 = xf[g1];
                    float w0, w1;
                    uint8_t pb0 = prow[(cs + c0) / 2];
                    uint8_t pb1 = prow[(cs + c1) / 2];
                    if (mask && mask[g0]) w0 = dqo_h2f(wrow[g0]);
                    else w0 = sf * ((float)(pb0 & 0xF) - zf);
                    if (mask && mask[g1]) w1 = dqo_h2f(wrow[g1]);
                    else w1 = sf * ((float)((pb1 >> 4) & 0xF) - zf);
                    float p0 = w0 * x0, p1 = w1 * x1;
                    float s = p0 + p1;
                    acc[lane] = acc[lane] + s;
                }
            }
        }
        float r = shfl_down_tree(acc);
        if (y32) y32[row] = r;
        if (y16) y16[row] = dqo_f2h(r);
    }
    free(xf);
}

/* Detection followed by the split GEMV: the whole of launch_split_gemv
 * (src/split_gemv.cu:160-198).  Returns the outlier count. */
int dqo_split_gemv(const uint8_t* packed, const uint16_t* scales, const uint16_t* zeros,
                   const uint16_t* fp16_w, const uint16_t* x, int d_out, int d_in,
                   float k, float* y32, uint16_t* y16, uint8_t* mask_out) {
    uint8_t* mask = mask_out ? mask_out : (uint8_t*)malloc((size_t)d_in);
    int n = dqo_detect(x, d_in, k, mask, NULL, NULL);
    dqo_split_gemv_masked(packed, scales, zeros, fp16_w, x, mask, d_out, d_in, y32, y16);
    if (!mask_out) free(mask);
    return n;
}

/* src/int4_gemv.cu:30-78: per lane two bytes, acc += w0*x0; acc += w1*x1. */
void dqo_int4_gemv(const uint8_t* packed, const uint16_t* scales, const uint16_t* zeros,
                   const uint16_t* x, int d_out, int d_in, float* y32, uint16_t* y16) {
    const int T = d_in / DQO_GROUP;
    float* xf = (float*)malloc(sizeof(float) * (size_t)d_in);
    for (int c = 0; c < d_in; ++c) xf[c] = dqo_h2f(x[c]);
    #pragma omp parallel for schedule(static)
    for (int row = 0; row < d_out; ++row) {
        float acc[32];
        for (int l = 0; l < 32; ++l) acc[l] = 0.f;
        const uint8_t* prow = packed + (size_t)row * (d_in / 2);
        for (int t = 0; t < T; ++t) {
            int cs = t * DQO_GROUP;
            float sf = dqo_h2f(scales[(size_t)row * T + t]);
            float zf = dqo_h2f(zeros[(size_t)row * T + t]);
            for (int lane = 0; lane < 32; ++lane) {
                for (int i = 0; i < 2; ++i) {
                    uint8_t pb = prow[cs / 2 + lane * 2 + i];
                    int c0 = lane * 4 + i * 2, c1 = c0 + 1;
                    float w0 = sf * ((float)(pb & 0xF) - zf);
                    float w1 = sf * ((float)((pb >> 4) & 0xF) - zf);
                    acc[lane] = acc[lane] + w0 * xf[cs + c0];
                    acc[lane] = acc[lane] + w1 * xf[cs + c1];
                }
            }
        }
        float r = shfl_down_tree(acc);
        if (y32) y32[row] = r;
        if (y16) y16[row] = dqo_f2h(r);
    }
    free(xf);
}

/* src/reference_gemv.cu:9-57: per lane four consecutive columns per tile. */
void dqo_reference_gemv(const uint16_t* w, const uint16_t* x, int d_out, int d_in,
                        float* y32, uint16_t* y16) {
    const int T = d_in / DQO_GROUP;
    float* xf = (float*)malloc(sizeof(float) * (size_t)d_in);
    for (int c = 0; c < d_in; ++c) xf[c] = dqo_h2f(x[c]);
    #pragma omp parallel for schedule(static)
    for (int row = 0; row < d_out; ++row) {
        float acc[32];
        for (int l = 0; l < 32; ++l) acc[l] = 0.f;
        const uint16_t* wr = w + (size_t)row * d_in;
        for (int t = 0; t < T; ++t) {
            int cs = t * DQO_GROUP;
            for (int lane = 0; lane < 32; ++lane)
                for (int i = 0; i < 4; ++i) {
                    int c = cs + lane * 4 + i;
                    acc[lane] = acc[lane] + dqo_h2f(wr[c]) * xf[c];
                }
        }
        float r = shfl_down_tree(acc);
        if (y32) y32[row] = r;
        if (y16) y16[row] = dqo_f2h(r);
    }
    free(xf);
}

/* Dense yardstick: y = W x in binary64 over the FP16 inputs. */
void dqo_dense_gemv_f64(const uint16_t* w, const uint16_t* x, int d_out, int d_in, double* y) {
    double* xd = (double*)malloc(sizeof(double) * (size_t)d_in);
    for (int c = 0; c < d_in; ++c) xd[c] = (double)dqo_h2f(x[c]);
    #pragma omp parallel for schedule(static)
    for (int row = 0; row < d_out; ++row) {
        const uint16_t* wr = w + (size_t)row * d_in;
        double s = 0.0;
        for (int c = 0; c < d_in; ++c) s += (double)dqo_h2f(wr[c]) * xd[c];
        y[row] = s;
    }
    free(xd);
}

int dqo_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void dqo_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/*
 * sf_oracle.c -- CPU restatement of the StrataFlow per-token MoE decode path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the product): see sf_oracle.h.
 *
 * Built with -ffp-contract=off so every float expression rounds exactly as
 * written (the synthetic generator and the weight quantizers are reproduced
 * bit for bit by the CUDA generator, which is compiled with -fmad=false).
 *
 * Citations: "engine.cpp" = src/model/engine/engine.cpp of the reference.
 * ggml b11379 is not vendored in the reference (.gitmodules:1-3); its CPU
 * kernels are restated from the published reference implementations
 * (ggml-quants.c *_ref functions, ggml-cpu ops.cpp) and named per function.
 */
#include "sf_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define QK_K 256
#define QK8_0 32

typedef struct { uint16_t d; int8_t qs[QK8_0]; } blk_q8_0;                        /* 34 B  */
typedef struct { uint16_t d, dmin; uint8_t scales[12]; uint8_t qs[QK_K / 2]; } blk_q4_K; /* 144 B */
typedef struct { uint8_t ql[QK_K / 2]; uint8_t qh[QK_K / 4]; int8_t scales[QK_K / 16]; uint16_t d; } blk_q6_K; /* 210 B */
typedef struct { float d; int8_t qs[QK_K]; int16_t bsums[QK_K / 16]; } blk_q8_K;  /* 292 B */

_Static_assert(sizeof(blk_q8_0) == 34, "q8_0");
_Static_assert(sizeof(blk_q4_K) == 144, "q4_K");
_Static_assert(sizeof(blk_q6_K) == 210, "q6_K");
_Static_assert(sizeof(blk_q8_K) == 292, "q8_K");

static int g_threads = 0;
void sfo_set_threads(int n) { g_threads = n; }
static int nthreads(void) {
#ifdef _OPENMP
    return g_threads > 0 ? g_threads : omp_get_max_threads();
#else
    return 1;
#endif
}

/* ---- fp16 <-> fp32, IEEE round-to-nearest-even (what F16C / numpy do) ---- */
float sfo_fp16_to_fp32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: normalise */
            int e = -1;
            do { man <<= 1; ++e; } while ((man & 0x400u) == 0);
            man &= 0x3FFu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t sfo_fp32_to_fp16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) { /* inf / nan */
        return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
    }
    if (ax >= 0x477FF000u) { /* rounds to >= 65520 -> inf */
        return (uint16_t)(sign | 0x7C00u);
    }
    if (ax < 0x38800000u) { /* result subnormal or zero (|f| < 2^-14) */
        if (ax < 0x33000000u) return sign; /* < 2^-25: rounds to 0 */
        const uint32_t e = ax >> 23;
        const uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
        const uint32_t shift = 126u - e; /* 14 + (113 - e) + ... */
        /* value = m * 2^(e-150); subnormal unit = 2^-24 -> q = m >> (126 - e) */
        const uint32_t q = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1u);
        uint32_t r = q + ((rem > half || (rem == half && (q & 1u))) ? 1u : 0u);
        return (uint16_t)(sign | r);
    }
    /* normal */
    uint32_t e = (ax >> 23) - 112u;
    uint32_t m = ax & 0x7FFFFFu;
    uint32_t q = (e << 10) | (m >> 13);
    const uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q += 1u; /* carry may bump exponent: still correct */
    return (uint16_t)(sign | q);
}

/* ggml's nearest_int: round half to even through the 1.5*2^23 trick, valid
 * for |fval| <= 4194303 (ggml-quants.c). */
static inline int nearest_int(float fval) {
    float val = fval + 12582912.f;
    int i;
    memcpy(&i, &val, sizeof(int));
    return (i & 0x007fffff) - 0x00400000;
}

size_t sfo_row_bytes(int type, int64_t n) {
    switch (type) {
    case SFO_F32: return (size_t)n * 4;
    case SFO_F16: return (size_t)n * 2;
    case SFO_Q8_0: return (size_t)(n / QK8_0) * sizeof(blk_q8_0);
    case SFO_Q4_K: return (size_t)(n / QK_K) * sizeof(blk_q4_K);
    case SFO_Q6_K: return (size_t)(n / QK_K) * sizeof(blk_q6_K);
    case SFO_Q8_K: return (size_t)(n / QK_K) * sizeof(blk_q8_K);
    default: return 0;
    }
}

static int block_size(int type) {
    switch (type) {
    case SFO_Q8_0: return QK8_0;
    case SFO_Q4_K: case SFO_Q6_K: case SFO_Q8_K: return QK_K;
    default: return 1;
    }
}

/* ---- dequantization (ggml-quants.c dequantize_row_*; gguf-py quants.py
 *      Q8_0:396, Q4_K:504, Q6_K:552 restate the same arithmetic) ---------- */
static void get_scale_min_k4(int j, const uint8_t *q, uint8_t *d, uint8_t *m) {
    if (j < 4) {
        *d = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *d = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j - 0] >> 6) << 4));
    }
}

int sfo_dequantize(int type, const void *src, float *y, int64_t n) {
    if (n % block_size(type)) return -1;
    switch (type) {
    case SFO_F32: memcpy(y, src, (size_t)n * 4); return 0;
    case SFO_F16: {
        const uint16_t *h = (const uint16_t *)src;
        for (int64_t i = 0; i < n; ++i) y[i] = sfo_fp16_to_fp32(h[i]);
        return 0;
    }
    case SFO_Q8_0: {
        const blk_q8_0 *x = (const blk_q8_0 *)src;
        for (int64_t i = 0; i < n / QK8_0; ++i) {
            const float d = sfo_fp16_to_fp32(x[i].d);
            for (int j = 0; j < QK8_0; ++j) y[i * QK8_0 + j] = x[i].qs[j] * d;
        }
        return 0;
    }
    case SFO_Q4_K: {
        const blk_q4_K *x = (const blk_q4_K *)src;
        for (int64_t i = 0; i < n / QK_K; ++i) {
            const float d = sfo_fp16_to_fp32(x[i].d);
            const float min = sfo_fp16_to_fp32(x[i].dmin);
            const uint8_t *q = x[i].qs;
            float *yy = y + i * QK_K;
            int is = 0;
            for (int j = 0; j < QK_K; j += 64) {
                uint8_t sc, m;
                get_scale_min_k4(is + 0, x[i].scales, &sc, &m);
                const float d1 = d * sc, m1 = min * m;
                get_scale_min_k4(is + 1, x[i].scales, &sc, &m);
                const float d2 = d * sc, m2 = min * m;
                for (int l = 0; l < 32; ++l) *yy++ = d1 * (q[l] & 0xF) - m1;
                for (int l = 0; l < 32; ++l) *yy++ = d2 * (q[l] >> 4) - m2;
                q += 32;
                is += 2;
            }
        }
        return 0;
    }
    case SFO_Q6_K: {
        const blk_q6_K *x = (const blk_q6_K *)src;
        for (int64_t i = 0; i < n / QK_K; ++i) {
            const float d = sfo_fp16_to_fp32(x[i].d);
            const uint8_t *ql = x[i].ql, *qh = x[i].qh;
            const int8_t *sc = x[i].scales;
            float *yy = y + i * QK_K;
            for (int nn = 0; nn < QK_K; nn += 128) {
                for (int l = 0; l < 32; ++l) {
                    const int is = l / 16;
                    const int8_t q1 = (int8_t)((ql[l + 0] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                    const int8_t q2 = (int8_t)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                    const int8_t q3 = (int8_t)((ql[l + 0] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                    const int8_t q4 = (int8_t)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                    yy[l + 0] = d * sc[is + 0] * q1;
                    yy[l + 32] = d * sc[is + 2] * q2;
                    yy[l + 64] = d * sc[is + 4] * q3;
                    yy[l + 96] = d * sc[is + 6] * q4;
                }
                yy += 128;
                ql += 64;
                qh += 32;
                sc += 8;
            }
        }
        return 0;
    }
    case SFO_Q8_K: {
        const blk_q8_K *x = (const blk_q8_K *)src;
        for (int64_t i = 0; i < n / QK_K; ++i)
            for (int j = 0; j < QK_K; ++j) y[i * QK_K + j] = x[i].d * x[i].qs[j];
        return 0;
    }
    default: return -1;
    }
}

/* ---- activation quantizers (ggml-quants.c quantize_row_q8_0_ref,
 *      quantize_row_q8_K_ref) ---------------------------------------------- */
int sfo_quantize_q8_0(const float *x, void *dst, int64_t k) {
    if (k % QK8_0) return -1;
    blk_q8_0 *y = (blk_q8_0 *)dst;
    for (int64_t i = 0; i < k / QK8_0; ++i) {
        float amax = 0.0f;
        for (int j = 0; j < QK8_0; ++j) {
            const float v = fabsf(x[i * QK8_0 + j]);
            amax = amax > v ? amax : v;
        }
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        y[i].d = sfo_fp32_to_fp16(d);
        for (int j = 0; j < QK8_0; ++j) y[i].qs[j] = (int8_t)roundf(x[i * QK8_0 + j] * id);
    }
    return 0;
}

int sfo_quantize_q8_K(const float *x, void *dst, int64_t k) {
    if (k % QK_K) return -1;
    blk_q8_K *y = (blk_q8_K *)dst;
    for (int64_t i = 0; i < k / QK_K; ++i) {
        const float *xx = x + i * QK_K;
        float max = 0, amax = 0;
        for (int j = 0; j < QK_K; ++j) {
            const float ax = fabsf(xx[j]);
            if (ax > amax) { amax = ax; max = xx[j]; }
        }
        if (amax == 0.0f) {
            y[i].d = 0;
            memset(y[i].qs, 0, QK_K);
            memset(y[i].bsums, 0, sizeof(y[i].bsums));
            continue;
        }
        const float iscale = -127.f / max;
        for (int j = 0; j < QK_K; ++j) {
            const int v = nearest_int(iscale * xx[j]);
            y[i].qs[j] = (int8_t)(v < 127 ? v : 127);
        }
        for (int j = 0; j < QK_K / 16; ++j) {
            int sum = 0;
            for (int ii = 0; ii < 16; ++ii) sum += y[i].qs[j * 16 + ii];
            y[i].bsums[j] = (int16_t)sum;
        }
        y[i].d = 1 / iscale;
    }
    return 0;
}

/* ---- the build's own weight quantizers (fixture generation only) ---------
 * Q4_K: ggml's block structure (8 sub-blocks of 32, 6-bit scales and mins
 * under f16 super-scales) with a direct min/max scale choice in place of
 * ggml's iterative make_qkx2_quants search.  Q6_K: 16 sub-blocks of 16, signed
 * 6-bit codes under int8 scales (the make_qx_quants sign convention).
 * Every step is a single IEEE op so the CUDA generator reproduces it exactly. */
static void quant_block_q4_K(const float *x, blk_q4_K *y) {
    float scales[8], mins[8];
    float max_scale = 0.0f, max_min = 0.0f;
    for (int j = 0; j < 8; ++j) {
        const float *xs = x + 32 * j;
        float mn = xs[0], mx = xs[0];
        for (int l = 1; l < 32; ++l) {
            if (xs[l] < mn) mn = xs[l];
            if (xs[l] > mx) mx = xs[l];
        }
        if (mn > 0.0f) mn = 0.0f;
        scales[j] = (mx - mn) / 15.0f;
        mins[j] = -mn;
        if (scales[j] > max_scale) max_scale = scales[j];
        if (mins[j] > max_min) max_min = mins[j];
    }
    const float inv_scale = max_scale > 0.0f ? 63.0f / max_scale : 0.0f;
    const float inv_min = max_min > 0.0f ? 63.0f / max_min : 0.0f;
    uint8_t ls[8], lm[8];
    for (int j = 0; j < 8; ++j) {
        int a = nearest_int(inv_scale * scales[j]);
        int b = nearest_int(inv_min * mins[j]);
        ls[j] = (uint8_t)(a > 63 ? 63 : (a < 0 ? 0 : a));
        lm[j] = (uint8_t)(b > 63 ? 63 : (b < 0 ? 0 : b));
    }
    memset(y->scales, 0, 12);
    for (int j = 0; j < 8; ++j) {
        if (j < 4) {
            y->scales[j] = ls[j];
            y->scales[j + 4] = lm[j];
        } else {
            y->scales[j + 4] = (uint8_t)((ls[j] & 0xF) | ((lm[j] & 0xF) << 4));
            y->scales[j - 4] |= (uint8_t)((ls[j] >> 4) << 6);
            y->scales[j - 0] |= (uint8_t)((lm[j] >> 4) << 6);
        }
    }
    y->d = sfo_fp32_to_fp16(max_scale / 63.0f);
    y->dmin = sfo_fp32_to_fp16(max_min / 63.0f);
    const float d = sfo_fp16_to_fp32(y->d), dmin = sfo_fp16_to_fp32(y->dmin);
    uint8_t L[QK_K];
    for (int j = 0; j < 8; ++j) {
        uint8_t sc, m;
        get_scale_min_k4(j, y->scales, &sc, &m);
        const float dd = d * sc, dm = dmin * m;
        for (int l = 0; l < 32; ++l) {
            int q = 0;
            if (dd != 0.0f) {
                float v = (x[32 * j + l] + dm) / dd;
                v = fminf(fmaxf(v, -1.0f), 16.0f);
                q = nearest_int(v);
                q = q < 0 ? 0 : (q > 15 ? 15 : q);
            }
            L[32 * j + l] = (uint8_t)q;
        }
    }
    for (int c = 0; c < 4; ++c)
        for (int l = 0; l < 32; ++l)
            y->qs[32 * c + l] = (uint8_t)(L[64 * c + l] | (L[64 * c + 32 + l] << 4));
}

static void quant_block_q6_K(const float *x, blk_q6_K *y) {
    float scales[16];
    float max_scale = 0.0f, max_abs = 0.0f;
    for (int j = 0; j < 16; ++j) {
        float amax = 0.0f, mx = 0.0f;
        for (int l = 0; l < 16; ++l) {
            const float ax = fabsf(x[16 * j + l]);
            if (ax > amax) { amax = ax; mx = x[16 * j + l]; }
        }
        scales[j] = amax > 0.0f ? mx / -32.0f : 0.0f;
        const float as = fabsf(scales[j]);
        if (as > max_abs) { max_abs = as; max_scale = scales[j]; }
    }
    memset(y, 0, sizeof(*y));
    uint8_t L[QK_K];
    if (max_abs == 0.0f) {
        for (int i = 0; i < QK_K; ++i) L[i] = 32;
    } else {
        const float iscale = -128.0f / max_scale;
        y->d = sfo_fp32_to_fp16(1.0f / iscale);
        for (int j = 0; j < 16; ++j) {
            int s = nearest_int(iscale * scales[j]);
            y->scales[j] = (int8_t)(s > 127 ? 127 : (s < -128 ? -128 : s));
        }
        const float d = sfo_fp16_to_fp32(y->d);
        for (int j = 0; j < 16; ++j) {
            const float dj = d * y->scales[j];
            for (int l = 0; l < 16; ++l) {
                int q = 0;
                if (dj != 0.0f) {
                    float v = x[16 * j + l] / dj;
                    v = fminf(fmaxf(v, -40.0f), 40.0f);
                    q = nearest_int(v);
                    q = q < -32 ? -32 : (q > 31 ? 31 : q);
                }
                L[16 * j + l] = (uint8_t)(q + 32);
            }
        }
    }
    for (int n = 0; n < 2; ++n) {
        for (int l = 0; l < 32; ++l) {
            const uint8_t q1 = L[128 * n + l + 0], q2 = L[128 * n + l + 32];
            const uint8_t q3 = L[128 * n + l + 64], q4 = L[128 * n + l + 96];
            y->ql[64 * n + l + 0] = (uint8_t)((q1 & 0xF) | ((q3 & 0xF) << 4));
            y->ql[64 * n + l + 32] = (uint8_t)((q2 & 0xF) | ((q4 & 0xF) << 4));
            y->qh[32 * n + l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
        }
    }
}

int sfo_quantize_weights(int type, const float *x, void *dst, int64_t nrows, int64_t ncols) {
    if (ncols % block_size(type)) return -1;
    const size_t rb = sfo_row_bytes(type, ncols);
    #pragma omp parallel for num_threads(nthreads()) schedule(static)
    for (int64_t r = 0; r < nrows; ++r) {
        const float *xr = x + r * ncols;
        uint8_t *yr = (uint8_t *)dst + (size_t)r * rb;
        switch (type) {
        case SFO_F32: memcpy(yr, xr, rb); break;
        case SFO_F16:
            for (int64_t i = 0; i < ncols; ++i) ((uint16_t *)yr)[i] = sfo_fp32_to_fp16(xr[i]);
            break;
        case SFO_Q8_0: sfo_quantize_q8_0(xr, yr, ncols); break;
        case SFO_Q4_K:
            for (int64_t b = 0; b < ncols / QK_K; ++b) quant_block_q4_K(xr + b * QK_K, (blk_q4_K *)yr + b);
            break;
        case SFO_Q6_K:
            for (int64_t b = 0; b < ncols / QK_K; ++b) quant_block_q6_K(xr + b * QK_K, (blk_q6_K *)yr + b);
            break;
        default: break;
        }
    }
    return 0;
}

/* ---- synthetic weights ---------------------------------------------------- */
static inline uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

uint64_t sfo_tensor_seed(uint64_t seed, int tid, int layer) {
    return splitmix64(seed * 0x100000001B3ull + (uint64_t)(tid + 1) * 0x9E3779B1ull +
                      (uint64_t)(layer + 1) * 0x85EBCA77ull);
}

/* z = (sum of twelve 16-bit uniforms - 6*65536) / 65536: mean 0, variance ~1.
 * Integer sum, exact int->float conversion and a power-of-two scale make the
 * value identical on any IEEE machine. */
static inline float synth_z(uint64_t seed, int64_t i) {
    uint32_t s = 0;
    for (int w = 0; w < 3; ++w) {
        const uint64_t r = splitmix64(seed + (uint64_t)i * 3u + (uint64_t)w);
        s += (uint32_t)(r & 0xFFFF) + (uint32_t)((r >> 16) & 0xFFFF) +
             (uint32_t)((r >> 32) & 0xFFFF) + (uint32_t)(r >> 48);
    }
    return (float)((int32_t)s - 393210) * (1.0f / 65536.0f);
}

void sfo_synth_f32(uint64_t seed, int64_t offset, int64_t n, float std_, float *dst) {
    #pragma omp parallel for num_threads(nthreads()) schedule(static)
    for (int64_t i = 0; i < n; ++i) dst[i] = synth_z(seed, offset + i) * std_;
}

/* ---- exp -------------------------------------------------------------------
 * exp(x) for float x by Cody & Waite's argument reduction (x = n ln2 + r with
 * ln2 split into a 16-bit head and a tail so n*head is exact) and the degree-7
 * Taylor polynomial of e^r on |r| <= ln2/2 (truncation < 8e-9 relative),
 * scaled by 2^n through the exponent field.  Every step is one IEEE-rounded
 * operation, so the CUDA kernels evaluate it to the same bits (they spell each
 * step with __fmul_rn / __fadd_rn).  Used where ggml calls expf (softmax,
 * SiLU); ggml's SIMD builds also use their own exp approximations. */
float sfo_expf(float x) {
    if (x != x) return x;
    if (x > 88.72283935546875f) return INFINITY;
    if (x < -103.97208404541015625f) return 0.0f;
    const float t = x * 1.44269502162933349609375f;
    const int n = nearest_int(t);
    const float fn = (float)n;
    float r = x - fn * 0.693145751953125f;
    r = r - fn * 1.428606765330187045037746429443359375e-06f;
    float p = 1.98412701138295233249664306640625e-04f;
    p = p * r + 1.38888892251998186111450195312500e-03f;
    p = p * r + 8.33333376795053482055664062500000e-03f;
    p = p * r + 4.16666679084300994873046875000000e-02f;
    p = p * r + 1.66666671633720397949218750000000e-01f;
    p = p * r + 0.5f;
    p = p * r + 1.0f;
    p = p * r + 1.0f;
    /* p * 2^n, n in [-150, 128]: two exact power-of-two factors */
    int n1 = n / 2, n2 = n - n / 2;
    uint32_t b1 = (uint32_t)(n1 + 127) << 23, b2 = (uint32_t)(n2 + 127) << 23;
    float f1, f2;
    memcpy(&f1, &b1, 4);
    memcpy(&f2, &b2, 4);
    return (p * f1) * f2;
}

/* ---- dot products ------------------------------------------------------------
 * Integer parts follow ggml's vec_dot_q4_K_q8_K / vec_dot_q6_K_q8_K /
 * vec_dot_q8_0_q8_0 exactly (sub-block int8 x int8 sums, 6-bit or int8 scales,
 * Q8_K bsums for the Q4_K mins).  ggml leaves the fp32 accumulation order of
 * the block partials to each SIMD backend (generic, AVX2, NEON differ); this
 * restatement fixes the order the B200 kernels use:
 *   - a row of K columns is cut into 128-column units (half a 256-block; four
 *     Q8_0 blocks), each giving one fp32 partial;
 *   - units are taken 32 at a time (one group); the group's partials are summed
 *     by the 5-level butterfly p[l] + p[l^16], ^8, ^4, ^2, ^1 (missing units
 *     count as 0);
 *   - group sums are added in order to 0.
 * dot_*_blockorder keep ggml's generic per-block order for comparison. */
static float unit_q4_K(const blk_q4_K *x, const blk_q8_K *y, int u) {
    const int b = u >> 1, h = u & 1;
    int32_t isum = 0, imin = 0;
    for (int j = 4 * h; j < 4 * h + 4; ++j) {
        uint8_t sc, m;
        get_scale_min_k4(j, x[b].scales, &sc, &m);
        const uint8_t *q = x[b].qs + 32 * (j / 2);
        const int8_t *a = y[b].qs + 32 * j;
        int32_t sacc = 0;
        if ((j & 1) == 0) {
            for (int l = 0; l < 32; ++l) sacc += (int32_t)(q[l] & 0xF) * a[l];
        } else {
            for (int l = 0; l < 32; ++l) sacc += (int32_t)(q[l] >> 4) * a[l];
        }
        isum += (int32_t)sc * sacc;
        imin += (int32_t)m * (y[b].bsums[2 * j] + y[b].bsums[2 * j + 1]);
    }
    const float d = sfo_fp16_to_fp32(x[b].d) * y[b].d;
    const float dmin = sfo_fp16_to_fp32(x[b].dmin) * y[b].d;
    return d * (float)isum - dmin * (float)imin;
}

static float unit_q6_K(const blk_q6_K *x, const blk_q8_K *y, int u) {
    const int b = u >> 1, h = u & 1;
    const uint8_t *ql = x[b].ql + 64 * h, *qh = x[b].qh + 32 * h;
    const int8_t *a = y[b].qs + 128 * h;
    int32_t sacc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int l = 0; l < 32; ++l) {
        const int q1 = ((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
        const int q2 = ((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
        const int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
        const int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
        const int is = l / 16;
        sacc[is + 0] += q1 * a[l];
        sacc[is + 2] += q2 * a[l + 32];
        sacc[is + 4] += q3 * a[l + 64];
        sacc[is + 6] += q4 * a[l + 96];
    }
    int32_t isum = 0;
    for (int j = 0; j < 8; ++j) isum += (int32_t)x[b].scales[8 * h + j] * sacc[j];
    return (sfo_fp16_to_fp32(x[b].d) * y[b].d) * (float)isum;
}

static float unit_q8_0(const blk_q8_0 *x, const blk_q8_0 *y, int u) {
    float acc = 0.0f;
    for (int j = 0; j < 4; ++j) {
        const blk_q8_0 *xb = x + 4 * u + j, *yb = y + 4 * u + j;
        int32_t sacc = 0;
        for (int l = 0; l < QK8_0; ++l) sacc += (int32_t)xb->qs[l] * yb->qs[l];
        acc = acc + (float)sacc * (sfo_fp16_to_fp32(xb->d) * sfo_fp16_to_fp32(yb->d));
    }
    return acc;
}

static float butterfly32(float p[32]) {
    float q[32];
    for (int o = 16; o > 0; o >>= 1) {
        for (int l = 0; l < 32; ++l) q[l] = p[l] + p[l ^ o];
        memcpy(p, q, sizeof(q));
    }
    return p[0];
}

static float dot_row_units(int type, const void *w, const void *xq, int64_t K) {
    const int U = (int)(K / 128);
    float acc = 0.0f;
    for (int g = 0; g * 32 < U; ++g) {
        const int ng = U - 32 * g < 32 ? U - 32 * g : 32;
        float p[32];
        for (int l = 0; l < 32; ++l) p[l] = 0.0f;
        for (int l = 0; l < ng; ++l) {
            const int u = 32 * g + l;
            switch (type) {
            case SFO_Q4_K: p[l] = unit_q4_K((const blk_q4_K *)w, (const blk_q8_K *)xq, u); break;
            case SFO_Q6_K: p[l] = unit_q6_K((const blk_q6_K *)w, (const blk_q8_K *)xq, u); break;
            case SFO_Q8_0: p[l] = unit_q8_0((const blk_q8_0 *)w, (const blk_q8_0 *)xq, u); break;
            default: break;
            }
        }
        acc = acc + butterfly32(p);
    }
    return acc;
}

static float dot_q4_K_q8_K(int64_t n, const blk_q4_K *x, const blk_q8_K *y) {
    float sumf = 0.0f;
    for (int64_t i = 0; i < n / QK_K; ++i) {
        int32_t isum = 0, isum_m = 0;
        for (int j = 0; j < 8; ++j) {
            uint8_t sc, m;
            get_scale_min_k4(j, x[i].scales, &sc, &m);
            const uint8_t *q = x[i].qs + 32 * (j / 2);
            const int8_t *a = y[i].qs + 32 * j;
            int32_t s = 0;
            if ((j & 1) == 0) {
                for (int l = 0; l < 32; ++l) s += (int32_t)(q[l] & 0xF) * a[l];
            } else {
                for (int l = 0; l < 32; ++l) s += (int32_t)(q[l] >> 4) * a[l];
            }
            isum += (int32_t)sc * s;
            isum_m += (int32_t)m * (y[i].bsums[2 * j] + y[i].bsums[2 * j + 1]);
        }
        const float d = sfo_fp16_to_fp32(x[i].d) * y[i].d;
        const float dmin = sfo_fp16_to_fp32(x[i].dmin) * y[i].d;
        sumf += d * (float)isum - dmin * (float)isum_m;
    }
    return sumf;
}

static float dot_q6_K_q8_K(int64_t n, const blk_q6_K *x, const blk_q8_K *y) {
    float sumf = 0.0f;
    for (int64_t i = 0; i < n / QK_K; ++i) {
        int32_t isum = 0;
        const uint8_t *ql = x[i].ql, *qh = x[i].qh;
        for (int h = 0; h < 2; ++h) {
            int32_t s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            const int8_t *a = y[i].qs + 128 * h;
            for (int l = 0; l < 32; ++l) {
                const int q1 = ((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                const int q2 = ((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                const int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                const int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                const int is = l / 16;
                s[is + 0] += q1 * a[l];
                s[is + 2] += q2 * a[l + 32];
                s[is + 4] += q3 * a[l + 64];
                s[is + 6] += q4 * a[l + 96];
            }
            for (int j = 0; j < 8; ++j) isum += (int32_t)x[i].scales[8 * h + j] * s[j];
            ql += 64;
            qh += 32;
        }
        sumf += (sfo_fp16_to_fp32(x[i].d) * y[i].d) * (float)isum;
    }
    return sumf;
}

static float dot_q8_0_q8_0(int64_t n, const blk_q8_0 *x, const blk_q8_0 *y) {
    float sumf = 0.0f;
    for (int64_t i = 0; i < n / QK8_0; ++i) {
        int32_t s = 0;
        for (int j = 0; j < QK8_0; ++j) s += (int32_t)x[i].qs[j] * y[i].qs[j];
        sumf += (float)s * (sfo_fp16_to_fp32(x[i].d) * sfo_fp16_to_fp32(y[i].d));
    }
    return sumf;
}

/* ggml_vec_dot_f32, generic form: float products summed in double */
static float dot_f32(int64_t n, const float *x, const float *y) {
    double s = 0.0;
    for (int64_t i = 0; i < n; ++i) s += (double)(x[i] * y[i]);
    return (float)s;
}

int sfo_mul_mat(int type, const void *w, int64_t nrows, int64_t ncols, const float *x, float *y,
                int fp32_mode) {
    const size_t rb = sfo_row_bytes(type, ncols);
    if (rb == 0 || ncols % block_size(type)) return -1;
    if (type == SFO_F32) {
        #pragma omp parallel for num_threads(nthreads()) schedule(static)
        for (int64_t r = 0; r < nrows; ++r) y[r] = dot_f32(ncols, (const float *)w + r * ncols, x);
        return 0;
    }
    if (fp32_mode == 1) {
        #pragma omp parallel num_threads(nthreads())
        {
            float *row = (float *)malloc((size_t)ncols * sizeof(float));
            #pragma omp for schedule(static)
            for (int64_t r = 0; r < nrows; ++r) {
                sfo_dequantize(type, (const uint8_t *)w + (size_t)r * rb, row, ncols);
                y[r] = dot_f32(ncols, row, x);
            }
            free(row);
        }
        return 0;
    }
    void *xq;
    if (type == SFO_Q8_0) {
        xq = malloc(sfo_row_bytes(SFO_Q8_0, ncols));
        sfo_quantize_q8_0(x, xq, ncols);
    } else {
        xq = malloc(sfo_row_bytes(SFO_Q8_K, ncols));
        sfo_quantize_q8_K(x, xq, ncols);
    }
    const int blockorder = fp32_mode == 2;
    #pragma omp parallel for num_threads(nthreads()) schedule(static)
    for (int64_t r = 0; r < nrows; ++r) {
        const void *wr = (const uint8_t *)w + (size_t)r * rb;
        if (!blockorder) {
            y[r] = dot_row_units(type, wr, xq, ncols);
            continue;
        }
        switch (type) {
        case SFO_Q4_K: y[r] = dot_q4_K_q8_K(ncols, (const blk_q4_K *)wr, (const blk_q8_K *)xq); break;
        case SFO_Q6_K: y[r] = dot_q6_K_q8_K(ncols, (const blk_q6_K *)wr, (const blk_q8_K *)xq); break;
        case SFO_Q8_0: y[r] = dot_q8_0_q8_0(ncols, (const blk_q8_0 *)wr, (const blk_q8_0 *)xq); break;
        default: y[r] = 0.0f; break;
        }
    }
    free(xq);
    return 0;
}

/* ---- elementwise ops ------------------------------------------------------ */
/* ggml_rms_norm (ggml-cpu ops.cpp rms_norm_f32: squares summed in double,
 * scale = 1/sqrtf(mean + eps)) followed by ggml_mul with the norm weight:
 * engine.cpp:1878-1879. */
void sfo_rms_norm(const float *x, const float *w, int64_t n, float eps, float *y) {
    double sum = 0.0;
    for (int64_t i = 0; i < n; ++i) sum += (double)(x[i] * x[i]);
    const float mean = (float)(sum / (double)n);
    const float scale = 1.0f / sqrtf(mean + eps);
    for (int64_t i = 0; i < n; ++i) {
        const float t = x[i] * scale;
        y[i] = w ? t * w[i] : t;
    }
}

/* ggml_rope_ext mode NORMAL (0), n_dims = head_dim, freq_scale 1, ext_factor 0,
 * attn_factor 1 (engine.cpp:1892-1897).  ggml builds the angle cache
 * iteratively: theta_0 = pos, theta_{i+1} = theta_i * theta_scale with
 * theta_scale = powf(base, -2/n_dims); pairs (2i, 2i+1) rotate. */
void sfo_rope_normal(float *x, int n_head, int head_dim, int pos, float freq_base) {
    const float theta_scale = powf(freq_base, -2.0f / (float)head_dim);
    float *cs = (float *)malloc(sizeof(float) * (size_t)head_dim);
    float theta = (float)pos;
    for (int i0 = 0; i0 < head_dim; i0 += 2) {
        cs[i0 + 0] = cosf(theta);
        cs[i0 + 1] = sinf(theta);
        theta *= theta_scale;
    }
    for (int h = 0; h < n_head; ++h) {
        float *v = x + (size_t)h * head_dim;
        for (int i0 = 0; i0 < head_dim; i0 += 2) {
            const float c = cs[i0], s = cs[i0 + 1];
            const float x0 = v[i0], x1 = v[i0 + 1];
            v[i0 + 0] = x0 * c - x1 * s;
            v[i0 + 1] = x0 * s + x1 * c;
        }
    }
    free(cs);
}

/* ggml_soft_max_ext (ggml-cpu ops.cpp soft_max_f32): scale, max-subtract,
 * expf, sum in double, multiply by (float)(1/sum).  The all-zero kq_mask the
 * engine passes (engine.cpp:2806-2808) adds nothing. */
void sfo_soft_max(const float *x, float *y, int64_t n, float scale) {
    float max = -INFINITY;
    for (int64_t i = 0; i < n; ++i) {
        y[i] = x[i] * scale;
        if (y[i] > max) max = y[i];
    }
    double sum = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        const float e = sfo_expf(y[i] - max);
        y[i] = e;
        sum += (double)e;
    }
    sum = 1.0 / sum;
    for (int64_t i = 0; i < n; ++i) y[i] *= (float)sum;
}

/* ggml_argsort_top_k, descending; ties resolve to the lower index. */
void sfo_top_k_desc(const float *x, int64_t n, int k, int32_t *ids) {
    for (int j = 0; j < k; ++j) {
        int32_t best = -1;
        for (int64_t i = 0; i < n; ++i) {
            int taken = 0;
            for (int t = 0; t < j; ++t) taken |= (ids[t] == (int32_t)i);
            if (taken) continue;
            if (best < 0 || x[i] > x[best]) best = (int32_t)i;
        }
        ids[j] = best;
    }
}

int32_t sfo_argmax(const float *v, int n) {
    int32_t best = 0;
    float best_v = -INFINITY;
    for (int i = 0; i < n; ++i) {
        if (v[i] > best_v) { best_v = v[i]; best = i; }
    }
    return best;
}

/* Token sampling of the generate loop (the reference declares
 * sf_sampling_params, include/strataflow/strataflow.h:193-199, and never
 * reads them: src/api/strataflow_api.cpp:308-335 always takes the argmax).
 * Defined here and on the device (csrc/sfk_sample.cu) as: temperature <= 0
 * -> the argmax (first maximum); else p_i = exp((l_i - max) * (1 / T)),
 * keep the top_k largest p (ties: lower index first; top_k <= 0: all), then
 * the shortest prefix in (p desc, index asc) order whose mass reaches
 * top_p times the kept mass (top_p >= 1: all), and return the first kept
 * index, in index order, whose running mass exceeds u times the kept mass,
 * u = splitmix64(seed + (step + 1) * golden) / 2^64 (53 bits). */
static uint64_t sfo_splitmix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
static const float *g_sort_p;
static int sfo_cmp_p_desc(const void *a, const void *b) {
    const int32_t i = *(const int32_t *)a, j = *(const int32_t *)b;
    const float pi = g_sort_p[i], pj = g_sort_p[j];
    if (pi > pj) return -1;
    if (pi < pj) return 1;
    return i < j ? -1 : (i > j);
}
int32_t sfo_sample(const float *logits, int64_t V, float temperature, int32_t top_k, float top_p, uint64_t seed,
                   int32_t step) {
    if (!(temperature > 0.0f)) return sfo_argmax(logits, (int)V);
    float mx = -INFINITY;
    for (int64_t i = 0; i < V; ++i) mx = logits[i] > mx ? logits[i] : mx;
    const float invT = 1.0f / temperature;
    float *p = (float *)malloc(sizeof(float) * (size_t)V);
    int32_t *idx = (int32_t *)malloc(sizeof(int32_t) * (size_t)V);
    uint8_t *keep = (uint8_t *)calloc((size_t)V, 1);
    for (int64_t i = 0; i < V; ++i) {
        p[i] = sfo_expf((logits[i] - mx) * invT);
        idx[i] = (int32_t)i;
    }
    g_sort_p = p;
    qsort(idx, (size_t)V, sizeof(int32_t), sfo_cmp_p_desc);
    const int64_t nk = (top_k > 0 && top_k < V) ? top_k : V;
    double mk = 0.0;
    for (int64_t j = 0; j < nk; ++j) mk += (double)p[idx[j]];
    int64_t nkeep = nk;
    if (top_p < 1.0f) {
        const double target = (double)top_p * mk;
        double a = 0.0;
        for (int64_t j = 0; j < nk; ++j) {
            a += (double)p[idx[j]];
            if (a >= target) { nkeep = j + 1; break; }
        }
    }
    for (int64_t j = 0; j < nkeep; ++j) keep[idx[j]] = 1;
    const uint64_t z = sfo_splitmix64(seed + (uint64_t)(step + 1) * 0x9E3779B97F4A7C15ull);
    const double u = (double)(z >> 11) * (1.0 / 9007199254740992.0);
    double total = 0.0;
    for (int64_t i = 0; i < V; ++i) if (keep[i]) total += (double)p[i];
    const double target = u * total;
    double a = 0.0;
    int32_t pick = -1, last = -1;
    for (int64_t i = 0; i < V && pick < 0; ++i) {
        if (!keep[i]) continue;
        last = (int32_t)i;
        a += (double)p[i];
        if (a > target) pick = (int32_t)i;
    }
    free(p);
    free(idx);
    free(keep);
    return pick >= 0 ? pick : last;
}

/* Router: engine.cpp:1913-1924 (mul_mat gate_inp, soft_max, argsort_top_k,
 * get_rows, sum_rows (double accumulation, ggml_vec_sum_f32), clamp, div). */
void sfo_router(const float *w_r, int n_expert, int d, const float *x, int k,
                int32_t *ids, float *weights, float *probs_out) {
    float *logits = (float *)malloc(sizeof(float) * (size_t)n_expert);
    float *probs = (float *)malloc(sizeof(float) * (size_t)n_expert);
    for (int e = 0; e < n_expert; ++e) logits[e] = dot_f32(d, w_r + (size_t)e * d, x);
    sfo_soft_max(logits, probs, n_expert, 1.0f);
    sfo_top_k_desc(probs, n_expert, k, ids);
    double s = 0.0;
    for (int j = 0; j < k; ++j) {
        weights[j] = probs[ids[j]];
        s += (double)weights[j];
    }
    float wsum = (float)s;
    if (wsum < 6.103515625e-5f) wsum = 6.103515625e-5f;
    for (int j = 0; j < k; ++j) weights[j] = weights[j] / wsum;
    if (probs_out) memcpy(probs_out, probs, sizeof(float) * (size_t)n_expert);
    free(logits);
    free(probs);
}

static inline float silu_f32(float x) { return x / (1.0f + sfo_expf(-x)); }

static int moe_ffn_impl(int type_gu, int type_down, const void *gate, const void *up, const void *down,
                        int n_expert, int d, int F, int b, int k,
                        const float *x, const float *res, const int32_t *ids, const float *wts,
                        float *out, float *gu_out, int fp32_mode, int ep_size);

int sfo_moe_ffn(int type_gu, int type_down, const void *gate, const void *up, const void *down,
                int n_expert, int d, int F, int b, int k,
                const float *x, const float *res, const int32_t *ids, const float *wts,
                float *out, float *gu_out, int fp32_mode) {
    return moe_ffn_impl(type_gu, type_down, gate, up, down, n_expert, d, F, b, k, x, res, ids, wts, out, gu_out,
                        fp32_mode, 1);
}

static int moe_ffn_impl(int type_gu, int type_down, const void *gate, const void *up, const void *down,
                        int n_expert, int d, int F, int b, int k,
                        const float *x, const float *res, const int32_t *ids, const float *wts,
                        float *out, float *gu_out, int fp32_mode, int ep_size) {
    const size_t gu_rb = sfo_row_bytes(type_gu, d), dn_rb = sfo_row_bytes(type_down, F);
    float *g = (float *)malloc(sizeof(float) * (size_t)F);
    float *u = (float *)malloc(sizeof(float) * (size_t)F);
    float *yk = (float *)malloc(sizeof(float) * (size_t)d * (size_t)k);
    for (int t = 0; t < b; ++t) {
        for (int j = 0; j < k; ++j) {
            const int e = ids[t * k + j];
            if (e < 0 || e >= n_expert) { free(g); free(u); free(yk); return -1; }
            /* engine.cpp:1967-1969: up, gate, swiglu_split(gate, up) */
            sfo_mul_mat(type_gu, (const uint8_t *)up + (size_t)e * F * gu_rb, F, d, x + (size_t)t * d, u, fp32_mode);
            sfo_mul_mat(type_gu, (const uint8_t *)gate + (size_t)e * F * gu_rb, F, d, x + (size_t)t * d, g, fp32_mode);
            for (int f = 0; f < F; ++f) g[f] = silu_f32(g[f]) * u[f];
            if (gu_out) memcpy(gu_out + ((size_t)t * k + j) * F, g, sizeof(float) * (size_t)F);
            /* engine.cpp:1970: down over the activation, then :1973 weight */
            sfo_mul_mat(type_down, (const uint8_t *)down + (size_t)e * d * dn_rb, d, F, g, yk + (size_t)j * d, fp32_mode);
            const float wgt = wts[t * k + j];
            for (int i = 0; i < d; ++i) yk[(size_t)j * d + i] *= wgt;
        }
        /* engine.cpp:1974-1986: moe_out = e0 + e1 + ...; then + ffn_inp */
        float *o = out + (size_t)t * d;
        if (ep_size > 1) {
            /* expert parallelism: rank r sums its own experts' outputs in slot
             * order from 0 (rank 0 then adds the residual); the partials are
             * added in rank order */
            const int el = n_expert / ep_size;
            for (int i = 0; i < d; ++i) {
                float tot = 0.0f;
                for (int r = 0; r < ep_size; ++r) {
                    float a = 0.0f;
                    for (int j = 0; j < k; ++j)
                        if (ids[t * k + j] / el == r) a = a + yk[(size_t)j * d + i];
                    if (r == 0 && res) a = a + res[(size_t)t * d + i];
                    tot = r == 0 ? a : tot + a;
                }
                o[i] = tot;
            }
            continue;
        }
        for (int i = 0; i < d; ++i) {
            float acc = yk[i];
            for (int j = 1; j < k; ++j) acc = acc + yk[(size_t)j * d + i];
            o[i] = res ? acc + res[(size_t)t * d + i] : acc;
        }
    }
    free(g);
    free(u);
    free(yk);
    return 0;
}

/* engine.cpp:1751-1761: kq = K.q per head (f32 accumulation), soft_max_ext with
 * scale 1/sqrtf(head_dim), kqv = V^T.kq; q head h reads kv head
 * h / (n_head / n_head_kv) (ggml mul_mat broadcast). */
void sfo_attn_decode(const float *q, const float *k, const float *v, int n_kv,
                     int n_head, int n_head_kv, int head_dim, float *out) {
    const int gqa = n_head / n_head_kv;
    const float scale = 1.0f / sqrtf((float)head_dim);
    float *s = (float *)malloc(sizeof(float) * (size_t)n_kv);
    float *p = (float *)malloc(sizeof(float) * (size_t)n_kv);
    for (int h = 0; h < n_head; ++h) {
        const int hk = h / gqa;
        const float *qh = q + (size_t)h * head_dim;
        for (int t = 0; t < n_kv; ++t)
            s[t] = dot_f32(head_dim, k + ((size_t)t * n_head_kv + hk) * head_dim, qh);
        sfo_soft_max(s, p, n_kv, scale);
        for (int i = 0; i < head_dim; ++i) {
            double acc = 0.0;
            for (int t = 0; t < n_kv; ++t)
                acc += (double)(v[((size_t)t * n_head_kv + hk) * head_dim + i] * p[t]);
            out[(size_t)h * head_dim + i] = (float)acc;
        }
    }
    free(s);
    free(p);
}

/* ---- whole model ------------------------------------------------------------ */
typedef struct {
    int type;
    int64_t ne[3];
    size_t bytes;
    uint8_t *data;
} sfo_tensor;

struct sfo_model {
    sfo_hparams hp;
    sfo_tensor t[SFO_T_COUNT][/*layer*/ 1 + 128];
};

struct sfo_seq {
    const sfo_model *m;
    float *k_cache, *v_cache; /* [n_layer][n_ctx][Hkv][hd] */
    float *hidden;            /* [n_layer][d] per-layer outputs of the last forward */
    int32_t *ids;             /* [n_layer][k] */
    double t_layers, t_head;  /* accumulated wall seconds */
    float *dbg;               /* [n_layer][5][max(d, Hq*hd)] intermediates */
    size_t dbg_stride;
};

static double now_s(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

void sfo_seq_timing(const sfo_seq *s, double *layers_s, double *head_s) {
    if (layers_s) *layers_s = s->t_layers;
    if (head_s) *head_s = s->t_head;
}

static int tensor_layered(int tid) { return tid >= SFO_T_ATTN_NORM; }

/* attention head width: n_embd / n_head (engine.cpp:1161) unless the model
 * states its own (head_dim > 0, e.g. 64 heads x 128 over d = 7168) */
static int hp_head_dim(const sfo_hparams *hp) { return hp->head_dim > 0 ? hp->head_dim : hp->n_embd / hp->n_head; }

static void tensor_shape(const sfo_hparams *hp, int tid, int *type, int64_t ne[3]) {
    const int64_t d = hp->n_embd, hd = hp_head_dim(hp);
    ne[0] = ne[1] = ne[2] = 1;
    switch (tid) {
    case SFO_T_TOK_EMBD: *type = hp->type_embd; ne[0] = d; ne[1] = hp->n_vocab; break;
    case SFO_T_OUTPUT_NORM: *type = SFO_F32; ne[0] = d; break;
    case SFO_T_OUTPUT: *type = hp->type_output; ne[0] = d; ne[1] = hp->n_vocab; break;
    case SFO_T_ATTN_NORM: *type = SFO_F32; ne[0] = d; break;
    case SFO_T_ATTN_Q: *type = hp->type_attn; ne[0] = d; ne[1] = hp->n_head * hd; break;
    case SFO_T_ATTN_K: case SFO_T_ATTN_V: *type = hp->type_attn; ne[0] = d; ne[1] = hp->n_head_kv * hd; break;
    case SFO_T_ATTN_OUT: *type = hp->type_attn; ne[0] = hp->n_head * hd; ne[1] = d; break;
    case SFO_T_FFN_NORM: *type = SFO_F32; ne[0] = d; break;
    case SFO_T_FFN_GATE_INP: *type = SFO_F32; ne[0] = d; ne[1] = hp->n_expert; break;
    case SFO_T_FFN_GATE_EXPS: case SFO_T_FFN_UP_EXPS:
        *type = hp->type_ffn_gu; ne[0] = d; ne[1] = hp->n_ff; ne[2] = hp->n_expert; break;
    case SFO_T_FFN_DOWN_EXPS:
        *type = hp->type_ffn_down; ne[0] = hp->n_ff; ne[1] = d; ne[2] = hp->n_expert; break;
    default: *type = -1; break;
    }
}

sfo_model *sfo_model_create(const sfo_hparams *hp) {
    if (hp->n_layer > 128 || hp->n_layer <= 0 || hp->n_head <= 0 || hp->n_head_kv <= 0 ||
        hp->n_head % hp->n_head_kv || (hp->head_dim <= 0 && hp->n_embd % hp->n_head) ||
        hp->n_expert_used > hp->n_expert)
        return NULL;
    sfo_model *m = (sfo_model *)calloc(1, sizeof(sfo_model));
    m->hp = *hp;
    for (int tid = 0; tid < SFO_T_COUNT; ++tid) {
        const int nl = tensor_layered(tid) ? hp->n_layer : 1;
        for (int l = 0; l < nl; ++l) {
            sfo_tensor *t = &m->t[tid][l];
            tensor_shape(hp, tid, &t->type, t->ne);
            t->bytes = sfo_row_bytes(t->type, t->ne[0]) * (size_t)t->ne[1] * (size_t)t->ne[2];
            t->data = (uint8_t *)calloc(1, t->bytes);
            if (!t->data) { sfo_model_free(m); return NULL; }
        }
    }
    return m;
}

void sfo_set_fp32_mode(sfo_model *m, int mode) {
    if (m) m->hp.fp32_mode = mode;
}

void sfo_model_free(sfo_model *m) {
    if (!m) return;
    for (int tid = 0; tid < SFO_T_COUNT; ++tid)
        for (int l = 0; l < 129; ++l) free(m->t[tid][l].data);
    free(m);
}

size_t sfo_tensor_bytes(const sfo_model *m, int tid, int layer, int *type, int64_t ne[3]) {
    if (tid < 0 || tid >= SFO_T_COUNT) return 0;
    if (tensor_layered(tid) ? (layer < 0 || layer >= m->hp.n_layer) : layer != 0) return 0;
    const sfo_tensor *t = &m->t[tid][layer];
    if (type) *type = t->type;
    if (ne) { ne[0] = t->ne[0]; ne[1] = t->ne[1]; ne[2] = t->ne[2]; }
    return t->bytes;
}

void *sfo_tensor_data(sfo_model *m, int tid, int layer) {
    if (!sfo_tensor_bytes(m, tid, layer, NULL, NULL)) return NULL;
    return m->t[tid][layer].data;
}

int sfo_model_synth(sfo_model *m, uint64_t seed) {
    for (int tid = 0; tid < SFO_T_COUNT; ++tid) {
        const int nl = tensor_layered(tid) ? m->hp.n_layer : 1;
        for (int l = 0; l < nl; ++l) {
            sfo_tensor *t = &m->t[tid][l];
            const int64_t n = t->ne[0] * t->ne[1] * t->ne[2];
            if (tid == SFO_T_OUTPUT_NORM || tid == SFO_T_ATTN_NORM || tid == SFO_T_FFN_NORM) {
                for (int64_t i = 0; i < n; ++i) ((float *)t->data)[i] = 1.0f; /* reference fixtures: norms = 1 */
                continue;
            }
            const uint64_t ts = sfo_tensor_seed(seed, tid, l);
            /* generate and quantize row-chunk by row-chunk to bound memory */
            const int64_t ncols = t->ne[0], nrows = t->ne[1] * t->ne[2];
            const int64_t chunk = 4096;
            float *buf = (float *)malloc(sizeof(float) * (size_t)(chunk * ncols));
            for (int64_t r0 = 0; r0 < nrows; r0 += chunk) {
                const int64_t nr = nrows - r0 < chunk ? nrows - r0 : chunk;
                sfo_synth_f32(ts, r0 * ncols, nr * ncols, 0.02f, buf);
                sfo_quantize_weights(t->type, buf, t->data + (size_t)r0 * sfo_row_bytes(t->type, ncols), nr, ncols);
            }
            free(buf);
        }
    }
    return 0;
}

sfo_seq *sfo_seq_create(const sfo_model *m) {
    const sfo_hparams *hp = &m->hp;
    const size_t hd = (size_t)hp_head_dim(hp);
    const size_t kv = (size_t)hp->n_layer * hp->n_ctx * hp->n_head_kv * hd;
    sfo_seq *s = (sfo_seq *)calloc(1, sizeof(sfo_seq));
    s->m = m;
    s->k_cache = (float *)calloc(kv, sizeof(float));
    s->v_cache = (float *)calloc(kv, sizeof(float));
    s->hidden = (float *)calloc((size_t)hp->n_layer * hp->n_embd, sizeof(float));
    s->ids = (int32_t *)calloc((size_t)hp->n_layer * (hp->n_expert_used > 0 ? hp->n_expert_used : 1), sizeof(int32_t));
    s->dbg_stride = (size_t)(hp->n_embd > hp->n_head * (int)hd ? hp->n_embd : hp->n_head * (int)hd);
    s->dbg = (float *)calloc((size_t)hp->n_layer * 5 * s->dbg_stride, sizeof(float));
    if (!s->k_cache || !s->v_cache || !s->hidden || !s->ids || !s->dbg) { sfo_seq_free(s); return NULL; }
    return s;
}

void sfo_seq_free(sfo_seq *s) {
    if (!s) return;
    free(s->k_cache);
    free(s->v_cache);
    free(s->hidden);
    free(s->ids);
    free(s->dbg);
    free(s);
}

void sfo_seq_reset(sfo_seq *s) {
    const sfo_hparams *hp = &s->m->hp;
    const size_t hd = (size_t)hp_head_dim(hp);
    const size_t kv = (size_t)hp->n_layer * hp->n_ctx * hp->n_head_kv * hd;
    memset(s->k_cache, 0, kv * sizeof(float));
    memset(s->v_cache, 0, kv * sizeof(float));
}

/* Timing support: positions 0..n_pos-1 of every layer's K/V cache receive
 * seeded pseudo-random values in [-1, 1) (rounded through f16 in the f16-KV
 * mode), as if a prompt had been fed, so a decode step at position n_pos
 * attends over a full context without running the prompt. */
int sfo_seq_fill_kv(sfo_seq *s, int n_pos, uint64_t seed) {
    const sfo_hparams *hp = &s->m->hp;
    if (n_pos < 0 || n_pos > hp->n_ctx) return -1;
    const size_t hd = (size_t)hp_head_dim(hp);
    const size_t row = (size_t)hp->n_head_kv * hd, per_layer = (size_t)hp->n_ctx * row;
    for (int il = 0; il < hp->n_layer; ++il)
        for (size_t i = 0; i < (size_t)n_pos * row; ++i) {
            const uint64_t z = splitmix64(seed ^ (((uint64_t)il << 40) + i));
            const float a = (float)((double)(z >> 40) / (double)(1ull << 24) * 2.0 - 1.0);
            const float b = (float)((double)(z & 0xFFFFFFull) / (double)(1ull << 24) * 2.0 - 1.0);
            s->k_cache[(size_t)il * per_layer + i] = hp->kv_f16 ? sfo_fp16_to_fp32(sfo_fp32_to_fp16(a)) : a;
            s->v_cache[(size_t)il * per_layer + i] = hp->kv_f16 ? sfo_fp16_to_fp32(sfo_fp32_to_fp16(b)) : b;
        }
    return 0;
}

const float *sfo_seq_hidden(const sfo_seq *s, int il) { return s->hidden + (size_t)il * s->m->hp.n_embd; }
const int32_t *sfo_seq_ids(const sfo_seq *s, int il) { return s->ids + (size_t)il * s->m->hp.n_expert_used; }
const float *sfo_seq_debug(const sfo_seq *s, int il, int which) {
    if (il < 0 || il >= s->m->hp.n_layer || which < 0 || which > 4) return NULL;
    return s->dbg + ((size_t)il * 5 + (size_t)which) * s->dbg_stride;
}
static void dbg_put(sfo_seq *s, int il, int which, const float *v, int n) {
    memcpy(s->dbg + ((size_t)il * 5 + (size_t)which) * s->dbg_stride, v, sizeof(float) * (size_t)n);
}

static inline float kv_round(float v, int f16) { return f16 ? sfo_fp16_to_fp32(sfo_fp32_to_fp16(v)) : v; }

/* engine::Engine::forward, engine.cpp:2498-3025, one token at `pos`. */
int32_t sfo_forward(const sfo_model *m, sfo_seq *s, int32_t token, int32_t pos, float *logits) {
    const sfo_hparams *hp = &m->hp;
    const int d = hp->n_embd, Hq = hp->n_head, Hkv = hp->n_head_kv, hd = hp_head_dim(hp);
    const int k = hp->n_expert_used, E = hp->n_expert, F = hp->n_ff;
    if (token < 0 || token >= hp->n_vocab || pos < 0 || pos >= hp->n_ctx) return -1;
    const int fp32 = hp->fp32_mode;

    float *hidden = (float *)malloc(sizeof(float) * (size_t)d);
    float *cur = (float *)malloc(sizeof(float) * (size_t)d);
    float *ffn_inp = (float *)malloc(sizeof(float) * (size_t)d);
    float *q = (float *)malloc(sizeof(float) * (size_t)Hq * hd);
    float *kc = (float *)malloc(sizeof(float) * (size_t)Hkv * hd);
    float *vc = (float *)malloc(sizeof(float) * (size_t)Hkv * hd);
    float *att = (float *)malloc(sizeof(float) * (size_t)Hq * hd);
    float *tmp = (float *)malloc(sizeof(float) * (size_t)d);

    const double t0 = now_s();
    /* embedding: ggml_get_rows(token_embd) (engine.cpp:2708-2723) */
    {
        const sfo_tensor *te = &m->t[SFO_T_TOK_EMBD][0];
        const size_t rb = sfo_row_bytes(te->type, d);
        sfo_dequantize(te->type, te->data + (size_t)token * rb, hidden, d);
    }

    const size_t kv_layer = (size_t)hp->n_ctx * Hkv * hd;
    const double t1 = now_s();
    for (int il = 0; il < hp->n_layer; ++il) {
        /* --- router segment: engine.cpp:1854-1947 --- */
        sfo_rms_norm(hidden, (const float *)m->t[SFO_T_ATTN_NORM][il].data, d, hp->rms_eps, cur);
        const sfo_tensor *wq = &m->t[SFO_T_ATTN_Q][il], *wk = &m->t[SFO_T_ATTN_K][il];
        const sfo_tensor *wv = &m->t[SFO_T_ATTN_V][il], *wo = &m->t[SFO_T_ATTN_OUT][il];
        sfo_mul_mat(wq->type, wq->data, Hq * hd, d, cur, q, fp32);
        sfo_mul_mat(wk->type, wk->data, Hkv * hd, d, cur, kc, fp32);
        sfo_mul_mat(wv->type, wv->data, Hkv * hd, d, cur, vc, fp32);
        sfo_rope_normal(q, Hq, hd, pos, hp->freq_base);
        sfo_rope_normal(kc, Hkv, hd, pos, hp->freq_base);
        /* KV write at column pos (engine.cpp:1646-1656) */
        float *Kl = s->k_cache + (size_t)il * kv_layer, *Vl = s->v_cache + (size_t)il * kv_layer;
        for (int i = 0; i < Hkv * hd; ++i) {
            Kl[(size_t)pos * Hkv * hd + i] = kv_round(kc[i], hp->kv_f16);
            Vl[(size_t)pos * Hkv * hd + i] = kv_round(vc[i], hp->kv_f16);
        }
        dbg_put(s, il, 4, q, Hq * hd);
        sfo_attn_decode(q, Kl, Vl, pos + 1, Hq, Hkv, hd, att);
        dbg_put(s, il, 0, att, Hq * hd);
        if (hp->ep_size > 1 && hp->ep_head_par) {
            /* heads split over the ranks: rank r projects its heads' columns
             * (a matrix of its own), rank 0 adds the residual, the partials
             * are added in rank order */
            const int N = hp->ep_size, Kl = Hq * hd / N;
            const size_t rbf = sfo_row_bytes(wo->type, Hq * hd), rbl = sfo_row_bytes(wo->type, Kl);
            uint8_t *ws = (uint8_t *)malloc((size_t)d * rbl);
            for (int r = 0; r < N; ++r) {
                for (int row = 0; row < d; ++row)
                    memcpy(ws + (size_t)row * rbl, (const uint8_t *)wo->data + (size_t)row * rbf + (size_t)r * rbl, rbl);
                sfo_mul_mat(wo->type, ws, d, Kl, att + (size_t)r * Kl, tmp, fp32);
                for (int i = 0; i < d; ++i) ffn_inp[i] = r == 0 ? tmp[i] + hidden[i] : ffn_inp[i] + tmp[i];
            }
            free(ws);
        } else {
            sfo_mul_mat(wo->type, wo->data, d, Hq * hd, att, tmp, fp32);
            for (int i = 0; i < d; ++i) ffn_inp[i] = tmp[i] + hidden[i];
        }
        sfo_rms_norm(ffn_inp, (const float *)m->t[SFO_T_FFN_NORM][il].data, d, hp->rms_eps, cur);
        int32_t *ids = s->ids + (size_t)il * k;
        float wts[64];
        sfo_router((const float *)m->t[SFO_T_FFN_GATE_INP][il].data, E, d, cur, k, ids, wts, NULL);
        dbg_put(s, il, 1, ffn_inp, d);
        dbg_put(s, il, 2, cur, d);
        dbg_put(s, il, 3, wts, k);
        /* --- expert segment: engine.cpp:1956-1989 --- */
        const sfo_tensor *tg = &m->t[SFO_T_FFN_GATE_EXPS][il], *tu = &m->t[SFO_T_FFN_UP_EXPS][il];
        const sfo_tensor *tdn = &m->t[SFO_T_FFN_DOWN_EXPS][il];
        moe_ffn_impl(tg->type, tdn->type, tg->data, tu->data, tdn->data, E, d, F, 1, k, cur, ffn_inp, ids, wts,
                     hidden, NULL, fp32, hp->ep_size);
        memcpy(s->hidden + (size_t)il * d, hidden, sizeof(float) * (size_t)d);
    }

    const double t2 = now_s();
    /* final norm + lm_head: engine.cpp:2988-3006 */
    sfo_rms_norm(hidden, (const float *)m->t[SFO_T_OUTPUT_NORM][0].data, d, hp->rms_eps, cur);
    const sfo_tensor *to = &m->t[SFO_T_OUTPUT][0];
    sfo_mul_mat(to->type, to->data, hp->n_vocab, d, cur, logits, fp32);

    free(hidden); free(cur); free(ffn_inp); free(q); free(kc); free(vc); free(att); free(tmp);
    const int32_t am = sfo_argmax(logits, hp->n_vocab);
    const double t3 = now_s();
    s->t_layers += t2 - t1;
    s->t_head += (t1 - t0) + (t3 - t2);
    return am;
}

/*
 * qmm_oracle.c -- CPU restatement of the reference's GGUF quantized-matmul
 * path.  TEST INFRASTRUCTURE ONLY: the checker for the CUDA path and the CPU
 * baseline timed beside it.  The product never links or calls this file.
 *
 * Reference paths are relative to openIE-dev/rce/compute/crates/.
 * Build: see oracle/Makefile (-O2 -ffp-contract=off, no fast-math).  Each
 * binary32 operation below is one operation of the reference, in the same
 * order; gcc on x86-64 (SSE, no x87) then reproduces it bit for bit.
 */
#include "qmm_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#if defined(__FP_FAST_FMAF) && !defined(ORACLE_ALLOW_FMA)
#error "the oracle must be built without FMA contraction (-ffp-contract=off)"
#endif

/* binary16 -> binary32, exactly; restates half_free
 * (rce-vm-backend-cpu/src/ml/kquant.rs:416-422), which the reference uses as
 * its exact stand-in for half::f16::to_f32 (half 2.7.1). */
float oracle_f16_to_f32(uint16_t h) {
    uint32_t s = ((uint32_t)(h >> 15)) << 31;
    int e = (h >> 10) & 0x1f;
    uint32_t m = h & 0x3ff;
    float mag;
    if (e == 0) {
        float two_m24;
        uint32_t b = 0x33800000u; /* 2^-24 */
        memcpy(&two_m24, &b, 4);
        mag = (float)m * two_m24;
    } else if (e == 31) {
        uint32_t b = 0x7f800000u | (m << 13);
        memcpy(&mag, &b, 4);
    } else {
        uint32_t b = ((uint32_t)(e - 15 + 127) << 23) | (m << 13);
        memcpy(&mag, &b, 4);
    }
    uint32_t bits;
    memcpy(&bits, &mag, 4);
    bits |= s;
    float out;
    memcpy(&out, &bits, 4);
    return out;
}

static inline float rd_f16(const uint8_t *p) {
    return oracle_f16_to_f32((uint16_t)(p[0] | (p[1] << 8)));
}

/* round_to_f16 (rce-vm-backend-cpu/src/ml/nn.rs:521-533): x rounded once to
 * the nearest binary16 value, ties to even, returned as f32. */
float oracle_round_to_f16(float x) {
    if (x == 0.0f || !isfinite(x)) return x;
    uint32_t bits;
    float ax = fabsf(x);
    memcpy(&bits, &ax, 4);
    int e = (int)((bits >> 23) & 0xff) - 127;
    int qe = (e >= -14) ? e - 10 : -24;
    double q = ldexp(1.0, qe);
    double r = nearbyint((double)x / q) * q; /* default rounding mode: ties to even */
    if (fabs(r) >= 65520.0) return x > 0 ? INFINITY : -INFINITY;
    return (float)r;
}

/* The binary16 bit pattern of round_to_f16(x). */
uint16_t oracle_f32_to_f16_bits(float x) {
    float r = oracle_round_to_f16(x);
    uint32_t b;
    memcpy(&b, &r, 4);
    uint16_t s = (uint16_t)((b >> 16) & 0x8000);
    if (isnan(r)) return 0x7e00;
    if (isinf(r)) return s | 0x7c00;
    float a = fabsf(r);
    if (a == 0.0f) return s;
    int e;
    double f = frexp((double)a, &e); /* a = f * 2^e, f in [0.5,1) */
    int exp16 = e - 1 + 15;
    if (exp16 <= 0) { /* subnormal: a = m * 2^-24 */
        return s | (uint16_t)llrint(ldexp((double)a, 24));
    }
    uint16_t mant = (uint16_t)llrint((f * 2.0 - 1.0) * 1024.0);
    return s | (uint16_t)(exp16 << 10) | mant;
}

/* q4_k_get_scale_min (rce-op-qmm/src/lib.rs:720-728; duplicate at
 * rce-ingest-gguf/src/dequant.rs:593-604): the 6-bit scale and min of
 * sub-block j from the 12 packed scale bytes. */
void oracle_q4k_get_scale_min(const uint8_t *scales, int j, uint8_t *sc, uint8_t *m) {
    if (j < 4) {
        *sc = scales[j] & 63;
        *m = scales[j + 4] & 63;
    } else {
        *sc = (uint8_t)((scales[j + 4] & 0x0F) | ((scales[j - 4] >> 6) << 4));
        *m = (uint8_t)((scales[j + 4] >> 4) | ((scales[j] >> 6) << 4));
    }
}

/* tensor_byte_size (rce-ingest-gguf/src/dequant.rs:18-58), the formats on
 * this path plus F32/F16. */
size_t oracle_tensor_byte_size(int dtype, size_t n) {
    switch (dtype) {
    case ORACLE_GGUF_F32: return n * 4;
    case ORACLE_GGUF_F16: return n * 2;
    case ORACLE_GGUF_Q4_0: return (n + 31) / 32 * 18;
    case ORACLE_GGUF_Q8_0: return (n + 31) / 32 * 34;
    case ORACLE_GGUF_Q4_K: return (n + 255) / 256 * 144;
    case ORACLE_GGUF_Q5_K: return (n + 255) / 256 * 176;
    case ORACLE_GGUF_Q6_K: return (n + 255) / 256 * 210;
    default: return 0;
    }
}

/* ---- dequantize_to_f32 (rce-ingest-gguf/src/dequant.rs:115-134) -------- */

/* dequant_q4_0 (dequant.rs:360-383). */
static void dequant_q4_0(const uint8_t *data, size_t nbytes, size_t n, float *out) {
    size_t nb = (n + 31) / 32;
    memset(out, 0, nb * 32 * sizeof(float));
    for (size_t b = 0; b < nb; b++) {
        size_t s = b * 18;
        if (s + 18 > nbytes) break;
        float scale = rd_f16(data + s);
        for (int j = 0; j < 16; j++) {
            uint8_t byte = data[s + 2 + j];
            int8_t v0 = (int8_t)((byte & 0x0F) - 8);
            int8_t v1 = (int8_t)(((byte >> 4) & 0x0F) - 8);
            out[b * 32 + j] = (float)v0 * scale;
            out[b * 32 + j + 16] = (float)v1 * scale;
        }
    }
}

/* dequant_q8_0 (dequant.rs:438-456). */
static void dequant_q8_0(const uint8_t *data, size_t nbytes, size_t n, float *out) {
    size_t nb = (n + 31) / 32;
    memset(out, 0, nb * 32 * sizeof(float));
    for (size_t b = 0; b < nb; b++) {
        size_t s = b * 34;
        if (s + 34 > nbytes) break;
        float scale = rd_f16(data + s);
        for (int i = 0; i < 32; i++) out[b * 32 + i] = (float)(int8_t)data[s + 2 + i] * scale;
    }
}

/* dequant_q4_k (dequant.rs:546-591). */
static void dequant_q4_k(const uint8_t *data, size_t nbytes, size_t n, float *out) {
    size_t nb = (n + 255) / 256;
    memset(out, 0, nb * 256 * sizeof(float));
    for (size_t b = 0; b < nb; b++) {
        size_t s = b * 144;
        if (s + 144 > nbytes) break;
        float d = rd_f16(data + s);
        float dmin = rd_f16(data + s + 2);
        const uint8_t *scales = data + s + 4;
        const uint8_t *qs = data + s + 16;
        for (int j = 0; j < 4; j++) {
            uint8_t sc1, m1, sc2, m2;
            oracle_q4k_get_scale_min(scales, j * 2, &sc1, &m1);
            oracle_q4k_get_scale_min(scales, j * 2 + 1, &sc2, &m2);
            float d1 = d * (float)sc1, min1 = dmin * (float)m1;
            float d2 = d * (float)sc2, min2 = dmin * (float)m2;
            for (int l = 0; l < 32; l++) {
                uint8_t byte = qs[j * 32 + l];
                float t1 = d1 * (float)(byte & 0x0F);
                out[b * 256 + j * 64 + l] = t1 - min1;
                float t2 = d2 * (float)((byte >> 4) & 0x0F);
                out[b * 256 + j * 64 + 32 + l] = t2 - min2;
            }
        }
    }
}

/* dequant_q5_k (dequant.rs:606-656): Q4_K's groups of 64 with a fifth bit,
 * bit 2j (low nibbles) or 2j + 1 (high) of qh[l], worth 16. */
static void dequant_q5_k(const uint8_t *data, size_t nbytes, size_t n, float *out) {
    size_t nb = (n + 255) / 256;
    memset(out, 0, nb * 256 * sizeof(float));
    for (size_t b = 0; b < nb; b++) {
        size_t s = b * 176;
        if (s + 176 > nbytes) break;
        float d = rd_f16(data + s);
        float dmin = rd_f16(data + s + 2);
        const uint8_t *scales = data + s + 4, *qh = data + s + 16, *qs = data + s + 48;
        for (int j = 0; j < 4; j++) {
            uint8_t sc1, m1, sc2, m2;
            oracle_q4k_get_scale_min(scales, j * 2, &sc1, &m1);
            oracle_q4k_get_scale_min(scales, j * 2 + 1, &sc2, &m2);
            float d1 = d * (float)sc1, min1 = dmin * (float)m1;
            float d2 = d * (float)sc2, min2 = dmin * (float)m2;
            for (int l = 0; l < 32; l++) {
                uint8_t byte = qs[j * 32 + l];
                unsigned h1 = (qh[l] & (1u << (2 * j))) ? 16u : 0u;
                unsigned h2 = (qh[l] & (1u << (2 * j + 1))) ? 16u : 0u;
                float t1 = d1 * (float)((byte & 0x0F) + h1);
                out[b * 256 + j * 64 + l] = t1 - min1;
                float t2 = d2 * (float)(((byte >> 4) & 0x0F) + h2);
                out[b * 256 + j * 64 + 32 + l] = t2 - min2;
            }
        }
    }
}

/* The six-bit code of element 128 o + 32 q + l of a Q6_K block (ql, qh as
 * in the block), minus 32: ql[64 o + 32 (q & 1) + l] supplies the low four
 * bits (low nibble for q < 2, high nibble above), qh[32 o + l] bits 2q, 2q+1
 * the high two. */
static int q6k_code(const uint8_t *ql, const uint8_t *qh, int o, int q, int l) {
    const uint8_t b = ql[64 * o + 32 * (q & 1) + l];
    const int lo = q < 2 ? (b & 0x0F) : (b >> 4);
    const int hi = (qh[32 * o + l] >> (2 * q)) & 0x03;
    return (lo | (hi << 4)) - 32;
}

/* dequant_q6_k (dequant.rs:658-698): per half o and l = 0..31, the four
 * elements l, l+32, l+64, l+96 of the half, value = (d * sc) * q with the
 * scale of the element's 16 (is = l / 16, + 2 per quarter). */
static void dequant_q6_k(const uint8_t *data, size_t nbytes, size_t n, float *out) {
    size_t nb = (n + 255) / 256;
    memset(out, 0, nb * 256 * sizeof(float));
    for (size_t b = 0; b < nb; b++) {
        size_t s = b * 210;
        if (s + 210 > nbytes) break;
        const uint8_t *ql = data + s, *qh = data + s + 128;
        const int8_t *sc = (const int8_t *)(data + s + 192);
        float d = rd_f16(data + s + 208);
        for (int o = 0; o < 2; o++)
            for (int l = 0; l < 32; l++) {
                int is = l / 16;
                for (int q = 0; q < 4; q++) {
                    float t = d * (float)sc[8 * o + is + 2 * q];
                    out[b * 256 + 128 * o + 32 * q + l] = t * (float)q6k_code(ql, qh, o, q, l);
                }
            }
    }
}

int oracle_dequant(const uint8_t *bytes, size_t nbytes, int dtype, size_t n, float *out) {
    switch (dtype) {
    case ORACLE_GGUF_Q6_K: dequant_q6_k(bytes, nbytes, n, out); return 0;
    case ORACLE_GGUF_Q5_K: dequant_q5_k(bytes, nbytes, n, out); return 0;
    case ORACLE_GGUF_Q4_0: dequant_q4_0(bytes, nbytes, n, out); return 0;
    case ORACLE_GGUF_Q8_0: dequant_q8_0(bytes, nbytes, n, out); return 0;
    case ORACLE_GGUF_Q4_K: dequant_q4_k(bytes, nbytes, n, out); return 0;
    default: return -1;
    }
}

/* ---- row dot products ---------------------------------------------------- */

/* One row of mm_1d_q4_0 (rce-op-qmm/src/lib.rs:496-522): per block,
 * sub accumulates (lo-8)*a[q] then (hi-8)*a[q+16] for q = 0..15, and
 * sumf += scale * sub. */
static float dot_row_q4_0(const float *a, const uint8_t *row, size_t k) {
    float sumf = 0.0f;
    for (size_t ib = 0; ib < k / 32; ib++) {
        const uint8_t *s = row + ib * 18;
        float scale = rd_f16(s);
        const float *ab = a + ib * 32;
        float sub = 0.0f;
        for (int q = 0; q < 16; q++) {
            uint8_t byte = s[2 + q];
            int8_t v0 = (int8_t)((byte & 0x0F) - 8);
            int8_t v1 = (int8_t)(((byte >> 4) & 0x0F) - 8);
            float p0 = (float)v0 * ab[q];
            sub = sub + p0;
            float p1 = (float)v1 * ab[q + 16];
            sub = sub + p1;
        }
        float t = scale * sub;
        sumf = sumf + t;
    }
    return sumf;
}

/* One row of mm_1d_q8_0 (rce-op-qmm/src/lib.rs:648-670) == dot_row_q8_0
 * (:316-328). */
static float dot_row_q8_0(const float *a, const uint8_t *row, size_t k) {
    float sumf = 0.0f;
    for (size_t ib = 0; ib < k / 32; ib++) {
        const uint8_t *s = row + ib * 34;
        float scale = rd_f16(s);
        const float *ab = a + ib * 32;
        float sub = 0.0f;
        for (int q = 0; q < 32; q++) {
            float p = (float)(int8_t)s[2 + q] * ab[q];
            sub = sub + p;
        }
        float t = scale * sub;
        sumf = sumf + t;
    }
    return sumf;
}

/* One row of mm_1d_q4_k (rce-op-qmm/src/lib.rs:730-781) == dot_row_q4_k
 * (:355-385): per group g of 64, four running sums over l = 0..31, then
 * sumf += ((d1*va_lo - min1*a_lo) + d2*va_hi) - min2*a_hi. */
static float dot_row_q4_k(const float *a, const uint8_t *row, size_t k) {
    float sumf = 0.0f;
    for (size_t ib = 0; ib < k / 256; ib++) {
        const uint8_t *s = row + ib * 144;
        float d = rd_f16(s);
        float dmin = rd_f16(s + 2);
        const uint8_t *scales = s + 4;
        const uint8_t *qs = s + 16;
        for (int g = 0; g < 4; g++) {
            const float *ab = a + ib * 256 + g * 64;
            uint8_t sc1, m1, sc2, m2;
            oracle_q4k_get_scale_min(scales, g * 2, &sc1, &m1);
            oracle_q4k_get_scale_min(scales, g * 2 + 1, &sc2, &m2);
            float d1 = d * (float)sc1, min1 = dmin * (float)m1;
            float d2 = d * (float)sc2, min2 = dmin * (float)m2;
            float va_lo = 0.0f, a_lo = 0.0f, va_hi = 0.0f, a_hi = 0.0f;
            for (int l = 0; l < 32; l++) {
                uint8_t byte = qs[g * 32 + l];
                float v_lo = (float)(byte & 0x0F);
                float v_hi = (float)((byte >> 4) & 0x0F);
                float al = ab[l];
                float ah = ab[32 + l];
                float p;
                p = v_lo * al; va_lo = va_lo + p;
                a_lo = a_lo + al;
                p = v_hi * ah; va_hi = va_hi + p;
                a_hi = a_hi + ah;
            }
            float t1 = d1 * va_lo;
            float t2 = min1 * a_lo;
            float t = t1 - t2;
            float t3 = d2 * va_hi;
            t = t + t3;
            float t4 = min2 * a_hi;
            t = t - t4;
            sumf = sumf + t;
        }
    }
    return sumf;
}

/* One row of mm_1d_q5_k (rce-op-qmm/src/lib.rs:783-832) == dot_row_q5_k
 * (:387-422): dot_row_q4_k's order, the code (nibble | fifth bit << 4) from
 * bit 2g / 2g + 1 of qh[l]. */
static float dot_row_q5_k(const float *a, const uint8_t *row, size_t k) {
    float sumf = 0.0f;
    for (size_t ib = 0; ib < k / 256; ib++) {
        const uint8_t *s = row + ib * 176;
        float d = rd_f16(s);
        float dmin = rd_f16(s + 2);
        const uint8_t *scales = s + 4, *qh = s + 16, *qs = s + 48;
        for (int g = 0; g < 4; g++) {
            const float *ab = a + ib * 256 + g * 64;
            uint8_t sc1, m1, sc2, m2;
            oracle_q4k_get_scale_min(scales, g * 2, &sc1, &m1);
            oracle_q4k_get_scale_min(scales, g * 2 + 1, &sc2, &m2);
            float d1 = d * (float)sc1, min1 = dmin * (float)m1;
            float d2 = d * (float)sc2, min2 = dmin * (float)m2;
            float va_lo = 0.0f, a_lo = 0.0f, va_hi = 0.0f, a_hi = 0.0f;
            for (int l = 0; l < 32; l++) {
                uint8_t byte = qs[g * 32 + l];
                unsigned h1 = ((qh[l] >> (2 * g)) & 1u) << 4;
                unsigned h2 = ((qh[l] >> (2 * g + 1)) & 1u) << 4;
                float v_lo = (float)((byte & 0x0F) | h1);
                float v_hi = (float)(((byte >> 4) & 0x0F) | h2);
                float al = ab[l];
                float ah = ab[32 + l];
                float p;
                p = v_lo * al; va_lo = va_lo + p;
                a_lo = a_lo + al;
                p = v_hi * ah; va_hi = va_hi + p;
                a_hi = a_hi + ah;
            }
            float t1 = d1 * va_lo;
            float t2 = min1 * a_lo;
            float t = t1 - t2;
            float t3 = d2 * va_hi;
            t = t + t3;
            float t4 = min2 * a_hi;
            t = t - t4;
            sumf = sumf + t;
        }
    }
    return sumf;
}

/* One row of mm_1d_q6_k (rce-op-qmm/src/lib.rs:1667-1705) == dot_row_q6_k
 * (:426-450): per super-block, half o and l = 0..31, four terms in the
 * order q1..q4, each ((d * sc) * q) * a added to the single running sum. */
static float dot_row_q6_k(const float *a, const uint8_t *row, size_t k) {
    float sumf = 0.0f;
    for (size_t ib = 0; ib < k / 256; ib++) {
        const uint8_t *s = row + ib * 210;
        const uint8_t *ql = s, *qh = s + 128;
        const int8_t *sc = (const int8_t *)(s + 192);
        float d = rd_f16(s + 208);
        for (int o = 0; o < 2; o++) {
            const float *ab = a + ib * 256 + 128 * o;
            for (int l = 0; l < 32; l++) {
                int is = l / 16;
                for (int q = 0; q < 4; q++) {
                    float t = d * (float)sc[8 * o + is + 2 * q];
                    t = t * (float)q6k_code(ql, qh, o, q, l);
                    t = t * ab[32 * q + l];
                    sumf = sumf + t;
                }
            }
        }
    }
    return sumf;
}

typedef float (*dot_fn)(const float *, const uint8_t *, size_t);

static int row_kernel(int dtype, dot_fn *fn, size_t *bb, size_t *blk) {
    switch (dtype) {
    case ORACLE_GGUF_Q4_0: *fn = dot_row_q4_0; *bb = 18; *blk = 32; return 0;
    case ORACLE_GGUF_Q8_0: *fn = dot_row_q8_0; *bb = 34; *blk = 32; return 0;
    case ORACLE_GGUF_Q4_K: *fn = dot_row_q4_k; *bb = 144; *blk = 256; return 0;
    case ORACLE_GGUF_Q6_K: *fn = dot_row_q6_k; *bb = 210; *blk = 256; return 0;
    case ORACLE_GGUF_Q5_K: *fn = dot_row_q5_k; *bb = 176; *blk = 256; return 0;
    default: return -1;
    }
}

typedef struct {
    const float *a;
    const uint8_t *w;
    dot_fn fn;
    size_t row_bytes, k, r0, r1;
    float *out;
} rows_job;

static void *rows_worker(void *p) {
    rows_job *j = (rows_job *)p;
    for (size_t r = j->r0; r < j->r1; r++) j->out[r] = j->fn(j->a, j->w + r * j->row_bytes, j->k);
    return NULL;
}

/* mm_1d restricted to rows [row0,row1): rayon's par_iter over output rows
 * becomes nthreads contiguous row ranges; per-row arithmetic is unchanged, so
 * the split has no numeric effect.  out is indexed by absolute row. */
int oracle_mm_1d_rows(const float *a, const uint8_t *w, int dtype, size_t n_rows,
                      size_t n_cols, size_t row0, size_t row1, float *out, int nthreads) {
    dot_fn fn;
    size_t bb, blk;
    if (row_kernel(dtype, &fn, &bb, &blk) != 0) return -1;
    if (n_cols % blk != 0 || row1 > n_rows || row0 > row1) return -2;
    size_t row_bytes = n_cols / blk * bb;
    size_t nr = row1 - row0;
    if (nthreads <= 1 || nr < 2) {
        for (size_t r = row0; r < row1; r++) out[r] = fn(a, w + r * row_bytes, n_cols);
        return 0;
    }
    if ((size_t)nthreads > nr) nthreads = (int)nr;
    pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)nthreads);
    rows_job *jobs = (rows_job *)malloc(sizeof(rows_job) * (size_t)nthreads);
    for (int t = 0; t < nthreads; t++) {
        jobs[t].a = a; jobs[t].w = w; jobs[t].fn = fn; jobs[t].row_bytes = row_bytes;
        jobs[t].k = n_cols; jobs[t].out = out;
        jobs[t].r0 = row0 + nr * (size_t)t / (size_t)nthreads;
        jobs[t].r1 = row0 + nr * (size_t)(t + 1) / (size_t)nthreads;
        pthread_create(&th[t], NULL, rows_worker, &jobs[t]);
    }
    for (int t = 0; t < nthreads; t++) pthread_join(th[t], NULL);
    free(th);
    free(jobs);
    return 0;
}

/* mm_1d (rce-op-qmm/src/lib.rs:216-270) for Q4_0 / Q8_0 / Q4_K; other
 * dtypes are out of scope and report -1 (the reference panics, :268). */
int oracle_mm_1d(const float *a, const uint8_t *w, int dtype, size_t n_rows, size_t n_cols,
                 float *out, int nthreads) {
    return oracle_mm_1d_rows(a, w, dtype, n_rows, n_cols, 0, n_rows, out, nthreads);
}

/* mm_batched (rce-op-qmm/src/lib.rs:967-1023): for these dtypes it is
 * t_rows independent mm_1d calls (:1015-1021). */
int oracle_mm_batched(const float *a, size_t t_rows, const uint8_t *w, int dtype,
                      size_t n_rows, size_t n_cols, float *out, int nthreads) {
    for (size_t t = 0; t < t_rows; t++) {
        int rc = oracle_mm_1d(a + t * n_cols, w, dtype, n_rows, n_cols, out + t * n_rows, nthreads);
        if (rc) return rc;
    }
    return 0;
}

/* ---- MoE (rce-op-moe/src/lib.rs) ---------------------------------------- */

/* moe_router steps 2-4 (rce-op-moe/src/lib.rs:49-72): max-subtracted softmax
 * over all experts (exp = libm expf, as Rust's f32::exp), sort descending,
 * keep top_k, optionally renormalise.  The reference sorts with
 * sort_unstable_by, whose order among equal probabilities is unspecified;
 * here ties keep the lower expert index first. */
void oracle_moe_softmax_topk(const float *logits, int n_experts, int top_k, int normalize,
                             int32_t *idx_out, float *w_out) {
    float maxl = -INFINITY;
    for (int e = 0; e < n_experts; e++) maxl = fmaxf(maxl, logits[e]);
    float *probs = (float *)malloc(sizeof(float) * (size_t)n_experts);
    int *idx = (int *)malloc(sizeof(int) * (size_t)n_experts);
    for (int e = 0; e < n_experts; e++) probs[e] = expf(logits[e] - maxl);
    float sum = 0.0f;
    for (int e = 0; e < n_experts; e++) sum = sum + probs[e];
    if (sum > 0.0f)
        for (int e = 0; e < n_experts; e++) probs[e] = probs[e] / sum;
    for (int e = 0; e < n_experts; e++) idx[e] = e;
    /* insertion sort, descending by prob; stable (lower index first on ties) */
    for (int i = 1; i < n_experts; i++) {
        int v = idx[i];
        int j = i - 1;
        while (j >= 0 && probs[idx[j]] < probs[v]) { idx[j + 1] = idx[j]; j--; }
        idx[j + 1] = v;
    }
    float s = 0.0f;
    for (int i = 0; i < top_k; i++) { idx_out[i] = idx[i]; w_out[i] = probs[idx[i]]; }
    if (normalize) {
        for (int i = 0; i < top_k; i++) s = s + w_out[i];
        if (s > 0.0f)
            for (int i = 0; i < top_k; i++) w_out[i] = w_out[i] / s;
    }
    free(probs);
    free(idx);
}

/* moe_router (rce-op-moe/src/lib.rs:35-73): the logits come from mm_1d of
 * the gate weight, then softmax / top-k / renormalise. */
int oracle_moe_router(const float *x, const uint8_t *gate_w, int gate_dtype, int n_experts,
                      size_t d_model, int top_k, int normalize, int32_t *idx, float *weights) {
    float *logits = (float *)malloc(sizeof(float) * (size_t)n_experts);
    int rc = oracle_mm_1d(x, gate_w, gate_dtype, (size_t)n_experts, d_model, logits, 1);
    if (rc == 0) oracle_moe_softmax_topk(logits, n_experts, top_k, normalize, idx, weights);
    free(logits);
    return rc;
}

/* moe_combine (rce-op-moe/src/lib.rs:98-110): out = 0; for each selected
 * expert in route order, out[i] += w * exp[i]. */
void oracle_moe_combine(const float *weights, int k, const float *outs, size_t d_model, float *out) {
    for (size_t i = 0; i < d_model; i++) out[i] = 0.0f;
    for (int j = 0; j < k; j++)
        for (size_t i = 0; i < d_model; i++) {
            float p = weights[j] * outs[(size_t)j * d_model + i];
            out[i] = out[i] + p;
        }
}

/* silu (rce-qwen36-moe/src/lib.rs:459-461). */
float oracle_silu(float x) {
    if (x >= 0.0f) {
        float den = 1.0f + expf(-x);
        return x / den;
    }
    float e = expf(x);
    float num = x * e;
    float den = 1.0f + e;
    return num / den;
}

/* Expert-grouped SwiGLU FFN: per token, route on the given logits, run each
 * routed expert as swiglu_expert_serial (rce-qwen36-moe/src/lib.rs:666-676:
 * g = W_gate x, u = W_up x, g = silu(g) * u, y = W_down g) and combine in
 * route order (:700-703).  Expert matmuls use the mm_1d row arithmetic. */
int oracle_moe_ffn(const float *x, size_t t_rows, size_t d_model, size_t d_ff,
                   const float *router_logits, int n_experts, int top_k,
                   const uint8_t *gate, const uint8_t *up, const uint8_t *down,
                   size_t gate_stride, size_t up_stride, size_t down_stride, int dtype,
                   float *out, int nthreads) {
    float *g = (float *)malloc(sizeof(float) * d_ff);
    float *u = (float *)malloc(sizeof(float) * d_ff);
    float *y = (float *)malloc(sizeof(float) * d_model);
    int32_t *idx = (int32_t *)malloc(sizeof(int32_t) * (size_t)top_k);
    float *wt = (float *)malloc(sizeof(float) * (size_t)top_k);
    int rc = 0;
    for (size_t t = 0; t < t_rows && rc == 0; t++) {
        const float *xt = x + t * d_model;
        float *ot = out + t * d_model;
        oracle_moe_softmax_topk(router_logits + t * (size_t)n_experts, n_experts, top_k, 1, idx, wt);
        for (size_t i = 0; i < d_model; i++) ot[i] = 0.0f;
        for (int j = 0; j < top_k && rc == 0; j++) {
            size_t e = (size_t)idx[j];
            rc |= oracle_mm_1d(xt, gate + e * gate_stride, dtype, d_ff, d_model, g, nthreads);
            rc |= oracle_mm_1d(xt, up + e * up_stride, dtype, d_ff, d_model, u, nthreads);
            for (size_t i = 0; i < d_ff; i++) {
                float s = oracle_silu(g[i]);
                g[i] = s * u[i];
            }
            rc |= oracle_mm_1d(g, down + e * down_stride, dtype, d_model, d_ff, y, nthreads);
            for (size_t i = 0; i < d_model; i++) {
                float p = wt[j] * y[i];
                ot[i] = ot[i] + p;
            }
        }
    }
    free(g); free(u); free(y); free(idx); free(wt);
    return rc;
}

/* sigmoid (rce-qwen36-moe/src/lib.rs:465-467). */
float oracle_sigmoid(float x) {
    if (x >= 0.0f) {
        float den = 1.0f + expf(-x);
        return 1.0f / den;
    }
    float e = expf(x);
    float den = 1.0f + e;
    return e / den;
}

/* The always-on shared expert of moe_ffn_forward (rce-qwen36-moe/src/lib.rs:
 * 694-705), added into out [t_rows][d_model] (which holds the routed
 * experts' combine): sh = swiglu_expert_serial(x, gate, up, down) with the
 * shared weights ([n_ff, d_model], [n_ff, d_model], [d_model, n_ff]),
 * g = sum_i gate_inp[i] * x[i] left to right, out[i] += sigmoid(g) * sh[i]. */
int oracle_moe_shared_expert(const float *x, size_t t_rows, size_t d_model, size_t n_ff, const float *gate_inp,
                             const uint8_t *gate, const uint8_t *up, const uint8_t *down, int dtype, float *out,
                             int nthreads) {
    float *g = malloc(n_ff * sizeof(float)), *u = malloc(n_ff * sizeof(float));
    float *sh = malloc(d_model * sizeof(float));
    int rc = (g && u && sh) ? 0 : -1;
    for (size_t t = 0; t < t_rows && rc == 0; t++) {
        const float *xt = x + t * d_model;
        float *ot = out + t * d_model;
        rc |= oracle_mm_1d(xt, gate, dtype, n_ff, d_model, g, nthreads);
        rc |= oracle_mm_1d(xt, up, dtype, n_ff, d_model, u, nthreads);
        for (size_t i = 0; i < n_ff; i++) {
            float s = oracle_silu(g[i]);
            g[i] = s * u[i];
        }
        rc |= oracle_mm_1d(g, down, dtype, d_model, n_ff, sh, nthreads);
        float acc = 0.0f;
        for (size_t i = 0; i < d_model; i++) {
            float p = gate_inp[i] * xt[i];
            acc = acc + p;
        }
        const float alpha = oracle_sigmoid(acc);
        for (size_t i = 0; i < d_model; i++) {
            float p = alpha * sh[i];
            ot[i] = ot[i] + p;
        }
    }
    free(g); free(u); free(sh);
    return rc;
}

/* quantize_block (rce-vm-backend-cpu/src/ml/nn.rs:541-563): GGUF's reference
 * quantizer for one block of 32.  q4: d = max / -8, q = min(15, floor(x id +
 * 8.5)) - 8; otherwise d = amax / 127, q = round-half-away(x id).  The scale
 * returned is d rounded to binary16 (as f32). */
void oracle_quantize_block(const float *x, int q4, int32_t *q, float *d_out) {
    float amax = 0.0f, max = 0.0f;
    for (int i = 0; i < 32; i++) {
        if (amax < fabsf(x[i])) { amax = fabsf(x[i]); max = x[i]; }
    }
    float d = q4 ? max / -8.0f : amax / 127.0f;
    float id = (d != 0.0f) ? 1.0f / d : 0.0f;
    for (int i = 0; i < 32; i++) {
        float v = x[i] * id;
        if (q4) {
            float t = v + 8.5f;
            int32_t f = (int32_t)floorf(t);
            q[i] = (f < 15 ? f : 15) - 8;
        } else {
            q[i] = (int32_t)roundf(v); /* roundf: half away from zero, like f32::round */
        }
    }
    *d_out = oracle_round_to_f16(d);
}

/* matmul_q (rce-vm-backend-cpu/src/ml/nn.rs:477-517): the normative order of
 * matmul_q8_0 / matmul_q4_0 on unpacked q [n][k] and d [n][k/32]. */
void oracle_spec_matmul_q(const float *x, size_t m, const int32_t *q, const float *d,
                          size_t n, size_t k, int q4, float *out) {
    size_t nb = k / 32;
    int order[32];
    for (int t = 0; t < 16; t++) {
        order[2 * t] = q4 ? t : 2 * t;
        order[2 * t + 1] = q4 ? t + 16 : 2 * t + 1;
    }
    for (size_t i = 0; i < m; i++) {
        const float *xr = x + i * k;
        for (size_t j = 0; j < n; j++) {
            const int32_t *qr = q + j * k;
            float sum = 0.0f;
            for (size_t b = 0; b < nb; b++) {
                float sub = 0.0f;
                for (int t = 0; t < 32; t++) {
                    size_t at = b * 32 + (size_t)order[t];
                    float p = (float)qr[at] * xr[at];
                    sub = sub + p;
                }
                float p = d[j * nb + b] * sub;
                sum = sum + p;
            }
            out[i * n + j] = sum;
        }
    }
}

/* matmul_k for Q4_K (rce-vm-backend-cpu/src/ml/kquant.rs:81-150): q [n][k]
 * in 0..15, s and o [n][k/32] (s = d*sc, o = dmin*m); per pair of
 * sub-blocks y += ((s u - o a) + s' u') - o' a'. */
void oracle_spec_matmul_q4k(const float *x, size_t m, const int32_t *q, const float *s,
                            const float *o, size_t n, size_t k, float *out) {
    size_t ns = k / 32;
    for (size_t i = 0; i < m; i++) {
        const float *xr = x + i * k;
        for (size_t j = 0; j < n; j++) {
            const int32_t *qr = q + j * k;
            const float *sr = s + j * ns;
            const float *orr = o + j * ns;
            float y = 0.0f;
            for (size_t g = 0; g < k / 64; g++) {
                size_t b1 = 2 * g, b2 = 2 * g + 1;
                float u1 = 0.0f, a1 = 0.0f, u2 = 0.0f, a2 = 0.0f;
                for (int t = 0; t < 32; t++) {
                    size_t p1 = b1 * 32 + (size_t)t, p2 = b2 * 32 + (size_t)t;
                    float p;
                    p = (float)qr[p1] * xr[p1]; u1 = u1 + p;
                    a1 = a1 + xr[p1];
                    p = (float)qr[p2] * xr[p2]; u2 = u2 + p;
                    a2 = a2 + xr[p2];
                }
                float t1 = sr[b1] * u1;
                float t2 = orr[b1] * a1;
                float acc = t1 - t2;
                float t3 = sr[b2] * u2;
                acc = acc + t3;
                float t4 = orr[b2] * a2;
                acc = acc - t4;
                y = y + acc;
            }
            out[i * n + j] = y;
        }
    }
}

void oracle_test_activations(int kind, float c1, float c0, size_t n, float *out) {
    for (size_t i = 0; i < n; i++) {
        float v = (float)i * c1;
        v = v + c0;
        out[i] = kind == 0 ? sinf(v) : cosf(v);
    }
}

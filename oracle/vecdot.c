/* ggml's CPU matrix-vector product for the weights the reference leaves to
 * ggml_mul_mat -- TEST INFRASTRUCTURE ONLY.
 *
 * The reference multiplies by a weight that is not on its int8 path with
 * ggml_mul_mat (src/nexterabert.cpp:1140-1142): the tied MLM decoder over the
 * quantized embedding table (:1995-1998), the classifier (:1314-1316), and any
 * float matrix.  ggml's CPU backend first converts the activation row to the
 * weight type's "vec_dot type" and then takes one dot product per weight row:
 *
 *   weight type                 activation becomes        block dot
 *   F32                         F32                       sum w*x
 *   F16 / BF16                  F16 / BF16 (round even)   sum w*x in fp32
 *   Q4_0 Q5_0 Q8_0              Q8_0 (32 per block)       d_w*d_x * isum
 *   Q4_1 Q5_1                   Q8_1 (32 per block)       d_w*d_x * isum + m_w*s_x
 *   Q2_K Q3_K Q4_K Q5_K Q6_K    Q8_K (256 per block)      d_x*d_w*isum - d_x*dmin_w*msum
 *
 * isum = sum over sub-blocks of (integer sub-scale * integer dot of the codes);
 * msum = sum over sub-blocks of (integer sub-min * sum of the activation codes).
 * ggml v0.9.9 is not vendored with the reference, so this restates its published
 * algorithm (ggml-quants.c quantize_row_q8_K_ref; the x86 quantize_row_q8_0 /
 * q8_1, which scale by 127/amax and round to nearest even; the generic vec_dot_*).
 * The integer parts are exact; ggml's SIMD kernels add the per-block floats in
 * another order, so results agree with ggml to fp32 rounding, not bit for bit:
 * parity here is unpinned and tests use a tolerance.
 */
#include "oracle.h"

#include <math.h>
#include <string.h>

static inline float h2f(const uint8_t * p) {
    uint16_t h;
    memcpy(&h, p, 2);
    return or_fp16_to_fp32(h);
}

/* fp32 -> fp16, round to nearest even (F16C's rounding) */
uint16_t or_fp32_to_fp16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t) (sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    if (ax >= 0x477ff000u) return (uint16_t) (sign | 0x7c00u);          /* rounds past 65504 */
    if (ax < 0x38800000u) {                                              /* fp16 subnormal or zero */
        if (ax < 0x33000000u) return (uint16_t) sign;                    /* below half the least subnormal */
        const uint32_t e = ax >> 23, m = (ax & 0x7fffffu) | 0x800000u;
        const int shift = 126 - (int) e;                                 /* 14 .. 24 */
        uint32_t q = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        return (uint16_t) (sign | q);
    }
    uint32_t r = ax - 0x38000000u;                                       /* rebias 127 -> 15 */
    const uint32_t rem = r & 0x1fffu;
    r >>= 13;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) ++r;
    return (uint16_t) (sign | r);
}

static float round_f16(float f) { return or_fp16_to_fp32(or_fp32_to_fp16(f)); }

static float round_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) {
        u = (u | 0x00400000u) & 0xffff0000u;          /* quiet NaN */
    } else {
        u = (u + (0x7fffu + ((u >> 16) & 1u))) & 0xffff0000u;
    }
    memcpy(&f, &u, 4);
    return f;
}

/* ------------------------------------------------------------------------- */
/* weight blocks as integer codes                                            */
/* ------------------------------------------------------------------------- */

enum { FAM_F32, FAM_F16, FAM_BF16, FAM_Q8_0, FAM_Q8_1, FAM_Q8_K, FAM_NONE };

int or_vec_dot_family(int type) {
    switch (type) {
        case OR_F32: return FAM_F32;
        case OR_F16: return FAM_F16;
        case OR_BF16: return FAM_BF16;
        case OR_Q4_0: case OR_Q5_0: case OR_Q8_0: return FAM_Q8_0;
        case OR_Q4_1: case OR_Q5_1: return FAM_Q8_1;
        case OR_Q2_K: case OR_Q3_K: case OR_Q4_K: case OR_Q5_K: case OR_Q6_K: return FAM_Q8_K;
        default: return FAM_NONE;
    }
}

/* One weight block: n codes q[] (the integers the block dot multiplies), in
 * sub-blocks of `sub` with integer scale sc[] and min mn[]; d, dmin (or m). */
typedef struct {
    int n, sub;
    int q[256];
    int sc[16], mn[16];
    float d, dmin;
} wblock;

static void k_scale_min(const uint8_t * s, int j, int * sc, int * mn) {
    if (j < 4) {
        *sc = s[j] & 63;
        *mn = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
        *mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

static size_t decode_block(int type, const uint8_t * b, wblock * w) {
    memset(w->sc, 0, sizeof(w->sc));
    memset(w->mn, 0, sizeof(w->mn));
    w->dmin = 0.0f;
    switch (type) {
        case OR_Q4_0:
            w->n = w->sub = 32; w->sc[0] = 1; w->d = h2f(b);
            for (int j = 0; j < 16; ++j) { w->q[j] = (b[2 + j] & 15) - 8; w->q[j + 16] = (b[2 + j] >> 4) - 8; }
            return 18;
        case OR_Q4_1:
            w->n = w->sub = 32; w->sc[0] = 1; w->d = h2f(b); w->dmin = h2f(b + 2);
            for (int j = 0; j < 16; ++j) { w->q[j] = b[4 + j] & 15; w->q[j + 16] = b[4 + j] >> 4; }
            return 20;
        case OR_Q5_0: {
            w->n = w->sub = 32; w->sc[0] = 1; w->d = h2f(b);
            uint32_t qh; memcpy(&qh, b + 2, 4);
            for (int i = 0; i < 32; ++i) {
                const int lo = i < 16 ? (b[6 + i] & 15) : (b[6 + i - 16] >> 4);
                w->q[i] = (lo | (int) (((qh >> i) & 1u) << 4)) - 16;
            }
            return 22;
        }
        case OR_Q5_1: {
            w->n = w->sub = 32; w->sc[0] = 1; w->d = h2f(b); w->dmin = h2f(b + 2);
            uint32_t qh; memcpy(&qh, b + 4, 4);
            for (int i = 0; i < 32; ++i) {
                const int lo = i < 16 ? (b[8 + i] & 15) : (b[8 + i - 16] >> 4);
                w->q[i] = lo | (int) (((qh >> i) & 1u) << 4);
            }
            return 24;
        }
        case OR_Q8_0:
            w->n = w->sub = 32; w->sc[0] = 1; w->d = h2f(b);
            for (int i = 0; i < 32; ++i) w->q[i] = (int8_t) b[2 + i];
            return 34;
        case OR_Q2_K: {
            const uint8_t * sc = b, * qs = b + 16;
            w->n = 256; w->sub = 16; w->d = h2f(b + 80); w->dmin = h2f(b + 82);
            for (int j = 0; j < 16; ++j) { w->sc[j] = sc[j] & 15; w->mn[j] = sc[j] >> 4; }
            for (int i = 0; i < 256; ++i) {
                const int h = i / 128, s = (i / 32) % 4, e = i % 32;
                w->q[i] = (qs[32 * h + e] >> (2 * s)) & 3;
            }
            return 84;
        }
        case OR_Q3_K: {
            const uint8_t * hm = b, * qs = b + 32, * sc = b + 96;
            w->n = 256; w->sub = 16; w->d = h2f(b + 108);
            for (int j = 0; j < 16; ++j) {
                const int lo = (sc[j % 8] >> (4 * (j / 8))) & 15;
                const int hi = (sc[8 + j % 4] >> (2 * (j / 4))) & 3;
                w->sc[j] = (lo | (hi << 4)) - 32;
            }
            for (int i = 0; i < 256; ++i) {
                const int h = i / 128, s = (i / 32) % 4, e = i % 32;
                const int ql = (qs[32 * h + e] >> (2 * s)) & 3;
                const int hb = (hm[i % 32] >> (i / 32)) & 1;
                w->q[i] = ql - ((hb ^ 1) << 2);
            }
            return 110;
        }
        case OR_Q4_K: {
            const uint8_t * s = b + 4, * qs = b + 16;
            w->n = 256; w->sub = 32; w->d = h2f(b); w->dmin = h2f(b + 2);
            for (int j = 0; j < 8; ++j) {
                k_scale_min(s, j, &w->sc[j], &w->mn[j]);
                for (int e = 0; e < 32; ++e) w->q[32 * j + e] = (qs[32 * (j / 2) + e] >> (4 * (j % 2))) & 15;
            }
            return 144;
        }
        case OR_Q5_K: {
            const uint8_t * s = b + 4, * qh = b + 16, * qs = b + 48;
            w->n = 256; w->sub = 32; w->d = h2f(b); w->dmin = h2f(b + 2);
            for (int j = 0; j < 8; ++j) {
                k_scale_min(s, j, &w->sc[j], &w->mn[j]);
                for (int e = 0; e < 32; ++e) {
                    w->q[32 * j + e] = ((qs[32 * (j / 2) + e] >> (4 * (j % 2))) & 15) | (((qh[e] >> j) & 1) << 4);
                }
            }
            return 176;
        }
        case OR_Q6_K: {
            const uint8_t * ql = b, * qh = b + 128;
            const int8_t * sc = (const int8_t *) (b + 192);
            w->n = 256; w->sub = 16; w->d = h2f(b + 208);
            for (int j = 0; j < 16; ++j) w->sc[j] = sc[j];
            for (int p = 0; p < 256; ++p) {
                const int h = p / 128, r = p % 128;
                const int lo = (ql[64 * h + (r % 64)] >> (4 * (r / 64))) & 15;
                const int hi = (qh[32 * h + (r % 32)] >> (2 * (r / 32))) & 3;
                w->q[p] = (lo | (hi << 4)) - 32;
            }
            return 210;
        }
        default: return 0;
    }
}

/* ------------------------------------------------------------------------- */
/* the activation in the vec_dot type                                        */
/* ------------------------------------------------------------------------- */
/* Layout of a quantized activation row of K values (or_act_bytes):
 *   Q8_0 / Q8_1: int8 q[K], then per 32-block float d (fp16-rounded), float s (Q8_1 only)
 *   Q8_K:        int8 q[K], then per 256-block float d, then int32 bsum[K/16]
 *   F16 / BF16:  float x rounded to the type; F32: float x */

size_t or_act_bytes(int type, int64_t K) {
    switch (or_vec_dot_family(type)) {
        case FAM_F32: case FAM_F16: case FAM_BF16: return sizeof(float) * (size_t) K;
        case FAM_Q8_0: return (size_t) K + sizeof(float) * (size_t) (K / 32);
        case FAM_Q8_1: return (size_t) K + 2 * sizeof(float) * (size_t) (K / 32);
        case FAM_Q8_K: return (size_t) K + sizeof(float) * (size_t) (K / 256) + sizeof(int32_t) * (size_t) (K / 16);
        default: return 0;
    }
}

/* x * 127/amax rounded to nearest even; the fp16-rounded d = amax/127 */
static void quant_q8_0(const float * x, int64_t K, int8_t * q, float * d, float * s) {
    for (int64_t b = 0; b < K / 32; ++b) {
        const float * xb = x + 32 * b;
        float amax = 0.0f;
        for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(xb[i]));
        const float db = amax / 127.0f;
        const float id = amax != 0.0f ? 127.0f / amax : 0.0f;
        int sum = 0;
        for (int i = 0; i < 32; ++i) {
            const float v = xb[i] * id;
            const int qi = (int) nearbyintf(v);
            q[32 * b + i] = (int8_t) qi;
            sum += qi;
        }
        d[b] = round_f16(db);
        if (s) s[b] = round_f16(db * (float) sum);
    }
}

/* quantize_row_q8_K_ref: scale by -127/max of the largest-magnitude value */
static void quant_q8_k(const float * x, int64_t K, int8_t * q, float * d, int32_t * bsum) {
    for (int64_t b = 0; b < K / 256; ++b) {
        const float * xb = x + 256 * b;
        float amax = 0.0f, mx = 0.0f;
        for (int i = 0; i < 256; ++i) {
            const float ax = fabsf(xb[i]);
            if (ax > amax) { amax = ax; mx = xb[i]; }
        }
        if (amax == 0.0f) {
            d[b] = 0.0f;
            memset(q + 256 * b, 0, 256);
            for (int j = 0; j < 16; ++j) bsum[16 * b + j] = 0;
            continue;
        }
        const float iscale = -127.0f / mx;
        for (int i = 0; i < 256; ++i) {
            const int v = (int) nearbyintf(iscale * xb[i]);
            q[256 * b + i] = (int8_t) (v < 127 ? v : 127);
        }
        for (int j = 0; j < 16; ++j) {
            int s = 0;
            for (int i = 0; i < 16; ++i) s += q[256 * b + 16 * j + i];
            bsum[16 * b + j] = s;
        }
        d[b] = 1.0f / iscale;
    }
}

int or_quantize_act(int type, const float * x, int64_t K, void * out) {
    uint8_t * o = (uint8_t *) out;
    switch (or_vec_dot_family(type)) {
        case FAM_F32: memcpy(o, x, sizeof(float) * (size_t) K); return 0;
        case FAM_F16:
            for (int64_t i = 0; i < K; ++i) ((float *) o)[i] = round_f16(x[i]);
            return 0;
        case FAM_BF16:
            for (int64_t i = 0; i < K; ++i) ((float *) o)[i] = round_bf16(x[i]);
            return 0;
        case FAM_Q8_0:
            if (K % 32) return -1;
            quant_q8_0(x, K, (int8_t *) o, (float *) (o + K), NULL);
            return 0;
        case FAM_Q8_1:
            if (K % 32) return -1;
            quant_q8_0(x, K, (int8_t *) o, (float *) (o + K), (float *) (o + K) + K / 32);
            return 0;
        case FAM_Q8_K:
            if (K % 256) return -1;
            quant_q8_k(x, K, (int8_t *) o, (float *) (o + K), (int32_t *) (o + K + sizeof(float) * (size_t) (K / 256)));
            return 0;
        default: return -1;
    }
}

/* one weight row (GGUF bytes) times one activation row from or_quantize_act */
float or_vec_dot(int type, const void * wrow, const void * xact, int64_t K) {
    const uint8_t * w = (const uint8_t *) wrow, * xa = (const uint8_t *) xact;
    const int fam = or_vec_dot_family(type);
    float acc = 0.0f;
    if (fam == FAM_F32 || fam == FAM_F16 || fam == FAM_BF16) {
        const float * x = (const float *) xa;
        for (int64_t i = 0; i < K; ++i) {
            float wv;
            if (fam == FAM_F32) {
                memcpy(&wv, w + 4 * i, 4);
            } else if (fam == FAM_F16) {
                wv = h2f(w + 2 * i);
            } else {
                const uint32_t bits = (uint32_t) (w[2 * i] | (w[2 * i + 1] << 8)) << 16;
                memcpy(&wv, &bits, 4);
            }
            acc += wv * x[i];
        }
        return acc;
    }
    const int8_t * q = (const int8_t *) xa;
    wblock wb;
    if (fam == FAM_Q8_0 || fam == FAM_Q8_1) {
        const float * dx = (const float *) (xa + K), * sx = dx + K / 32;
        for (int64_t b = 0; b < K / 32; ++b) {
            w += decode_block(type, w, &wb);
            int isum = 0;
            for (int i = 0; i < 32; ++i) isum += wb.q[i] * q[32 * b + i];
            acc += (wb.d * dx[b]) * (float) isum;
            if (fam == FAM_Q8_1) acc += wb.dmin * sx[b];
        }
        return acc;
    }
    const float * dx = (const float *) (xa + K);
    const int32_t * bsum = (const int32_t *) (xa + K + sizeof(float) * (size_t) (K / 256));
    for (int64_t b = 0; b < K / 256; ++b) {
        w += decode_block(type, w, &wb);
        int isum = 0, msum = 0;
        for (int j = 0; j < 256 / wb.sub; ++j) {
            int s = 0, xs = 0;
            for (int i = 0; i < wb.sub; ++i) s += wb.q[wb.sub * j + i] * q[256 * b + wb.sub * j + i];
            for (int i = 0; i < wb.sub / 16; ++i) xs += bsum[16 * b + (wb.sub / 16) * j + i];
            isum += wb.sc[j] * s;
            msum += wb.mn[j] * xs;
        }
        acc += (dx[b] * wb.d) * (float) isum;
        acc -= (dx[b] * wb.dmin) * (float) msum;
    }
    return acc;
}

/* out[m][n] = W[n] . x[m] for M activation rows and N weight rows */
int or_mul_mat(int type, const void * w, int64_t N, int64_t K, const float * x, int64_t M, float * out) {
    const size_t ab = or_act_bytes(type, K);
    if (!ab) return -1;
    size_t rs;
    switch (type) {
        case OR_F32: rs = 4 * (size_t) K; break;
        case OR_F16: case OR_BF16: rs = 2 * (size_t) K; break;
        case OR_Q4_0: rs = 18 * (size_t) (K / 32); break;
        case OR_Q4_1: rs = 20 * (size_t) (K / 32); break;
        case OR_Q5_0: rs = 22 * (size_t) (K / 32); break;
        case OR_Q5_1: rs = 24 * (size_t) (K / 32); break;
        case OR_Q8_0: rs = 34 * (size_t) (K / 32); break;
        case OR_Q2_K: rs = 84 * (size_t) (K / 256); break;
        case OR_Q3_K: rs = 110 * (size_t) (K / 256); break;
        case OR_Q4_K: rs = 144 * (size_t) (K / 256); break;
        case OR_Q5_K: rs = 176 * (size_t) (K / 256); break;
        case OR_Q6_K: rs = 210 * (size_t) (K / 256); break;
        default: return -1;
    }
    uint8_t act[4 * 8192 + 8192];
    if (ab > sizeof(act)) return -1;
    for (int64_t m = 0; m < M; ++m) {
        if (or_quantize_act(type, x + m * K, K, act) != 0) return -1;
        for (int64_t n = 0; n < N; ++n) out[m * N + n] = or_vec_dot(type, (const uint8_t *) w + rs * (size_t) n, act, K);
    }
    return 0;
}

void or_gelu_erf(const float * x, int64_t n, float * out) {
    for (int64_t i = 0; i < n; ++i) {
        const float xi = x[i];
        out[i] = 0.5f * xi * (1.0f + erff(xi * 0.70710678118654752f));
    }
}

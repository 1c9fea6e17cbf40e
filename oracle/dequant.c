/* GGUF block dequantization for the CPU oracle (test infrastructure).
 *
 * The reference expands weights through ggml's `to_float` / `ggml_fp16_to_fp32_row`
 * (src/nexterabert.cpp:1026-1028) and dequantizes the embedding through ggml's
 * get_rows (:1272).  ggml v0.9.9 is not vendored with the reference, so its C
 * arithmetic cannot be read or run here.  This file restates the published
 * block layouts with the operation order of gguf-py 0.19.0
 * (gguf/quants.py, `dequantize_blocks` of each type): every product and
 * difference is a separate fp32 rounding, no fused multiply-add.  The tests pin
 * this file bit-exactly against gguf-py.
 */
#include "oracle.h"

#include <string.h>

float or_fp16_to_fp32(uint16_t h) {
    const uint32_t sign = (uint32_t) (h & 0x8000) << 16;
    uint32_t exp = (h >> 10) & 0x1f, man = h & 0x3ff, bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {                       /* subnormal: renormalise */
            exp = 127 - 15 + 1;
            while (!(man & 0x400)) { man <<= 1; --exp; }
            man &= 0x3ff;
            bits = sign | (exp << 23) | (man << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static inline float h2f(const uint8_t * p) {
    uint16_t h;
    memcpy(&h, p, 2);
    return or_fp16_to_fp32(h);
}

/* mul / sub / add helpers keep each step a separate rounding even if the
 * compiler is allowed to contract (the oracle is built with -ffp-contract=off) */
static inline float fmul(float a, float b) { volatile float r = a * b; return r; }

static void deq_q4_0(const uint8_t * b, float * y) {
    const float d = h2f(b);
    const uint8_t * qs = b + 2;
    for (int j = 0; j < 16; ++j) {
        y[j]      = fmul(d, (float) ((int) (qs[j] & 15) - 8));
        y[j + 16] = fmul(d, (float) ((int) (qs[j] >> 4) - 8));
    }
}

static void deq_q4_1(const uint8_t * b, float * y) {
    const float d = h2f(b), m = h2f(b + 2);
    const uint8_t * qs = b + 4;
    for (int j = 0; j < 16; ++j) {
        y[j]      = fmul(d, (float) (qs[j] & 15)) + m;
        y[j + 16] = fmul(d, (float) (qs[j] >> 4)) + m;
    }
}

static void deq_q5_0(const uint8_t * b, float * y) {
    const float d = h2f(b);
    uint32_t qh;
    memcpy(&qh, b + 2, 4);
    const uint8_t * qs = b + 6;
    for (int i = 0; i < 32; ++i) {
        const int lo = i < 16 ? (qs[i] & 15) : (qs[i - 16] >> 4);
        const int q  = lo | (int) (((qh >> i) & 1u) << 4);
        y[i] = fmul(d, (float) (q - 16));
    }
}

static void deq_q5_1(const uint8_t * b, float * y) {
    const float d = h2f(b), m = h2f(b + 2);
    uint32_t qh;
    memcpy(&qh, b + 4, 4);
    const uint8_t * qs = b + 8;
    for (int i = 0; i < 32; ++i) {
        const int lo = i < 16 ? (qs[i] & 15) : (qs[i - 16] >> 4);
        const int q  = lo | (int) (((qh >> i) & 1u) << 4);
        y[i] = fmul(d, (float) q) + m;
    }
}

static void deq_q8_0(const uint8_t * b, float * y) {
    const float d = h2f(b);
    const int8_t * qs = (const int8_t *) (b + 2);
    for (int i = 0; i < 32; ++i) y[i] = fmul((float) qs[i], d);
}

static void deq_q2_k(const uint8_t * b, float * y) {
    const uint8_t * sc = b, * qs = b + 16;
    const float d = h2f(b + 80), dmin = h2f(b + 82);
    for (int i = 0; i < 256; ++i) {
        const int h = i / 128, s = (i / 32) % 4, e = i % 32, sub = i / 16;
        const int q = (qs[32 * h + e] >> (2 * s)) & 3;
        const float dl = fmul(d, (float) (sc[sub] & 15));
        const float ml = fmul(dmin, (float) (sc[sub] >> 4));
        y[i] = fmul(dl, (float) q) - ml;
    }
}

static void deq_q3_k(const uint8_t * b, float * y) {
    const uint8_t * hm = b, * qs = b + 32, * sc = b + 96;
    const float d = h2f(b + 108);
    int scale[16];
    for (int i = 0; i < 16; ++i) {
        const int lo = (sc[i % 8] >> (4 * (i / 8))) & 15;
        const int hi = (sc[8 + i % 4] >> (2 * (i / 4))) & 3;
        scale[i] = (int) (int8_t) (uint8_t) (lo | (hi << 4)) - 32;
    }
    for (int i = 0; i < 256; ++i) {
        const int h = i / 128, s = (i / 32) % 4, e = i % 32;
        const int ql = (qs[32 * h + e] >> (2 * s)) & 3;
        const int hb = (hm[i % 32] >> (i / 32)) & 1;
        const int q  = ql - ((hb ^ 1) << 2);
        const float dl = fmul(d, (float) scale[i / 16]);
        y[i] = fmul(dl, (float) q);
    }
}

static void k_scale_min(const uint8_t * s, int j, int * sc, int * mn) {
    if (j < 4) {
        *sc = s[j] & 63;
        *mn = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
        *mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

static void deq_q4_k(const uint8_t * b, float * y) {
    const float d = h2f(b), dmin = h2f(b + 2);
    const uint8_t * s = b + 4, * qs = b + 16;
    for (int j = 0; j < 8; ++j) {
        int sc, mn;
        k_scale_min(s, j, &sc, &mn);
        const float d1 = fmul(d, (float) sc), m1 = fmul(dmin, (float) mn);
        const int i4 = j / 2, sh = 4 * (j % 2);
        for (int e = 0; e < 32; ++e) {
            const int q = (qs[32 * i4 + e] >> sh) & 15;
            y[32 * j + e] = fmul(d1, (float) q) - m1;
        }
    }
}

static void deq_q5_k(const uint8_t * b, float * y) {
    const float d = h2f(b), dmin = h2f(b + 2);
    const uint8_t * s = b + 4, * qh = b + 16, * qs = b + 48;
    for (int j = 0; j < 8; ++j) {
        int sc, mn;
        k_scale_min(s, j, &sc, &mn);
        const float d1 = fmul(d, (float) sc), m1 = fmul(dmin, (float) mn);
        const int i4 = j / 2, sh = 4 * (j % 2);
        for (int e = 0; e < 32; ++e) {
            const int q = ((qs[32 * i4 + e] >> sh) & 15) | (((qh[e] >> j) & 1) << 4);
            y[32 * j + e] = fmul(d1, (float) q) - m1;
        }
    }
}

static void deq_q6_k(const uint8_t * b, float * y) {
    const uint8_t * ql = b, * qh = b + 128;
    const int8_t * sc = (const int8_t *) (b + 192);
    const float d = h2f(b + 208);
    for (int p = 0; p < 256; ++p) {
        const int h = p / 128, r = p % 128;
        const int lo = (ql[64 * h + (r % 64)] >> (4 * (r / 64))) & 15;
        const int hi = (qh[32 * h + (r % 32)] >> (2 * (r / 32))) & 3;
        const int q  = (lo | (hi << 4)) - 32;
        const float d1 = fmul(d, (float) sc[p / 16]);
        y[p] = fmul(d1, (float) q);
    }
}

int or_dequant_row(int type, const void * src, float * y, int64_t n) {
    const uint8_t * b = (const uint8_t *) src;
    switch (type) {
        case OR_F32: memcpy(y, src, sizeof(float) * (size_t) n); return 0;
        case OR_F16:
            for (int64_t i = 0; i < n; ++i) y[i] = h2f(b + 2 * i);
            return 0;
        case OR_BF16:
            for (int64_t i = 0; i < n; ++i) {
                uint32_t bits = (uint32_t) (b[2 * i] | (b[2 * i + 1] << 8)) << 16;
                memcpy(&y[i], &bits, 4);
            }
            return 0;
        default: break;
    }
    int64_t bs;
    size_t ts;
    void (*fn)(const uint8_t *, float *);
    switch (type) {
        case OR_Q4_0: bs = 32;  ts = 18;  fn = deq_q4_0; break;
        case OR_Q4_1: bs = 32;  ts = 20;  fn = deq_q4_1; break;
        case OR_Q5_0: bs = 32;  ts = 22;  fn = deq_q5_0; break;
        case OR_Q5_1: bs = 32;  ts = 24;  fn = deq_q5_1; break;
        case OR_Q8_0: bs = 32;  ts = 34;  fn = deq_q8_0; break;
        case OR_Q2_K: bs = 256; ts = 84;  fn = deq_q2_k; break;
        case OR_Q3_K: bs = 256; ts = 110; fn = deq_q3_k; break;
        case OR_Q4_K: bs = 256; ts = 144; fn = deq_q4_k; break;
        case OR_Q5_K: bs = 256; ts = 176; fn = deq_q5_k; break;
        case OR_Q6_K: bs = 256; ts = 210; fn = deq_q6_k; break;
        default: return -1;
    }
    if (n % bs) return -1;
    for (int64_t i = 0; i < n / bs; ++i) fn(b + (size_t) i * ts, y + i * bs);
    return 0;
}

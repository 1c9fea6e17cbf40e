/* CPU oracle: scalar restatement of the reference's encoder arithmetic.
 * TEST INFRASTRUCTURE ONLY -- see oracle.h for what may use it and how it is pinned.
 *
 * Every function names the reference lines it follows (src/nexterabert.cpp of
 * Rikka-Botan/NexteraBERT.cpp).  The AVX2 code there keeps 8-lane (or 32-lane)
 * accumulators and reduces them with fixed horizontal-add trees; the scalar
 * loops below keep the same accumulators in arrays and reduce them in the same
 * order, so results are identical to the last bit.  Build with
 * -ffp-contract=off: a fused multiply-add appears only where the reference
 * writes one (fmaf), never by compiler contraction.
 */
#include "oracle.h"
#include "gguf_min.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

void or_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void) n;
#endif
}

static inline float vmin(float a, float b) { return a < b ? a : b; }   /* _mm256_min_ps(a, b) */
static inline float vmax(float a, float b) { return a > b ? a : b; }   /* _mm256_max_ps(a, b) */

/* ------------------------------------------------------------------------- */
/* SIMD helpers, one lane at a time (nexterabert.cpp:81-198)                  */
/* ------------------------------------------------------------------------- */

/* exp256 (:81-99): Cephes-style range reduction and polynomial */
float or_exp8(float x) {
    x = vmin(x, 88.3762626647949f);
    x = vmax(x, -87.3f);
    const float fx = rintf(x * 1.44269504088896341f);
    x = fmaf(-fx, 0.693359375f, x);
    x = fmaf(-fx, -2.12194440e-4f, x);
    const float z = x * x;
    float y = 1.9875691500e-4f;
    y = fmaf(y, x, 1.3981999507e-3f);
    y = fmaf(y, x, 8.3334519073e-3f);
    y = fmaf(y, x, 4.1665795894e-2f);
    y = fmaf(y, x, 1.6666665459e-1f);
    y = fmaf(y, x, 5.0000001201e-1f);
    y = fmaf(y, z, x + 1.0f);
    const uint32_t e = (uint32_t) ((int32_t) fx + 127) << 23;
    float p;
    memcpy(&p, &e, 4);
    return y * p;
}

/* tanh256 (:103-117) */
float or_tanh8(float x) {
    const float ax = fabsf(x);
    const float t = or_exp8(ax * -2.0f);
    float big = (1.0f - t) / (1.0f + t);
    if (signbit(x)) big = -big;                     /* or with the sign of x; big >= 0 */
    const float x2 = x * x;
    float p = -17.0f / 315.0f;
    p = fmaf(p, x2, 2.0f / 15.0f);
    p = fmaf(p, x2, -1.0f / 3.0f);
    p = fmaf(p, x2, 1.0f);
    const float small = p * x;
    return ax < 0.1f ? small : big;
}

/* sigmoid256 (:119-122) */
float or_sigmoid8(float x) {
    return 1.0f / (1.0f + or_exp8(0.0f - x));
}

/* hsum256 (:124-129) of 8 lanes */
static inline float hsum8(const float * v) {
    return ((v[0] + v[4]) + (v[2] + v[6])) + ((v[1] + v[5]) + (v[3] + v[7]));
}

/* dot_f32 (:133-151): four 8-lane accumulators over 32-wide steps, then 8-wide
 * steps into the first one, a horizontal sum, then a scalar tail */
float or_dot_f32(const float * a, const float * b, int n) {
    float acc[32] = {0};
    int i = 0;
    for (; i + 32 <= n; i += 32) {
        for (int L = 0; L < 32; ++L) acc[L] = fmaf(a[i + L], b[i + L], acc[L]);
    }
    for (; i + 8 <= n; i += 8) {
        for (int l = 0; l < 8; ++l) acc[l] = fmaf(a[i + l], b[i + l], acc[l]);
    }
    float v[8];
    for (int l = 0; l < 8; ++l) v[l] = (acc[l] + acc[8 + l]) + (acc[16 + l] + acc[24 + l]);
    float s = hsum8(v);
    for (; i < n; ++i) s += a[i] * b[i];
    return s;
}

/* axpy_f32 (:154-163): y += w * x */
static void axpy_f32(float * y, float w, const float * x, int n) {
    int i = 0;
    for (; i + 8 <= n; i += 8) {
        for (int l = 0; l < 8; ++l) y[i + l] = fmaf(w, x[i + l], y[i + l]);
    }
    for (; i < n; ++i) y[i] += w * x[i];
}

/* addmul_f32 (:166-175): y += a * b */
static void addmul_f32(float * y, const float * a, const float * b, int n) {
    int i = 0;
    for (; i + 8 <= n; i += 8) {
        for (int l = 0; l < 8; ++l) y[i + l] = fmaf(a[i + l], b[i + l], y[i + l]);
    }
    for (; i < n; ++i) y[i] += a[i] * b[i];
}

/* softmax_exp (:178-198): s[i] = exp(s[i] - max) in place, returns the sum */
static float softmax_exp(float * s, int n) {
    float m = s[0];
    for (int i = 1; i < n; ++i) m = (m < s[i]) ? s[i] : m;     /* std::max(m, s[i]) */
    int i = 0;
    float vs[8] = {0};
    for (; i + 8 <= n; i += 8) {
        for (int l = 0; l < 8; ++l) {
            const float e = or_exp8(s[i + l] - m);
            s[i + l] = e;
            vs[l] = vs[l] + e;
        }
    }
    float sum = hsum8(vs);
    for (; i < n; ++i) {
        s[i] = expf(s[i] - m);
        sum += s[i];
    }
    return sum;
}

/* ------------------------------------------------------------------------- */
/* int8 linear                                                               */
/* ------------------------------------------------------------------------- */

/* quantize_row (:378-403), one token: u8 = sat(rint(x * 127/amax) + 128); stored as u8 - 128 */
static void quantize_row(const float * xr, int8_t * q, float * sx, int n_in) {
    const int n_blk = (n_in + OR_I8_BLOCK - 1) / OR_I8_BLOCK;
    for (int B = 0; B < n_blk; ++B) {
        const int i0 = B * OR_I8_BLOCK, i1 = n_in < i0 + OR_I8_BLOCK ? n_in : i0 + OR_I8_BLOCK;
        float amax = 0.0f;
        for (int i = i0; i < i1; ++i) amax = vmax(amax, fabsf(xr[i]));
        sx[B] = amax / (float) OR_ACT_MAX;
        const float inv = amax > 0.0f ? (float) OR_ACT_MAX / amax : 0.0f;
        for (int i = i0; i < i1; ++i) {
            const float v = xr[i] * inv;
            int32_t c = (fabsf(v) < 2147483520.0f) ? (int32_t) rintf(v) : INT32_MIN;   /* cvtps_epi32 */
            int64_t u = (int64_t) c + 128;                                            /* + ACT_OFF */
            if (u < 0) u = 0;                                                         /* packs + packus */
            if (u > 255) u = 255;
            q[i] = (int8_t) (u - 128);
        }
    }
}

void or_quantize_rows(const float * x, int T, int n_in, int8_t * q, float * sx) {
    const int n_blk = (n_in + OR_I8_BLOCK - 1) / OR_I8_BLOCK;
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; ++t) {
        quantize_row(x + (size_t) t * n_in, q + (size_t) t * n_in, sx + (size_t) t * n_blk, n_in);
    }
}

/* build_i8_weight (:1010-1049) */
int or_build_i8_weight(int type, const void * data, int n_in, int n_out,
                       int8_t * w, float * scale, int32_t * off) {
    const int n_blk = (n_in + OR_I8_BLOCK - 1) / OR_I8_BLOCK;
    const size_t row_bytes = gm_row_size(type, n_in);
    if (!row_bytes) return -1;
    int bad = 0;
#pragma omp parallel
    {
        float * row = (float *) malloc(sizeof(float) * (size_t) n_in);
#pragma omp for schedule(static)
        for (int r = 0; r < n_out; ++r) {
            if (or_dequant_row(type, (const uint8_t *) data + (size_t) r * row_bytes, row, n_in) != 0) {
                bad = 1;
                continue;
            }
            int8_t * q = w + (size_t) r * n_in;
            for (int B = 0; B < n_blk; ++B) {
                const int i0 = B * OR_I8_BLOCK, i1 = n_in < i0 + OR_I8_BLOCK ? n_in : i0 + OR_I8_BLOCK;
                float amax = 0.0f;
                for (int i = i0; i < i1; ++i) amax = fmaxf(amax, fabsf(row[i]));
                const float inv = amax > 0.0f ? 127.0f / amax : 0.0f;
                int32_t sum = 0;
                for (int i = i0; i < i1; ++i) {
                    q[i] = (int8_t) lroundf(row[i] * inv);
                    sum += q[i];
                }
                scale[(size_t) B * n_out + r] = amax / 127.0f;
                off[(size_t) B * n_out + r]   = -128 * sum;
            }
        }
        free(row);
    }
    return bad ? -1 : 0;
}

/* op_linear_i8 / i8_kernel_3x4 / i8_kernel_4x1 (:881-1007):
 *   f = sum_B fma(float(S_B) * sx[t,B], sw[B,r], f)   with S_B = sum_i w8 * (u8 - 128)
 * in ascending B from f = 0; the residual is added last (res + f). */
void or_linear_i8(const int8_t * xq, const float * sx, int T, const int8_t * w, const float * sw,
                  int n_in, int n_out, const float * res, float * out, int32_t * block_sums) {
    const int n_blk = (n_in + OR_I8_BLOCK - 1) / OR_I8_BLOCK;
#pragma omp parallel for schedule(dynamic, 4)
    for (int t = 0; t < T; ++t) {
        const int8_t * xr = xq + (size_t) t * n_in;
        for (int r = 0; r < n_out; ++r) {
            const int8_t * wr = w + (size_t) r * n_in;
            float f = 0.0f;
            for (int B = 0; B < n_blk; ++B) {
                const int i0 = B * OR_I8_BLOCK, i1 = n_in < i0 + OR_I8_BLOCK ? n_in : i0 + OR_I8_BLOCK;
                int32_t s = 0;
                for (int i = i0; i < i1; ++i) s += (int32_t) wr[i] * (int32_t) xr[i];
                if (block_sums) block_sums[((size_t) t * n_out + r) * n_blk + B] = s;
                f = fmaf((float) s * sx[(size_t) t * n_blk + B], sw[(size_t) B * n_out + r], f);
            }
            out[(size_t) t * n_out + r] = res ? res[(size_t) t * n_out + r] + f : f;
        }
    }
}

/* ------------------------------------------------------------------------- */
/* row ops                                                                   */
/* ------------------------------------------------------------------------- */

/* op_rms_norm (:464-482) */
void or_rms_norm(const float * x, const float * gain, float eps, int T, int C, float * out) {
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; ++t) {
        const float * xr = x + (size_t) t * C;
        float * o = out + (size_t) t * C;
        const float inv = 1.0f / sqrtf(or_dot_f32(xr, xr, C) / (float) C + eps);
        for (int i = 0; i < C; ++i) o[i] = (xr[i] * inv) * gain[i];
    }
}

/* op_relu_sqr (:485-505) */
void or_relu_sqr(const float * x, int T, int C, float * out) {
    const size_t n = (size_t) T * C;
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; ++i) {
        const float r = x[i] > 0.0f ? x[i] : 0.0f;
        out[i] = r * r;
    }
}

/* op_gate (:508-523): sigmoid(g) * y; the scalar tail uses y / (1 + exp(-g)) */
void or_gate(const float * g, const float * y, int T, int C, float * out) {
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; ++t) {
        const float * gr = g + (size_t) t * C, * yr = y + (size_t) t * C;
        float * o = out + (size_t) t * C;
        int i = 0;
        for (; i + 8 <= C; i += 8) {
            for (int l = 0; l < 8; ++l) o[i + l] = or_sigmoid8(gr[i + l]) * yr[i + l];
        }
        for (; i < C; ++i) o[i] = yr[i] / (1.0f + expf(-gr[i]));
    }
}

/* op_dwconv (:528-544) */
void or_dwconv(const float * x, const float * r, const float * taps, int k,
               const int32_t * row_doc, const int32_t * doc_start, const int32_t * doc_len,
               int T, int C, float * out) {
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; ++t) {
        const int d = row_doc[t], lo = doc_start[d], hi = lo + doc_len[d];
        float * o = out + (size_t) t * C;
        if (r) memcpy(o, r + (size_t) t * C, sizeof(float) * (size_t) C);
        else   memset(o, 0, sizeof(float) * (size_t) C);
        for (int j = 0; j < k; ++j) {
            const int tt = t + j - k / 2;
            if (tt < lo || tt >= hi) continue;
            addmul_f32(o, taps + (size_t) j * C, x + (size_t) tt * C, C);
        }
    }
}

/* op_lily_state (:548-579) */
void or_lily_state(const float * a, const float * x, const float * b, const float * taps, int k,
                   const int32_t * row_doc, const int32_t * doc_start, const int32_t * doc_len,
                   int T, int C, float * out) {
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; ++t) {
        const int d = row_doc[t], lo = doc_start[d], hi = lo + doc_len[d];
        int j0 = lo - (t - k / 2), j1 = hi - (t - k / 2);
        if (j0 < 0) j0 = 0;
        if (j1 > k) j1 = k;
        const float * br = b + (size_t) t * C;
        float * o = out + (size_t) t * C;
        int i = 0;
        for (; i + 8 <= C; i += 8) {
            for (int l = 0; l < 8; ++l) {
                float acc = 0.0f;
                for (int j = j0; j < j1; ++j) {
                    const size_t tt = (size_t) (t + j - k / 2);
                    acc = fmaf(taps[(size_t) j * C + i + l], a[tt * C + i + l] * x[tt * C + i + l], acc);
                }
                o[i + l] = acc * br[i + l];
            }
        }
        for (; i < C; ++i) {
            float acc = 0.0f;
            for (int j = j0; j < j1; ++j) {
                const size_t tt = (size_t) (t + j - k / 2);
                acc += taps[(size_t) j * C + i] * a[tt * C + i] * x[tt * C + i];
            }
            o[i] = acc * br[i];
        }
    }
}

/* op_qk_prep (:590-625): DyT beta*tanh(alpha*x) per head channel, then RoPE at
 * the document-relative position: y1 = a*cos + b*sin, y2 = b*cos - a*sin */
void or_qk_prep(const float * x, const float * alpha, const float * beta,
                const float * cos_t, const float * sin_t,
                const int32_t * row_doc, const int32_t * doc_start,
                int T, int H, int D, int head_major, float * out) {
    const int half = D / 2;
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; ++t) {
        const int pos = t - doc_start[row_doc[t]];
        const float * c = cos_t + (size_t) pos * half, * s = sin_t + (size_t) pos * half;
        const float * xr = x + (size_t) t * H * D;
        for (int h = 0; h < H; ++h) {
            const float * x1 = xr + (size_t) h * D, * x2 = x1 + half;
            float * y1 = head_major ? out + ((size_t) h * T + t) * D : out + (size_t) t * H * D + (size_t) h * D;
            float * y2 = y1 + half;
            int i = 0;
            for (; i + 8 <= half; i += 8) {
                for (int l = 0; l < 8; ++l) {
                    const int j = i + l;
                    const float a = beta[j] * or_tanh8(alpha[j] * x1[j]);
                    const float b = beta[half + j] * or_tanh8(alpha[half + j] * x2[j]);
                    y1[j] = fmaf(a, c[j], b * s[j]);
                    y2[j] = fmaf(-a, s[j], b * c[j]);
                }
            }
            for (; i < half; ++i) {
                const float a = beta[i] * tanhf(alpha[i] * x1[i]);
                const float b = beta[half + i] * tanhf(alpha[half + i] * x2[i]);
                y1[i] = a * c[i] + b * s[i];
                y2[i] = b * c[i] - a * s[i];
            }
        }
    }
}

/* op_head_major (:628-639): [T][H][D] -> [H][T][D] */
void or_head_major(const float * x, int T, int H, int D, float * out) {
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; ++t) {
        for (int h = 0; h < H; ++h) {
            memcpy(out + ((size_t) h * T + t) * D, x + (size_t) t * H * D + (size_t) h * D, sizeof(float) * (size_t) D);
        }
    }
}

/* op_block_mean (:642-660): mean over each block's real tokens of h (* g) */
void or_block_mean(const float * h, const float * g, int C, int block,
                   const int32_t * doc_start, const int32_t * doc_len,
                   const int32_t * bdoc_start, const int32_t * brow_doc, int n_brows, float * out) {
#pragma omp parallel for schedule(static)
    for (int b = 0; b < n_brows; ++b) {
        const int d = brow_doc[b], bi = b - bdoc_start[d];
        const int ts = doc_start[d] + bi * block;
        int n = doc_len[d] - bi * block;
        if (n > block) n = block;
        float * o = out + (size_t) b * C;
        memset(o, 0, sizeof(float) * (size_t) C);
        for (int i = 0; i < n; ++i) {
            if (g) addmul_f32(o, h + (size_t) (ts + i) * C, g + (size_t) (ts + i) * C, C);
            else   axpy_f32(o, 1.0f, h + (size_t) (ts + i) * C, C);
        }
        const float inv = 1.0f / (float) n;
        for (int c = 0; c < C; ++c) o[c] *= inv;
    }
}

/* op_upsample_add (:679-690) */
void or_upsample_add(const float * y, const float * r, int C, int block, int T,
                     const int32_t * row_doc, const int32_t * doc_start, const int32_t * bdoc_start,
                     float * out) {
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; ++t) {
        const int d = row_doc[t];
        const float * yb = y + (size_t) (bdoc_start[d] + (t - doc_start[d]) / block) * C;
        const float * rr = r + (size_t) t * C;
        float * o = out + (size_t) t * C;
        for (int c = 0; c < C; ++c) o[c] = yb[c] + rr[c];
    }
}

/* ------------------------------------------------------------------------- */
/* attention (:698-852)                                                      */
/* ------------------------------------------------------------------------- */

/* NEXTERA_DOT64 (:710-714): lane l accumulates q[8r+l]*k[8r+l], r = 0..7 */
static inline void dot64_lanes(const float * q, const float * k, float * a) {
    for (int l = 0; l < 8; ++l) {
        float s = q[l] * k[l];
        for (int r = 1; r < 8; ++r) s = fmaf(q[8 * r + l], k[8 * r + l], s);
        a[l] = s;
    }
}

/* scores_d64 (:704-730): groups of 8 keys reduce ((a0+a1)+(a2+a3))+((a4+a5)+(a6+a7));
 * keys past the last whole group use hsum256 */
static void scores_d64(const float * q, const float * k, size_t stride, int j0, int j1, float scale, float * sc) {
    float a[8];
    int j = j0;
    for (; j + 8 <= j1; j += 8) {
        for (int kk = 0; kk < 8; ++kk) {
            dot64_lanes(q, k + (size_t) (j + kk) * stride, a);
            const float t = ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
            sc[j + kk] = t * scale;
        }
    }
    for (; j < j1; ++j) {
        dot64_lanes(q, k + (size_t) j * stride, a);
        sc[j] = scale * hsum8(a);
    }
}

/* values_d64 (:733-754): acc += sum_j (w[j] * inv) * v[j], keys in order */
static void values_d64(const float * w, float inv, const float * v, size_t stride, int j0, int j1, float * acc) {
    for (int j = j0; j < j1; ++j) {
        const float * vp = v + (size_t) j * stride;
        const float c = w[j] * inv;
        for (int d = 0; d < 64; ++d) acc[d] = fmaf(c, vp[d], acc[d]);
    }
}

/* attend (:759-774) */
static void attend(const float * q, const float * k, const float * v, size_t stride, int n, int D,
                   float scale, float * sc, float * out) {
    if (D == 64) {
        scores_d64(q, k, stride, 0, n, scale, sc);
        const float inv = 1.0f / softmax_exp(sc, n);
        memset(out, 0, sizeof(float) * 64);
        values_d64(sc, inv, v, stride, 0, n, out);
        return;
    }
    for (int j = 0; j < n; ++j) sc[j] = scale * or_dot_f32(q, k + (size_t) j * stride, D);
    const float inv = 1.0f / softmax_exp(sc, n);
    memset(out, 0, sizeof(float) * (size_t) D);
    for (int j = 0; j < n; ++j) axpy_f32(out, sc[j] * inv, v + (size_t) j * stride, D);
}

/* op_attention (:785-852).  Its blocked branch for documents of >= 2048 keys
 * groups keys exactly as the unblocked one (key blocks start at multiples of
 * 1024, :701-703) and sums values in the same key order, so it is bit-identical
 * to this single path. */
void or_attention(const float * q, const float * k, const float * v, int T, int H, int G, int D,
                  int half, const float * scale, const int32_t * row_doc, const int32_t * doc_start,
                  const int32_t * doc_len, float * out) {
    const int rep = H / G, CQ = D * H;
    int max_len = 0;
    for (int t = 0; t < T; ++t) {
        const int L = doc_len[row_doc[t]];
        if (L > max_len) max_len = L;
    }
#pragma omp parallel
    {
        float * sc = (float *) malloc(sizeof(float) * ((size_t) max_len + 8));
#pragma omp for schedule(dynamic, 8)
        for (int t = 0; t < T; ++t) {
            const int d = row_doc[t];
            for (int h = 0; h < H; ++h) {
                const size_t go = (size_t) (h / rep) * T * D;
                int lo = doc_start[d], hi = lo + doc_len[d];
                if (half >= 0) {
                    if (lo < t - half) lo = t - half;
                    if (hi > t + half + 1) hi = t + half + 1;
                }
                attend(q + (size_t) t * CQ + (size_t) h * D, k + go + (size_t) lo * D, v + go + (size_t) lo * D,
                       (size_t) D, hi - lo, D, scale[d], sc, out + (size_t) t * CQ + (size_t) h * D);
            }
        }
        free(sc);
    }
}

/* ggml_norm + ggml_mul + ggml_add (:1292-1293).  ggml itself is not available;
 * this restates LayerNorm as mean and variance accumulated in double, y =
 * (x - mean) * 1/sqrt(var + eps) in fp32.  Unpinned against ggml. */
void or_layer_norm(const float * x, const float * w, const float * b, float eps, int T, int C, float * out) {
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; ++t) {
        const float * xr = x + (size_t) t * C;
        float * y = out + (size_t) t * C;
        double sum = 0.0;
        for (int i = 0; i < C; ++i) sum += (double) xr[i];
        const float mean = (float) (sum / C);
        double sum2 = 0.0;
        for (int i = 0; i < C; ++i) {
            const float v = xr[i] - mean;
            y[i] = v;
            sum2 += (double) (v * v);
        }
        const float variance = (float) (sum2 / C);
        const float scale = 1.0f / sqrtf(variance + eps);
        for (int i = 0; i < C; ++i) y[i] *= scale;
        if (w) for (int i = 0; i < C; ++i) y[i] = y[i] * w[i];
        if (b) for (int i = 0; i < C; ++i) y[i] = y[i] + b[i];
    }
}

/* run_forward's pooling (:1903-1918): sequential sum over the document's rows,
 * then 1/n or, with normalize, 1/||sum|| (the L2 norm of the sum replaces 1/n) */
void or_pool(const float * hidden, const int32_t * lengths, int n_seqs, int C, int normalize, float * pooled) {
    size_t s = 0;
    for (int d = 0; d < n_seqs; ++d) {
        float * pv = pooled + (size_t) d * C;
        memset(pv, 0, sizeof(float) * (size_t) C);
        const int n = lengths[d];
        for (int t = 0; t < n; ++t) axpy_f32(pv, 1.0f, hidden + (s + (size_t) t) * C, C);
        float scale = 1.0f / (float) n;
        if (normalize) {
            const float nrm = sqrtf(or_dot_f32(pv, pv, C));
            scale = nrm > 0.0f ? 1.0f / nrm : 0.0f;
        }
        for (int i = 0; i < C; ++i) pv[i] *= scale;
        s += (size_t) n;
    }
}

/* build_rope (:1322-1338) */
void or_rope_table(int n_pos, float base, int head_dim, float * cos_t, float * sin_t) {
    const int half = head_dim / 2;
    float * inv = (float *) malloc(sizeof(float) * (size_t) half);
    for (int i = 0; i < half; ++i) inv[i] = 1.0f / powf(base, (float) (2 * i) / (float) head_dim);
    for (int t = 0; t < n_pos; ++t) {
        for (int i = 0; i < half; ++i) {
            const float a = (float) t * inv[i];
            cos_t[(size_t) t * half + i] = cosf(a);
            sin_t[(size_t) t * half + i] = sinf(a);
        }
    }
    free(inv);
}

/* ------------------------------------------------------------------------- */
/* whole model                                                               */
/* ------------------------------------------------------------------------- */

enum { MIX_LILY, MIX_SWA, MIX_ATTN, MIX_HRA };
enum { SS_SSSMAX, SS_SSMAX, SS_NONE };

typedef struct {
    char *    name;
    int       type;
    int64_t   ne[4];
    void *    raw;            /* file bytes */
    /* int8 path */
    int       is_i8, n_in, n_out;
    int8_t *  w;
    float *   scale;
    int32_t * off;
    float *   taps;           /* conv kernels, tap-major [k][C] */
    int       k;
} or_tensor;

struct or_model {
    int n_vocab, n_embd, n_layer, n_inter, n_head, n_kv_head, head_dim;
    int lily_kernel, hra_block, swa_window, ntk_train_len, ssmax, n_types;
    float rope_base, swa_rope_base, ssmax_base, rms_eps, ln_eps;
    int * block_types;
    int n_tensors;
    or_tensor * t;
};

static or_tensor * find(const or_model * m, const char * name) {
    for (int i = 0; i < m->n_tensors; ++i) {
        if (strcmp(m->t[i].name, name) == 0) return &m->t[i];
    }
    return NULL;
}

static or_tensor * need(const or_model * m, const char * name) {
    or_tensor * t = find(m, name);
    if (!t) {
        fprintf(stderr, "oracle: missing tensor '%s'\n", name);
        abort();
    }
    return t;
}

static uint32_t kv_u32(const gm_file * g, const char * key, uint32_t def) {
    const int64_t i = gm_find_key(g, key);
    return i < 0 ? def : (uint32_t) g->kv[i].v.u;
}
static float kv_f32(const gm_file * g, const char * key, float def) {
    const int64_t i = gm_find_key(g, key);
    return i < 0 ? def : (float) g->kv[i].v.f;
}
static const char * kv_str(const gm_file * g, const char * key, const char * def) {
    const int64_t i = gm_find_key(g, key);
    return i < 0 || !g->kv[i].str ? def : g->kv[i].str;
}

static int ends_with(const char * s, const char * suf) {
    const size_t n = strlen(s), m = strlen(suf);
    return n >= m && strcmp(s + n - m, suf) == 0;
}

or_model * or_load(const char * path) {
    gm_file * g = gm_open(path);
    if (!g) return NULL;
    if (strcmp(kv_str(g, "general.architecture", ""), "nexterabert") != 0) {
        fprintf(stderr, "oracle: not a nexterabert GGUF\n");
        gm_close(g);
        return NULL;
    }
    or_model * m = (or_model *) calloc(1, sizeof(or_model));
    m->n_vocab    = (int) kv_u32(g, "nexterabert.vocab_size", 0);
    m->n_embd     = (int) kv_u32(g, "nexterabert.embedding_length", 0);
    m->n_layer    = (int) kv_u32(g, "nexterabert.block_count", 0);
    m->n_inter    = (int) kv_u32(g, "nexterabert.feed_forward_length", 0);
    m->n_head     = (int) kv_u32(g, "nexterabert.attention.head_count", 0);
    m->n_kv_head  = (int) kv_u32(g, "nexterabert.attention.head_count_kv", 0);
    m->head_dim   = m->n_embd / m->n_head;
    m->lily_kernel = (int) kv_u32(g, "nexterabert.lily.kernel_size", 5);
    m->hra_block  = (int) kv_u32(g, "nexterabert.hra.block_size", 4);
    m->swa_window = (int) kv_u32(g, "nexterabert.swa.window", 256);
    m->ntk_train_len = (int) kv_u32(g, "nexterabert.rope.ntk_train_length", 0);
    m->rope_base  = kv_f32(g, "nexterabert.rope.freq_base", 100000.0f);
    m->swa_rope_base = kv_f32(g, "nexterabert.swa.rope.freq_base", 10000.0f);
    m->ssmax_base = kv_f32(g, "nexterabert.ssmax.base", 0.1f);
    m->rms_eps    = kv_f32(g, "nexterabert.rms_norm_epsilon", 1e-8f);
    m->ln_eps     = kv_f32(g, "nexterabert.layer_norm_epsilon", 1e-5f);
    const char * mode = kv_str(g, "nexterabert.ssmax.mode", "sssmax");
    m->ssmax = strcmp(mode, "none") == 0 ? SS_NONE : strcmp(mode, "ssmax") == 0 ? SS_SSMAX : SS_SSSMAX;
    m->block_types = (int *) calloc((size_t) m->n_layer + 1, sizeof(int));
    const int64_t bi = gm_find_key(g, "nexterabert.block_types");
    if (bi < 0 || (int) g->kv[bi].arr_n != m->n_layer) {
        fprintf(stderr, "oracle: bad block_types\n");
        gm_close(g);
        or_free(m);
        return NULL;
    }
    for (int l = 0; l < m->n_layer; ++l) {
        const char * s = g->kv[bi].arr_str[l];
        m->block_types[l] = strcmp(s, "lily") == 0 ? MIX_LILY : strcmp(s, "swa") == 0 ? MIX_SWA
                          : strcmp(s, "attn") == 0 ? MIX_ATTN : MIX_HRA;
    }
    FILE * fp = fopen(path, "rb");
    m->n_tensors = (int) g->n_tensors;
    m->t = (or_tensor *) calloc((size_t) m->n_tensors, sizeof(or_tensor));
    int ok = 1;
    for (int i = 0; ok && i < m->n_tensors; ++i) {
        const gm_tensor * gt = &g->tensors[i];
        or_tensor * t = &m->t[i];
        t->name = strdup(gt->name);
        t->type = gt->type;
        memcpy(t->ne, gt->ne, sizeof(t->ne));
        t->raw = malloc(gt->nbytes ? gt->nbytes : 1);
        if (fseeko(fp, (off_t) (g->data_offset + gt->offset), SEEK_SET) != 0 ||
            fread(t->raw, 1, gt->nbytes, fp) != gt->nbytes) {
            fprintf(stderr, "oracle: failed to read '%s'\n", gt->name);
            ok = 0;
            break;
        }
        /* placement: nexterabert.cpp:1663-1667 */
        const int gemm = strcmp(t->name, "embedding.weight") != 0 && strcmp(t->name, "mlm.decoder.weight") != 0
                         && strcmp(t->name, "token_type_embeddings.weight") != 0
                         && gt->n_dims == 2 && gm_is_quantized(t->type);
        if (gemm && gt->ne[0] % 32 == 0 && gt->ne[1] % 4 == 0) {
            t->is_i8 = 1;
            t->n_in = (int) gt->ne[0];
            t->n_out = (int) gt->ne[1];
            const int n_blk = (t->n_in + OR_I8_BLOCK - 1) / OR_I8_BLOCK;
            t->w = (int8_t *) malloc((size_t) t->n_in * t->n_out);
            t->scale = (float *) malloc(sizeof(float) * (size_t) n_blk * t->n_out);
            t->off = (int32_t *) malloc(sizeof(int32_t) * (size_t) n_blk * t->n_out);
            if (or_build_i8_weight(t->type, t->raw, t->n_in, t->n_out, t->w, t->scale, t->off) != 0) ok = 0;
        }
        /* conv kernels -> tap-major (:1702-1711) */
        if (ends_with(t->name, ".depthwise.weight") || ends_with(t->name, ".kernel")) {
            const int k = (int) gt->ne[0], C = (int) gt->ne[1];
            const float * src = (const float *) t->raw;
            t->k = k;
            t->taps = (float *) malloc(sizeof(float) * (size_t) k * C);
            for (int ch = 0; ch < C; ++ch) {
                for (int j = 0; j < k; ++j) t->taps[(size_t) j * C + ch] = src[(size_t) ch * k + j];
            }
        }
    }
    fclose(fp);
    or_tensor * tt = find(m, "token_type_embeddings.weight");
    m->n_types = tt ? (int) tt->ne[1] : 0;
    gm_close(g);
    if (!ok) {
        or_free(m);
        return NULL;
    }
    return m;
}

void or_free(or_model * m) {
    if (!m) return;
    for (int i = 0; i < m->n_tensors; ++i) {
        or_tensor * t = &m->t[i];
        free(t->name); free(t->raw); free(t->w); free(t->scale); free(t->off); free(t->taps);
    }
    free(m->t);
    free(m->block_types);
    free(m);
}

int or_n_embd(const or_model * m) { return m->n_embd; }

int or_get_i8(const or_model * m, const char * name, int * n_in, int * n_out,
              const int8_t ** w, const float ** scale, const int32_t ** off) {
    or_tensor * t = find(m, name);
    if (!t || !t->is_i8) return -1;
    *n_in = t->n_in; *n_out = t->n_out; *w = t->w; *scale = t->scale; *off = t->off;
    return 0;
}

/* per-forward state */
typedef struct {
    int n_docs, T;
    int32_t * start, * len, * row_doc;   /* token layout */
    int32_t * bstart, * blen, * brow_doc;
    int nb;                              /* block rows */
    float * rope_c[2], * rope_s[2];
} fwd;

/* a quantized activation */
typedef struct { int8_t * q; float * sx; int T, C; } qact;

static qact quant(const float * x, int T, int C) {
    qact a;
    const int n_blk = (C + OR_I8_BLOCK - 1) / OR_I8_BLOCK;
    a.q = (int8_t *) malloc((size_t) T * C);
    a.sx = (float *) malloc(sizeof(float) * (size_t) T * n_blk);
    a.T = T;
    a.C = C;
    or_quantize_rows(x, T, C, a.q, a.sx);
    return a;
}

static void qfree(qact a) { free(a.q); free(a.sx); }

static float * linear(const or_model * m, const char * name, qact x, const float * res) {
    or_tensor * w = need(m, name);
    if (!w->is_i8) {
        fprintf(stderr, "oracle: '%s' is not on the int8 path (float files are not supported)\n", name);
        abort();
    }
    if (w->n_in != x.C) {
        fprintf(stderr, "oracle: '%s' expects %d inputs, got %d\n", name, w->n_in, x.C);
        abort();
    }
    float * y = (float *) malloc(sizeof(float) * (size_t) x.T * w->n_out);
    or_linear_i8(x.q, x.sx, x.T, w->w, w->scale, w->n_in, w->n_out, res, y, NULL);
    return y;
}

static const float * fdata(const or_model * m, const char * name) {
    return (const float *) need(m, name)->raw;
}

static float * rms(const or_model * m, const char * name, const float * x, int T) {
    float * o = (float *) malloc(sizeof(float) * (size_t) T * m->n_embd);
    or_rms_norm(x, fdata(m, name), m->rms_eps, T, m->n_embd, o);
    return o;
}

/* ssmax_scale (:1174-1181) */
static float ssmax_scale(const or_model * m, const char * pre, int n) {
    char nm[256];
    if (m->ssmax == SS_NONE) return 1.0f;
    snprintf(nm, sizeof nm, "%sscalable_factor.s", pre);
    const float s = fdata(m, nm)[0];
    const float ln = logf((float) (n > 1 ? n : 1));
    if (m->ssmax == SS_SSMAX) return s * ln;
    snprintf(nm, sizeof nm, "%sscalable_factor.b", pre);
    const float b = fdata(m, nm)[0];
    return s * ln + m->ssmax_base + (b > 0.0f ? b : 0.0f);
}

/* builder::attention (:1184-1206) over rows of layout (start, len, row_doc, T) */
static float * attention(const or_model * m, const char * pre, qact h, const int32_t * start, const int32_t * len,
                         const int32_t * row_doc, int n_docs, int T, const float * rc, const float * rs,
                         int half, int ssmax) {
    const int H = m->n_head, G = m->n_kv_head, D = m->head_dim;
    char nm[256], na[256], nb[256];
    snprintf(nm, sizeof nm, "%sc_q.weight", pre);
    float * ql = linear(m, nm, h, NULL);
    float * q = (float *) malloc(sizeof(float) * (size_t) T * H * D);
    snprintf(na, sizeof na, "%sq_norm.alpha", pre);
    snprintf(nb, sizeof nb, "%sq_norm.beta", pre);
    or_qk_prep(ql, fdata(m, na), fdata(m, nb), rc, rs, row_doc, start, T, H, D, 0, q);
    free(ql);
    snprintf(nm, sizeof nm, "%sc_k.weight", pre);
    float * kl = linear(m, nm, h, NULL);
    float * k = (float *) malloc(sizeof(float) * (size_t) T * G * D);
    snprintf(na, sizeof na, "%sk_norm.alpha", pre);
    snprintf(nb, sizeof nb, "%sk_norm.beta", pre);
    or_qk_prep(kl, fdata(m, na), fdata(m, nb), rc, rs, row_doc, start, T, G, D, 1, k);
    free(kl);
    snprintf(nm, sizeof nm, "%sc_v.weight", pre);
    float * vl = linear(m, nm, h, NULL);
    float * v = (float *) malloc(sizeof(float) * (size_t) T * G * D);
    or_head_major(vl, T, G, D, v);
    free(vl);
    float * scale = (float *) malloc(sizeof(float) * (size_t) n_docs);
    const float base = 1.0f / sqrtf((float) D);
    for (int d = 0; d < n_docs; ++d) scale[d] = base * (ssmax ? ssmax_scale(m, pre, len[d]) : 1.0f);
    float * y = (float *) malloc(sizeof(float) * (size_t) T * H * D);
    or_attention(q, k, v, T, H, G, D, half, scale, row_doc, start, len, y);
    free(q); free(k); free(v); free(scale);
    return y;
}

/* builder::gated_out (:1209-1214): x + c_proj(sigmoid(c_gate(y)) * z) */
static float * gated_out(const or_model * m, const char * pre, const float * y, const float * z, const float * x, int T) {
    const int C = m->n_embd;
    char nm[256];
    qact yq = quant(y, T, C);
    snprintf(nm, sizeof nm, "%sc_gate.weight", pre);
    float * gl = linear(m, nm, yq, NULL);
    qfree(yq);
    float * gz = (float *) malloc(sizeof(float) * (size_t) T * C);
    or_gate(gl, z, T, C, gz);
    free(gl);
    qact gq = quant(gz, T, C);
    free(gz);
    snprintf(nm, sizeof nm, "%sc_proj.weight", pre);
    float * out = linear(m, nm, gq, x);
    qfree(gq);
    return out;
}

static float * mix_attn(const or_model * m, const fwd * f, const char * pre, const char * norm, const float * x, int swa) {
    float * hn = rms(m, norm, x, f->T);
    qact h = quant(hn, f->T, m->n_embd);
    free(hn);
    int half = -1;
    if (swa) { half = m->swa_window / 2; if (half < 1) half = 1; }
    float * y = attention(m, pre, h, f->start, f->len, f->row_doc, f->n_docs, f->T,
                          f->rope_c[swa ? 1 : 0], f->rope_s[swa ? 1 : 0], half, !swa);
    qfree(h);
    float * out = gated_out(m, pre, y, y, x, f->T);
    free(y);
    return out;
}

static float * mix_lily(const or_model * m, const fwd * f, const char * pre, const char * norm, const float * x) {
    const int T = f->T, C = m->n_embd;
    char nm[256];
    float * hn = rms(m, norm, x, T);
    qact h = quant(hn, T, C);
    free(hn);
    snprintf(nm, sizeof nm, "%sltc_conv.in_proj.weight", pre);
    float * z = linear(m, nm, h, NULL);
    const int r = need(m, nm)->n_out;
    snprintf(nm, sizeof nm, "%sltc_conv.A.weight", pre);
    float * rr = linear(m, nm, h, NULL);
    snprintf(nm, sizeof nm, "%sltc_conv.kernel", pre);
    or_tensor * kt = need(m, nm);
    float * lr = (float *) malloc(sizeof(float) * (size_t) T * r);
    or_dwconv(z, rr, kt->taps, kt->k, f->row_doc, f->start, f->len, T, r, lr);
    free(z); free(rr);
    qact lq = quant(lr, T, r);
    free(lr);
    snprintf(nm, sizeof nm, "%sltc_conv.out_proj.weight", pre);
    float * a = linear(m, nm, lq, NULL);
    qfree(lq);
    snprintf(nm, sizeof nm, "%sx_proj.weight", pre);
    float * xp = linear(m, nm, h, NULL);
    snprintf(nm, sizeof nm, "%sB_proj.weight", pre);
    float * b = linear(m, nm, h, NULL);
    qfree(h);
    snprintf(nm, sizeof nm, "%sstate_conv.depthwise.weight", pre);
    or_tensor * st_t = need(m, nm);
    float * st = (float *) malloc(sizeof(float) * (size_t) T * C);
    or_lily_state(a, xp, b, st_t->taps, st_t->k, f->row_doc, f->start, f->len, T, C, st);
    free(a); free(xp); free(b);
    qact sq = quant(st, T, C);
    free(st);
    snprintf(nm, sizeof nm, "%sc_proj.weight", pre);
    float * out = linear(m, nm, sq, x);
    qfree(sq);
    return out;
}

static float * mix_hra(const or_model * m, const fwd * f, const char * pre, const char * norm, const float * x) {
    const int T = f->T, C = m->n_embd;
    char nm[256];
    float * hn = rms(m, norm, x, T);
    qact h = quant(hn, T, C);
    free(hn);
    snprintf(nm, sizeof nm, "%sqkv_in.weight", pre);
    float * i = linear(m, nm, h, NULL);
    snprintf(nm, sizeof nm, "%sqkv_conv.depthwise.weight", pre);
    or_tensor * ct = need(m, nm);
    float * ci = (float *) malloc(sizeof(float) * (size_t) T * C);
    or_dwconv(i, NULL, ct->taps, ct->k, f->row_doc, f->start, f->len, T, C, ci);
    free(i);
    snprintf(nm, sizeof nm, "%sqkv_gate.weight", pre);
    float * gt = linear(m, nm, h, NULL);
    float * hb = (float *) malloc(sizeof(float) * (size_t) f->nb * C);
    or_block_mean(ci, gt, C, m->hra_block, f->start, f->len, f->bstart, f->brow_doc, f->nb, hb);
    free(ci); free(gt);
    qact hbq = quant(hb, f->nb, C);
    free(hb);
    float * yb = attention(m, pre, hbq, f->bstart, f->blen, f->brow_doc, f->n_docs, f->nb,
                           f->rope_c[0], f->rope_s[0], -1, 1);
    qfree(hbq);
    snprintf(nm, sizeof nm, "%sc_C.weight", pre);
    float * cc = linear(m, nm, h, NULL);
    qfree(h);
    float * y = (float *) malloc(sizeof(float) * (size_t) T * C);
    or_upsample_add(yb, cc, C, m->hra_block, T, f->row_doc, f->start, f->bstart, y);
    free(yb); free(cc);
    snprintf(nm, sizeof nm, "%sc_o.depthwise.weight", pre);
    or_tensor * ot = need(m, nm);
    float * co = (float *) malloc(sizeof(float) * (size_t) T * C);
    or_dwconv(y, NULL, ot->taps, ot->k, f->row_doc, f->start, f->len, T, C, co);
    float * out = gated_out(m, pre, y, co, x, T);
    free(y); free(co);
    return out;
}

int or_encode(or_model * m, const int32_t * tokens, const int32_t * types, const int32_t * lengths,
              int n_seqs, float * hidden, float * pooled, int normalize, int n_layers) {
    const int C = m->n_embd;
    if (n_seqs <= 0) return 1;
    fwd f;
    memset(&f, 0, sizeof f);
    int max_len = 0;
    for (int i = 0; i < n_seqs; ++i) {
        if (lengths[i] <= 0) return 1;
        if (lengths[i] > max_len) max_len = lengths[i];
    }
    /* layout::build for tokens and HRA blocks (:236-243, :1351-1354) */
    f.n_docs = n_seqs;
    f.start = (int32_t *) malloc(sizeof(int32_t) * (size_t) n_seqs);
    f.len = (int32_t *) malloc(sizeof(int32_t) * (size_t) n_seqs);
    f.bstart = (int32_t *) malloc(sizeof(int32_t) * (size_t) n_seqs);
    f.blen = (int32_t *) malloc(sizeof(int32_t) * (size_t) n_seqs);
    for (int i = 0; i < n_seqs; ++i) {
        f.start[i] = f.T; f.len[i] = lengths[i]; f.T += lengths[i];
        f.blen[i] = (lengths[i] + m->hra_block - 1) / m->hra_block;
        f.bstart[i] = f.nb; f.nb += f.blen[i];
    }
    f.row_doc = (int32_t *) malloc(sizeof(int32_t) * (size_t) f.T);
    f.brow_doc = (int32_t *) malloc(sizeof(int32_t) * (size_t) f.nb);
    for (int i = 0; i < n_seqs; ++i) {
        for (int t = 0; t < f.len[i]; ++t) f.row_doc[f.start[i] + t] = i;
        for (int b = 0; b < f.blen[i]; ++b) f.brow_doc[f.bstart[i] + b] = i;
    }
    for (int i = 0; i < f.T; ++i) {
        if (tokens[i] < 0 || tokens[i] >= m->n_vocab) {
            fprintf(stderr, "oracle: token id %d out of range\n", tokens[i]);
            free(f.start); free(f.len); free(f.bstart); free(f.blen); free(f.row_doc); free(f.brow_doc);
            return 1;
        }
        if (types && m->n_types > 0 && (types[i] < 0 || types[i] >= m->n_types)) {
            free(f.start); free(f.len); free(f.bstart); free(f.blen); free(f.row_doc); free(f.brow_doc);
            return 1;
        }
    }
    /* rope tables (:1356-1368) */
    float base = m->rope_base;
    if (m->ntk_train_len > 0 && max_len > m->ntk_train_len) {
        if (n_seqs > 1) {
            free(f.start); free(f.len); free(f.bstart); free(f.blen); free(f.row_doc); free(f.brow_doc);
            return 1;
        }
        const double d = m->head_dim;
        base = (float) ((double) base * pow((double) max_len / m->ntk_train_len, d / (d - 2.0)));
    }
    const int half = m->head_dim / 2;
    for (int r = 0; r < 2; ++r) {
        f.rope_c[r] = (float *) malloc(sizeof(float) * (size_t) max_len * half);
        f.rope_s[r] = (float *) malloc(sizeof(float) * (size_t) max_len * half);
    }
    or_rope_table(max_len, base, m->head_dim, f.rope_c[0], f.rope_s[0]);
    or_rope_table(max_len, m->swa_rope_base, m->head_dim, f.rope_c[1], f.rope_s[1]);

    /* embedding (:1272-1273) */
    const int T = f.T;
    float * x = (float *) malloc(sizeof(float) * (size_t) T * C);
    {
        or_tensor * e = need(m, "embedding.weight");
        const size_t rb = gm_row_size(e->type, C);
        or_tensor * tt = (types && m->n_types > 0) ? need(m, "token_type_embeddings.weight") : NULL;
        const size_t trb = tt ? gm_row_size(tt->type, C) : 0;
#pragma omp parallel
        {
            float * tmp = (float *) malloc(sizeof(float) * (size_t) C);
#pragma omp for schedule(static)
            for (int t = 0; t < T; ++t) {
                or_dequant_row(e->type, (const uint8_t *) e->raw + rb * (size_t) tokens[t], x + (size_t) t * C, C);
                if (tt) {
                    or_dequant_row(tt->type, (const uint8_t *) tt->raw + trb * (size_t) types[t], tmp, C);
                    for (int c = 0; c < C; ++c) x[(size_t) t * C + c] = x[(size_t) t * C + c] + tmp[c];
                }
            }
            free(tmp);
        }
    }
    const int n_layer = n_layers >= 0 ? (n_layers < m->n_layer ? n_layers : m->n_layer) : m->n_layer;
    char pre[128], norm[160], nm[256];
    for (int l = 0; l < n_layer; ++l) {
        snprintf(pre, sizeof pre, "blocks.%d.attn.", l);
        snprintf(norm, sizeof norm, "blocks.%d.attn_norm.weight", l);
        float * nx = NULL;
        switch (m->block_types[l]) {
            case MIX_LILY: nx = mix_lily(m, &f, pre, norm, x); break;
            case MIX_SWA:  nx = mix_attn(m, &f, pre, norm, x, 1); break;
            case MIX_ATTN: nx = mix_attn(m, &f, pre, norm, x, 0); break;
            default:       nx = mix_hra(m, &f, pre, norm, x); break;
        }
        free(x);
        x = nx;
        /* MLP (:1284-1289) */
        snprintf(nm, sizeof nm, "blocks.%d.mlp_norm.weight", l);
        float * hn = rms(m, nm, x, T);
        qact h = quant(hn, T, C);
        free(hn);
        snprintf(nm, sizeof nm, "blocks.%d.mlp.c_fc.weight", l);
        float * u = linear(m, nm, h, NULL);
        const int I = need(m, nm)->n_out;
        qfree(h);
        or_relu_sqr(u, T, I, u);
        qact rq = quant(u, T, I);
        free(u);
        snprintf(nm, sizeof nm, "blocks.%d.mlp.c_proj.weight", l);
        nx = linear(m, nm, rq, x);
        qfree(rq);
        free(x);
        x = nx;
    }
    if (n_layers < 0) {
        or_layer_norm(x, fdata(m, "out_norm.weight"), fdata(m, "out_norm.bias"), m->ln_eps, T, C, x);
    }
    if (hidden) memcpy(hidden, x, sizeof(float) * (size_t) T * C);
    if (pooled) or_pool(x, lengths, n_seqs, C, normalize, pooled);
    free(x);
    for (int r = 0; r < 2; ++r) { free(f.rope_c[r]); free(f.rope_s[r]); }
    free(f.start); free(f.len); free(f.bstart); free(f.blen); free(f.row_doc); free(f.brow_doc);
    return 0;
}

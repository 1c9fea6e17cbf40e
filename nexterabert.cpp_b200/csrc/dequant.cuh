// Per-element decoding of GGUF block formats on the device.
//
// Each value is decoded independently with the same fp32 operation order as
// the oracle's restatement of ggml's dequantization (gguf-py 0.19.0 order: every
// product and difference rounded separately), so the expanded int8 weights and
// the embedding rows match the CPU path bit for bit.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

namespace nxk {

enum : int { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8,
             T_Q2_K = 10, T_Q3_K = 11, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14, T_BF16 = 30 };

__host__ __device__ inline int blck_size(int t) {
    switch (t) {
        case T_F32: case T_F16: case T_BF16: return 1;
        case T_Q4_0: case T_Q4_1: case T_Q5_0: case T_Q5_1: case T_Q8_0: return 32;
        case T_Q2_K: case T_Q3_K: case T_Q4_K: case T_Q5_K: case T_Q6_K: return 256;
        default: return 0;
    }
}

__host__ __device__ inline int type_size(int t) {
    switch (t) {
        case T_F32: return 4;
        case T_F16: case T_BF16: return 2;
        case T_Q4_0: return 18;
        case T_Q4_1: return 20;
        case T_Q5_0: return 22;
        case T_Q5_1: return 24;
        case T_Q8_0: return 34;
        case T_Q2_K: return 84;
        case T_Q3_K: return 110;
        case T_Q4_K: return 144;
        case T_Q5_K: return 176;
        case T_Q6_K: return 210;
        default: return 0;
    }
}

__device__ __forceinline__ float ld_h2f(const uint8_t * p) {
    const unsigned short h = (unsigned short) (p[0] | (p[1] << 8));
    return __half2float(__ushort_as_half(h));
}

__device__ __forceinline__ void k_scale_min(const uint8_t * s, int j, int & sc, int & mn) {
    if (j < 4) {
        sc = s[j] & 63;
        mn = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
        mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

// value e (0-based) of a row stored as blocks of `type`
__device__ __forceinline__ float deq_elem(int type, const uint8_t * row, int e) {
    switch (type) {
        case T_F32: {
            float v;
            memcpy(&v, row + 4 * (size_t) e, 4);
            return v;
        }
        case T_F16: return ld_h2f(row + 2 * (size_t) e);
        case T_BF16: {
            const uint32_t b = (uint32_t) (row[2 * e] | (row[2 * e + 1] << 8)) << 16;
            return __uint_as_float(b);
        }
        case T_Q4_0: {
            const uint8_t * b = row + (size_t) (e / 32) * 18;
            const int i = e % 32;
            const int q = i < 16 ? (b[2 + i] & 15) : (b[2 + i - 16] >> 4);
            return __fmul_rn(ld_h2f(b), (float) (q - 8));
        }
        case T_Q4_1: {
            const uint8_t * b = row + (size_t) (e / 32) * 20;
            const int i = e % 32;
            const int q = i < 16 ? (b[4 + i] & 15) : (b[4 + i - 16] >> 4);
            return __fadd_rn(__fmul_rn(ld_h2f(b), (float) q), ld_h2f(b + 2));
        }
        case T_Q5_0: {
            const uint8_t * b = row + (size_t) (e / 32) * 22;
            const int i = e % 32;
            const uint32_t qh = (uint32_t) b[2] | ((uint32_t) b[3] << 8) | ((uint32_t) b[4] << 16) | ((uint32_t) b[5] << 24);
            const int lo = i < 16 ? (b[6 + i] & 15) : (b[6 + i - 16] >> 4);
            const int q = lo | (int) (((qh >> i) & 1u) << 4);
            return __fmul_rn(ld_h2f(b), (float) (q - 16));
        }
        case T_Q5_1: {
            const uint8_t * b = row + (size_t) (e / 32) * 24;
            const int i = e % 32;
            const uint32_t qh = (uint32_t) b[4] | ((uint32_t) b[5] << 8) | ((uint32_t) b[6] << 16) | ((uint32_t) b[7] << 24);
            const int lo = i < 16 ? (b[8 + i] & 15) : (b[8 + i - 16] >> 4);
            const int q = lo | (int) (((qh >> i) & 1u) << 4);
            return __fadd_rn(__fmul_rn(ld_h2f(b), (float) q), ld_h2f(b + 2));
        }
        case T_Q8_0: {
            const uint8_t * b = row + (size_t) (e / 32) * 34;
            return __fmul_rn((float) (int8_t) b[2 + e % 32], ld_h2f(b));
        }
        case T_Q2_K: {
            const uint8_t * b = row + (size_t) (e / 256) * 84;
            const int i = e % 256, h = i / 128, s = (i / 32) % 4, ee = i % 32, sub = i / 16;
            const int q = (b[16 + 32 * h + ee] >> (2 * s)) & 3;
            const float dl = __fmul_rn(ld_h2f(b + 80), (float) (b[sub] & 15));
            const float ml = __fmul_rn(ld_h2f(b + 82), (float) (b[sub] >> 4));
            return __fsub_rn(__fmul_rn(dl, (float) q), ml);
        }
        case T_Q3_K: {
            const uint8_t * b = row + (size_t) (e / 256) * 110;
            const int i = e % 256, h = i / 128, s = (i / 32) % 4, ee = i % 32, sub = i / 16;
            const uint8_t * sc = b + 96;
            const int lo = (sc[sub % 8] >> (4 * (sub / 8))) & 15;
            const int hi = (sc[8 + sub % 4] >> (2 * (sub / 4))) & 3;
            const int scale = (int) (int8_t) (uint8_t) (lo | (hi << 4)) - 32;
            const int ql = (b[32 + 32 * h + ee] >> (2 * s)) & 3;
            const int hb = (b[i % 32] >> (i / 32)) & 1;
            const int q = ql - ((hb ^ 1) << 2);
            return __fmul_rn(__fmul_rn(ld_h2f(b + 108), (float) scale), (float) q);
        }
        case T_Q4_K: {
            const uint8_t * b = row + (size_t) (e / 256) * 144;
            const int i = e % 256, j = i / 32, ee = i % 32;
            int sc, mn;
            k_scale_min(b + 4, j, sc, mn);
            const float d1 = __fmul_rn(ld_h2f(b), (float) sc), m1 = __fmul_rn(ld_h2f(b + 2), (float) mn);
            const int q = (b[16 + 32 * (j / 2) + ee] >> (4 * (j % 2))) & 15;
            return __fsub_rn(__fmul_rn(d1, (float) q), m1);
        }
        case T_Q5_K: {
            const uint8_t * b = row + (size_t) (e / 256) * 176;
            const int i = e % 256, j = i / 32, ee = i % 32;
            int sc, mn;
            k_scale_min(b + 4, j, sc, mn);
            const float d1 = __fmul_rn(ld_h2f(b), (float) sc), m1 = __fmul_rn(ld_h2f(b + 2), (float) mn);
            const int q = ((b[48 + 32 * (j / 2) + ee] >> (4 * (j % 2))) & 15) | (((b[16 + ee] >> j) & 1) << 4);
            return __fsub_rn(__fmul_rn(d1, (float) q), m1);
        }
        case T_Q6_K: {
            const uint8_t * b = row + (size_t) (e / 256) * 210;
            const int p = e % 256, h = p / 128, r = p % 128;
            const int lo = (b[64 * h + (r % 64)] >> (4 * (r / 64))) & 15;
            const int hi = (b[128 + 32 * h + (r % 32)] >> (2 * (r / 32))) & 3;
            const int q = (lo | (hi << 4)) - 32;
            const float d1 = __fmul_rn(ld_h2f(b + 208), (float) (int8_t) b[192 + p / 16]);
            return __fmul_rn(d1, (float) q);
        }
        default: return 0.0f;
    }
}

} // namespace nxk

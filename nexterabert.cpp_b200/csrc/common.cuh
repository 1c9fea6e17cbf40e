// Device arithmetic that reproduces the reference CPU runtime's fp32 results.
//
// The reference (src/nexterabert.cpp) computes with AVX2 intrinsics in a fixed
// order: fused multiply-adds where it writes _mm256_fmadd_ps, 8- and 32-lane
// accumulators reduced by fixed horizontal-add trees, and its own Cephes-style
// exp (exp256, :81-99) under tanh and sigmoid.  The helpers below perform the
// same IEEE operations in the same order with explicit round-to-nearest
// intrinsics (never a contracted multiply-add), so the row ops built on them
// are bit-identical to the reference.  Translation units are compiled with
// -fmad=false as a second guard.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace nxk {

constexpr int I8_BLOCK = 256;
constexpr int ACT_MAX  = 127;

// one lane of exp256 (:81-99)
__device__ __forceinline__ float exp8(float x) {
    x = fminf(x, 88.3762626647949f);
    x = fmaxf(x, -87.3f);
    const float fx = rintf(__fmul_rn(x, 1.44269504088896341f));
    x = __fmaf_rn(-fx, 0.693359375f, x);
    x = __fmaf_rn(-fx, -2.12194440e-4f, x);
    const float z = __fmul_rn(x, x);
    float y = 1.9875691500e-4f;
    y = __fmaf_rn(y, x, 1.3981999507e-3f);
    y = __fmaf_rn(y, x, 8.3334519073e-3f);
    y = __fmaf_rn(y, x, 4.1665795894e-2f);
    y = __fmaf_rn(y, x, 1.6666665459e-1f);
    y = __fmaf_rn(y, x, 5.0000001201e-1f);
    y = __fmaf_rn(y, z, __fadd_rn(x, 1.0f));
    const int e = (__float2int_rn(fx) + 127) << 23;
    return __fmul_rn(y, __int_as_float(e));
}

// two lanes of exp256 at once: the same operations as exp8 on each component (the packed
// multiply, add and fused multiply-add round each component as the scalar forms do)
// NONPOS: the arguments are known to be <= 0, where exp256's upper clamp is the identity.
template <bool NONPOS = false>
__device__ __forceinline__ float2 exp8x2(float2 x) {
    if (!NONPOS) {
        x.x = fminf(x.x, 88.3762626647949f);
        x.y = fminf(x.y, 88.3762626647949f);
    }
    x.x = fmaxf(x.x, -87.3f);
    x.y = fmaxf(x.y, -87.3f);
    const float2 t = __fmul2_rn(x, make_float2(1.44269504088896341f, 1.44269504088896341f));
    const float2 fx = make_float2(rintf(t.x), rintf(t.y));
    const float2 nfx = make_float2(-fx.x, -fx.y);
    x = __ffma2_rn(nfx, make_float2(0.693359375f, 0.693359375f), x);
    x = __ffma2_rn(nfx, make_float2(-2.12194440e-4f, -2.12194440e-4f), x);
    const float2 z = __fmul2_rn(x, x);
    float2 y = make_float2(1.9875691500e-4f, 1.9875691500e-4f);
    y = __ffma2_rn(y, x, make_float2(1.3981999507e-3f, 1.3981999507e-3f));
    y = __ffma2_rn(y, x, make_float2(8.3334519073e-3f, 8.3334519073e-3f));
    y = __ffma2_rn(y, x, make_float2(4.1665795894e-2f, 4.1665795894e-2f));
    y = __ffma2_rn(y, x, make_float2(1.6666665459e-1f, 1.6666665459e-1f));
    y = __ffma2_rn(y, x, make_float2(5.0000001201e-1f, 5.0000001201e-1f));
    y = __ffma2_rn(y, z, __fadd2_rn(x, make_float2(1.0f, 1.0f)));
    const float2 p2 = make_float2(__int_as_float((__float2int_rn(fx.x) + 127) << 23),
                                  __int_as_float((__float2int_rn(fx.y) + 127) << 23));
    return __fmul2_rn(y, p2);
}

// one lane of tanh256 (:103-117)
__device__ __forceinline__ float tanh8(float x) {
    const float ax = fabsf(x);
    const float t = exp8(__fmul_rn(ax, -2.0f));
    float big = __fdiv_rn(__fsub_rn(1.0f, t), __fadd_rn(1.0f, t));
    big = __int_as_float(__float_as_int(big) | (__float_as_int(x) & (int) 0x80000000));
    const float x2 = __fmul_rn(x, x);
    float p = -17.0f / 315.0f;
    p = __fmaf_rn(p, x2, 2.0f / 15.0f);
    p = __fmaf_rn(p, x2, -1.0f / 3.0f);
    p = __fmaf_rn(p, x2, 1.0f);
    const float small = __fmul_rn(p, x);
    return ax < 0.1f ? small : big;
}

// one lane of sigmoid256 (:119-122)
__device__ __forceinline__ float sigmoid8(float x) {
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, exp8(__fsub_rn(0.0f, x))));
}

// The reference's dot_f32 (:133-151) of a row whose length is a multiple of 32,
// when lane L of a warp has accumulated the fma chain over elements 32*i + L:
// its four 8-lane accumulators are lanes 0-7, 8-15, 16-23, 24-31.  Reduction:
// v = (s0 + s1) + (s2 + s3) per lane of 8, then hsum256 =
// ((v0+v4) + (v2+v6)) + ((v1+v5) + (v3+v7)).  Result broadcast to all lanes.
__device__ __forceinline__ float warp_dot_tree(float acc) {
    float w = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 8));
    float v = __fadd_rn(w, __shfl_down_sync(0xffffffffu, w, 16));
    float x = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 4));
    float y = __fadd_rn(x, __shfl_down_sync(0xffffffffu, x, 2));
    float z = __fadd_rn(y, __shfl_down_sync(0xffffffffu, y, 1));
    return __shfl_sync(0xffffffffu, z, 0);
}

__device__ __forceinline__ float warp_max(float v) {
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// quantize_row (:378-403) for one value once the block's amax is known:
// u8 = saturate(rint(x * 127/amax) + 128); returned as the signed code u8 - 128.
__device__ __forceinline__ float act_inv(float amax) {
    return amax > 0.0f ? __fdiv_rn((float) ACT_MAX, amax) : 0.0f;
}
__device__ __forceinline__ float act_scale(float amax) { return __fdiv_rn(amax, (float) ACT_MAX); }
__device__ __forceinline__ int8_t act_code(float x, float inv) {
    const float v = __fmul_rn(x, inv);
    int c = fabsf(v) < 2147483520.0f ? __float2int_rn(v) : (int) 0x80000000;   // cvtps_epi32
    long long u = (long long) c + 128;
    u = u < 0 ? 0 : (u > 255 ? 255 : u);                                        // packs + packus
    return (int8_t) (u - 128);
}

// exact int32 -> fp32 for |s| <= 2^22 (block sums are within 256 * 127 * 128)
__device__ __forceinline__ float i2f_exact(int32_t s) {
    return __fsub_rn(__int_as_float(s + 0x4B400000), 12582912.0f);
}

// 16-byte asynchronous global -> shared copies (both addresses 16-byte aligned)
__device__ __forceinline__ void cp_async16(void * dst, const void * src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                 :: "r"((uint32_t) __cvta_generic_to_shared(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }

} // namespace nxk

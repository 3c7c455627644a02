// Portable exponential for the decoder's softmax and SiLU.
//
// The reference's exp inside oneDNN's swish and std::exp in its attention softmax are library code whose last-bit
// behaviour is not specified, so no device exp can reproduce them bit for bit. The decoder instead fixes its own
// exp, written from the mathematics, and the CPU oracle evaluates the identical sequence of IEEE f32 operations:
//  - Cody-Waite argument reduction: x = n ln2 + r, n = rint(x log2 e), with ln2 split into a 12-bit head
//    (0x1.62ep-1, so n * head is exact for |n| <= 2^12) and the f32 tail 0x1.0bfbe8p-15;
//  - e^r from its Taylor series to degree 7 in Horner form (|r| <= ln2 / 2: truncation below 6e-9 relative);
//  - scaling by 2^n through the exponent field, in two steps where the result is subnormal.
// Measured against exp in double over [-110, 95]: at most 1.2 ulp. The library is compiled with --fmad=false, so no
// multiply-add here is contracted.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace cppinf::device {

__device__ __forceinline__ float pexp(float x) {
    if (x != x) {
        return x;
    }
    if (x > 88.8f) {
        return __int_as_float(0x7f800000);
    }
    if (x < -104.0f) {
        return 0.0f;
    }
    const float n = rintf(x * 0x1.715476p+0f);
    const float r = (x - n * 0x1.62ep-1f) - n * 0x1.0bfbe8p-15f;
    float p = 0x1.a01a02p-13f;
    p = p * r + 0x1.6c16c2p-10f;
    p = p * r + 0x1.111112p-7f;
    p = p * r + 0x1.555556p-5f;
    p = p * r + 0x1.555556p-3f;
    p = p * r + 0.5f;
    p = p * r + 1.0f;
    p = p * r + 1.0f;
    int e = static_cast<int>(n);
    if (e > 127) {
        p = p * 2.0f;
        e -= 1;
    }
    if (e < -126) {
        p = p * 0x1p-64f;
        e += 64;
    }
    return p * __int_as_float((e + 127) << 23);
}

// x / (1 + exp(-x)): the reference's SiLU (oneDNN eltwise_swish with alpha 1, src/ops/nn_ops.cpp:44-48).
__device__ __forceinline__ float silu_pexp(float x) {
    return x / (1.0f + pexp(-x));
}

}  // namespace cppinf::device

// Activations fused into the GEMM epilogues: the FFN's gelu_tanh
// (src/layers/linear.jl:61-68) after the up-projection, and its derivative
// applied to the down-projection's dX.
//
// Forward (ACT_GELU_TANH): the reference rounds the up-projection output to
// the activation dtype (`hidden`), evaluates
//     gelu(x) = 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))
// in fp32 on that rounded value and rounds again.  The epilogue does the same
// and also writes the rounded `hidden` for the backward.
// Backward (ACT_GELU_TANH_GRAD): the gradient reaching gelu's output is the
// down-projection's dX, rounded to the activation dtype; the gradient of
// `hidden` is that value times gelu'(hidden) in fp32, rounded.
//
// Evaluation: with u = sqrt(2/pi) (x + 0.044715 x^3) and the identity
// 1 + tanh(u) = 2 s, s = 1 / (1 + exp(-2u)) (the logistic function of 2u),
//     gelu(x)  = x s
//     gelu'(x) = s + 2 x s (1 - s) sqrt(2/pi) (1 + 3 * 0.044715 x^2)
// (1 - tanh^2 = 4 s (1 - s)).  exp and the reciprocal are single
// approximate instructions (ex2.approx, rcp.approx): relative error about
// 1e-6 against the fp32 tanh form for |x| < 10, far below one rounding step
// of bf16 (2^-9) or fp16 (2^-12), so the rounded results agree except where
// a value lies within that error of a rounding boundary.  The epilogue
// evaluates this for every output element while sharing the SM's issue
// slots with the dequantising warps, so its instruction count is what costs.
#pragma once
#include "common.cuh"

namespace reels {

enum EpiAct : int { ACT_NONE = 0, ACT_GELU_TANH = 1, ACT_GELU_TANH_GRAD = 2 };

// Float32(sqrt(Float32(2 / pi))), as linear.jl:65 evaluates it.
constexpr float kGeluK0 = 0.7978845238685608f;
constexpr float kGeluK1 = 0.044715f;

// 2^x and 1/x on the multi-function unit, subnormal results flushed (the
// flush never triggers below: 1 + e >= 1 and the capped 2^a <= 2^115).
__device__ __forceinline__ float ex2_ftz(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float rcp_ftz(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// s = 1 / (1 + exp(-2u)) for u = sqrt(2/pi) (x + 0.044715 x^3), with
// exp(-2u) = 2^(-2 log2(e) u) and the argument capped at 115 (2^115 ~ e^80).
__device__ __forceinline__ float gelu_logistic(float x) {
    constexpr float kArg = -2.0f * 1.4426950408889634f * kGeluK0;
    const float a = kArg * fmaf(kGeluK1 * x, x * x, x);
    return rcp_ftz(1.0f + ex2_ftz(fminf(a, 115.0f)));
}

__device__ __forceinline__ float gelu_tanh_f32(float x) { return x * gelu_logistic(x); }

// gelu'(x) = s + 2 x s (1 - s) sqrt(2/pi) (1 + 3 * 0.044715 x^2)
//          = s (1 + (1 - s) x (2 sqrt(2/pi) + 6 * 0.044715 sqrt(2/pi) x^2))
__device__ __forceinline__ float gelu_tanh_grad_f32(float x) {
    constexpr float kA = 2.0f * kGeluK0, kB = 6.0f * kGeluK1 * kGeluK0;
    const float s = gelu_logistic(x);
    const float w = x * fmaf(kB, x * x, kA);
    return s * fmaf(1.0f - s, w, 1.0f);
}

// The value an element takes after rounding to the activation dtype.
template <int DT>
__device__ __forceinline__ float round_act(float x) {
    return Elem<DT>::to_f(Elem<DT>::from_f(x));
}

// The two values of a packed pair (low half first), without taking the
// register's address.
template <int DT>
__device__ __forceinline__ void unpack2(uint32_t w, float &a, float &b) {
    if constexpr (DT == DT_BF16) {
        a = __uint_as_float(w << 16);
        b = __uint_as_float(w & 0xffff0000u);
    } else {
        a = __half2float(__ushort_as_half((unsigned short)(w & 0xffffu)));
        b = __half2float(__ushort_as_half((unsigned short)(w >> 16)));
    }
}

// Two values already rounded to DT as one packed pair (a in the low half).
template <int DT>
__device__ __forceinline__ uint32_t pack_rounded(float a, float b) {
    if constexpr (DT == DT_BF16) return __byte_perm(__float_as_uint(a), __float_as_uint(b), 0x7632);
    else return Elem<DT>::pack2(a, b);
}

}  // namespace reels

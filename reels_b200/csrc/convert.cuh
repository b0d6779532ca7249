// Int8 -> 16-bit conversions used by the weight-dequant warps.
//
// Each helper turns 8 int8 weights (two 32-bit words, element 0 in the low
// byte) into 8 16-bit values packed as a uint4 in element order.  The unscaled
// forms are exact: every int8 in [-127, 127] is representable in bf16 and in
// fp16, and the bit tricks below only add and subtract exactly representable
// powers of two.
#pragma once
#include "common.cuh"

namespace reels {

// bf16, exact.  For a byte b (two's complement q), take
//   hi = bf16(0x43 << 8 | (b & 0x7f)) = 128 + (b & 0x7f)
//   lo = bf16(0x43 << 8 | (b & 0x80)) = 128 or 256
// then q = hi - lo; both operands and the difference are exact in bf16.
__device__ __forceinline__ uint32_t bytes01_to_bf16x2(uint32_t w, uint32_t sel) {
    // sel picks [byte i, 0x43, byte i+1, 0x43] from (w, 0x43)
    uint32_t x = __byte_perm(w, 0x43u, sel);
    uint32_t hi = x & 0xFF7FFF7Fu;
    uint32_t lo = x & 0xFF80FF80u;
    __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162 *>(&hi);
    __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162 *>(&lo);
    __nv_bfloat162 d = __hsub2(a, b);
    return *reinterpret_cast<uint32_t *>(&d);
}

__device__ __forceinline__ uint4 i8x8_to_bf16(uint2 v) {
    uint4 o;
    o.x = bytes01_to_bf16x2(v.x, 0x4140u);
    o.y = bytes01_to_bf16x2(v.x, 0x4342u);
    o.z = bytes01_to_bf16x2(v.y, 0x4140u);
    o.w = bytes01_to_bf16x2(v.y, 0x4342u);
    return o;
}

// fp16, exact: 0x64 << 8 | (q + 128) is the fp16 value 1024 + q + 128;
// subtracting 1152 (0x6480) leaves q.
__device__ __forceinline__ uint32_t bytes01_to_f16x2(uint32_t wx, uint32_t sel) {
    uint32_t x = __byte_perm(wx, 0x64u, sel);
    const uint32_t bias = 0x64806480u;
    __half2 a = *reinterpret_cast<__half2 *>(&x);
    __half2 b = *reinterpret_cast<const __half2 *>(&bias);
    __half2 d = __hsub2(a, b);
    return *reinterpret_cast<uint32_t *>(&d);
}

__device__ __forceinline__ uint4 i8x8_to_f16(uint2 v) {
    uint32_t a = v.x ^ 0x80808080u, b = v.y ^ 0x80808080u;
    uint4 o;
    o.x = bytes01_to_f16x2(a, 0x4140u);
    o.y = bytes01_to_f16x2(a, 0x4342u);
    o.z = bytes01_to_f16x2(b, 0x4140u);
    o.w = bytes01_to_f16x2(b, 0x4342u);
    return o;
}

// Scaled path: byte i of (w ^ 0x80808080) placed under the exponent of
// 2^23 gives the float 2^23 + q + 128 exactly; adding -(2^23 + 128) leaves q.
// fp32(q) * scale rounded once to the 16-bit type; scale per element.
// Packed f32x2 add/multiply (sm_100) halve the instruction count; the add
// is exact (it recovers q), so the only rounding is the product's.
template <int DT>
__device__ __forceinline__ uint32_t scaled_pair(uint32_t wx, uint32_t i, float s0, float s1) {
    const float2 magic = make_float2(-8388736.0f, -8388736.0f);
    float2 f = make_float2(__int_as_float(__byte_perm(wx, 0x4B000000u, 0x7540u | i)),
                           __int_as_float(__byte_perm(wx, 0x4B000000u, 0x7540u | (i + 1))));
    f = __fmul2_rn(__fadd2_rn(f, magic), make_float2(s0, s1));
    return Elem<DT>::pack2(f.x, f.y);
}

template <int DT>
__device__ __forceinline__ uint4 i8x8_scaled(uint2 v, const float (&sc)[8]) {
    const uint32_t a = v.x ^ 0x80808080u, b = v.y ^ 0x80808080u;
    uint4 o;
    o.x = scaled_pair<DT>(a, 0, sc[0], sc[1]);
    o.y = scaled_pair<DT>(a, 2, sc[2], sc[3]);
    o.z = scaled_pair<DT>(b, 0, sc[4], sc[5]);
    o.w = scaled_pair<DT>(b, 2, sc[6], sc[7]);
    return o;
}

// Same with one scale for all eight elements.
template <int DT>
__device__ __forceinline__ uint4 i8x8_scaled1(uint2 v, float s) {
    const uint32_t a = v.x ^ 0x80808080u, b = v.y ^ 0x80808080u;
    uint4 o;
    o.x = scaled_pair<DT>(a, 0, s, s);
    o.y = scaled_pair<DT>(a, 2, s, s);
    o.z = scaled_pair<DT>(b, 0, s, s);
    o.w = scaled_pair<DT>(b, 2, s, s);
    return o;
}

template <int DT>
__device__ __forceinline__ uint4 i8x8_exact(uint2 v) {
    if constexpr (DT == DT_BF16) return i8x8_to_bf16(v);
    else return i8x8_to_f16(v);
}

}  // namespace reels

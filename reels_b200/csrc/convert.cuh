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

// Exact fp32 value of byte i of (w ^ 0x80808080): the word 0x4B0000xx is the
// float 2^23 + xx, and xx = q + 128, so subtracting 2^23 + 128 leaves q.
__device__ __forceinline__ float byte_to_f32(uint32_t wx, uint32_t i) {
    return __int_as_float(__byte_perm(wx, 0x4B000000u, 0x7540u | i)) - 8388736.0f;
}

// fp32(q) * scale rounded once to the 16-bit type; scale per element.
template <int DT>
__device__ __forceinline__ uint4 i8x8_scaled(uint2 v, const float (&sc)[8]) {
    uint32_t a = v.x ^ 0x80808080u, b = v.y ^ 0x80808080u;
    float f[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        f[i] = byte_to_f32(a, i) * sc[i];
        f[i + 4] = byte_to_f32(b, i) * sc[i + 4];
    }
    uint4 o;
    o.x = Elem<DT>::pack2(f[0], f[1]);
    o.y = Elem<DT>::pack2(f[2], f[3]);
    o.z = Elem<DT>::pack2(f[4], f[5]);
    o.w = Elem<DT>::pack2(f[6], f[7]);
    return o;
}

// Same with one scale for all eight elements.
template <int DT>
__device__ __forceinline__ uint4 i8x8_scaled1(uint2 v, float s) {
    uint32_t a = v.x ^ 0x80808080u, b = v.y ^ 0x80808080u;
    float f[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        f[i] = byte_to_f32(a, i) * s;
        f[i + 4] = byte_to_f32(b, i) * s;
    }
    uint4 o;
    o.x = Elem<DT>::pack2(f[0], f[1]);
    o.y = Elem<DT>::pack2(f[2], f[3]);
    o.z = Elem<DT>::pack2(f[4], f[5]);
    o.w = Elem<DT>::pack2(f[6], f[7]);
    return o;
}

template <int DT>
__device__ __forceinline__ uint4 i8x8_exact(uint2 v) {
    if constexpr (DT == DT_BF16) return i8x8_to_bf16(v);
    else return i8x8_to_f16(v);
}

}  // namespace reels

// Dequantisation helpers shared by the tensor-core GEMM kernels.
//
// One packed word holds 8 consecutive k of one column (k = 0..7 at bits 4k,
// int4 two's complement, vulkan-runtime/shaders/q4gemm.comp:104-116).  The
// nibbles are unpacked exactly with the 2^23 magic number ((u ^ 8) = v + 8 in
// [0, 15], float(0x4B000000 | (v + 8)) = 2^23 + v + 8), multiplied by the
// group scale in fp32 (one rounding: the reference's w = float(v) * scale,
// q4gemm.comp:116-122) and rounded to the 16-bit MMA operand type.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>
#include <type_traits>

namespace q4 {

template <typename T16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    if constexpr (std::is_same<T16, __half>::value) {
        __half2 h = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&h);
    } else {
        __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&h);
    }
}

// Eight weights of one column times s (both lanes of s2) as four 16-bit pairs
// (k, k+1), processed as packed f32x2.
template <typename T16>
__device__ __forceinline__ uint4 dequant_word(uint32_t q, float2 s2) {
    const uint32_t lo = (q ^ 0x88888888u) & 0x0F0F0F0Fu;         // k = 0, 2, 4, 6
    const uint32_t hi = ((q >> 4) ^ 0x08080808u) & 0x0F0F0F0Fu;  // k = 1, 3, 5, 7
    const float2 nbias = make_float2(-8388616.0f, -8388616.0f);   // -(2^23 + 8)
    uint32_t out[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        // byte_perm selector 0x744b: byte b -> byte 0, zeros -> bytes 1-2,
        // 0x4B (the exponent byte of 2^23) -> byte 3.
        const float2 mg = make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7440u | static_cast<uint32_t>(b))),
                                      __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7440u | static_cast<uint32_t>(b))));
        const float2 w = __fmul2_rn(__fadd2_rn(mg, nbias), s2);
        out[b] = pack2<T16>(w.x, w.y);
    }
    return make_uint4(out[0], out[1], out[2], out[3]);
}

// Eight weights of one column as four f16 pairs (k, k+1) in f16x2
// arithmetic: per byte b (nibbles k = 2b, 2b+1), one PRMT puts the byte in
// both halves, one LOP3 keeps the low nibble in the low half and the high
// nibble in the high half with the sign bit flipped (u ^ 8 = v + 8) under the
// f16 exponent of 1024, i.e. (1032 + v0, 1152 + 16 v1); one HFMA2 with
// (1, 1/16) and (-1032, -72) gives (v0, v1) exactly.  The group scale s
// arrives split as s = s_hi + s_lo (two f16 values, split_scale_f16), and
// w = fma(v, s_hi, RN16(v * s_lo)) rounds v * s once to f16: the argument of
// that final rounding differs from v * s by about 2^-21 relative, so the
// result is RN16(v * s) except when v * s lies within that distance of a
// rounding midpoint.  20 instructions per word against ~36 for the fp32 path.
// (Rounding the scale to f16 first and then the product, RN16(v * RN16(s)),
// would cost one instruction less per pair but doubles the weight's rounding
// error: on a 128 x 64 x 256 product with N(0,1) activations and scales in
// [0.01, 0.05], the elementwise error |y - ref| / max(1, |ref|) grows from
// 1.9e-3 to 2.6e-3.)
__device__ __forceinline__ uint4 dequant_word_f16x2(uint32_t q, __half2 s_hi, __half2 s_lo) {
    const __half2 mul = __halves2half2(__ushort_as_half(0x3C00u), __ushort_as_half(0x2C00u));  // 1, 1/16
    const __half2 add = __halves2half2(__ushort_as_half(0xE408u), __ushort_as_half(0xD480u));  // -1032, -72
    uint32_t out[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        const uint32_t both = __byte_perm(q, 0u, 0x4040u | (static_cast<uint32_t>(b) << 8) | static_cast<uint32_t>(b));
        const uint32_t t = ((both ^ 0x00800008u) & 0x00F0000Fu) | 0x64006400u;
        const __half2 v = __hfma2(*reinterpret_cast<const __half2*>(&t), mul, add);
        const __half2 w = __hfma2(v, s_hi, __hmul2(v, s_lo));
        out[b] = *reinterpret_cast<const uint32_t*>(&w);
    }
    return make_uint4(out[0], out[1], out[2], out[3]);
}

// s = hi + lo in f16 (both lanes), hi = RN16(s), lo = RN16(s - hi).
__device__ __forceinline__ void split_scale_f16(float s, __half2& hi, __half2& lo) {
    const __half h = __float2half_rn(s);
    hi = __half2half2(h);
    lo = __float2half2_rn(s - __half2float(h));
}

// f16 operands take the f16x2 path, bf16 operands the fp32 one.
template <typename T16>
__device__ __forceinline__ uint4 dequant_f16x2_or(uint32_t q, float2 s2, __half2 s_hi, __half2 s_lo) {
    if constexpr (std::is_same<T16, __half>::value) {
        return dequant_word_f16x2(q, s_hi, s_lo);
    } else {
        return dequant_word<T16>(q, s2);
    }
}

__device__ __forceinline__ float exp2i(int e) { return __int_as_float((127 + e) << 23); }

}  // namespace q4

// codec.cuh -- device-side 8-bit codecs.
//
// compat_*: bit-exact restatement of the reference FP8E4M3 / FP8E5M2 classes
//   (include/cuda/quantize/fp8_types.hpp:64-115 and :147-207), written on the
//   float's integer fields instead of frexp/round/ldexp.  For a normal float
//   with biased exponent E and mantissa M, frexp gives mant = (2^23+M)/2^24
//   and exponent E-126, so:
//     E4M3: exp = E-120; normal mantissa round-half-away of M/2^20 with the
//           carry dropped (fp8_types.hpp:94); exp in [-3,0] keeps
//           (2^23+M) >> (19+exp) masked to 7 bits (:78-84); exp >= 15 -> Inf.
//     E5M2: exp = E-112; rounding of M/2^21 with the carry propagated
//           (:177-186); exp in [-2,0] keeps (2^23+M) >> (20+exp) (:161-167).
//   Float subnormals fall below the smallest kept exponent and give +-0.
// ocp_*: OCP E4M3FN / E5M2 with round-to-nearest-even and saturation, done by
//   the hardware conversion (cvt.rn.satfinite.{e4m3,e5m2}x2.f32).
// int8: cvt.rni (round to nearest even) and clamp to [-127, 127]
//   (int8_kernels.cu:30-35).
#pragma once

#include <cfloat>
#include <cuda_fp16.h>
#include <stdint.h>

namespace nq {
namespace dev {

enum Fmt : int { kE4M3 = 0, kE5M2 = 1, kINT8 = 2 };

template <int F>
struct FmtTraits;
template <>
struct FmtTraits<kE4M3> { static constexpr float qmax = 448.0f; };
template <>
struct FmtTraits<kE5M2> { static constexpr float qmax = 57344.0f; };
template <>
struct FmtTraits<kINT8> { static constexpr float qmax = 127.0f; };

__device__ __forceinline__ uint32_t compat_e4m3_encode(float f) {
    const uint32_t u = __float_as_uint(f);
    const uint32_t sign = (u >> 31) << 7;
    const uint32_t E = (u >> 23) & 0xFFu, M = u & 0x7FFFFFu;
    if (E == 0xFFu) return M ? 0x7Du : (sign | 0x7Cu);
    const int exp = static_cast<int>(E) - 120;
    if (exp < -3) return sign;  // zero, float subnormals and tiny values
    if (exp <= 0) return sign | (((0x800000u | M) >> (19 + exp)) & 0x7Fu);
    if (exp >= 15) return sign | 0x7Cu;
    const uint32_t r = (M + (1u << 19)) >> 20;
    return sign | (static_cast<uint32_t>(exp) << 3) | (r & 7u);
}

__device__ __forceinline__ uint32_t compat_e5m2_encode(float f) {
    const uint32_t u = __float_as_uint(f);
    const uint32_t sign = (u >> 31) << 7;
    const uint32_t E = (u >> 23) & 0xFFu, M = u & 0x7FFFFFu;
    if (E == 0xFFu) return M ? 0x7Du : (sign | 0x7Cu);
    int exp = static_cast<int>(E) - 112;
    if (exp < -2) return sign;
    if (exp <= 0) return sign | (((0x800000u | M) >> (20 + exp)) & 0x7Fu);
    if (exp >= 31) return sign | 0x7Cu;
    uint32_t r = (M + (1u << 20)) >> 21;
    if (r >= 4u) {
        r = 0;
        ++exp;
        if (exp >= 31) return sign | 0x7Cu;
    }
    return sign | (static_cast<uint32_t>(exp) << 2) | r;
}

// fp8_types.hpp:99-115: exponent field 0 is read as a normal number.
__device__ __forceinline__ float compat_e4m3_decode(uint32_t b) {
    if ((b & 0x7Fu) == 0) return __uint_as_float((b & 0x80u) << 24);  // +-0
    if (b == 0x7Cu) return __uint_as_float(0x7F800000u);
    if (b == 0xFCu) return __uint_as_float(0xFF800000u);
    if (b == 0x7Du) return __uint_as_float(0x7FC00000u);
    const uint32_t e = (b >> 3) & 0xFu, m = b & 7u;
    return __uint_as_float(((b & 0x80u) << 24) | ((e + 120u) << 23) | (m << 20));
}
// fp8_types.hpp:191-207
__device__ __forceinline__ float compat_e5m2_decode(uint32_t b) {
    if ((b & 0x7Fu) == 0) return __uint_as_float((b & 0x80u) << 24);
    if (b == 0x7Cu) return __uint_as_float(0x7F800000u);
    if (b == 0xFCu) return __uint_as_float(0xFF800000u);
    if (b == 0x7Du) return __uint_as_float(0x7FC00000u);
    const uint32_t e = (b >> 2) & 0x1Fu, m = b & 3u;
    return __uint_as_float(((b & 0x80u) << 24) | ((e + 112u) << 23) | (m << 21));
}

// Two floats -> two OCP codes, lo in bits [0,8), hi in bits [8,16).
template <int F>
__device__ __forceinline__ uint32_t ocp_encode2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t ocp_encode2<kE4M3>(float lo, float hi) {
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
    return r;
}
template <>
__device__ __forceinline__ uint32_t ocp_encode2<kE5M2>(float lo, float hi) {
    uint16_t r;
    asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
    return r;
}
__device__ __forceinline__ uint32_t int8_encode(float v) {
    int q = __float2int_rn(v);
    q = max(-127, min(127, q));
    return static_cast<uint32_t>(q) & 0xFFu;
}
template <>
__device__ __forceinline__ uint32_t ocp_encode2<kINT8>(float lo, float hi) {
    return int8_encode(lo) | (int8_encode(hi) << 8);
}

// Two OCP codes (lo byte, hi byte of `pair`) -> two floats.
template <int F>
__device__ __forceinline__ float2 ocp_decode2(uint32_t pair);
template <>
__device__ __forceinline__ float2 ocp_decode2<kE4M3>(uint32_t pair) {
    uint32_t h2;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(static_cast<uint16_t>(pair)));
    return __half22float2(*reinterpret_cast<__half2*>(&h2));
}
template <>
__device__ __forceinline__ float2 ocp_decode2<kE5M2>(uint32_t pair) {
    uint32_t h2;
    asm("cvt.rn.f16x2.e5m2x2 %0, %1;" : "=r"(h2) : "h"(static_cast<uint16_t>(pair)));
    return __half22float2(*reinterpret_cast<__half2*>(&h2));
}
template <>
__device__ __forceinline__ float2 ocp_decode2<kINT8>(uint32_t pair) {
    return make_float2(static_cast<float>(static_cast<int8_t>(pair & 0xFFu)),
                       static_cast<float>(static_cast<int8_t>((pair >> 8) & 0xFFu)));
}

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t h) { return __uint_as_float(h << 16); }

// fp32 -> bf16 bits, round to nearest even (hardware cvt.rn.bf16x2.f32).
__device__ __forceinline__ uint32_t f32x2_to_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// Per-row / per-column scaling: scale = amax / qmax (1 for an all-zero row)
// and q = encode(x * inv) with inv = qmax / amax, one IEEE division per row.
// When qmax / amax overflows (amax < qmax / FLT_MAX) the row is divided by
// its scale instead, so a row of tiny values never meets an infinite
// multiplier.  The choice is uniform over a row, so it costs no divergence.
struct RowScale {
    float s, inv;
    bool mul;
};
template <int F>
__device__ __forceinline__ RowScale row_scale(float a) {
    constexpr float q = FmtTraits<F>::qmax;
    if (!(a > 0.0f)) return RowScale{1.0f, 1.0f, true};
    const float inv = q / a;
    return RowScale{a / q, inv, inv <= FLT_MAX};
}
template <bool MUL>
__device__ __forceinline__ float scale_apply(float x, const RowScale& r) {
    return MUL ? x * r.inv : x / r.s;
}

// Element e of a 16-byte vector of fp32 (4) or bf16 (8) values.
template <class In>
__device__ __forceinline__ float vec_elem(const uint4& q, int e) {
    constexpr int EPV = 16 / sizeof(In);
    const uint32_t w = e < EPV / 4 ? q.x : (e < EPV / 2 ? q.y : (e < 3 * EPV / 4 ? q.z : q.w));
    if (sizeof(In) == 2) return __uint_as_float((e & 1) ? (w & 0xFFFF0000u) : (w << 16));
    return __uint_as_float(w);
}
template <int F, class In, bool MUL>
__device__ __forceinline__ void encode_vec(const uint4& q, uint8_t* out, const RowScale& r) {
    constexpr int EPV = 16 / sizeof(In);
    uint32_t codes[EPV / 2];
#pragma unroll
    for (int e = 0; e < EPV; e += 2)
        codes[e / 2] = ocp_encode2<F>(scale_apply<MUL>(vec_elem<In>(q, e), r),
                                           scale_apply<MUL>(vec_elem<In>(q, e + 1), r));
    if (EPV == 8) *reinterpret_cast<uint2*>(out) = make_uint2(codes[0] | (codes[1] << 16), codes[2] | (codes[3] << 16));
    else *reinterpret_cast<uint32_t*>(out) = codes[0] | (codes[1] << 16);
}

}  // namespace dev
}  // namespace nq

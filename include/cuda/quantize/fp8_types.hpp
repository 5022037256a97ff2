// fp8_types.hpp -- drop-in for pplmx/nova include/cuda/quantize/fp8_types.hpp.
//
// FP8E4M3 / FP8E5M2 keep the reference's public surface (uint8_t value,
// explicit float constructor, explicit operator float, from_bits, to_bits,
// POS_INF / NEG_INF / NAN_VAL / NEG_ZERO / MAX_NORMAL / MIN_NORMAL / EXP_BIAS /
// MANTISSA_BITS, fp8_types.hpp:35-208) and produce bit-identical codes: the
// codec is computed on the float's integer fields (exponent E, mantissa M).
//   E4M3: exp = E - 120; exp in [-3, 0] keeps ((2^23 + M) >> (19 + exp)) & 0x7F
//         (the reference's subnormal path, :78-84); exp >= 15 gives Inf (:86);
//         otherwise the mantissa is M / 2^20 rounded half away from zero with
//         the carry dropped (:94).
//   E5M2: exp = E - 112; exp in [-2, 0] keeps ((2^23 + M) >> (20 + exp)) & 0x7F;
//         exp >= 31 gives Inf; M / 2^21 rounded half away, carry propagated
//         (:179-186).
// Decoding reads every code other than 0, 0x80, 0x7C, 0xFC, 0x7D as
// (1 + m / 2^mbits) * 2^(e - bias), exponent field 0 included (:99-115).
// The tensor-core paths of libnova_q use OCP E4M3FN / E5M2 (nova_q.h).
#ifndef NOVA_B200_FP8_TYPES_HPP
#define NOVA_B200_FP8_TYPES_HPP

#include <cstdint>
#include <cstring>
#include <type_traits>

#if defined(__CUDACC__)
#define NOVA_HD __host__ __device__
#else
#define NOVA_HD
#endif

namespace nova {
namespace quantize {

namespace fp8_detail {
NOVA_HD inline uint32_t bits_of(float f) {
#if defined(__CUDA_ARCH__)
    return __float_as_uint(f);
#else
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return u;
#endif
}
NOVA_HD inline float float_of(uint32_t u) {
#if defined(__CUDA_ARCH__)
    return __uint_as_float(u);
#else
    float f;
    std::memcpy(&f, &u, 4);
    return f;
#endif
}
}  // namespace fp8_detail

class FP8E4M3 {
public:
    uint8_t value;

    NOVA_HD FP8E4M3() : value(0) {}
    NOVA_HD explicit FP8E4M3(float f) : value(encode(f)) {}
    NOVA_HD explicit operator float() const { return decode(value); }
    NOVA_HD static FP8E4M3 from_bits(uint8_t bits) {
        FP8E4M3 r;
        r.value = bits;
        return r;
    }
    NOVA_HD uint8_t to_bits() const { return value; }

    static constexpr uint8_t POS_INF = 0x7C;
    static constexpr uint8_t NEG_INF = 0xFC;
    static constexpr uint8_t NAN_VAL = 0x7D;
    static constexpr uint8_t NEG_ZERO = 0x80;
    static constexpr float MAX_NORMAL = 240.0f;
    static constexpr float MIN_NORMAL = 0.015625f;
    static constexpr int EXP_BIAS = 7;
    static constexpr int MANTISSA_BITS = 3;

private:
    NOVA_HD static uint8_t encode(float f) {
        const uint32_t u = fp8_detail::bits_of(f);
        const uint32_t sign = (u >> 31) << 7;
        const uint32_t E = (u >> 23) & 0xFFu, M = u & 0x7FFFFFu;
        if (E == 0xFFu) return static_cast<uint8_t>(M ? NAN_VAL : (sign | POS_INF));
        const int exp = static_cast<int>(E) - 120;
        if (exp < -3) return static_cast<uint8_t>(sign);
        if (exp <= 0) return static_cast<uint8_t>(sign | (((0x800000u | M) >> (19 + exp)) & 0x7Fu));
        if (exp >= 15) return static_cast<uint8_t>(sign | POS_INF);
        const uint32_t r = (M + (1u << 19)) >> 20;
        return static_cast<uint8_t>(sign | (static_cast<uint32_t>(exp) << 3) | (r & 7u));
    }
    NOVA_HD static float decode(uint8_t b) {
        if ((b & 0x7Fu) == 0) return fp8_detail::float_of(static_cast<uint32_t>(b & 0x80u) << 24);
        if (b == POS_INF) return fp8_detail::float_of(0x7F800000u);
        if (b == NEG_INF) return fp8_detail::float_of(0xFF800000u);
        if (b == NAN_VAL) return fp8_detail::float_of(0x7FC00000u);
        const uint32_t e = (b >> 3) & 0xFu, m = b & 7u;
        return fp8_detail::float_of((static_cast<uint32_t>(b & 0x80u) << 24) | ((e + 120u) << 23) | (m << 20));
    }
};

class FP8E5M2 {
public:
    uint8_t value;

    NOVA_HD FP8E5M2() : value(0) {}
    NOVA_HD explicit FP8E5M2(float f) : value(encode(f)) {}
    NOVA_HD explicit operator float() const { return decode(value); }
    NOVA_HD static FP8E5M2 from_bits(uint8_t bits) {
        FP8E5M2 r;
        r.value = bits;
        return r;
    }
    NOVA_HD uint8_t to_bits() const { return value; }

    static constexpr uint8_t POS_INF = 0x7C;
    static constexpr uint8_t NEG_INF = 0xFC;
    static constexpr uint8_t NAN_VAL = 0x7D;
    static constexpr uint8_t NEG_ZERO = 0x80;
    static constexpr float MAX_NORMAL = 57344.0f;
    static constexpr float MIN_NORMAL = 5.9604644775390625e-5f;
    static constexpr int EXP_BIAS = 15;
    static constexpr int MANTISSA_BITS = 2;

private:
    NOVA_HD static uint8_t encode(float f) {
        const uint32_t u = fp8_detail::bits_of(f);
        const uint32_t sign = (u >> 31) << 7;
        const uint32_t E = (u >> 23) & 0xFFu, M = u & 0x7FFFFFu;
        if (E == 0xFFu) return static_cast<uint8_t>(M ? NAN_VAL : (sign | POS_INF));
        int exp = static_cast<int>(E) - 112;
        if (exp < -2) return static_cast<uint8_t>(sign);
        if (exp <= 0) return static_cast<uint8_t>(sign | (((0x800000u | M) >> (20 + exp)) & 0x7Fu));
        if (exp >= 31) return static_cast<uint8_t>(sign | POS_INF);
        uint32_t r = (M + (1u << 20)) >> 21;
        if (r >= 4u) {
            r = 0;
            if (++exp >= 31) return static_cast<uint8_t>(sign | POS_INF);
        }
        return static_cast<uint8_t>(sign | (static_cast<uint32_t>(exp) << 2) | r);
    }
    NOVA_HD static float decode(uint8_t b) {
        if ((b & 0x7Fu) == 0) return fp8_detail::float_of(static_cast<uint32_t>(b & 0x80u) << 24);
        if (b == POS_INF) return fp8_detail::float_of(0x7F800000u);
        if (b == NEG_INF) return fp8_detail::float_of(0xFF800000u);
        if (b == NAN_VAL) return fp8_detail::float_of(0x7FC00000u);
        const uint32_t e = (b >> 2) & 0x1Fu, m = b & 3u;
        return fp8_detail::float_of((static_cast<uint32_t>(b & 0x80u) << 24) | ((e + 112u) << 23) | (m << 21));
    }
};

template <typename T>
struct is_fp8_type : std::false_type {};
template <>
struct is_fp8_type<FP8E4M3> : std::true_type {};
template <>
struct is_fp8_type<FP8E5M2> : std::true_type {};
template <typename T>
inline constexpr bool is_fp8_type_v = is_fp8_type<T>::value;

static_assert(sizeof(FP8E4M3) == 1 && sizeof(FP8E5M2) == 1, "FP8 types are one byte, as in the reference");

}  // namespace quantize
}  // namespace nova

#endif

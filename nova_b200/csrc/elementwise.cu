// elementwise.cu -- quantize / dequantize kernels (HBM-bound).
//
// Every kernel streams its input with 128-bit loads and writes 128-bit
// stores: one thread handles 16 elements per step (64 B of fp32 in and 16 B
// of codes out for a quantize), on a grid-stride loop over a grid sized to the
// SM count.  Tails (n % 16) and unaligned pointers take a scalar loop with the
// same arithmetic, so the result never depends on the path.  Also here: QAT
// fake quantize (fp32 -> fp32) and the activations on FP8 codes.
#include <algorithm>

#include "codec.cuh"
#include "nq_internal.h"

namespace nq {
namespace {

using dev::Fmt;

__device__ __forceinline__ bool dev_aligned16(const void* p) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// ---- vector load / store of 16 elements --------------------------------------
__device__ __forceinline__ void load16(const float* p, float (&x)[16]) {
    const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float4 v = __ldg(q + i);
        x[4 * i] = v.x; x[4 * i + 1] = v.y; x[4 * i + 2] = v.z; x[4 * i + 3] = v.w;
    }
}
__device__ __forceinline__ void load16(const uint16_t* p, float (&x)[16]) {  // bf16 bits
    const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        uint4 v = __ldg(q + i);
        uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            x[8 * i + 2 * j] = __uint_as_float(w[j] << 16);
            x[8 * i + 2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
        }
    }
}
__device__ __forceinline__ float load1(const float* p) { return __ldg(p); }
__device__ __forceinline__ float load1(const uint16_t* p) {
    return __uint_as_float(static_cast<uint32_t>(__ldg(p)) << 16);
}
__device__ __forceinline__ void store16_codes(uint8_t* p, const uint32_t (&c)[16]) {
    uint4 v;
    v.x = c[0] | (c[1] << 8) | (c[2] << 16) | (c[3] << 24);
    v.y = c[4] | (c[5] << 8) | (c[6] << 16) | (c[7] << 24);
    v.z = c[8] | (c[9] << 8) | (c[10] << 16) | (c[11] << 24);
    v.w = c[12] | (c[13] << 8) | (c[14] << 16) | (c[15] << 24);
    *reinterpret_cast<uint4*>(p) = v;
}
__device__ __forceinline__ void load16_codes(const uint8_t* p, uint32_t (&c)[16]) {
    uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
    uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 16; ++i) c[i] = (w[i >> 2] >> (8 * (i & 3))) & 0xFFu;
}
__device__ __forceinline__ void store16(float* p, const float (&y)[16]) {
    float4* q = reinterpret_cast<float4*>(p);
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = make_float4(y[4 * i], y[4 * i + 1], y[4 * i + 2], y[4 * i + 3]);
}

// ---- element ops ---------------------------------------------------------------
// Each op maps one input value to one output; quantize ops produce a code.
struct CompatE4M3 {
    __device__ uint32_t operator()(float x) const { return dev::compat_e4m3_encode(x); }
};
struct CompatE5M2 {
    __device__ uint32_t operator()(float x) const { return dev::compat_e5m2_encode(x); }
};
// int8_kernels.cu:29-35: IEEE division (no fast math), RNE, clamp +-127
struct Int8Sym {
    float scale;
    __device__ uint32_t operator()(float x) const { return dev::int8_encode(x / scale); }
};
struct Int8Asym {
    float scale, zp;
    __device__ uint32_t operator()(float x) const { return dev::int8_encode((x - zp) / scale); }
};
// int8_kernels.cu:182-193: s = range/254, q = rn((x - min)/s - 127), 0 if range < 1e-6
struct Int8Calib {
    float min_val, range;
    __device__ uint32_t operator()(float x) const {
        if (range < 1e-6f) return 0u;
        const float s = range / 254.0f;
        return dev::int8_encode(__fsub_rn((x - min_val) / s, 127.0f));
    }
};
// quantize_tensor.hpp:176-182: std::round (half away from zero), clamp +-127
struct Int8RoundAway {
    float scale;
    __device__ uint32_t operator()(float x) const {
        float r = roundf(x / scale);
        r = fmaxf(-127.0f, fminf(127.0f, r));
        return static_cast<uint32_t>(static_cast<int>(r)) & 0xFFu;
    }
};

template <class Op, class In>
__global__ void __launch_bounds__(256) k_quant(const In* __restrict__ src, uint8_t* __restrict__ dst,
                                               size_t n, int vec, Op op) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    const size_t t0 = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const size_t nvec = vec ? n / 16 : 0;
    for (size_t v = t0; v < nvec; v += stride) {
        float x[16];
        load16(src + v * 16, x);
        uint32_t c[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) c[i] = op(x[i]);
        store16_codes(dst + v * 16, c);
    }
    for (size_t i = nvec * 16 + t0; i < n; i += stride) dst[i] = static_cast<uint8_t>(op(load1(src + i)));
}

// Reference-codec FP8 encode by table.  The code of a float that is not NaN
// depends only on its sign, exponent and top 7 mantissa bits (bits 31..16): the
// rounding of fp8_types.hpp:90-95 / :177-186 looks at mantissa bits 22..19
// (E4M3) or 22..20 (E5M2), the reduced range at bits 22..16 / 22..18.  Only
// exponents [LO, HI) need the encoder -- below them the code is 0, from HI on
// 0x7C -- so a table of (HI - LO + 2) rows of 128 bytes in shared memory (2.5 KB
// for E4M3, 4.2 KB for E5M2), indexed by the clamped exponent and the 7 bits and
// ORed with the sign, replaces the ~20 integer operations of
// dev::compat_e4m3_encode per element.  Measured on B200 at 224 Mi elements:
// 71% of HBM with the integer encode, 77% with a 32 KB table over bits 30..16
// (six CTAs per SM), 87.5% with this one (eight).  NaN (code 0x7D, no sign) is
// tested apart, since its low mantissa bits decide it.
template <int F>
__global__ void __launch_bounds__(256) k_quant_compat_lut(const float* __restrict__ src, uint8_t* __restrict__ dst,
                                                          size_t n, int vec) {
    constexpr int LO = F == dev::kE4M3 ? 117 : 110;
    constexpr int HI = F == dev::kE4M3 ? 135 : 143;
    constexpr int ROWS = HI - LO + 2;  // row 0: exponents below LO (code 0); last: HI and above (0x7C)
    __shared__ __align__(16) uint8_t lut[ROWS * 128];
    for (int i = threadIdx.x; i < ROWS * 128; i += blockDim.x) {
        const int r = i >> 7, m = i & 127;
        uint32_t v = r == 0 ? 0u : 0x7Cu;
        if (r > 0 && r < ROWS - 1) {
            const float f = __uint_as_float((static_cast<uint32_t>(r - 1 + LO) << 23) | (static_cast<uint32_t>(m) << 16));
            v = F == dev::kE4M3 ? dev::compat_e4m3_encode(f) : dev::compat_e5m2_encode(f);
        }
        lut[i] = static_cast<uint8_t>(v);
    }
    __syncthreads();
    auto enc = [&](float x) -> uint32_t {
        const uint32_t u = __float_as_uint(x);
        const int e = static_cast<int>((u >> 23) & 0xFFu);
        const int r = min(max(e - (LO - 1), 0), ROWS - 1);
        const uint32_t c = static_cast<uint32_t>(lut[(r << 7) | ((u >> 16) & 0x7Fu)]) | ((u >> 24) & 0x80u);
        return x != x ? 0x7Du : c;
    };
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    const size_t t0 = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const size_t nvec = vec ? n / 16 : 0;
    for (size_t v = t0; v < nvec; v += stride) {
        float x[16];
        load16(src + v * 16, x);
        uint32_t c[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) c[i] = enc(x[i]);
        store16_codes(dst + v * 16, c);
    }
    for (size_t i = nvec * 16 + t0; i < n; i += stride) dst[i] = static_cast<uint8_t>(enc(load1(src + i)));
}

// Scaled OCP / INT8 quantize, the scale read from device memory.
template <int F, class In>
__global__ void __launch_bounds__(256) k_quant_scaled(const In* __restrict__ src,
                                                      uint8_t* __restrict__ dst, size_t n, int vec,
                                                      const float* __restrict__ d_scale) {
    const float s = __ldg(d_scale);
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    const size_t t0 = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const size_t nvec = vec ? n / 16 : 0;
    for (size_t v = t0; v < nvec; v += stride) {
        float x[16];
        load16(src + v * 16, x);
        uint32_t c[16];
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
            uint32_t p = dev::ocp_encode2<F>(x[i] / s, x[i + 1] / s);
            c[i] = p & 0xFFu;
            c[i + 1] = p >> 8;
        }
        store16_codes(dst + v * 16, c);
    }
    for (size_t i = nvec * 16 + t0; i < n; i += stride)
        dst[i] = static_cast<uint8_t>(dev::ocp_encode2<F>(load1(src + i) / s, 0.0f) & 0xFFu);
}

// ---- dequantize ---------------------------------------------------------------
struct DecCompatE4M3 {
    float scale;
    __device__ float operator()(uint32_t c) const { return dev::compat_e4m3_decode(c) * scale; }
};
struct DecCompatE5M2 {
    float scale;
    __device__ float operator()(uint32_t c) const { return dev::compat_e5m2_decode(c) * scale; }
};
// int8_kernels.cu:53-57
struct DecInt8Sym {
    float scale;
    __device__ float operator()(uint32_t c) const {
        return static_cast<float>(static_cast<int8_t>(c)) * scale;
    }
};
struct DecInt8Asym {
    float scale, zp;
    __device__ float operator()(uint32_t c) const {
        return __fmul_rn(__fadd_rn(static_cast<float>(static_cast<int8_t>(c)), zp), scale);
    }
};
template <int F>
struct DecOcp {
    float scale;
    __device__ float operator()(uint32_t c) const { return dev::ocp_decode2<F>(c).x * scale; }
};

// Writes are four times the reads: each lane turns 4 codes (one 4-byte load)
// into one float4 store, so every warp store instruction covers 512
// contiguous bytes; four groups per step keep loads in flight.
template <class Op>
__global__ void __launch_bounds__(256) k_dequant(const uint8_t* __restrict__ src,
                                                 float* __restrict__ dst, size_t n, int vec, Op op) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    const size_t t0 = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const size_t ng = vec ? n / 4 : 0;
    const uint32_t* s4 = reinterpret_cast<const uint32_t*>(src);
    float4* d4 = reinterpret_cast<float4*>(dst);
    size_t g = t0;
    for (; g + 3 * stride < ng; g += 4 * stride) {
        uint32_t w[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) w[u] = __ldg(s4 + g + u * stride);
#pragma unroll
        for (int u = 0; u < 4; ++u)
            d4[g + u * stride] = make_float4(op(w[u] & 0xFFu), op((w[u] >> 8) & 0xFFu), op((w[u] >> 16) & 0xFFu), op(w[u] >> 24));
    }
    for (; g < ng; g += stride) {
        const uint32_t w = __ldg(s4 + g);
        d4[g] = make_float4(op(w & 0xFFu), op((w >> 8) & 0xFFu), op((w >> 16) & 0xFFu), op(w >> 24));
    }
    for (size_t i = ng * 4 + t0; i < n; i += stride) dst[i] = op(__ldg(src + i));
}

template <class Op>
__global__ void __launch_bounds__(256) k_dequant_scaled(const uint8_t* __restrict__ src,
                                                        float* __restrict__ dst, size_t n, int vec,
                                                        const float* __restrict__ d_scale) {
    Op op{__ldg(d_scale)};
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    const size_t t0 = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const size_t nvec = vec ? n / 16 : 0;
    for (size_t v = t0; v < nvec; v += stride) {
        uint32_t c[16];
        load16_codes(src + v * 16, c);
        float y[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) y[i] = op(c[i]);
        store16(dst + v * 16, y);
    }
    for (size_t i = nvec * 16 + t0; i < n; i += stride) dst[i] = op(__ldg(src + i));
}

// ---- batched (fp8_kernels.cu:83-122): grid.y = tensor, grid.x strides ------------
__global__ void __launch_bounds__(256) k_quant_batched(const float* const* src, uint8_t* const* dst,
                                                       const size_t* sizes, const float* scales) {
    const int b = blockIdx.y;
    const float* s = src[b];
    uint8_t* d = dst[b];
    const size_t n = sizes[b];
    const float mul = scales[b];
    const bool vec = dev_aligned16(s) && dev_aligned16(d);
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    const size_t t0 = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const size_t nvec = vec ? n / 16 : 0;
    for (size_t v = t0; v < nvec; v += stride) {
        float x[16];
        load16(s + v * 16, x);
        uint32_t c[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) c[i] = dev::compat_e4m3_encode(x[i] * mul);
        store16_codes(d + v * 16, c);
    }
    for (size_t i = nvec * 16 + t0; i < n; i += stride)
        d[i] = static_cast<uint8_t>(dev::compat_e4m3_encode(__ldg(s + i) * mul));
}

__global__ void __launch_bounds__(256) k_dequant_batched(const uint8_t* const* src, float* const* dst,
                                                         const size_t* sizes, const float* scales) {
    const int b = blockIdx.y;
    const uint8_t* s = src[b];
    float* d = dst[b];
    const size_t n = sizes[b];
    const float mul = scales[b];
    const bool vec = dev_aligned16(s) && dev_aligned16(d);
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    const size_t t0 = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const size_t nvec = vec ? n / 16 : 0;
    for (size_t v = t0; v < nvec; v += stride) {
        uint32_t c[16];
        load16_codes(s + v * 16, c);
        float y[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) y[i] = dev::compat_e4m3_decode(c[i]) * mul;
        store16(d + v * 16, y);
    }
    for (size_t i = nvec * 16 + t0; i < n; i += stride) d[i] = dev::compat_e4m3_decode(__ldg(s + i)) * mul;
}

// FakeQuantize::forward of QAT (qat.hpp:64-72) over an array: scale floored at
// 1e-6, q = clamp(round_half_away((x - zp) / scale), +-127), y = q * scale + zp,
// each step rounded once (no FMA), as the reference's host expression.
__device__ __forceinline__ float fake_quant1(float x, float s, float zp) {
    const float r = roundf(__fdiv_rn(__fsub_rn(x, zp), s));
    const float c = fmaxf(-127.0f, fminf(127.0f, r));
    return __fadd_rn(__fmul_rn(c, s), zp);
}
__global__ void __launch_bounds__(256) k_fake_quant(const float* __restrict__ src, float* __restrict__ dst, size_t n,
                                                    int vec, float s, float zp) {
    const size_t t0 = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    const size_t n4 = vec ? n / 4 : 0;
    for (size_t v = t0; v < n4; v += stride) {
        const float4 x = __ldg(reinterpret_cast<const float4*>(src) + v);
        reinterpret_cast<float4*>(dst)[v] =
            make_float4(fake_quant1(x.x, s, zp), fake_quant1(x.y, s, zp), fake_quant1(x.z, s, zp), fake_quant1(x.w, s, zp));
    }
    for (size_t i = n4 * 4 + t0; i < n; i += stride) dst[i] = fake_quant1(__ldg(src + i), s, zp);
}

// Element-wise activations on FP8 codes of the reference codec
// (fp8_activation.hpp:26-59 of pplmx/nova): decode, activate in fp32 with the
// reference's expressions, re-encode; relu returns negative inputs as +0 and
// every other input code unchanged.  16 codes per thread step.
template <bool E4M3, int OP>
__device__ __forceinline__ uint32_t fp8_act1(uint32_t c, float alpha) {
    const float x = E4M3 ? dev::compat_e4m3_decode(c) : dev::compat_e5m2_decode(c);
    float y;
    if (OP == NQ_ACT_RELU) {
        if (!(x < 0.0f)) return c;
        y = 0.0f;
    } else if (OP == NQ_ACT_GELU) {
        const float cdf = 0.5f * (1.0f + erff(x * 0.7071067811865476f));
        y = x * cdf;
    } else if (OP == NQ_ACT_SIGMOID) {
        y = 1.0f / (1.0f + expf(-x));
    } else {
        y = x >= 0.0f ? x : alpha * x;
    }
    return E4M3 ? dev::compat_e4m3_encode(y) : dev::compat_e5m2_encode(y);
}
template <bool E4M3, int OP>
__global__ void __launch_bounds__(256) k_fp8_act(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, size_t n,
                                                 int vec, float alpha) {
    const size_t t0 = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    const size_t n16 = vec ? n / 16 : 0;
    for (size_t v = t0; v < n16; v += stride) {
        uint4 q = __ldg(reinterpret_cast<const uint4*>(src) + v);
        uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint32_t o = 0;
#pragma unroll
            for (int b = 0; b < 4; ++b) o |= fp8_act1<E4M3, OP>((w[j] >> (8 * b)) & 0xFFu, alpha) << (8 * b);
            w[j] = o;
        }
        reinterpret_cast<uint4*>(dst)[v] = make_uint4(w[0], w[1], w[2], w[3]);
    }
    for (size_t i = n16 * 16 + t0; i < n; i += stride)
        dst[i] = static_cast<uint8_t>(fp8_act1<E4M3, OP>(__ldg(src + i), alpha));
}

// bf16 -> fp32, 8 values per thread step when both pointers are 16-byte aligned.
__global__ void __launch_bounds__(256) k_bf16_to_f32(const uint16_t* __restrict__ src, float* __restrict__ dst,
                                                     size_t n, int vec) {
    const size_t t0 = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    const size_t n8 = vec ? n / 8 : 0;
    for (size_t v = t0; v < n8; v += stride) {
        const uint4 q = __ldg(reinterpret_cast<const uint4*>(src) + v);
        float4* o = reinterpret_cast<float4*>(dst) + 2 * v;
        o[0] = make_float4(__uint_as_float(q.x << 16), __uint_as_float(q.x & 0xFFFF0000u),
                           __uint_as_float(q.y << 16), __uint_as_float(q.y & 0xFFFF0000u));
        o[1] = make_float4(__uint_as_float(q.z << 16), __uint_as_float(q.z & 0xFFFF0000u),
                           __uint_as_float(q.w << 16), __uint_as_float(q.w & 0xFFFF0000u));
    }
    for (size_t i = n8 * 8 + t0; i < n; i += stride) dst[i] = __uint_as_float(static_cast<uint32_t>(__ldg(src + i)) << 16);
}

// ---- launch helpers ------------------------------------------------------------------
nq_status_t grid_for(size_t n, int* grid) {
    DeviceInfo di;
    nq_status_t st = current_device(&di);
    if (st != NQ_SUCCESS) return st;
    const size_t work = (n + 15) / 16;
    const size_t want = (work + 255) / 256;
    const size_t cap = static_cast<size_t>(di.sm_count) * 8;  // 8 x 256 threads per SM
    *grid = static_cast<int>(std::max<size_t>(1, std::min(want, cap)));
    return NQ_SUCCESS;
}

template <class Op, class In>
nq_status_t launch_quant(const In* src, uint8_t* dst, size_t n, Op op, cudaStream_t s, const char* what) {
    if (n == 0) return NQ_SUCCESS;
    if (!src || !dst) return fail(NQ_ERROR_INVALID_VALUE, std::string(what) + ": null pointer");
    int grid;
    nq_status_t st = grid_for(n, &grid);
    if (st != NQ_SUCCESS) return st;
    const int vec = aligned16(src) && aligned16(dst);
    k_quant<Op, In><<<grid, 256, 0, s>>>(src, dst, n, vec, op);
    NQ_LAUNCH_CHECK(what);
    return NQ_SUCCESS;
}

// Tables pay off once every CTA has a few thousand elements to encode.
constexpr size_t kCompatLutMin = size_t(1) << 22;

template <int F>
nq_status_t launch_quant_compat(const float* src, uint8_t* dst, size_t n, cudaStream_t s, const char* what) {
    if (n < kCompatLutMin) {
        if (F == dev::kE4M3) return launch_quant(src, dst, n, CompatE4M3{}, s, what);
        return launch_quant(src, dst, n, CompatE5M2{}, s, what);
    }
    if (!src || !dst) return fail(NQ_ERROR_INVALID_VALUE, std::string(what) + ": null pointer");
    int grid;
    nq_status_t st = grid_for(n, &grid);
    if (st != NQ_SUCCESS) return st;
    const int vec = aligned16(src) && aligned16(dst);
    k_quant_compat_lut<F><<<grid, 256, 0, s>>>(src, dst, n, vec);
    NQ_LAUNCH_CHECK(what);
    return NQ_SUCCESS;
}

template <class Op>
nq_status_t launch_dequant(const uint8_t* src, float* dst, size_t n, Op op, cudaStream_t s, const char* what) {
    if (n == 0) return NQ_SUCCESS;
    if (!src || !dst) return fail(NQ_ERROR_INVALID_VALUE, std::string(what) + ": null pointer");
    int grid;
    nq_status_t st = grid_for(n, &grid);
    if (st != NQ_SUCCESS) return st;
    const int vec = aligned16(src) && aligned16(dst);
    k_dequant<Op><<<grid, 256, 0, s>>>(src, dst, n, vec, op);
    NQ_LAUNCH_CHECK(what);
    return NQ_SUCCESS;
}

template <int F>
nq_status_t launch_quant_scaled(const void* src, nq_dtype_t dt, uint8_t* dst, size_t n,
                                const float* d_scale, cudaStream_t s, int grid) {
    const int vec = aligned16(src) && aligned16(dst);
    if (dt == NQ_F32)
        k_quant_scaled<F, float><<<grid, 256, 0, s>>>(static_cast<const float*>(src), dst, n, vec, d_scale);
    else
        k_quant_scaled<F, uint16_t><<<grid, 256, 0, s>>>(static_cast<const uint16_t*>(src), dst, n, vec,
                                                         d_scale);
    NQ_LAUNCH_CHECK("nq_quantize_scaled");
    return NQ_SUCCESS;
}

}  // namespace

// Used by reduce.cu's calibrate+quantize pipeline.
nq_status_t quantize_scaled_impl(const void* src, nq_dtype_t dt, uint8_t* dst, size_t n, nq_format_t fmt,
                                 const float* d_scale, cudaStream_t s) {
    if (n == 0) return NQ_SUCCESS;
    if (!src || !dst || !d_scale) return fail(NQ_ERROR_INVALID_VALUE, "nq_quantize_scaled: null pointer");
    if (dt != NQ_F32 && dt != NQ_BF16) return fail(NQ_ERROR_INVALID_VALUE, "nq_quantize_scaled: src dtype");
    int grid;
    nq_status_t st = grid_for(n, &grid);
    if (st != NQ_SUCCESS) return st;
    switch (fmt) {
        case NQ_E4M3: return launch_quant_scaled<dev::kE4M3>(src, dt, dst, n, d_scale, s, grid);
        case NQ_E5M2: return launch_quant_scaled<dev::kE5M2>(src, dt, dst, n, d_scale, s, grid);
        case NQ_INT8: return launch_quant_scaled<dev::kINT8>(src, dt, dst, n, d_scale, s, grid);
    }
    return fail(NQ_ERROR_INVALID_VALUE, "nq_quantize_scaled: format");
}

}  // namespace nq

using nq::fail;

extern "C" {

nq_status_t nq_quantize_f32_to_fp8e4m3(const float* src, uint8_t* dst, size_t n, nq_stream_t s) {
    return nq::launch_quant_compat<nq::dev::kE4M3>(src, dst, n, s, "nq_quantize_f32_to_fp8e4m3");
}
nq_status_t nq_quantize_f32_to_fp8e5m2(const float* src, uint8_t* dst, size_t n, nq_stream_t s) {
    return nq::launch_quant_compat<nq::dev::kE5M2>(src, dst, n, s, "nq_quantize_f32_to_fp8e5m2");
}
nq_status_t nq_dequantize_fp8e4m3_to_f32(const uint8_t* src, float* dst, size_t n, float scale,
                                         nq_stream_t s) {
    return nq::launch_dequant(src, dst, n, nq::DecCompatE4M3{scale}, s, "nq_dequantize_fp8e4m3_to_f32");
}
nq_status_t nq_dequantize_fp8e5m2_to_f32(const uint8_t* src, float* dst, size_t n, float scale,
                                         nq_stream_t s) {
    return nq::launch_dequant(src, dst, n, nq::DecCompatE5M2{scale}, s, "nq_dequantize_fp8e5m2_to_f32");
}

nq_status_t nq_quantize_batched_f32_to_fp8e4m3(const float* const* src, uint8_t* const* dst, int batch,
                                               const size_t* sizes, const float* scales, nq_stream_t s) {
    if (batch == 0) return NQ_SUCCESS;
    if (batch < 0 || batch > 65535 || !src || !dst || !sizes || !scales)
        return fail(NQ_ERROR_INVALID_VALUE, "nq_quantize_batched_f32_to_fp8e4m3: bad arguments");
    nq::DeviceInfo di;
    nq_status_t st = nq::current_device(&di);
    if (st != NQ_SUCCESS) return st;
    dim3 grid(std::max(1, di.sm_count * 8 / batch), batch);
    nq::k_quant_batched<<<grid, 256, 0, s>>>(src, dst, sizes, scales);
    NQ_LAUNCH_CHECK("nq_quantize_batched_f32_to_fp8e4m3");
    return NQ_SUCCESS;
}

nq_status_t nq_dequantize_batched_fp8e4m3_to_f32(const uint8_t* const* src, float* const* dst, int batch,
                                                 const size_t* sizes, const float* scales, nq_stream_t s) {
    if (batch == 0) return NQ_SUCCESS;
    if (batch < 0 || batch > 65535 || !src || !dst || !sizes || !scales)
        return fail(NQ_ERROR_INVALID_VALUE, "nq_dequantize_batched_fp8e4m3_to_f32: bad arguments");
    nq::DeviceInfo di;
    nq_status_t st = nq::current_device(&di);
    if (st != NQ_SUCCESS) return st;
    dim3 grid(std::max(1, di.sm_count * 8 / batch), batch);
    nq::k_dequant_batched<<<grid, 256, 0, s>>>(src, dst, sizes, scales);
    NQ_LAUNCH_CHECK("nq_dequantize_batched_fp8e4m3_to_f32");
    return NQ_SUCCESS;
}

nq_status_t nq_quantize_f32_to_int8(const float* src, int8_t* dst, size_t n, float scale, float zero_point,
                                    int symmetric, nq_stream_t s) {
    uint8_t* d = reinterpret_cast<uint8_t*>(dst);
    if (symmetric) return nq::launch_quant(src, d, n, nq::Int8Sym{scale}, s, "nq_quantize_f32_to_int8");
    return nq::launch_quant(src, d, n, nq::Int8Asym{scale, zero_point}, s, "nq_quantize_f32_to_int8");
}

nq_status_t nq_dequantize_int8_to_f32(const int8_t* src, float* dst, size_t n, float scale, float zero_point,
                                      int symmetric, nq_stream_t s) {
    const uint8_t* q = reinterpret_cast<const uint8_t*>(src);
    if (symmetric) return nq::launch_dequant(q, dst, n, nq::DecInt8Sym{scale}, s, "nq_dequantize_int8_to_f32");
    return nq::launch_dequant(q, dst, n, nq::DecInt8Asym{scale, zero_point}, s, "nq_dequantize_int8_to_f32");
}

nq_status_t nq_quantize_f32_to_int8_with_calibration(const float* src, int8_t* dst, size_t n, float min_val,
                                                     float max_val, nq_stream_t s) {
    return nq::launch_quant(src, reinterpret_cast<uint8_t*>(dst), n, nq::Int8Calib{min_val, max_val - min_val}, s,
                            "nq_quantize_f32_to_int8_with_calibration");
}

nq_status_t nq_quantize_f32_to_int8_round_away(const float* src, int8_t* dst, size_t n, float scale,
                                               nq_stream_t s) {
    return nq::launch_quant(src, reinterpret_cast<uint8_t*>(dst), n, nq::Int8RoundAway{scale}, s,
                            "nq_quantize_f32_to_int8_round_away");
}

nq_status_t nq_fp8_activation(const uint8_t* src, uint8_t* dst, size_t n, nq_format_t fmt, nq_activation_t op,
                              float alpha, nq_stream_t s) {
    if (n == 0) return NQ_SUCCESS;
    if (!src || !dst) return fail(NQ_ERROR_INVALID_VALUE, "nq_fp8_activation: null pointer");
    if (fmt != NQ_E4M3 && fmt != NQ_E5M2) return fail(NQ_ERROR_INVALID_VALUE, "nq_fp8_activation: format");
    if (op < NQ_ACT_RELU || op > NQ_ACT_LEAKY_RELU) return fail(NQ_ERROR_INVALID_VALUE, "nq_fp8_activation: op");
    int grid;
    nq_status_t st = nq::grid_for(n, &grid);
    if (st != NQ_SUCCESS) return st;
    const int vec = nq::aligned16(src) && nq::aligned16(dst);
#define NQ_ACT(E, OP) nq::k_fp8_act<E, OP><<<grid, 256, 0, s>>>(src, dst, n, vec, alpha)
    if (fmt == NQ_E4M3) {
        switch (op) {
            case NQ_ACT_RELU: NQ_ACT(true, NQ_ACT_RELU); break;
            case NQ_ACT_GELU: NQ_ACT(true, NQ_ACT_GELU); break;
            case NQ_ACT_SIGMOID: NQ_ACT(true, NQ_ACT_SIGMOID); break;
            default: NQ_ACT(true, NQ_ACT_LEAKY_RELU); break;
        }
    } else {
        switch (op) {
            case NQ_ACT_RELU: NQ_ACT(false, NQ_ACT_RELU); break;
            case NQ_ACT_GELU: NQ_ACT(false, NQ_ACT_GELU); break;
            case NQ_ACT_SIGMOID: NQ_ACT(false, NQ_ACT_SIGMOID); break;
            default: NQ_ACT(false, NQ_ACT_LEAKY_RELU); break;
        }
    }
#undef NQ_ACT
    NQ_LAUNCH_CHECK("nq_fp8_activation");
    return NQ_SUCCESS;
}

nq_status_t nq_fake_quantize_int8(const float* src, float* dst, size_t n, float scale, float zero_point,
                                  nq_stream_t s) {
    if (n == 0) return NQ_SUCCESS;
    if (!src || !dst) return fail(NQ_ERROR_INVALID_VALUE, "nq_fake_quantize_int8: null pointer");
    int grid;
    nq_status_t st = nq::grid_for(n, &grid);
    if (st != NQ_SUCCESS) return st;
    const float sc = scale < 1e-6f ? 1e-6f : scale;  // FakeQuantize::forward's floor (qat.hpp:65-66)
    nq::k_fake_quant<<<grid, 256, 0, s>>>(src, dst, n, nq::aligned16(src) && nq::aligned16(dst), sc, zero_point);
    NQ_LAUNCH_CHECK("nq_fake_quantize_int8");
    return NQ_SUCCESS;
}

nq_status_t nq_quantize_scaled(const void* src, nq_dtype_t src_dtype, uint8_t* dst, size_t n, nq_format_t fmt,
                               const float* d_scale, nq_stream_t s) {
    return nq::quantize_scaled_impl(src, src_dtype, dst, n, fmt, d_scale, s);
}

nq_status_t nq_dequantize_scaled(const uint8_t* src, float* dst, size_t n, nq_format_t fmt, const float* d_scale,
                                 nq_stream_t s) {
    if (n == 0) return NQ_SUCCESS;
    if (!src || !dst || !d_scale) return fail(NQ_ERROR_INVALID_VALUE, "nq_dequantize_scaled: null pointer");
    int grid;
    nq_status_t st = nq::grid_for(n, &grid);
    if (st != NQ_SUCCESS) return st;
    const int vec = nq::aligned16(src) && nq::aligned16(dst);
    switch (fmt) {
        case NQ_E4M3: nq::k_dequant_scaled<nq::DecOcp<nq::dev::kE4M3>><<<grid, 256, 0, s>>>(src, dst, n, vec, d_scale); break;
        case NQ_E5M2: nq::k_dequant_scaled<nq::DecOcp<nq::dev::kE5M2>><<<grid, 256, 0, s>>>(src, dst, n, vec, d_scale); break;
        case NQ_INT8: nq::k_dequant_scaled<nq::DecInt8Sym><<<grid, 256, 0, s>>>(src, dst, n, vec, d_scale); break;
        default: return fail(NQ_ERROR_INVALID_VALUE, "nq_dequantize_scaled: format");
    }
    NQ_LAUNCH_CHECK("nq_dequantize_scaled");
    return NQ_SUCCESS;
}

nq_status_t nq_convert_bf16_to_f32(const void* src, float* dst, size_t n, nq_stream_t s) {
    if (n == 0) return NQ_SUCCESS;
    if (!src || !dst) return fail(NQ_ERROR_INVALID_VALUE, "nq_convert_bf16_to_f32: null pointer");
    int grid;
    nq_status_t st = nq::grid_for(n, &grid);
    if (st != NQ_SUCCESS) return st;
    const int vec = nq::aligned16(src) && nq::aligned16(dst);
    nq::k_bf16_to_f32<<<grid, 256, 0, s>>>(static_cast<const uint16_t*>(src), dst, n, vec);
    NQ_LAUNCH_CHECK("nq_convert_bf16_to_f32");
    return NQ_SUCCESS;
}

}  // extern "C"

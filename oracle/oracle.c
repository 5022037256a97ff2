/*
 * oracle.c -- CPU restatement of pplmx/nova's cuda::quantize path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for tests/, smoke() and bench.py's
 * CPU baseline.  The product never links or calls it.
 *
 * Compiled with -O2 -ffp-contract=off so that every float operation is one
 * IEEE round-to-nearest operation, like the device code it is compared
 * with; where the reference's device code is contracted to an FMA by nvcc
 * (its default -fmad=true), the restatement calls fmaf explicitly.
 */
#include "oracle.h"

#include <float.h>
#include <stdlib.h>
#include <math.h>
#include <pthread.h>
#include <string.h>

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* ======================================================================
 * Compat codec: bit-exact restatement of the reference encoder/decoder.
 *
 * E4M3 encode, include/cuda/quantize/fp8_types.hpp:64-97:
 *   sign from f<0 or -0 (:65-66); zero -> sign (:67); Inf -> sign|0x7C (:71);
 *   NaN -> 0x7D without sign (:72); frexp, exp += bias-1 (:74-76);
 *   exp <= 0: below -3 -> sign, else truncate mant*2^(5-exp) and keep 7 bits
 *   (:78-84, the bits overflow into the exponent field: a reference bug that
 *   is reproduced, not fixed); exp >= 15 -> Inf (:86-88);
 *   mantissa round half away (std::round) and the carry is DROPPED (& 7, :94).
 * Here frexp of a normal float with biased exponent E and mantissa M gives
 *   mant = (2^23+M)/2^24, exponent E-126, so exp = E-120 and
 *   (2*mant-1)*8 = M/2^20; all quantities are computed on the integers.
 * ==================================================================== */
uint8_t orc_e4m3_compat_encode(float f) {
    uint32_t u = f2u(f);
    uint32_t sign = (u >> 31) ? 0x80u : 0u;
    uint32_t E = (u >> 23) & 0xFF, M = u & 0x7FFFFF;
    if (E == 0 && M == 0) return (uint8_t)sign;           /* +-0           */
    if (E == 0xFF) return M ? 0x7D : (uint8_t)(sign | 0x7C); /* NaN / Inf   */
    if (E == 0) return (uint8_t)sign;                     /* f32 denormal: exp < -3 */
    int exp = (int)E - 120;
    if (exp <= 0) {
        if (exp < -3) return (uint8_t)sign;
        uint32_t m = (0x800000u | M) >> (19 + exp);
        return (uint8_t)(sign | (m & 0x7F));
    }
    if (exp >= 15) return (uint8_t)(sign | 0x7C);
    uint32_t r = (M + (1u << 19)) >> 20;                  /* half away from zero */
    return (uint8_t)(sign | ((uint32_t)exp << 3) | (r & 7));
}

/* E4M3 decode, fp8_types.hpp:99-115: 0 / 0x80 / 0x7C / 0xFC / 0x7D special,
   every other code (exponent field 0 included) is (1+m/8)*2^(e-7). */
float orc_e4m3_compat_decode(uint8_t b) {
    if (b == 0) return 0.0f;
    if (b == 0x80) return -0.0f;
    if (b == 0x7C) return INFINITY;
    if (b == 0xFC) return -INFINITY;
    if (b == 0x7D) return NAN;
    int e = (b >> 3) & 0xF, m = b & 7;
    float v = ldexpf(1.0f + (float)m / 8.0f, e - 7);
    return (b & 0x80) ? -v : v;
}

/* E5M2 encode, fp8_types.hpp:147-189: as E4M3 with bias 15 (exp = E-112),
   subnormal shift (2^23+M) >> (20+exp) for exp in [-2,0] (:161-167),
   Inf at exp >= 31 (:169-171), and the mantissa carry IS propagated
   (:179-186). */
uint8_t orc_e5m2_compat_encode(float f) {
    uint32_t u = f2u(f);
    uint32_t sign = (u >> 31) ? 0x80u : 0u;
    uint32_t E = (u >> 23) & 0xFF, M = u & 0x7FFFFF;
    if (E == 0 && M == 0) return (uint8_t)sign;
    if (E == 0xFF) return M ? 0x7D : (uint8_t)(sign | 0x7C);
    if (E == 0) return (uint8_t)sign;
    int exp = (int)E - 112;
    if (exp <= 0) {
        if (exp < -2) return (uint8_t)sign;
        uint32_t m = (0x800000u | M) >> (20 + exp);
        return (uint8_t)(sign | (m & 0x7F));
    }
    if (exp >= 31) return (uint8_t)(sign | 0x7C);
    uint32_t r = (M + (1u << 20)) >> 21;
    if (r >= 4) {
        r = 0;
        ++exp;
        if (exp >= 31) return (uint8_t)(sign | 0x7C);
    }
    return (uint8_t)(sign | ((uint32_t)exp << 2) | r);
}

/* E5M2 decode, fp8_types.hpp:191-207 */
float orc_e5m2_compat_decode(uint8_t b) {
    if (b == 0) return 0.0f;
    if (b == 0x80) return -0.0f;
    if (b == 0x7C) return INFINITY;
    if (b == 0xFC) return -INFINITY;
    if (b == 0x7D) return NAN;
    int e = (b >> 2) & 0x1F, m = b & 3;
    float v = ldexpf(1.0f + (float)m / 4.0f, e - 15);
    return (b & 0x80) ? -v : v;
}

/* ======================================================================
 * OCP codec (OCP 8-bit FP spec; PTX cvt.rn.satfinite.{e4m3,e5m2}x2.f32):
 * round to nearest even on the integer significand, then saturate the
 * magnitude to the largest finite code.  NaN -> 0x7F; +-Inf saturates.
 * ==================================================================== */
static uint8_t ocp_encode(float f, int mbits, int bias, int emin, uint32_t maxcode) {
    uint32_t u = f2u(f);
    uint32_t sign = (u >> 31) ? 0x80u : 0u;
    uint32_t E = (u >> 23) & 0xFF, M = u & 0x7FFFFF;
    if (E == 0xFF) return M ? 0x7F : (uint8_t)(sign | maxcode);
    if (E == 0) return (uint8_t)sign;          /* |f| < 2^-126: rounds to zero */
    int te = (int)E - 127;
    if (te < emin) te = emin;
    int shift = (te - mbits) - ((int)E - 150);  /* >= 23 - mbits > 0 */
    uint32_t mant = 0x800000u | M;
    uint32_t q;
    if (shift >= 32) {
        q = 0;
    } else {
        q = mant >> shift;
        uint32_t rem = mant & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1u))) ++q;
    }
    if (q >= (2u << mbits)) { q >>= 1; ++te; }
    uint32_t code;
    if (q < (1u << mbits)) {
        code = q;                                /* subnormal or zero */
    } else {
        code = ((uint32_t)(te + bias) << mbits) | (q - (1u << mbits));
    }
    if (code > maxcode) code = maxcode;
    return (uint8_t)(sign | code);
}

static float ocp_decode(uint8_t b, int mbits, int bias, int e4m3) {
    uint32_t mag = b & 0x7F;
    float s = (b & 0x80) ? -1.0f : 1.0f;
    int e = (int)(mag >> mbits), m = (int)(mag & ((1u << mbits) - 1));
    if (e4m3) {
        if (mag == 0x7F) return NAN;
    } else if (e == 31) {
        return m ? NAN : s * INFINITY;
    }
    if (e == 0) return s * ldexpf((float)m, 1 - bias - mbits);
    return s * ldexpf((float)((1 << mbits) + m), e - bias - mbits);
}

uint8_t orc_e4m3_ocp_encode(float f) { return ocp_encode(f, 3, 7, -6, 0x7E); }
float orc_e4m3_ocp_decode(uint8_t b) { return ocp_decode(b, 3, 7, 1); }
uint8_t orc_e5m2_ocp_encode(float f) { return ocp_encode(f, 2, 15, -14, 0x7B); }
float orc_e5m2_ocp_decode(uint8_t b) { return ocp_decode(b, 2, 15, 0); }

/* bf16 round to nearest even (NaN -> quiet NaN keeping the sign) */
uint16_t orc_f32_to_bf16(float f) {
    uint32_t u = f2u(f);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
float orc_bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

/* ======================================================================
 * Element-wise kernels
 * ==================================================================== */

/* quantize_f32_kernel, src/cuda/quantize/fp8_kernels.cu:12-17 (no scale) */
void orc_quantize_f32_to_fp8_compat(const float* src, uint8_t* dst, size_t n, int fmt) {
    for (size_t i = 0; i < n; ++i)
        dst[i] = fmt == ORC_FMT_E5M2 ? orc_e5m2_compat_encode(src[i])
                                     : orc_e4m3_compat_encode(src[i]);
}

/* dequantize_fp8_kernel, fp8_kernels.cu:19-25: dec(src) * scale */
void orc_dequantize_fp8_compat(const uint8_t* src, float* dst, size_t n, float scale, int fmt) {
    for (size_t i = 0; i < n; ++i) {
        float d = fmt == ORC_FMT_E5M2 ? orc_e5m2_compat_decode(src[i])
                                      : orc_e4m3_compat_decode(src[i]);
        dst[i] = d * scale;
    }
}

/* quantize_batched_f32_kernel, fp8_kernels.cu:83-102: FP8E4M3(src * scale[b]);
   the batch scale MULTIPLIES (:96). */
void orc_quantize_scaled_fp8_compat(const float* src, uint8_t* dst, size_t n, float mul) {
    for (size_t i = 0; i < n; ++i) dst[i] = orc_e4m3_compat_encode(src[i] * mul);
}

/* round to nearest even, saturating float -> int32 (cvt.rni.s32.f32) */
static int32_t f2i_rn_sat(float v) {
    if (v != v) return 0;
    if (v >= 2147483648.0f) return INT32_MAX;
    if (v <= -2147483648.0f) return INT32_MIN;
    float r = nearbyintf(v);   /* default FE_TONEAREST = ties to even */
    return (int32_t)r;
}
/* truncating, saturating float -> int32 (cvt.rzi.s32.f32) */
static int32_t f2i_rz_sat(float v) {
    if (v != v) return 0;
    if (v >= 2147483648.0f) return INT32_MAX;
    if (v <= -2147483648.0f) return INT32_MIN;
    return (int32_t)v;
}
static inline int32_t clamp127(int32_t q) { return q < -127 ? -127 : (q > 127 ? 127 : q); }

/* quantize_f32_to_int8_kernel, int8_kernels.cu:15-37:
   sym clamp(rn(x/s)), asym clamp(rn((x-zp)/s)), IEEE division. */
void orc_quantize_f32_to_int8(const float* src, int8_t* dst, size_t n, float scale,
                              float zero_point, int symmetric) {
    for (size_t i = 0; i < n; ++i) {
        float v = symmetric ? src[i] / scale : (src[i] - zero_point) / scale;
        dst[i] = (int8_t)clamp127(f2i_rn_sat(v));
    }
}

/* dequantize_int8_to_f32_kernel, int8_kernels.cu:39-60: q*s / (q+zp)*s */
void orc_dequantize_int8_to_f32(const int8_t* src, float* dst, size_t n, float scale,
                                float zero_point, int symmetric) {
    for (size_t i = 0; i < n; ++i)
        dst[i] = symmetric ? (float)src[i] * scale : ((float)src[i] + zero_point) * scale;
}

/* quantize_with_scale_from_histogram_kernel, int8_kernels.cu:171-194:
   range < 1e-6 -> 0; s = range/254; q = clamp(rn((x-min)/s - 127)).
   nvcc fuses nothing here: (x-min)/s is a division, then one subtraction. */
void orc_quantize_int8_with_calibration(const float* src, int8_t* dst, size_t n,
                                        float min_val, float max_val) {
    float range = max_val - min_val;
    for (size_t i = 0; i < n; ++i) {
        if (range < 1e-6f) { dst[i] = 0; continue; }
        float s = range / 254.0f;
        float v = (src[i] - min_val) / s - 127.0f;
        dst[i] = (int8_t)clamp127(f2i_rn_sat(v));
    }
}

/* QuantizedTensor<int8_t>::FromFloat rounding, quantize_tensor.hpp:176-182:
   std::round (half away) of x/s, clamped to +-127 */
void orc_quantize_int8_half_away(const float* src, int8_t* dst, size_t n, float scale) {
    for (size_t i = 0; i < n; ++i) {
        float r = roundf(src[i] / scale);
        r = fmaxf(-127.0f, fminf(127.0f, r));
        dst[i] = (int8_t)r;
    }
}

static uint8_t enc_fmt(float v, int fmt) {
    if (fmt == ORC_FMT_E4M3) return orc_e4m3_ocp_encode(v);
    if (fmt == ORC_FMT_E5M2) return orc_e5m2_ocp_encode(v);
    return (uint8_t)(int8_t)clamp127(f2i_rn_sat(v));
}
static float dec_fmt(uint8_t c, int fmt) {
    if (fmt == ORC_FMT_E4M3) return orc_e4m3_ocp_decode(c);
    if (fmt == ORC_FMT_E5M2) return orc_e5m2_ocp_decode(c);
    return (float)(int8_t)c;
}
static float qmax_fmt(int fmt) {
    return fmt == ORC_FMT_E4M3 ? 448.0f : (fmt == ORC_FMT_E5M2 ? 57344.0f : 127.0f);
}

/* Scaled quantize of the extension API: q = encode(x / scale), IEEE division,
   RNE, saturating (INT8: clamp to +-127 as int8_kernels.cu:35). */
void orc_quantize_ocp(const float* src, uint8_t* dst, size_t n, float scale, int fmt) {
    for (size_t i = 0; i < n; ++i) dst[i] = enc_fmt(src[i] / scale, fmt);
}
void orc_dequantize_ocp(const uint8_t* src, float* dst, size_t n, float scale, int fmt) {
    for (size_t i = 0; i < n; ++i) dst[i] = dec_fmt(src[i], fmt) * scale;
}

/* ======================================================================
 * Reductions and calibration
 * ==================================================================== */

/* IEEE minNum/maxNum with -0 < +0, as PTX min.f32/max.f32 (fminf/fmaxf) */
static inline float mn(float a, float b) {
    if (a != a) return b;
    if (b != b) return a;
    if (a == b) return (f2u(a) >> 31) ? a : b;
    return a < b ? a : b;
}
static inline float mx(float a, float b) {
    if (a != a) return b;
    if (b != b) return a;
    if (a == b) return (f2u(a) >> 31) ? b : a;
    return a > b ? a : b;
}

/* compute_minmax, int8_kernels.cu:131-169 + host finish :324-410:
   fminf/fmaxf over all elements starting from +-FLT_MAX (NaN ignored);
   n == 0 gives 0,0 (:331-335). */
void orc_compute_minmax(const float* data, size_t n, float* min_val, float* max_val) {
    if (n == 0) { *min_val = 0.0f; *max_val = 0.0f; return; }
    float lo = FLT_MAX, hi = -FLT_MAX;
    for (size_t i = 0; i < n; ++i) { lo = mn(lo, data[i]); hi = mx(hi, data[i]); }
    *min_val = lo;
    *max_val = hi;
}

float orc_amax(const float* data, size_t n) {
    float a = 0.0f;
    for (size_t i = 0; i < n; ++i) a = mx(a, fabsf(data[i]));
    return a;
}

/* build_histogram_kernel, int8_kernels.cu:97-129: bin = (int)((x-min)/range
   *(bins-1)) clamped, only when range > 1e-6.  The reference flushes only
   256 bins and indexes smem[256] out of bounds for larger counts; this
   restatement keeps the intended result for every bin count (identical to
   the reference for bins <= 256). */
void orc_build_histogram(const float* data, uint32_t* hist, size_t n, float min_val,
                         float max_val, int num_bins) {
    memset(hist, 0, sizeof(uint32_t) * (size_t)num_bins);
    float range = max_val - min_val;
    if (!(range > 1e-6f)) return;
    float mul = (float)(num_bins - 1);
    for (size_t i = 0; i < n; ++i) {
        int32_t b = f2i_rz_sat((data[i] - min_val) / range * mul);
        if (b < 0) b = 0;
        if (b > num_bins - 1) b = num_bins - 1;
        hist[b]++;
    }
}

/* MinMaxCalibrator::calibrate, src/cuda/quantize/calibrator.cpp:17-40 */
void orc_minmax_calibrate(const float* data, size_t n, int symmetric, float out[5]) {
    float lo, hi, scale, zp;
    orc_compute_minmax(data, n, &lo, &hi);
    if (symmetric) {
        float a = fmaxf(fabsf(lo), fabsf(hi));
        scale = a / 127.0f;
        zp = 0.0f;
    } else {
        scale = (hi - lo) / 254.0f;
        zp = -lo / scale - 127.0f;
    }
    if (scale < 1e-6f) scale = 1e-6f;
    out[0] = scale; out[1] = zp; out[2] = (float)(symmetric != 0); out[3] = lo; out[4] = hi;
}

/* HistogramCalibrator::find_threshold_percentile, calibrator.cpp:109-129:
   target = (u64)(float(total) * p / 100); first bin whose running count
   reaches it; threshold = min + (i + 0.5) * range / bins. */
float orc_histogram_threshold(const uint32_t* hist, int num_bins, float min_val,
                              float max_val, float percentile) {
    uint64_t total = 0;
    for (int i = 0; i < num_bins; ++i) total += hist[i];
    uint64_t target = (uint64_t)((float)total * percentile / 100.0f);
    float range = max_val - min_val;
    float bin_width = range / (float)num_bins;
    uint64_t cum = 0;
    for (int i = 0; i < num_bins; ++i) {
        cum += hist[i];
        if (cum >= target) return min_val + ((float)i + 0.5f) * bin_width;
    }
    return max_val;
}

/* HistogramCalibrator::calibrate, calibrator.cpp:65-107 */
void orc_histogram_calibrate(const float* data, size_t n, int num_bins, float percentile,
                             int symmetric, uint32_t* hist_out, float out[5]) {
    float lo, hi;
    orc_compute_minmax(data, n, &lo, &hi);
    orc_build_histogram(data, hist_out, n, lo, hi, num_bins);
    float thr = orc_histogram_threshold(hist_out, num_bins, lo, hi, percentile);
    float a = fmaxf(fabsf(thr), fabsf(-thr));
    float scale = a / 127.0f;
    if (scale < 1e-6f) scale = 1e-6f;
    out[0] = scale; out[1] = 0.0f; out[2] = (float)(symmetric != 0); out[3] = lo; out[4] = hi;
}

/* MSECalibrator::calibrate, calibrator.cpp:158-190: candidate scales
   0.001 * 2^i up to max-min, float MSE over the first min(n, 10000)
   elements with std::round (half away). */
void orc_mse_calibrate(const float* data, size_t n, int symmetric, float out[5]) {
    float lo, hi;
    orc_compute_minmax(data, n, &lo, &hi);
    float best_mse = FLT_MAX, best = 1.0f;
    size_t cnt = n < 10000 ? n : 10000;
    for (float cs = 0.001f; cs <= (hi - lo); cs *= 2.0f) {
        float mse = 0.0f;
        for (size_t i = 0; i < cnt; ++i) {
            float q = roundf(data[i] / cs) * cs;
            float e = (data[i] - q) * (data[i] - q);
            mse += e;
        }
        mse /= (float)cnt;
        if (mse < best_mse) { best_mse = mse; best = cs; }
    }
    out[0] = best; out[1] = 0.0f; out[2] = (float)(symmetric != 0); out[3] = lo; out[4] = hi;
}

static float row_scale_of(float amax, int fmt) {
    return amax > 0.0f ? amax / qmax_fmt(fmt) : 1.0f;
}
/* Per-row / per-column scaling of the product kernels (reduce.cu row_scale):
   q = enc(x * inv) with inv = qmax / amax (1 for an all-zero row); when that
   quotient overflows, the row is divided by its scale instead. */
static float row_apply(float x, float amax, float scale, int fmt) {
    if (!(amax > 0.0f)) return x * 1.0f;
    const float inv = qmax_fmt(fmt) / amax;
    return inv <= FLT_MAX ? x * inv : x / scale;
}

void orc_quantize_rows(const void* src, int src_bf16, uint8_t* dst, float* scales,
                       size_t rows, size_t cols, int fmt) {
    for (size_t r = 0; r < rows; ++r) {
        float a = 0.0f;
        for (size_t c = 0; c < cols; ++c) {
            float v = src_bf16 ? orc_bf16_to_f32(((const uint16_t*)src)[r * cols + c])
                               : ((const float*)src)[r * cols + c];
            a = mx(a, fabsf(v));
        }
        float s = row_scale_of(a, fmt);
        scales[r] = s;
        for (size_t c = 0; c < cols; ++c) {
            float v = src_bf16 ? orc_bf16_to_f32(((const uint16_t*)src)[r * cols + c])
                               : ((const float*)src)[r * cols + c];
            dst[r * cols + c] = enc_fmt(row_apply(v, a, s, fmt), fmt);
        }
    }
}

void orc_quantize_cols(const float* src, uint8_t* dst, float* scales, size_t rows,
                       size_t cols, int fmt) {
    float* amax = (float*)malloc((cols ? cols : 1) * sizeof(float));
    for (size_t c = 0; c < cols; ++c) {
        float a = 0.0f;
        for (size_t r = 0; r < rows; ++r) a = mx(a, fabsf(src[r * cols + c]));
        amax[c] = a;
        scales[c] = row_scale_of(a, fmt);
    }
    for (size_t r = 0; r < rows; ++r)
        for (size_t c = 0; c < cols; ++c)
            dst[r * cols + c] = enc_fmt(row_apply(src[r * cols + c], amax[c], scales[c], fmt), fmt);
    free(amax);
}

/* ======================================================================
 * GEMMs
 * ==================================================================== */

/* fp8_gemm_naive_kernel, src/cuda/quantize/fp8_gemm.cu:64-86:
   sum += (dec(a)*sa) * (dec(b)*sb) over k in order; nvcc contracts the
   accumulation into an FMA; C = sum * so.  fmt selects the decoder
   (FP8E5M2GEMM reinterprets its bytes as E4M3, fp8_gemm.cu:247-249). */
static void fp8_ref_rows(const uint8_t* a, const uint8_t* b, float* c, int m, int k, int n,
                         float sa, float sb, float so, int fmt, int r0, int r1) {
    (void)m;
    for (int i = r0; i < r1; ++i)
        for (int j = 0; j < n; ++j) {
            float sum = 0.0f;
            for (int p = 0; p < k; ++p) {
                float av = (fmt == ORC_FMT_E5M2 ? orc_e5m2_compat_decode(a[(size_t)i * k + p])
                                                : orc_e4m3_compat_decode(a[(size_t)i * k + p])) * sa;
                float bv = (fmt == ORC_FMT_E5M2 ? orc_e5m2_compat_decode(b[(size_t)p * n + j])
                                                : orc_e4m3_compat_decode(b[(size_t)p * n + j])) * sb;
                sum = fmaf(av, bv, sum);
            }
            c[(size_t)i * n + j] = sum * so;
        }
}

void orc_fp8_gemm_reference(const uint8_t* a, const uint8_t* b, float* c, int m, int k,
                            int n, float sa, float sb, float so, int fmt) {
    fp8_ref_rows(a, b, c, m, k, n, sa, sb, so, fmt, 0, m);
}

typedef struct {
    const uint8_t *a, *b; float* c; int m, k, n; float sa, sb, so; int r0, r1;
    float lut[256];
} ref_job_t;

static void* ref_job_run(void* p) {
    ref_job_t* j = (ref_job_t*)p;
    /* Same arithmetic as fp8_ref_rows; the decode goes through a 256-entry
       table of the same decoder outputs, so every product is identical. */
    for (int i = j->r0; i < j->r1; ++i)
        for (int col = 0; col < j->n; ++col) {
            float sum = 0.0f;
            for (int p = 0; p < j->k; ++p) {
                float av = j->lut[j->a[(size_t)i * j->k + p]] * j->sa;
                float bv = j->lut[j->b[(size_t)p * j->n + col]] * j->sb;
                sum = fmaf(av, bv, sum);
            }
            j->c[(size_t)i * j->n + col] = sum * j->so;
        }
    return NULL;
}

int orc_fp8_gemm_reference_rows_mt(const uint8_t* a, const uint8_t* b, float* c, int m,
                                   int k, int n, float sa, float sb, float so, int row0,
                                   int rows, int threads) {
    (void)m;
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    if (threads > rows) threads = rows;
    static ref_job_t jobs[256];
    pthread_t th[256];
    for (int t = 0; t < threads; ++t) {
        ref_job_t* j = &jobs[t];
        j->a = a; j->b = b; j->c = c; j->m = m; j->k = k; j->n = n;
        j->sa = sa; j->sb = sb; j->so = so;
        j->r0 = row0 + (int)((long long)rows * t / threads);
        j->r1 = row0 + (int)((long long)rows * (t + 1) / threads);
        for (int v = 0; v < 256; ++v) j->lut[v] = orc_e4m3_compat_decode((uint8_t)v);
        pthread_create(&th[t], NULL, ref_job_run, j);
    }
    for (int t = 0; t < threads; ++t) pthread_join(th[t], NULL);
    return threads;
}

void orc_gemm_fp8_acc(const uint8_t* a, const uint8_t* b, float* acc, int m, int k, int n,
                      int fmt_a, int fmt_b, int b_kn) {
    float la[256], lb[256];
    for (int v = 0; v < 256; ++v) { la[v] = dec_fmt((uint8_t)v, fmt_a); lb[v] = dec_fmt((uint8_t)v, fmt_b); }
    for (int i = 0; i < m; ++i)
        for (int j = 0; j < n; ++j) {
            float s = 0.0f;
            for (int p = 0; p < k; ++p) {
                float bv = b_kn ? lb[b[(size_t)p * n + j]] : lb[b[(size_t)j * k + p]];
                s = fmaf(la[a[(size_t)i * k + p]], bv, s);
            }
            acc[(size_t)i * n + j] = s;
        }
}

void orc_gemm_i8_acc(const int8_t* a, const int8_t* b, int32_t* acc, int m, int k, int n,
                     int b_kn) {
    for (int i = 0; i < m; ++i)
        for (int j = 0; j < n; ++j) {
            int32_t s = 0;
            for (int p = 0; p < k; ++p) {
                int32_t bv = b_kn ? b[(size_t)p * n + j] : b[(size_t)j * k + p];
                s += (int32_t)a[(size_t)i * k + p] * bv;
            }
            acc[(size_t)i * n + j] = s;
        }
}

/* Scale-folded epilogue of the extension GEMMs (no reference counterpart:
   the reference GEMM only has scale_a*scale_b*scale_out, fp8_gemm.cu:80-85).
   Order: ((acc * alpha) * row[m]) * col[n] + bias[n], one rounding each. */
void orc_epilogue(const void* acc, int acc_i32, void* out, int out_kind, int m, int n,
                  float alpha, const float* row_scale, const float* col_scale,
                  const float* bias) {
    for (int i = 0; i < m; ++i)
        for (int j = 0; j < n; ++j) {
            size_t idx = (size_t)i * n + j;
            float v = acc_i32 ? (float)((const int32_t*)acc)[idx] : ((const float*)acc)[idx];
            v = v * alpha;
            if (row_scale) v = v * row_scale[i];
            if (col_scale) v = v * col_scale[j];
            if (bias) v = v + bias[j];
            if (out_kind == 1) ((uint16_t*)out)[idx] = orc_f32_to_bf16(v);
            else ((float*)out)[idx] = v;
        }
}

/* QuantizedMatmul::forward, include/cuda/quantize/quantize_ops.hpp:54-81 */
void orc_quantized_matmul(const int8_t* a, const int8_t* b, int8_t* out, int m, int k,
                          int n, float sa, float sb) {
    float os = sa * sb;
    for (int i = 0; i < m; ++i)
        for (int j = 0; j < n; ++j) {
            int32_t s = 0;
            for (int p = 0; p < k; ++p) s += (int32_t)a[i * k + p] * (int32_t)b[p * n + j];
            float q = (float)s * os;
            q = fmaxf(-127.0f, fminf(127.0f, q));
            out[i * n + j] = (int8_t)roundf(q);
        }
}

/* QuantizedTensor<int8_t>::FromFloat, quantize_tensor.hpp:160-191 */
int orc_quantized_tensor_from_float(const float* data, size_t n, float scale, int8_t* q,
                                    float* scale_out) {
    if (n == 0) return 0;
    if (scale <= 0.0f) {
        float m = 0.0f;
        for (size_t i = 0; i < n; ++i) m = fmaxf(m, fabsf(data[i]));
        scale = m / 127.0f;
    }
    if (scale == 0.0f) scale = 1.0f;
    orc_quantize_int8_half_away(data, q, n, scale);
    *scale_out = scale;
    return 1;
}

/* silu_and_mul_kernel, src/cuda/neural/activations.cu:80-92: g/(1+exp(-g))*u */
float orc_silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

void orc_swiglu_epilogue(const float* acc, void* out, int out_bf16, int m, int n, float alpha,
                         const float* row_scale, const float* col_scale, const float* bias) {
    const int no = n / 2;
    for (int i = 0; i < m; ++i)
        for (int j = 0; j < no; ++j) {
            const int gc = (j / 128) * 256 + (j % 128), uc = gc + 128;
            float g = acc[(size_t)i * n + gc] * alpha, u = acc[(size_t)i * n + uc] * alpha;
            if (row_scale) { g = g * row_scale[i]; u = u * row_scale[i]; }
            if (col_scale) { g = g * col_scale[gc]; u = u * col_scale[uc]; }
            if (bias) { g = g + bias[gc]; u = u + bias[uc]; }
            const float h = g / (1.0f + expf(-g)) * u;
            if (out_bf16) ((uint16_t*)out)[(size_t)i * no + j] = orc_f32_to_bf16(h);
            else ((float*)out)[(size_t)i * no + j] = h;
        }
}

/* FakeQuantize::forward (qat.hpp:64-72): scale floored at 1e-6, q =
   clamp(round_half_away((x - zp) / scale), +-127), y = q * scale + zp with a
   separate multiply and add (compiled with -ffp-contract=off). */
void orc_fake_quantize_int8(const float* src, float* dst, size_t n, float scale, float zero_point) {
    const float s = scale < 1e-6f ? 1e-6f : scale;
    for (size_t i = 0; i < n; ++i) {
        float r = roundf((src[i] - zero_point) / s);
        float c = r < 127.0f ? r : 127.0f;     /* NaN -> 127, as std::min(127, NaN) */
        c = -127.0f < c ? c : -127.0f;
        const float m = c * s;
        dst[i] = m + zero_point;
    }
}

/* FP8 activations of fp8_activation.hpp:26-59 on reference-codec codes: decode,
   activate in fp32 (libm erff / expf), re-encode; relu keeps non-negative
   codes (and NaN codes) unchanged and maps negative ones to +0.
   op 0 relu, 1 gelu, 2 sigmoid, 3 leaky relu; fmt 0 E4M3, 1 E5M2. */
void orc_fp8_activation(const uint8_t* src, uint8_t* dst, size_t n, int fmt, int op, float alpha) {
    for (size_t i = 0; i < n; ++i) {
        const float x = fmt == 0 ? orc_e4m3_compat_decode(src[i]) : orc_e5m2_compat_decode(src[i]);
        float y;
        if (op == 0) {
            if (!(x < 0.0f)) {
                dst[i] = src[i];
                continue;
            }
            y = 0.0f;
        } else if (op == 1) {
            const float cdf = 0.5f * (1.0f + erff(x * 0.7071067811865476f));
            y = x * cdf;
        } else if (op == 2) {
            y = 1.0f / (1.0f + expf(-x));
        } else {
            y = x >= 0.0f ? x : alpha * x;
        }
        dst[i] = fmt == 0 ? orc_e4m3_compat_encode(y) : orc_e5m2_compat_encode(y);
    }
}

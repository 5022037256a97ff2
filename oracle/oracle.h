/*
 * oracle.h -- CPU restatement of pplmx/nova's cuda::quantize path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (nova_b200/, include/)
 * links, loads or calls this code.  It is the checker that tests/, the
 * __graft_entry__.smoke() check and bench.py's cpu_baseline / reference arm
 * use.  Every function cites the reference file:line it restates
 * (paths relative to the pplmx/nova source tree).
 *
 * Parity pins (see tests/test_oracle_*.py):
 *   - the compat FP8 codec is checked exhaustively against the reference's
 *     own FP8E4M3/FP8E5M2 classes compiled from the reference headers
 *     (oracle/Makefile -> oracle/_ref/libnova_ref_host.so) and against the
 *     codes the reference tests pin (tests/quantize/fp8_types_test.cpp:59-83);
 *   - INT8 FromFloat / QuantizedMatmul are checked against the reference's
 *     own quantize_tensor.hpp / quantize_ops.hpp compiled the same way;
 *   - GPU kernels of the reference (int8_kernels.cu, fp8_kernels.cu,
 *     fp8_gemm.cu) are compiled into oracle/_ref/libnova_ref_gpu.so and
 *     compared with this file on the GPU box (tests/test_ref_gpu_pin.py).
 *   - the OCP codec follows the OCP 8-bit floating point specification
 *     (E4M3FN: bias 7, max 448, NaN 0x7F, no Inf; E5M2: bias 15, max 57344)
 *     with round-to-nearest-even and saturation to the largest finite value,
 *     i.e. PTX cvt.rn.satfinite; it is cross-checked against torch's
 *     float8 casts on in-range inputs.
 */
#ifndef NOVA_ORACLE_H
#define NOVA_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- scalar codecs ---------------------------------------------------- */
uint8_t orc_e4m3_compat_encode(float f);
float orc_e4m3_compat_decode(uint8_t b);
uint8_t orc_e5m2_compat_encode(float f);
float orc_e5m2_compat_decode(uint8_t b);
uint8_t orc_e4m3_ocp_encode(float f);
float orc_e4m3_ocp_decode(uint8_t b);
uint8_t orc_e5m2_ocp_encode(float f);
float orc_e5m2_ocp_decode(uint8_t b);
uint16_t orc_f32_to_bf16(float f);
float orc_bf16_to_f32(uint16_t h);

/* fmt codes shared with the product ABI: 0 = E4M3, 1 = E5M2, 2 = INT8 */
#define ORC_FMT_E4M3 0
#define ORC_FMT_E5M2 1
#define ORC_FMT_INT8 2

/* ---- element-wise kernels --------------------------------------------- */
void orc_quantize_f32_to_fp8_compat(const float* src, uint8_t* dst, size_t n, int fmt);
void orc_dequantize_fp8_compat(const uint8_t* src, float* dst, size_t n, float scale, int fmt);
void orc_quantize_scaled_fp8_compat(const float* src, uint8_t* dst, size_t n, float mul);
void orc_quantize_f32_to_int8(const float* src, int8_t* dst, size_t n, float scale,
                              float zero_point, int symmetric);
void orc_dequantize_int8_to_f32(const int8_t* src, float* dst, size_t n, float scale,
                                float zero_point, int symmetric);
void orc_quantize_int8_with_calibration(const float* src, int8_t* dst, size_t n,
                                        float min_val, float max_val);
void orc_quantize_int8_half_away(const float* src, int8_t* dst, size_t n, float scale);
void orc_quantize_ocp(const float* src, uint8_t* dst, size_t n, float scale, int fmt);
void orc_dequantize_ocp(const uint8_t* src, float* dst, size_t n, float scale, int fmt);

/* ---- reductions / calibration ----------------------------------------- */
void orc_compute_minmax(const float* data, size_t n, float* min_val, float* max_val);
float orc_amax(const float* data, size_t n);
void orc_build_histogram(const float* data, uint32_t* hist, size_t n, float min_val,
                         float max_val, int num_bins);
/* out = {scale, zero_point, symmetric, min, max} */
void orc_minmax_calibrate(const float* data, size_t n, int symmetric, float out[5]);
float orc_histogram_threshold(const uint32_t* hist, int num_bins, float min_val,
                              float max_val, float percentile);
void orc_histogram_calibrate(const float* data, size_t n, int num_bins, float percentile,
                             int symmetric, uint32_t* hist_out, float out[5]);
void orc_mse_calibrate(const float* data, size_t n, int symmetric, float out[5]);

/* per-row scales: scale[r] = amax(row r)/qmax (1.0 when the row is all zero),
   q = encode(x * (qmax / amax)) -- one division per row; a row whose
   qmax / amax overflows uses q = encode(x / scale[r]).  src is fp32
   (src_bf16 == 0) or bf16 bits. */
void orc_quantize_rows(const void* src, int src_bf16, uint8_t* dst, float* scales,
                       size_t rows, size_t cols, int fmt);
/* per-column scales of a row-major rows x cols matrix (same arithmetic per column) */
void orc_quantize_cols(const float* src, uint8_t* dst, float* scales, size_t rows,
                       size_t cols, int fmt);

/* ---- GEMMs ------------------------------------------------------------ */
/* the reference's naive FP8 kernel: compat decode, sequential k, FMA */
void orc_fp8_gemm_reference(const uint8_t* a, const uint8_t* b, float* c, int m, int k,
                            int n, float sa, float sb, float so, int fmt);
/* OCP-decoded fp32 accumulators, sequential k; b_kn = 1: B is K x N row-major,
   b_kn = 0: B is N x K row-major */
void orc_gemm_fp8_acc(const uint8_t* a, const uint8_t* b, float* acc, int m, int k, int n,
                      int fmt_a, int fmt_b, int b_kn);
void orc_gemm_i8_acc(const int8_t* a, const int8_t* b, int32_t* acc, int m, int k, int n,
                     int b_kn);
/* epilogue: v = acc * alpha [* row_scale[m]] [* col_scale[n]] [+ bias[n]];
   out_kind 0 = fp32, 1 = bf16 bits.  acc_i32 selects the accumulator type. */
void orc_epilogue(const void* acc, int acc_i32, void* out, int out_kind, int m, int n,
                  float alpha, const float* row_scale, const float* col_scale,
                  const float* bias);
/* reference host INT8 matmul: quantize_ops.hpp:54-81 */
void orc_quantized_matmul(const int8_t* a, const int8_t* b, int8_t* out, int m, int k,
                          int n, float sa, float sb);
/* reference QuantizedTensor<int8_t>::FromFloat: quantize_tensor.hpp:160-191 */
int orc_quantized_tensor_from_float(const float* data, size_t n, float scale, int8_t* q,
                                    float* scale_out);

/* SwiGLU of the TP MLP (activations.cu:80-92 restated on fp32 values) */
float orc_silu_mul(float g, float u);
/* Fused SwiGLU GEMM epilogue: acc is m x n fp32 with gate/up packed in
   alternating 128-column blocks; out (m x n/2, fp32 or bf16 bits) holds
   silu(g) * u of the scaled values (orc_epilogue's arithmetic for g and u). */
void orc_swiglu_epilogue(const float* acc, void* out, int out_bf16, int m, int n, float alpha,
                         const float* row_scale, const float* col_scale, const float* bias);

/* FP8 activations on reference-codec codes (fp8_activation.hpp:26-59):
   op 0 relu, 1 gelu, 2 sigmoid, 3 leaky relu (alpha); fmt 0 E4M3, 1 E5M2 */
void orc_fp8_activation(const uint8_t* src, uint8_t* dst, size_t n, int fmt, int op, float alpha);
/* QAT FakeQuantize::forward over an array (qat.hpp:64-72) */
void orc_fake_quantize_int8(const float* src, float* dst, size_t n, float scale, float zero_point);

/* bounded multi-threaded run of orc_fp8_gemm_reference over rows
   [row0, row0+rows); returns the number of threads used */
int orc_fp8_gemm_reference_rows_mt(const uint8_t* a, const uint8_t* b, float* c, int m,
                                   int k, int n, float sa, float sb, float so, int row0,
                                   int rows, int threads);

#ifdef __cplusplus
}
#endif
#endif

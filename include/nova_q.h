/*
 * nova_q.h -- C ABI of the B200 (sm_100a) quantized-inference path.
 *
 * This is the drop-in boundary for pplmx/nova's cuda::quantize subsystem.
 * Every entry point takes plain pointers, sizes and a cudaStream_t, returns
 * an nq_status_t, and is implemented by hand-written sm_100a CUDA kernels in
 * libnova_q.so.  The C++ API of the reference (FP8GEMM, MinMaxCalibrator,
 * quantize_f32_to_int8, ...) is provided as thin inline shims over these
 * functions in include/cuda/quantize/*.hpp (same include paths as the
 * reference).
 *
 * Each declaration names the reference interface it replaces
 * (file:line relative to the pplmx/nova source tree).
 *
 * Conventions
 *   - Device pointers unless stated otherwise.  The library never frees
 *     caller memory.
 *   - Asynchronous on `stream` unless stated otherwise.  Entry points that
 *     return values to the host (compute_minmax, build_histogram) synchronise
 *     `stream`, as the reference does.
 *   - Errors: a non-zero status; nq_last_error() returns a thread-local
 *     message for the last failing call on this thread.  The reference prints
 *     launch errors to stderr and continues (e.g. int8_kernels.cu:214-217);
 *     the C++ shims keep that behaviour where the reference had it.
 *   - Format codes: NQ_E4M3 / NQ_E5M2 are OCP FP8 (E4M3FN max 448, E5M2 max
 *     57344) encoded round-to-nearest-even with saturation; NQ_INT8 is
 *     symmetric int8 clamped to [-127, 127].  The reference's own FP8 codec
 *     (IEEE-like, max 240, Inf 0x7C, NaN 0x7D) is available bit-exactly
 *     through the *_fp8e4m3 / *_fp8e5m2 entry points that mirror its API.
 */
#ifndef NOVA_Q_H
#define NOVA_Q_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* nq_stream_t; /* identical to cudaStream_t */

typedef enum {
    NQ_SUCCESS = 0,
    NQ_ERROR_INVALID_VALUE = 1,  /* null pointer, bad size or enum         */
    NQ_ERROR_UNSUPPORTED = 2,    /* shape / alignment the path cannot take */
    NQ_ERROR_CUDA = 3,           /* a CUDA runtime or driver call failed   */
    NQ_ERROR_OUT_OF_MEMORY = 4,
    NQ_ERROR_NO_DEVICE = 5,      /* no sm_100 device is current            */
    NQ_ERROR_DEVICE_TIMEOUT = 6  /* a kernel's bounded wait ran out        */
} nq_status_t;

typedef enum { NQ_E4M3 = 0, NQ_E5M2 = 1, NQ_INT8 = 2 } nq_format_t;
/* NQ_S8: int8 requantized output, clamp(v, +-127) then round half away from
   zero (QuantizedMatmul::forward, quantize_ops.hpp:73-77). */
typedef enum { NQ_F32 = 0, NQ_BF16 = 1, NQ_S32 = 2, NQ_S8 = 3 } nq_dtype_t;
/* B operand layout of a GEMM: NQ_B_KN is K x N row-major (the layout of
   FP8GEMM::forward, fp8_gemm.cu:81); NQ_B_NK is N x K row-major (a
   "packed" weight, the layout of a torch Linear weight). */
typedef enum { NQ_B_KN = 0, NQ_B_NK = 1 } nq_b_layout_t;

/* ---- runtime ----------------------------------------------------------- */
const char* nq_status_string(nq_status_t s);
const char* nq_last_error(void);
int nq_version(void);
/* Reads (and with clear != 0 resets) the device-side error word of the
   current device: bit 0 = a bounded wait in a kernel timed out.  Clearing also
   resets the library's per-stream completion flags of that device, which a
   wait that ran out may have left raised. */
nq_status_t nq_device_error_flags(uint32_t* flags, int clear);
/* Upper bound, in ns, of a kernel's wait on counts sent by other GPUs (the
   fused all-reduce below; default 5 s, 0 restores the default).  Applies to
   kernels launched after the call, process-wide.  A wait that runs out sets
   bit 0 of the device error word and the kernel returns.  The reference
   bounds its NCCL waits the same way (safe_stream_wait deadline,
   src/cuda/nccl/nccl_error.cpp:13-83). */
nq_status_t nq_set_peer_wait_limit(uint64_t ns);
uint64_t nq_peer_wait_limit(void);

/* ---- FP8 element-wise, reference codec ------------------------------------
 * Replace src/cuda/quantize/fp8_kernels.cu:29-40 / include/cuda/quantize/
 * fp8_kernels.hpp:30-59.  Codes are bit-identical to FP8E4M3(float) /
 * FP8E5M2(float) of include/cuda/quantize/fp8_types.hpp:64-97,147-189. */
nq_status_t nq_quantize_f32_to_fp8e4m3(const float* src, uint8_t* dst, size_t n, nq_stream_t s);
nq_status_t nq_quantize_f32_to_fp8e5m2(const float* src, uint8_t* dst, size_t n, nq_stream_t s);
/* fp8_kernels.hpp:46 / :48 (dst = decode(src) * scale) */
nq_status_t nq_dequantize_fp8e4m3_to_f32(const uint8_t* src, float* dst, size_t n, float scale,
                                         nq_stream_t s);
nq_status_t nq_dequantize_fp8e5m2_to_f32(const uint8_t* src, float* dst, size_t n, float scale,
                                         nq_stream_t s);
/* fp8_kernels.hpp:50-52: dst[b][i] = FP8E4M3(src[b][i] * scales[b]); the
   pointer arrays, sizes and scales are device arrays, as in the reference. */
nq_status_t nq_quantize_batched_f32_to_fp8e4m3(const float* const* src, uint8_t* const* dst,
                                               int batch, const size_t* sizes,
                                               const float* scales, nq_stream_t s);
/* fp8_kernels.hpp:54-56: dst[b][i] = decode(src[b][i]) * scales[b] */
nq_status_t nq_dequantize_batched_fp8e4m3_to_f32(const uint8_t* const* src, float* const* dst,
                                                 int batch, const size_t* sizes,
                                                 const float* scales, nq_stream_t s);

/* ---- INT8 element-wise -------------------------------------------------------
 * include/cuda/quantize/int8_kernels.hpp:51-55 (and the _async twin :63-67):
 * sym q = clamp(rn(x/scale), +-127); asym q = clamp(rn((x-zp)/scale), +-127). */
nq_status_t nq_quantize_f32_to_int8(const float* src, int8_t* dst, size_t n, float scale,
                                    float zero_point, int symmetric, nq_stream_t s);
/* int8_kernels.hpp:57-61: sym q*scale, asym (q+zp)*scale */
nq_status_t nq_dequantize_int8_to_f32(const int8_t* src, float* dst, size_t n, float scale,
                                      float zero_point, int symmetric, nq_stream_t s);
/* int8_kernels.hpp:75-79 (int8_kernels.cu:171-194) */
nq_status_t nq_quantize_f32_to_int8_with_calibration(const float* src, int8_t* dst, size_t n,
                                                     float min_val, float max_val, nq_stream_t s);
/* Element-wise activations on FP8 codes of the reference codec, the kernels of
   include/cuda/quantize/fp8_activation.hpp (:26-59, :62-98): decode, activate
   in fp32, re-encode (relu: negative inputs become +0, other codes pass
   unchanged; gelu x*0.5*(1+erf(x/sqrt2)); sigmoid 1/(1+exp(-x)); leaky relu
   x >= 0 ? x : alpha*x).  fmt NQ_E4M3 or NQ_E5M2. */
typedef enum { NQ_ACT_RELU = 0, NQ_ACT_GELU = 1, NQ_ACT_SIGMOID = 2, NQ_ACT_LEAKY_RELU = 3 } nq_activation_t;
nq_status_t nq_fp8_activation(const uint8_t* src, uint8_t* dst, size_t n, nq_format_t fmt,
                              nq_activation_t op, float alpha, nq_stream_t s);
/* FakeQuantize::forward of quantization-aware training (qat.hpp:64-72) over a
   device array: scale floored at 1e-6, q = clamp(round_half_away((x - zp) /
   scale), +-127), dst = q * scale + zp (multiply, then add). */
nq_status_t nq_fake_quantize_int8(const float* src, float* dst, size_t n, float scale,
                                  float zero_point, nq_stream_t s);
/* QuantizedTensor<int8_t>::FromFloat rounding (quantize_tensor.hpp:176-182):
   q = clamp(round_half_away(x/scale), +-127). */
nq_status_t nq_quantize_f32_to_int8_round_away(const float* src, int8_t* dst, size_t n,
                                               float scale, nq_stream_t s);

/* dst = (float)src for n bf16 values (exact).  No reference counterpart: the
   drop-in TP layers return the bf16 output of the fused all-reduce as the fp32
   the reference's forward(float*) writes. */
nq_status_t nq_convert_bf16_to_f32(const void* src, float* dst, size_t n, nq_stream_t s);

/* ---- reductions and calibration ----------------------------------------------
 * int8_kernels.hpp:88-92 (int8_kernels.cu:324-410).  `data` may be host or
 * device memory, as may `min_val` / `max_val`.  Synchronises `s`.  NaNs are
 * ignored; n == 0 gives 0, 0. */
nq_status_t nq_compute_minmax(const float* data, size_t n, float* min_val, float* max_val,
                              nq_stream_t s);
/* int8_kernels.hpp:81-86 (int8_kernels.cu:275-322).  `data` host or device,
   `histogram` device with num_bins entries, zeroed here.  Synchronises `s`.
   Unlike the reference kernel, any num_bins in [1, 65536] is counted
   correctly (the reference kept only 256 shared bins). */
nq_status_t nq_build_histogram(const float* data, uint32_t* histogram, size_t n, float min_val,
                               float max_val, int num_bins, nq_stream_t s);

/* Device-resident, asynchronous min/max: d_out[0] = min, d_out[1] = max. */
nq_status_t nq_minmax_async(const float* data, size_t n, float* d_out, nq_stream_t s);
/* amax of |x| and the per-tensor scale for `fmt`: d_out[0] = amax,
   d_out[1] = amax / qmax (448, 57344 or 127), 1.0 when amax == 0.
   src_dtype NQ_F32 or NQ_BF16. */
nq_status_t nq_amax_scale_async(const void* data, nq_dtype_t src_dtype, size_t n,
                                nq_format_t fmt, float* d_out, nq_stream_t s);
/* Per-channel min/max of a rows x cols row-major matrix (one channel per
   row, the layout PerChannelCalibrator::calibrate_per_channel walks,
   calibrator.cpp:233-253) in one launch. */
nq_status_t nq_minmax_rows(const float* data, int rows, int cols, float* d_min, float* d_max,
                           nq_stream_t s);

/* ---- scaled quantize (OCP FP8 / INT8, RNE, saturating) ---------------------
 * q = encode(x / scale) with an IEEE division; `d_scale` is a device scalar
 * (e.g. written by nq_amax_scale_async, no host round trip). */
nq_status_t nq_quantize_scaled(const void* src, nq_dtype_t src_dtype, uint8_t* dst, size_t n,
                               nq_format_t fmt, const float* d_scale, nq_stream_t s);
/* dst = decode(q) * scale (f32 out) */
nq_status_t nq_dequantize_scaled(const uint8_t* src, float* dst, size_t n, nq_format_t fmt,
                                 const float* d_scale, nq_stream_t s);
/* amax -> scale -> quantize, two launches, no host synchronisation.
   d_amax_scale receives {amax, scale}. */
nq_status_t nq_calibrate_quantize(const void* src, nq_dtype_t src_dtype, uint8_t* dst, size_t n,
                                  nq_format_t fmt, float* d_amax_scale, nq_stream_t s);
/* Per-row dynamic quantization (per token of activations, or per output
   channel of an N x K weight): scales[r] = amax(row r)/qmax (1.0 for an
   all-zero row), q = encode(x * (qmax / amax(row r))), the reciprocal taken
   once per row (a row whose qmax / amax overflows float uses
   q = encode(x / scales[r])).  One launch. */
nq_status_t nq_quantize_rows(const void* src, nq_dtype_t src_dtype, uint8_t* dst, float* scales,
                             int rows, int cols, nq_format_t fmt, nq_stream_t s);
/* Per-column scales of a rows x cols (K x N) row-major fp32 matrix: the
   per-output-channel scales of a weight in FP8GEMM's B layout (the
   arithmetic of nq_quantize_rows, per column). */
nq_status_t nq_quantize_cols(const float* src, uint8_t* dst, float* scales, int rows, int cols,
                             nq_format_t fmt, nq_stream_t s);

/* Allocation-free twin of nq_quantize_cols, for callers that must not
   allocate device memory during the call (an engine that owns all of HBM
   through its own allocator, a plugin host that only hands over input and
   output buffers, a loop where cudaMalloc's implicit synchronisation is not
   allowed).  No counterpart in the reference.  Same results as
   nq_quantize_cols; the per-column amax scratch is a fixed 256 KiB device
   array inside libnova_q that every GPU loading the library holds until
   process exit, so cols is limited to 65536 (larger widths return
   NQ_ERROR_UNSUPPORTED).  The first call on a device looks up that array's
   address (cudaGetSymbolAddress) with the device current: make that first
   call before any stream capture.  All calls share the one array, so calls
   that overlap on the GPU (other streams, other threads) race; serialise
   them.  Nothing is allocated or freed: the scratch is cleared with
   cudaMemsetAsync on `s` at the start of every call. */
nq_status_t nq_quantize_cols_noalloc(const float* src, uint8_t* dst, float* scales, int rows,
                                     int cols, nq_format_t fmt, nq_stream_t s);

/* ---- GEMM -------------------------------------------------------------------
 * out[m, n] = epi( sum_k A[m, k] * B[k, n] )
 *   A: M x K row-major codes (K-major), B: per b_layout.
 *   FP8 (a/b_format E4M3/E5M2, any mix): fp32 accumulation on tcgen05
 *   kind::f8f6f4.  INT8 (both NQ_INT8): exact int32 accumulation on
 *   tcgen05 kind::i8.
 *   epi(acc) = ((acc * alpha) [* row_scale[m]]) [* col_scale[n]] [+ bias[n]],
 *   each step one fp32 rounding, then converted to out_dtype (NQ_F32,
 *   NQ_BF16 round-to-nearest-even, NQ_S8 clamp-and-round, or NQ_S32 = raw
 *   int32 accumulators, INT8 only).
 * Shapes with K % 16, N % 16 or pointers not 16-byte aligned run a SIMT
 * kernel with the same arithmetic. */
/* Epilogue functions applied after the scales:
   NQ_EPI_SWIGLU: the N columns of B hold gate and up weights packed in
   alternating 128-column blocks ([g_0 | u_0 | g_1 | u_1 | ...], block j of
   the output = columns 256j..256j+255 of B); the output is M x N/2 with
   out[:, 128j + c] = silu(g) * u, silu(g) = g / (1 + exp(-g)), g and u the
   scaled values of packed columns 256j + c and 256j + 128 + c (the fused form
   of silu_and_mul, activations.cu:80-92).  Needs N % 256 == 0 and the
   tensor-core path; col_scale and bias are indexed by packed column. */
typedef enum { NQ_EPI_NONE = 0, NQ_EPI_SWIGLU = 1 } nq_epilogue_t;

typedef struct {
    int m, n, k;
    nq_format_t a_format, b_format;
    nq_b_layout_t b_layout;
    nq_dtype_t out_dtype;
    float alpha;
    const float* row_scale; /* [m] device, or NULL */
    const float* col_scale; /* [n] device, or NULL */
    const float* bias;      /* [n] device, or NULL */
    nq_epilogue_t epilogue; /* NQ_EPI_NONE unless stated */
} nq_gemm_desc_t;

nq_status_t nq_gemm(const nq_gemm_desc_t* desc, const void* a, const void* b, void* out,
                    nq_stream_t s);
/* W8A8 GEMM with the per-token dynamic quantization of the activations fused
   into the kernel (a row-parallel or up-projection layer fed bf16
   activations).  x: m x k bf16, row-major.  The kernel quantizes every row of
   x exactly as nq_quantize_rows(x, NQ_BF16, a_codes, a_scales, m, k, NQ_E4M3)
   does -- bit-identical codes and scales, written to a_codes (m x k) and
   a_scales (m) -- and multiplies the codes by B with a_scales as the
   epilogue's row scale, in ONE launch: the grid's warps quantize the rows
   first and publish each 128-row block, and a tile's A loads wait (bounded)
   for its block.  desc: a_format NQ_E4M3, b_format E4M3 or E5M2, row_scale
   NULL, out_dtype NQ_BF16 or NQ_F32, epilogue NONE or SWIGLU; k, n multiples
   of 16 and 16-byte aligned pointers.  No reference counterpart: the
   reference's FP8GEMM::forward (fp8_gemm.cu:164-188) takes codes already
   quantized per tensor. */
nq_status_t nq_gemm_quant_a(const nq_gemm_desc_t* desc, const void* x, uint8_t* a_codes, float* a_scales,
                            const void* b, void* out, nq_stream_t s);
/* The same GEMM on the CUDA cores only (one thread per output, sequential-k
   fp32 FMA or int32 accumulation): an exactly ordered variant for checking
   and for shapes far below one tensor-core tile. */
nq_status_t nq_gemm_simt(const nq_gemm_desc_t* desc, const void* a, const void* b, void* out,
                         nq_stream_t s);

/* ---- GEMMs fused with the all-reduce of a row-parallel layer ------------------
 * RowParallelLayer::forward (tensor_parallel_layers.cpp:370-416) is a GEMM on
 * the rank's K shard followed by ncclAllReduce(sum) of the M x N output
 * (:406).  Here the all-reduce runs inside the GEMM kernels, over NVLink:
 *
 *  signal  the GEMM's output is a partial: its bf16 tiles go to the `out`
 *          argument (this rank's partial buffer); once a 256 x 256 tile's
 *          stores are complete a signaller warp adds 1 to the tile's counter
 *          on the tile's owner rank (tile % tp);
 *  job     the kernel's reducer warps (5 per CTA pair, beside the GEMM's own
 *          warps) sum the tiles of an m x n output that this rank owns, once
 *          all tp ranks have signalled them, and write the bf16 sum to every
 *          rank's output buffer:
 *            multicast (mc_partial / mc_out / mc_done non-NULL):
 *              multimem.ld_reduce (fp32 accumulation in the NVSwitch, one bf16
 *              rounding) and multimem.st;
 *            peer (multicast NULL): loads of the tp partials through the
 *              peer pointers, fp32 sum in rank order, one bf16 rounding,
 *              stores to every peer;
 *          each reducer warp then counts itself on every rank's completion
 *          counter (nq_allreduce_done_per_job);
 *  finish  with `done` set the kernel returns only once this rank's
 *          completion counter reaches done_target (its output buffer holds
 *          every reduced tile).
 *
 * nq_gemm_allreduce runs a GEMM with any of the three; with all three on the
 * GEMM's own output it is the whole row-parallel layer in one kernel.  A job
 * on an EARLIER output lets a token chunk's all-reduce overlap the next
 * chunk's GEMMs (the SwiGLU gate/up GEMM included).  nq_allreduce_finish runs
 * a job and / or finish without a GEMM.
 *
 * All buffers are symmetric allocations (same size on every rank, mapped into
 * every peer); job pointers address the job's first row.  Counters only
 * grow: zero before the first use; the n-th use of a counter set passes
 * epoch = n modulo 2^32 and a job waits for its tiles' counters to reach
 * epoch * tp.  Counters and targets are compared modulo 2^32 (the signed
 * difference), so they may wrap.  Every rank makes the same sequence of
 * calls.  Waits on other GPUs give up after nq_peer_wait_limit() ns (5 s by
 * default) and set the device error word (nq_device_error_flags).  A signalling GEMM
 * needs out_dtype NQ_BF16, epilogue NQ_EPI_NONE, n % 256 == 0; jobs need
 * n % 256 == 0; 1 <= tp <= NQ_MAX_TP. */
#define NQ_MAX_TP 8
typedef struct {
    int tp, rank;
    uint32_t epoch;                      /* 1 for the first use of the counters, then 2, ... (mod 2^32) */
    /* signal */
    int signal;                          /* 1: the GEMM's output is a partial */
    uint32_t* signal_flags[NQ_MAX_TP];   /* every rank's counters of the output's tiles */
    /* job */
    int m, n;                            /* the output to reduce; m == 0: no job */
    uint32_t* flags;                     /* this rank's counters of the job's tiles */
    void* mc_partial;                    /* multicast partial buffers, or NULL */
    void* mc_out;                        /* multicast output buffers, or NULL */
    uint32_t* mc_done;                   /* multicast completion counters, or NULL */
    void* peer_partial[NQ_MAX_TP];       /* peer path: every rank's partial buffer */
    void* peer_out[NQ_MAX_TP];           /* peer path: every rank's output buffer */
    uint32_t* peer_done[NQ_MAX_TP];      /* peer path: every rank's completion counter */
    /* finish (done non-NULL) */
    uint32_t* done;                      /* this rank's completion counter, or NULL: no finish */
    uint32_t done_target;                /* wait until *done reaches it (modulo 2^32) */
} nq_allreduce_desc_t;

/* Tiles (counters) of an m x n output. */
int nq_gemm_allreduce_counters(int m, int n);
/* Completion counts one job of an m x n output adds on every rank: 5 per tile,
   4 when the kernel hosting the job also signals its own output (one of its
   reducer warps is then the signaller). */
int nq_allreduce_done_per_job(int m, int n, int in_signalling_kernel);
nq_status_t nq_gemm_allreduce(const nq_gemm_desc_t* desc, const nq_allreduce_desc_t* ar,
                              const void* a, const void* b, void* out, nq_stream_t s);
nq_status_t nq_allreduce_finish(const nq_allreduce_desc_t* ar, nq_stream_t s);

/* FP8GEMM::forward / forward_async, include/cuda/quantize/fp8_gemm.hpp:55-69
   (fp8_gemm.cu:164-198): fp32 out = scale_out * sum (a*scale_a)(b*scale_b),
   A M x K, B K x N, E4M3 codes read as OCP E4M3FN by the tensor cores. */
nq_status_t nq_fp8_gemm_forward(const uint8_t* a, const uint8_t* b, float* out, int m, int k,
                                int n, float scale_a, float scale_b, float scale_out,
                                nq_stream_t s);
/* FP8E5M2GEMM::forward, fp8_gemm.hpp:101-107 (fp8_gemm.cu:232-258); the
   operands are decoded as E5M2 (the reference reinterpreted them as E4M3). */
nq_status_t nq_fp8e5m2_gemm_forward(const uint8_t* a, const uint8_t* b, float* out, int m, int k,
                                    int n, float scale_a, float scale_b, float scale_out,
                                    nq_stream_t s);
/* Gradients of C = (A.B)*scale_a*scale_b for FP8 operands, with the transposes
   FP8GEMM::backward omits (fp8_gemm.cu:200-230 passes A and B untransposed):
     grad_a (M x K) = scale_grad*scale_b * grad_out (M x N) . B^T
     grad_b (K x N) = scale_a*scale_grad * A^T . grad_out
   A M x K and B K x N E4M3, grad_out M x N in grad_format (E4M3, or E5M2 for
   the usual gradient range), fp32 outputs; either output may be NULL to skip
   it.  grad_b transposes A once into pool scratch. */
nq_status_t nq_fp8_gemm_backward(const uint8_t* grad_out, nq_format_t grad_format, const uint8_t* a,
                                 const uint8_t* b, float* grad_a, float* grad_b, int m, int k, int n,
                                 float scale_grad, float scale_a, float scale_b, nq_stream_t s);
/* QuantizedMatmul::mixed_precision, quantize_ops.hpp:83-102 (W8 A32):
   out[i,j] = sum_p a[i,p] * (b[p,j] * scale_b[p]) in order, one rounding per
   multiply and add (the reference host loop); all pointers device. */
nq_status_t nq_mixed_precision_matmul(const float* a, const int8_t* b, const float* scale_b,
                                      float* out, int m, int k, int n, nq_stream_t s);

/* FP8GEMM::get_workspace_size, fp8_gemm.cu:152-162 (same formula; the
   kernels here need no workspace). */
size_t nq_fp8_gemm_workspace_size(int m, int k, int n);

#ifdef __cplusplus
}
#endif
#endif /* NOVA_Q_H */

// reduce.cu -- min/max, amax, histograms and per-row / per-column scaled
// quantization (all HBM-bound).
//
// Whole-tensor reductions are single launches: every block reduces its
// grid-stride share with 128-bit loads and warp shuffles, writes one partial to
// stream-ordered scratch, and the last block to arrive (atomic ticket) folds the
// partials and writes the result to device memory -- no host round trip, unlike
// the reference's host-side finish (int8_kernels.cu:379-389).
//
// Per-row quantize stages whole rows in shared memory with 1-D bulk copies:
// one warp per row up to 12 KB (k_quant_rows_warp), one block per row up to
// 100 KB (k_quant_rows_bulk), a two-pass kernel otherwise (k_quant_rows).
#include <algorithm>
#include <cfloat>
#include <cstring>
#include <mutex>
#include <string>
#include <type_traits>

#include "codec.cuh"
#include "nq_internal.h"
#include "ptx.cuh"

namespace nq {

nq_status_t quantize_scaled_impl(const void* src, nq_dtype_t dt, uint8_t* dst, size_t n, nq_format_t fmt,
                                 const float* d_scale, cudaStream_t s);

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
// Block-wide min and max (all threads get the result).
__device__ __forceinline__ float2 block_minmax(float lo, float hi) {
    __shared__ float s_lo[32], s_hi[32];
    lo = warp_min(lo);
    hi = warp_max(hi);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) { s_lo[w] = lo; s_hi[w] = hi; }
    __syncthreads();
    const int nw = blockDim.x >> 5;
    lo = l < nw ? s_lo[l] : FLT_MAX;
    hi = l < nw ? s_hi[l] : -FLT_MAX;
    lo = warp_min(lo);
    hi = warp_max(hi);
    __syncthreads();
    return make_float2(lo, hi);
}

template <class In>
__device__ __forceinline__ void load4(const In* p, float (&x)[4]);
template <>
__device__ __forceinline__ void load4<float>(const float* p, float (&x)[4]) {
    float4 v = __ldg(reinterpret_cast<const float4*>(p));
    x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
}
template <>
__device__ __forceinline__ void load4<uint16_t>(const uint16_t* p, float (&x)[4]) {
    uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
    x[0] = __uint_as_float(v.x << 16); x[1] = __uint_as_float(v.x & 0xFFFF0000u);
    x[2] = __uint_as_float(v.y << 16); x[3] = __uint_as_float(v.y & 0xFFFF0000u);
}
__device__ __forceinline__ float ld1(const float* p) { return __ldg(p); }
__device__ __forceinline__ float ld1(const uint16_t* p) { return __uint_as_float(static_cast<uint32_t>(__ldg(p)) << 16); }

// ABS = false: (min, max) of x.  ABS = true: (0-based) max of |x| in .y.
// out: ABS=false -> out[0]=min, out[1]=max (or two separate pointers);
//      ABS=true  -> out[0]=amax, out[1]=amax/qmax (1 if amax == 0).
template <bool ABS, class In>
__global__ void __launch_bounds__(kThreads) k_minmax(const In* __restrict__ src, size_t n, int vec,
                                                     float* __restrict__ partials,
                                                     unsigned int* __restrict__ ticket, float* out_lo,
                                                     float* out_hi, float qmax) {
    float lo = FLT_MAX, hi = ABS ? 0.0f : -FLT_MAX;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    const size_t t0 = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const size_t n4 = vec ? n / 4 : 0;
    // two independent 16-byte loads in flight per thread per step
    size_t v = t0;
    for (; v + stride < n4; v += 2 * stride) {
        float x[4], y[4];
        load4<In>(src + v * 4, x);
        load4<In>(src + (v + stride) * 4, y);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if (ABS) {
                hi = fmaxf(hi, fmaxf(fabsf(x[i]), fabsf(y[i])));
            } else {
                lo = fminf(lo, fminf(x[i], y[i]));
                hi = fmaxf(hi, fmaxf(x[i], y[i]));
            }
        }
    }
    for (; v < n4; v += stride) {
        float x[4];
        load4<In>(src + v * 4, x);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if (ABS) hi = fmaxf(hi, fabsf(x[i]));
            else { lo = fminf(lo, x[i]); hi = fmaxf(hi, x[i]); }
        }
    }
    for (size_t i = n4 * 4 + t0; i < n; i += stride) {
        const float x = ld1(src + i);
        if (ABS) hi = fmaxf(hi, fabsf(x));
        else { lo = fminf(lo, x); hi = fmaxf(hi, x); }
    }
    float2 r = block_minmax(lo, hi);
    __shared__ bool s_last;
    if (threadIdx.x == 0) {
        partials[2 * blockIdx.x] = r.x;
        partials[2 * blockIdx.x + 1] = r.y;
        __threadfence();
        const unsigned int t = atomicAdd(ticket, 1u);
        s_last = (t == gridDim.x - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    lo = FLT_MAX;
    hi = ABS ? 0.0f : -FLT_MAX;
    for (unsigned int b = threadIdx.x; b < gridDim.x; b += blockDim.x) {
        lo = fminf(lo, __ldcg(partials + 2 * b));
        hi = fmaxf(hi, __ldcg(partials + 2 * b + 1));
    }
    r = block_minmax(lo, hi);
    if (threadIdx.x == 0) {
        if (ABS) {
            out_lo[0] = r.y;
            out_lo[1] = r.y > 0.0f ? r.y / qmax : 1.0f;
        } else {
            *out_lo = r.x;
            *out_hi = r.y;
        }
        *ticket = 0u;
    }
}

// One block per row: min and max of the row (PerChannelCalibrator channels).
__global__ void __launch_bounds__(kThreads) k_minmax_rows(const float* __restrict__ src, int cols,
                                                          float* __restrict__ d_min, float* __restrict__ d_max) {
    const float* row = src + static_cast<size_t>(blockIdx.x) * cols;
    float lo = FLT_MAX, hi = -FLT_MAX;
    const bool vec = ((reinterpret_cast<uintptr_t>(row) & 15u) == 0);
    const int n4 = vec ? cols / 4 : 0;
    for (int v = threadIdx.x; v < n4; v += blockDim.x) {
        float x[4];
        load4<float>(row + 4 * v, x);
#pragma unroll
        for (int i = 0; i < 4; ++i) { lo = fminf(lo, x[i]); hi = fmaxf(hi, x[i]); }
    }
    for (int i = n4 * 4 + threadIdx.x; i < cols; i += blockDim.x) {
        const float x = __ldg(row + i);
        lo = fminf(lo, x);
        hi = fmaxf(hi, x);
    }
    float2 r = block_minmax(lo, hi);
    if (threadIdx.x == 0) {
        d_min[blockIdx.x] = r.x;
        d_max[blockIdx.x] = r.y;
    }
}

// Histogram with a block-private shared copy of all bins (int8_kernels.cu:
// 97-129 restated for any bin count): bin = (int)((x-min)/range*(bins-1)),
// truncating and saturating like cvt.rzi, clamped to [0, bins-1].
template <bool SHARED>
__global__ void __launch_bounds__(kThreads) k_histogram(const float* __restrict__ src, size_t n, int vec,
                                                        uint32_t* __restrict__ hist, float min_val, float range,
                                                        int bins) {
    extern __shared__ uint32_t s_hist[];
    uint32_t* h = SHARED ? s_hist : hist;
    if (SHARED) {
        for (int i = threadIdx.x; i < bins; i += blockDim.x) s_hist[i] = 0;
        __syncthreads();
    }
    const float mul = static_cast<float>(bins - 1);
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    const size_t t0 = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const size_t n4 = vec ? n / 4 : 0;
    auto bin_of = [&](float x) {
        int b = __float2int_rz((x - min_val) / range * mul);
        return max(0, min(bins - 1, b));
    };
    for (size_t v = t0; v < n4; v += stride) {
        float x[4];
        load4<float>(src + 4 * v, x);
#pragma unroll
        for (int i = 0; i < 4; ++i) atomicAdd(h + bin_of(x[i]), 1u);
    }
    for (size_t i = n4 * 4 + t0; i < n; i += stride) atomicAdd(h + bin_of(__ldg(src + i)), 1u);
    if (SHARED) {
        __syncthreads();
        for (int i = threadIdx.x; i < bins; i += blockDim.x)
            if (s_hist[i]) atomicAdd(hist + i, s_hist[i]);
    }
}

using dev::encode_vec;
using dev::row_scale;
using dev::RowScale;
using dev::scale_apply;
using dev::vec_elem;

// Per-row scaled quantize, any width and alignment: one block per row; the
// second pass re-reads the row (from L1/L2).
template <int F, class In>
__global__ void __launch_bounds__(kThreads) k_quant_rows(const In* __restrict__ src, uint8_t* __restrict__ dst,
                                                         float* __restrict__ scales, int cols) {
    const size_t r = blockIdx.x;
    const In* row = src + r * static_cast<size_t>(cols);
    uint8_t* out = dst + r * static_cast<size_t>(cols);
    const bool vec = (cols % 16 == 0) && ((reinterpret_cast<uintptr_t>(row) & 15u) == 0) &&
                     ((reinterpret_cast<uintptr_t>(out) & 15u) == 0);
    const int n4 = vec ? cols / 4 : 0;
    float a = 0.0f;
    for (int v = threadIdx.x; v < n4; v += blockDim.x) {
        float x[4];
        load4<In>(row + 4 * v, x);
#pragma unroll
        for (int i = 0; i < 4; ++i) a = fmaxf(a, fabsf(x[i]));
    }
    for (int i = n4 * 4 + threadIdx.x; i < cols; i += blockDim.x) a = fmaxf(a, fabsf(ld1(row + i)));
    a = block_minmax(FLT_MAX, a).y;
    const RowScale rs = row_scale<F>(a);
    if (threadIdx.x == 0) scales[r] = rs.s;
    auto pass = [&](auto mul_tag) {
        constexpr bool MUL = decltype(mul_tag)::value;
        for (int v = threadIdx.x; v < n4; v += blockDim.x) {
            float x[4];
            load4<In>(row + 4 * v, x);
            const uint32_t p0 = dev::ocp_encode2<F>(scale_apply<MUL>(x[0], rs), scale_apply<MUL>(x[1], rs));
            const uint32_t p1 = dev::ocp_encode2<F>(scale_apply<MUL>(x[2], rs), scale_apply<MUL>(x[3], rs));
            reinterpret_cast<uint32_t*>(out)[v] = p0 | (p1 << 16);
        }
        for (int i = n4 * 4 + threadIdx.x; i < cols; i += blockDim.x)
            out[i] = static_cast<uint8_t>(dev::ocp_encode2<F>(scale_apply<MUL>(ld1(row + i), rs), 0.0f) & 0xFFu);
    };
    if (rs.mul) pass(std::true_type{});
    else pass(std::false_type{});
}

// Per-row scaled quantize with rows staged whole in shared memory by 1-D bulk
// copies: a persistent grid, block b owning rows b, b + gridDim.x, ...; a
// ring of `stages` row buffers keeps the next rows streaming in from HBM
// while the current one is reduced and encoded (one HBM read per element,
// and a block never idles on a single row's load latency).  Row bytes
// (cols * sizeof(In)) must be a multiple of 16 and src 16-byte aligned.
template <int F, class In>
__global__ void __launch_bounds__(kThreads) k_quant_rows_bulk(const In* __restrict__ src, uint8_t* __restrict__ dst,
                                                              float* __restrict__ scales, int rows, int cols,
                                                              int stages, uint32_t* err) {
    extern __shared__ __align__(128) uint8_t q_smem[];
    constexpr int EPV = 16 / sizeof(In);
    const uint32_t rb = static_cast<uint32_t>(cols) * sizeof(In);
    uint64_t* full = reinterpret_cast<uint64_t*>(q_smem + static_cast<size_t>(stages) * rb);
    const int nv = cols / EPV;
    dev::pdl_launch_dependents();  // launched with programmatic stream serialization
    if (threadIdx.x == 0) {
        for (int k = 0; k < stages; ++k) dev::mbar_init(&full[k], 1);
        dev::fence_mbar_init();
    }
    __syncthreads();
    dev::pdl_wait();  // the rows may come from the previous kernel
    const char* base = reinterpret_cast<const char*>(src);
    auto row_of = [&](int i) { return static_cast<long long>(blockIdx.x) + static_cast<long long>(i) * gridDim.x; };
    auto issue = [&](int i) {
        const long long r = row_of(i);
        if (r >= rows) return;
        const int st = i % stages;
        dev::mbar_arrive_expect_tx(&full[st], rb);
        dev::bulk_load_1d(q_smem + static_cast<size_t>(st) * rb, base + r * rb, rb, &full[st]);
    };
    if (threadIdx.x == 0)
        for (int i = 0; i < stages; ++i) issue(i);
    int i = 0;
    bool ok = true;
    for (;; ++i) {
        const long long r = row_of(i);
        if (r >= rows) break;
        const int st = i % stages;
        ok = dev::mbar_wait(&full[st], static_cast<uint32_t>(i / stages) & 1u, err);
        if (!__syncthreads_and(ok)) {
            ok = false;
            break;
        }
        const uint4* buf = reinterpret_cast<const uint4*>(q_smem + static_cast<size_t>(st) * rb);
        float a = 0.0f;
        for (int v = threadIdx.x; v < nv; v += kThreads) {
            const uint4 q = buf[v];
#pragma unroll
            for (int e = 0; e < EPV; ++e) a = fmaxf(a, fabsf(vec_elem<In>(q, e)));
        }
        a = block_minmax(FLT_MAX, a).y;
        const RowScale rs = row_scale<F>(a);
        if (threadIdx.x == 0) scales[r] = rs.s;
        uint8_t* out = dst + r * cols;
        if (rs.mul) {
            for (int v = threadIdx.x; v < nv; v += kThreads) encode_vec<F, In, true>(buf[v], out + v * EPV, rs);
        } else {
            for (int v = threadIdx.x; v < nv; v += kThreads) encode_vec<F, In, false>(buf[v], out + v * EPV, rs);
        }
        __syncthreads();  // every thread is done with buffer st
        if (threadIdx.x == 0) issue(i + stages);
    }
    if (!ok && threadIdx.x == 0) {
        // a wait gave up: let the copies still in flight land before the block exits
        for (int j = i; j < i + stages && row_of(j) < rows; ++j)
            dev::mbar_wait(&full[j % stages], static_cast<uint32_t>(j / stages) & 1u, nullptr);
    }
}

// Per-row scaled quantize, one warp per row, for rows of up to 12 KB: each
// warp streams its rows (global warp w takes rows w, w + warps, ...) through a
// private ring of `stages` row buffers filled by 1-D bulk copies, and reduces
// the row amax with shuffles -- no block barrier per row, so short rows from
// many warps are in flight at once.  Row bytes must be a multiple of 16 and
// src 16-byte aligned.
template <int F, class In>
__global__ void __launch_bounds__(kThreads) k_quant_rows_warp(const In* __restrict__ src, uint8_t* __restrict__ dst,
                                                              float* __restrict__ scales, int rows, int cols,
                                                              int stages, uint32_t* err) {
    extern __shared__ __align__(128) uint8_t q_smem[];
    constexpr int EPV = 16 / sizeof(In);
    constexpr int kWarps = kThreads / 32;
    const uint32_t rb = static_cast<uint32_t>(cols) * sizeof(In);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    uint8_t* ring = q_smem + static_cast<size_t>(warp) * stages * rb;
    uint64_t* full = reinterpret_cast<uint64_t*>(q_smem + static_cast<size_t>(kWarps) * stages * rb) + warp * stages;
    const int nv = cols / EPV;
    dev::pdl_launch_dependents();  // launched with programmatic stream serialization
    if (lane == 0) {
        for (int k = 0; k < stages; ++k) dev::mbar_init(&full[k], 1);
        dev::fence_mbar_init();
    }
    __syncwarp();
    dev::pdl_wait();  // the rows may come from the previous kernel
    const long long gw = static_cast<long long>(blockIdx.x) * kWarps + warp;
    const long long nw = static_cast<long long>(gridDim.x) * kWarps;
    const char* base = reinterpret_cast<const char*>(src);
    auto issue = [&](int i) {
        const long long r = gw + i * nw;
        if (r >= rows) return;
        const int st = i % stages;
        dev::mbar_arrive_expect_tx(&full[st], rb);
        dev::bulk_load_1d(ring + static_cast<size_t>(st) * rb, base + r * rb, rb, &full[st]);
    };
    if (lane == 0)
        for (int i = 0; i < stages; ++i) issue(i);
    int i = 0;
    bool ok = true;
    for (;; ++i) {
        const long long r = gw + i * nw;
        if (r >= rows) break;
        const int st = i % stages;
        ok = dev::mbar_wait(&full[st], static_cast<uint32_t>(i / stages) & 1u, err);
        if (!__all_sync(0xffffffffu, ok)) {
            ok = false;
            break;
        }
        const uint4* buf = reinterpret_cast<const uint4*>(ring + static_cast<size_t>(st) * rb);
        float a = 0.0f;
        for (int v = lane; v < nv; v += 32) {
            const uint4 q = buf[v];
#pragma unroll
            for (int e = 0; e < EPV; ++e) a = fmaxf(a, fabsf(vec_elem<In>(q, e)));
        }
        a = warp_max(a);
        const RowScale rs = row_scale<F>(a);
        if (lane == 0) scales[r] = rs.s;
        uint8_t* out = dst + r * cols;
        if (rs.mul) {
            for (int v = lane; v < nv; v += 32) encode_vec<F, In, true>(buf[v], out + v * EPV, rs);
        } else {
            for (int v = lane; v < nv; v += 32) encode_vec<F, In, false>(buf[v], out + v * EPV, rs);
        }
        __syncwarp();  // every lane is done with buffer st
        if (lane == 0) issue(i + stages);
    }
    if (!ok && lane == 0) {
        for (int j = i; j < i + stages && gw + j * nw < rows; ++j)
            dev::mbar_wait(&full[j % stages], static_cast<uint32_t>(j / stages) & 1u, nullptr);
    }
}

// Per-column amax of a rows x cols matrix: grid.x over column groups of 4 x
// 256, grid.y over row chunks; partial maxima of |x| (>= 0, so their float bit
// patterns order like unsigned ints) are merged with atomicMax.
__global__ void __launch_bounds__(kThreads) k_col_amax(const float* __restrict__ src, int rows, int cols,
                                                       int rows_per_chunk, uint32_t* __restrict__ amax_bits) {
    const int c4 = blockIdx.x * blockDim.x + threadIdx.x;  // group of 4 columns
    const int c = c4 * 4;
    if (c >= cols) return;
    const int r0 = blockIdx.y * rows_per_chunk;
    const int r1 = min(rows, r0 + rows_per_chunk);
    float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const bool vec = (cols % 4 == 0) && ((reinterpret_cast<uintptr_t>(src) & 15u) == 0);
    for (int r = r0; r < r1; ++r) {
        const float* p = src + static_cast<size_t>(r) * cols + c;
        if (vec) {
            float x[4];
            load4<float>(p, x);
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = fmaxf(a[i], fabsf(x[i]));
        } else {
            for (int i = 0; i < 4 && c + i < cols; ++i) a[i] = fmaxf(a[i], fabsf(__ldg(p + i)));
        }
    }
    for (int i = 0; i < 4 && c + i < cols; ++i) atomicMax(amax_bits + c + i, __float_as_uint(a[i]));
}

template <int F>
__global__ void __launch_bounds__(kThreads) k_quant_cols(const float* __restrict__ src, uint8_t* __restrict__ dst,
                                                         const uint32_t* __restrict__ amax_bits,
                                                         float* __restrict__ scales, int rows, int cols) {
    const size_t total = static_cast<size_t>(rows) * cols;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int c = static_cast<int>(i % cols);
        const RowScale rs = row_scale<F>(__uint_as_float(__ldg(amax_bits + c)));
        if (i < static_cast<size_t>(cols)) scales[c] = rs.s;
        const float x = __ldg(src + i);
        dst[i] = static_cast<uint8_t>(dev::ocp_encode2<F>(rs.mul ? x * rs.inv : x / rs.s, 0.0f) & 0xFFu);
    }
}

// ---- host helpers -----------------------------------------------------------------
}  // namespace

constexpr size_t kBulkRowSmem = 200 * 1024;  // ring budget of one block of k_quant_rows_bulk

// Ring depth: 4 rows up to 16 KB rows, else as many as fit 200 KB (>= 2);
// grid: every block that fits on the device at once (persistent).
template <int F>
nq_status_t launch_quant_rows_bulk(const void* src, nq_dtype_t dt, uint8_t* dst, float* scales, int rows, int cols,
                                   const DeviceInfo& di, cudaStream_t s) {
    const size_t rb = static_cast<size_t>(cols) * (dt == NQ_F32 ? 4 : 2);
    const int stages = rb <= 16384 ? 4 : static_cast<int>(std::min<size_t>(4, kBulkRowSmem / rb));
    const int smem = static_cast<int>(stages * rb + 8 * stages);
    auto launch = [&](auto kern, const auto* typed_src) -> nq_status_t {
        static std::mutex mu;
        static std::atomic<uint64_t> attr_set{0};
        nq_status_t st = once_per_device(attr_set, mu, di.device, [&]() -> nq_status_t {
            NQ_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(kBulkRowSmem + 64)),
                          "cudaFuncSetAttribute(quantize_rows)");
            return NQ_SUCCESS;
        });
        if (st != NQ_SUCCESS) return st;
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem) != cudaSuccess || per_sm < 1) {
            cudaGetLastError();
            per_sm = 1;
        }
        const int grid = static_cast<int>(std::min<long long>(rows, static_cast<long long>(di.sm_count) * per_sm));
        NQ_CHECK_CUDA(launch_pdl(kern, dim3(grid), dim3(kThreads), smem, s, typed_src, dst, scales, rows, cols, stages,
                                 device_error_word()),
                      "nq_quantize_rows (bulk)");
        return NQ_SUCCESS;
    };
    if (dt == NQ_F32) return launch(k_quant_rows_bulk<F, float>, static_cast<const float*>(src));
    return launch(k_quant_rows_bulk<F, uint16_t>, static_cast<const uint16_t*>(src));
}

constexpr size_t kWarpRowMax = 12 * 1024;  // rows up to this size take k_quant_rows_warp

// Ring depth per warp: about 24 KB of rows (2 .. 8 stages); grid: every block
// that fits on the device at once, at most one warp per row.
template <int F>
nq_status_t launch_quant_rows_warp(const void* src, nq_dtype_t dt, uint8_t* dst, float* scales, int rows, int cols,
                                   const DeviceInfo& di, cudaStream_t s) {
    const size_t rb = static_cast<size_t>(cols) * (dt == NQ_F32 ? 4 : 2);
    const int stages = static_cast<int>(std::max<size_t>(2, std::min<size_t>(8, (24 * 1024) / rb)));
    constexpr int warps = kThreads / 32;
    const int smem = static_cast<int>(warps * stages * rb + warps * stages * 8);
    auto launch = [&](auto kern, const auto* typed_src) -> nq_status_t {
        static std::mutex mu;
        static std::atomic<uint64_t> attr_set{0};
        nq_status_t st = once_per_device(attr_set, mu, di.device, [&]() -> nq_status_t {
            NQ_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024),
                          "cudaFuncSetAttribute(quantize_rows)");
            return NQ_SUCCESS;
        });
        if (st != NQ_SUCCESS) return st;
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem) != cudaSuccess || per_sm < 1) {
            cudaGetLastError();
            per_sm = 1;
        }
        const long long want = (static_cast<long long>(rows) + warps - 1) / warps;
        const int grid = static_cast<int>(std::max<long long>(1, std::min<long long>(want, static_cast<long long>(di.sm_count) * per_sm)));
        NQ_CHECK_CUDA(launch_pdl(kern, dim3(grid), dim3(kThreads), smem, s, typed_src, dst, scales, rows, cols, stages,
                                 device_error_word()),
                      "nq_quantize_rows (warp)");
        return NQ_SUCCESS;
    };
    if (dt == NQ_F32) return launch(k_quant_rows_warp<F, float>, static_cast<const float*>(src));
    return launch(k_quant_rows_warp<F, uint16_t>, static_cast<const uint16_t*>(src));
}

namespace {

bool is_device_pointer(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

int reduce_grid(size_t n, int sm_count) {
    const size_t want = (n / 4 + kThreads - 1) / kThreads;
    return static_cast<int>(std::max<size_t>(1, std::min<size_t>(want, static_cast<size_t>(sm_count) * 4)));
}

// Launches the single-pass reduction with pool scratch.
template <bool ABS, class In>
nq_status_t launch_minmax(const In* src, size_t n, float* out_lo, float* out_hi, float qmax, cudaStream_t s,
                          const char* what) {
    DeviceInfo di;
    nq_status_t st = current_device(&di);
    if (st != NQ_SUCCESS) return st;
    const int grid = reduce_grid(n, di.sm_count);
    void* scratch = nullptr;
    const size_t bytes = 256 + sizeof(float) * 2 * static_cast<size_t>(grid);
    st = scratch_alloc(&scratch, bytes, s);
    if (st != NQ_SUCCESS) return st;
    unsigned int* ticket = static_cast<unsigned int*>(scratch);
    float* partials = reinterpret_cast<float*>(static_cast<char*>(scratch) + 256);
    cudaError_t e = cudaMemsetAsync(ticket, 0, sizeof(unsigned int), s);
    if (e == cudaSuccess) {
        const int vec = aligned16(src);
        k_minmax<ABS, In><<<grid, kThreads, 0, s>>>(src, n, vec, partials, ticket, out_lo, out_hi, qmax);
        e = cudaGetLastError();
    }
    scratch_free(scratch, s);
    return cuda_status(e, what);
}

float qmax_of(nq_format_t f) { return f == NQ_E4M3 ? 448.0f : (f == NQ_E5M2 ? 57344.0f : 127.0f); }

}  // namespace

nq_status_t amax_scale_impl(const void* data, nq_dtype_t dt, size_t n, nq_format_t fmt, float* d_out,
                            cudaStream_t s) {
    if (!d_out || (n && !data)) return fail(NQ_ERROR_INVALID_VALUE, "nq_amax_scale_async: null pointer");
    if (fmt != NQ_E4M3 && fmt != NQ_E5M2 && fmt != NQ_INT8)
        return fail(NQ_ERROR_INVALID_VALUE, "nq_amax_scale_async: format");
    if (n == 0) {
        const float v[2] = {0.0f, 1.0f};
        return cuda_status(cudaMemcpyAsync(d_out, v, sizeof(v), cudaMemcpyHostToDevice, s), "nq_amax_scale_async");
    }
    if (dt == NQ_F32)
        return launch_minmax<true, float>(static_cast<const float*>(data), n, d_out, nullptr, qmax_of(fmt), s,
                                          "nq_amax_scale_async");
    if (dt == NQ_BF16)
        return launch_minmax<true, uint16_t>(static_cast<const uint16_t*>(data), n, d_out, nullptr, qmax_of(fmt),
                                             s, "nq_amax_scale_async");
    return fail(NQ_ERROR_INVALID_VALUE, "nq_amax_scale_async: src dtype");
}

}  // namespace nq

using nq::fail;

extern "C" {

nq_status_t nq_minmax_async(const float* data, size_t n, float* d_out, nq_stream_t s) {
    if (!d_out || (n && !data)) return fail(NQ_ERROR_INVALID_VALUE, "nq_minmax_async: null pointer");
    if (n == 0) return nq::cuda_status(cudaMemsetAsync(d_out, 0, 2 * sizeof(float), s), "nq_minmax_async");
    return nq::launch_minmax<false, float>(data, n, d_out, d_out + 1, 0.0f, s, "nq_minmax_async");
}

nq_status_t nq_compute_minmax(const float* data, size_t n, float* min_val, float* max_val, nq_stream_t s) {
    if (!min_val || !max_val) return fail(NQ_ERROR_INVALID_VALUE, "nq_compute_minmax: null output");
    const bool out_dev = nq::is_device_pointer(min_val) && nq::is_device_pointer(max_val);
    if (n == 0) {  // int8_kernels.cu:331-335
        if (out_dev) {
            NQ_CHECK_CUDA(cudaMemsetAsync(min_val, 0, sizeof(float), s), "nq_compute_minmax");
            NQ_CHECK_CUDA(cudaMemsetAsync(max_val, 0, sizeof(float), s), "nq_compute_minmax");
            NQ_CHECK_CUDA(cudaStreamSynchronize(s), "nq_compute_minmax");
        } else {
            *min_val = 0.0f;
            *max_val = 0.0f;
        }
        return NQ_SUCCESS;
    }
    if (!data) return fail(NQ_ERROR_INVALID_VALUE, "nq_compute_minmax: null data");
    // Host input: stage it through pooled device memory (int8_kernels.cu:337-357).
    const float* d_data = data;
    void* staged = nullptr;
    void* res = nullptr;
    nq_status_t st = NQ_SUCCESS;
    if (!nq::is_device_pointer(data)) {
        st = nq::scratch_alloc(&staged, n * sizeof(float), s);
        if (st != NQ_SUCCESS) return st;
        cudaError_t e = cudaMemcpyAsync(staged, data, n * sizeof(float), cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) { nq::scratch_free(staged, s); return nq::cuda_status(e, "nq_compute_minmax: H2D"); }
        d_data = static_cast<const float*>(staged);
    }
    float* lo = min_val;
    float* hi = max_val;
    if (!out_dev) {
        st = nq::scratch_alloc(&res, 2 * sizeof(float), s);
        if (st != NQ_SUCCESS) { nq::scratch_free(staged, s); return st; }
        lo = static_cast<float*>(res);
        hi = lo + 1;
    }
    st = nq::launch_minmax<false, float>(d_data, n, lo, hi, 0.0f, s, "nq_compute_minmax");
    float h[2] = {0.0f, 0.0f};
    if (st == NQ_SUCCESS && !out_dev)
        st = nq::cuda_status(cudaMemcpyAsync(h, res, sizeof(h), cudaMemcpyDeviceToHost, s), "nq_compute_minmax: D2H");
    nq::scratch_free(staged, s);
    nq::scratch_free(res, s);
    cudaError_t e = cudaStreamSynchronize(s);
    if (st != NQ_SUCCESS) return st;
    if (e != cudaSuccess) return nq::cuda_status(e, "nq_compute_minmax: synchronize");
    if (!out_dev) {
        *min_val = h[0];
        *max_val = h[1];
    }
    return NQ_SUCCESS;
}

nq_status_t nq_build_histogram(const float* data, uint32_t* histogram, size_t n, float min_val, float max_val,
                               int num_bins, nq_stream_t s) {
    if (!histogram || num_bins < 1 || num_bins > 65536)
        return fail(NQ_ERROR_INVALID_VALUE, "nq_build_histogram: bad histogram or num_bins");
    if (n && !data) return fail(NQ_ERROR_INVALID_VALUE, "nq_build_histogram: null data");
    nq::DeviceInfo di;
    nq_status_t st = nq::current_device(&di);
    if (st != NQ_SUCCESS) return st;
    NQ_CHECK_CUDA(cudaMemsetAsync(histogram, 0, sizeof(uint32_t) * num_bins, s), "nq_build_histogram: memset");
    const float range = max_val - min_val;
    if (n == 0 || !(range > 1e-6f)) {
        NQ_CHECK_CUDA(cudaStreamSynchronize(s), "nq_build_histogram");
        return NQ_SUCCESS;
    }
    const float* d_data = data;
    void* staged = nullptr;
    if (!nq::is_device_pointer(data)) {
        st = nq::scratch_alloc(&staged, n * sizeof(float), s);
        if (st != NQ_SUCCESS) return st;
        cudaError_t e = cudaMemcpyAsync(staged, data, n * sizeof(float), cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) { nq::scratch_free(staged, s); return nq::cuda_status(e, "nq_build_histogram: H2D"); }
        d_data = static_cast<const float*>(staged);
    }
    const int grid = nq::reduce_grid(n, di.sm_count);
    const int vec = nq::aligned16(d_data);
    const size_t smem = sizeof(uint32_t) * static_cast<size_t>(num_bins);
    cudaError_t e;
    if (smem <= 48 * 1024) {
        nq::k_histogram<true><<<grid, nq::kThreads, smem, s>>>(d_data, n, vec, histogram, min_val, range, num_bins);
    } else if (smem <= 200 * 1024) {
        cudaFuncSetAttribute(nq::k_histogram<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        nq::k_histogram<true><<<grid, nq::kThreads, smem, s>>>(d_data, n, vec, histogram, min_val, range, num_bins);
    } else {
        nq::k_histogram<false><<<grid, nq::kThreads, 0, s>>>(d_data, n, vec, histogram, min_val, range, num_bins);
    }
    e = cudaGetLastError();
    nq::scratch_free(staged, s);
    cudaError_t e2 = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return nq::cuda_status(e, "nq_build_histogram: launch");
    return nq::cuda_status(e2, "nq_build_histogram: synchronize");
}

nq_status_t nq_amax_scale_async(const void* data, nq_dtype_t src_dtype, size_t n, nq_format_t fmt, float* d_out,
                                nq_stream_t s) {
    return nq::amax_scale_impl(data, src_dtype, n, fmt, d_out, s);
}

nq_status_t nq_minmax_rows(const float* data, int rows, int cols, float* d_min, float* d_max, nq_stream_t s) {
    if (rows < 0 || cols < 0) return fail(NQ_ERROR_INVALID_VALUE, "nq_minmax_rows: negative size");
    if (rows == 0) return NQ_SUCCESS;
    if (!data || !d_min || !d_max) return fail(NQ_ERROR_INVALID_VALUE, "nq_minmax_rows: null pointer");
    nq::DeviceInfo di;
    nq_status_t st = nq::current_device(&di);
    if (st != NQ_SUCCESS) return st;
    nq::k_minmax_rows<<<rows, nq::kThreads, 0, s>>>(data, cols, d_min, d_max);
    NQ_LAUNCH_CHECK("nq_minmax_rows");
    return NQ_SUCCESS;
}

nq_status_t nq_calibrate_quantize(const void* src, nq_dtype_t src_dtype, uint8_t* dst, size_t n, nq_format_t fmt,
                                  float* d_amax_scale, nq_stream_t s) {
    nq_status_t st = nq::amax_scale_impl(src, src_dtype, n, fmt, d_amax_scale, s);
    if (st != NQ_SUCCESS) return st;
    return nq::quantize_scaled_impl(src, src_dtype, dst, n, fmt, d_amax_scale + 1, s);
}

nq_status_t nq_quantize_rows(const void* src, nq_dtype_t src_dtype, uint8_t* dst, float* scales, int rows,
                             int cols, nq_format_t fmt, nq_stream_t s) {
    if (rows < 0 || cols < 0) return fail(NQ_ERROR_INVALID_VALUE, "nq_quantize_rows: negative size");
    if (rows == 0 || cols == 0) return NQ_SUCCESS;
    if (!src || !dst || !scales) return fail(NQ_ERROR_INVALID_VALUE, "nq_quantize_rows: null pointer");
    if (src_dtype != NQ_F32 && src_dtype != NQ_BF16) return fail(NQ_ERROR_INVALID_VALUE, "nq_quantize_rows: dtype");
    nq::DeviceInfo di;
    nq_status_t st = nq::current_device(&di);
    if (st != NQ_SUCCESS) return st;
    using namespace nq::dev;
    const size_t row_bytes = static_cast<size_t>(cols) * (src_dtype == NQ_F32 ? 4 : 2);
    const bool staged = row_bytes % 16 == 0 && nq::aligned16(src) &&
                        reinterpret_cast<uintptr_t>(dst) % (src_dtype == NQ_F32 ? 4 : 8) == 0;
    // rows up to 12 KB: one warp per row, bulk-staged per-warp ring
    if (staged && row_bytes <= nq::kWarpRowMax) {
        switch (fmt) {
            case NQ_E4M3: return nq::launch_quant_rows_warp<kE4M3>(src, src_dtype, dst, scales, rows, cols, di, s);
            case NQ_E5M2: return nq::launch_quant_rows_warp<kE5M2>(src, src_dtype, dst, scales, rows, cols, di, s);
            case NQ_INT8: return nq::launch_quant_rows_warp<kINT8>(src, src_dtype, dst, scales, rows, cols, di, s);
            default: return fail(NQ_ERROR_INVALID_VALUE, "nq_quantize_rows: format");
        }
    }
    // rows of 12 KB .. 100 KB: one block per row, bulk-staged ring, persistent grid
    if (staged && 2 * row_bytes <= nq::kBulkRowSmem) {
        switch (fmt) {
            case NQ_E4M3: return nq::launch_quant_rows_bulk<kE4M3>(src, src_dtype, dst, scales, rows, cols, di, s);
            case NQ_E5M2: return nq::launch_quant_rows_bulk<kE5M2>(src, src_dtype, dst, scales, rows, cols, di, s);
            case NQ_INT8: return nq::launch_quant_rows_bulk<kINT8>(src, src_dtype, dst, scales, rows, cols, di, s);
            default: return fail(NQ_ERROR_INVALID_VALUE, "nq_quantize_rows: format");
        }
    }
#define NQ_QROWS(F)                                                                                       \
    (src_dtype == NQ_F32                                                                                  \
         ? nq::k_quant_rows<F, float><<<rows, nq::kThreads, 0, s>>>(static_cast<const float*>(src), dst,  \
                                                                    scales, cols)                         \
         : nq::k_quant_rows<F, uint16_t><<<rows, nq::kThreads, 0, s>>>(static_cast<const uint16_t*>(src), \
                                                                       dst, scales, cols))
    switch (fmt) {
        case NQ_E4M3: NQ_QROWS(kE4M3); break;
        case NQ_E5M2: NQ_QROWS(kE5M2); break;
        case NQ_INT8: NQ_QROWS(kINT8); break;
        default: return fail(NQ_ERROR_INVALID_VALUE, "nq_quantize_rows: format");
    }
#undef NQ_QROWS
    NQ_LAUNCH_CHECK("nq_quantize_rows");
    return NQ_SUCCESS;
}

nq_status_t nq_quantize_cols(const float* src, uint8_t* dst, float* scales, int rows, int cols, nq_format_t fmt,
                             nq_stream_t s) {
    if (rows < 0 || cols < 0) return fail(NQ_ERROR_INVALID_VALUE, "nq_quantize_cols: negative size");
    if (rows == 0 || cols == 0) return NQ_SUCCESS;
    if (!src || !dst || !scales) return fail(NQ_ERROR_INVALID_VALUE, "nq_quantize_cols: null pointer");
    if (fmt != NQ_E4M3 && fmt != NQ_E5M2 && fmt != NQ_INT8)
        return fail(NQ_ERROR_INVALID_VALUE, "nq_quantize_cols: format");
    nq::DeviceInfo di;
    nq_status_t st = nq::current_device(&di);
    if (st != NQ_SUCCESS) return st;
    void* amax = nullptr;
    st = nq::scratch_alloc(&amax, sizeof(uint32_t) * static_cast<size_t>(cols), s);
    if (st != NQ_SUCCESS) return st;
    cudaError_t e = cudaMemsetAsync(amax, 0, sizeof(uint32_t) * static_cast<size_t>(cols), s);
    if (e == cudaSuccess) {
        const int groups = (cols + 4 * nq::kThreads - 1) / (4 * nq::kThreads);
        const int chunks = std::max(1, std::min(rows, (di.sm_count * 8 + groups - 1) / groups));
        const int rpc = (rows + chunks - 1) / chunks;
        dim3 g1(groups, (rows + rpc - 1) / rpc);
        nq::k_col_amax<<<g1, nq::kThreads, 0, s>>>(src, rows, cols, rpc, static_cast<uint32_t*>(amax));
        const size_t total = static_cast<size_t>(rows) * cols;
        const int g2 = static_cast<int>(std::min<size_t>((total + nq::kThreads - 1) / nq::kThreads,
                                                         static_cast<size_t>(di.sm_count) * 8));
        const uint32_t* ab = static_cast<const uint32_t*>(amax);
        switch (fmt) {
            case NQ_E4M3: nq::k_quant_cols<nq::dev::kE4M3><<<g2, nq::kThreads, 0, s>>>(src, dst, ab, scales, rows, cols); break;
            case NQ_E5M2: nq::k_quant_cols<nq::dev::kE5M2><<<g2, nq::kThreads, 0, s>>>(src, dst, ab, scales, rows, cols); break;
            default: nq::k_quant_cols<nq::dev::kINT8><<<g2, nq::kThreads, 0, s>>>(src, dst, ab, scales, rows, cols); break;
        }
        e = cudaGetLastError();
    }
    nq::scratch_free(amax, s);
    return nq::cuda_status(e, "nq_quantize_cols");
}

}  // extern "C"

// ---- allocation-free per-column quantize ---------------------------------------
// Some callers cannot allocate device memory while they run: an engine that
// reserved all of HBM up front for its own allocator, a plugin host that hands
// a plugin only its input and output buffers, or a latency-critical loop where
// cudaMalloc's implicit synchronisation is not allowed.  For them,
// nq_quantize_cols_noalloc keeps its per-column amax scratch in this fixed
// array instead of the library's memory pool.  Every GPU that loads the
// library holds it (65536 x 4 B = 256 KiB) until the process exits.
static constexpr int kNoAllocMaxCols = 65536;
static __device__ __align__(256) uint32_t g_noalloc_col_amax[kNoAllocMaxCols];

namespace nq {
namespace {

// Host code may not pass the symbol itself to a kernel (on the host it names
// a stand-in, not device memory): its device address is looked up once per
// device, with that device current, and cached.  Later calls read the cached
// address without a lock; only a device's first call takes the mutex.
nq_status_t noalloc_scratch(uint32_t** out) {
    static std::mutex mu;
    static std::atomic<uint32_t*> addr[64];
    int dev = -1;
    NQ_CHECK_CUDA(cudaGetDevice(&dev), "nq_quantize_cols_noalloc: cudaGetDevice");
    if (dev < 0 || dev >= 64) return fail(NQ_ERROR_NO_DEVICE, "nq_quantize_cols_noalloc: device ordinal out of range");
    uint32_t* a = addr[dev].load(std::memory_order_acquire);
    if (!a) {
        std::lock_guard<std::mutex> lk(mu);
        a = addr[dev].load(std::memory_order_relaxed);
        if (!a) {
            void* p = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_col_amax);
            if (e != cudaSuccess) return cuda_status(e, "nq_quantize_cols_noalloc: cudaGetSymbolAddress");
            a = static_cast<uint32_t*>(p);
            addr[dev].store(a, std::memory_order_release);
        }
    }
    *out = a;
    return NQ_SUCCESS;
}
}  // namespace
}  // namespace nq

extern "C" {

nq_status_t nq_quantize_cols_noalloc(const float* src, uint8_t* dst, float* scales, int rows, int cols,
                                     nq_format_t fmt, nq_stream_t s) {
    if (rows < 0 || cols < 0) return fail(NQ_ERROR_INVALID_VALUE, "nq_quantize_cols_noalloc: negative size");
    if (cols > kNoAllocMaxCols)
        return fail(NQ_ERROR_UNSUPPORTED, "nq_quantize_cols_noalloc: cols = " + std::to_string(cols) +
                                              " exceeds the fixed scratch of " + std::to_string(kNoAllocMaxCols) +
                                              " columns; use nq_quantize_cols");
    if (rows == 0 || cols == 0) return NQ_SUCCESS;
    if (!src || !dst || !scales) return fail(NQ_ERROR_INVALID_VALUE, "nq_quantize_cols_noalloc: null pointer");
    if (fmt != NQ_E4M3 && fmt != NQ_E5M2 && fmt != NQ_INT8)
        return fail(NQ_ERROR_INVALID_VALUE, "nq_quantize_cols_noalloc: format");
    nq::DeviceInfo di;
    nq_status_t st = nq::current_device(&di);
    if (st != NQ_SUCCESS) return st;
    uint32_t* amax = nullptr;
    st = nq::noalloc_scratch(&amax);
    if (st != NQ_SUCCESS) return st;
    // The array keeps the previous call's maxima: clear the columns used.
    NQ_CHECK_CUDA(cudaMemsetAsync(amax, 0, sizeof(uint32_t) * static_cast<size_t>(cols), s),
                  "nq_quantize_cols_noalloc: clear scratch");
    const int groups = (cols + 4 * nq::kThreads - 1) / (4 * nq::kThreads);
    const int chunks = std::max(1, std::min(rows, (di.sm_count * 8 + groups - 1) / groups));
    const int rpc = (rows + chunks - 1) / chunks;
    dim3 g1(groups, (rows + rpc - 1) / rpc);
    nq::k_col_amax<<<g1, nq::kThreads, 0, s>>>(src, rows, cols, rpc, amax);
    const size_t total = static_cast<size_t>(rows) * cols;
    const int g2 = static_cast<int>(
        std::min<size_t>((total + nq::kThreads - 1) / nq::kThreads, static_cast<size_t>(di.sm_count) * 8));
    switch (fmt) {
        case NQ_E4M3: nq::k_quant_cols<nq::dev::kE4M3><<<g2, nq::kThreads, 0, s>>>(src, dst, amax, scales, rows, cols); break;
        case NQ_E5M2: nq::k_quant_cols<nq::dev::kE5M2><<<g2, nq::kThreads, 0, s>>>(src, dst, amax, scales, rows, cols); break;
        default: nq::k_quant_cols<nq::dev::kINT8><<<g2, nq::kThreads, 0, s>>>(src, dst, amax, scales, rows, cols); break;
    }
    NQ_LAUNCH_CHECK("nq_quantize_cols_noalloc");
    return NQ_SUCCESS;
}

}  // extern "C"

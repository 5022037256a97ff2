// gemm.cu -- FP8 (kind::f8f6f4) and INT8 (kind::i8) GEMMs on the sm_100a
// tensor cores, with the scale / bias / bf16 / int8 / SwiGLU epilogues fused,
// and the GEMM-fused all-reduce of a row-parallel layer.
//
// Kernel k_gemm_tc2 (M > 128, and every SwiGLU / all-reduce GEMM): a cluster
//   of two CTAs computes 256 x 256 tiles with tcgen05.mma.cta_group::2; warp 0
//   of each CTA loads its half of A and B by TMA (5-stage ring), warp 1 of the
//   first CTA issues the MMAs, warps 2..9 of both CTAs drain TMEM through the
//   epilogue and TMA stores; persistent grid, banded tile order.  The AR
//   variant adds reducer warps (ar_job) and a signaller (ar_signal_tiles).
// Kernel k_gemm_tc (M <= 128; persistent, one CTA per SM, 192 threads):
//   warp 0 TMA producer ([128 x 128 B] A and [128 B x 256] B per stage,
//   4-stage ring), warp 1 MMA issuer (M=128, N=256), warps 2..5 epilogue.
// Kernel k_gemm_decode (M <= 32 against large weights): operands swapped so
//   128 weight rows are the MMA's M side, stream-K over weight slices with a
//   deterministic fixup.
// B is read either K x N row-major (FP8GEMM::forward's layout, the MN-major
// operand form of tcgen05) or N x K row-major (K-major, a packed weight).
// Every wait is bounded (ptx.cuh); a timeout sets the device error word.
//
// Kernel k_gemm_simt: one thread per output, sequential-k FMA (int32 for
// INT8), for shapes the TMA path cannot take (K or N not a multiple of 16,
// unaligned pointers) and tiny problems.
#include <algorithm>
#include <atomic>
#include <cstring>
#include <mutex>
#include <string>
#include <utility>

#include "codec.cuh"
#include "nq_internal.h"
#include "ptx.cuh"

namespace nq {
namespace {

using namespace dev;

constexpr int BM = 128, BN = 256, BK = 128;  // BK in elements (= bytes)
constexpr int STAGES = 4;
constexpr int A_STAGE = BM * BK;        // 16 KB
constexpr int B_STAGE = BN * BK;        // 32 KB
constexpr int TMEM_COLS = 2 * BN;       // two accumulators
constexpr int GEMM_THREADS = 192;
constexpr int SMEM_BYTES = 1024 + STAGES * (A_STAGE + B_STAGE) + 256;

struct Epi {
    void* out;
    int ldo;  // elements per output row
    nq_dtype_t out_dtype;
    float alpha;
    const float* row_scale;
    const float* col_scale;
    const float* bias;
};

// Device view of nq_allreduce_desc_t (signal / job / finish of the fused
// all-reduce; pointers as bytes).
struct ArParams {
    int tp, rank;
    uint32_t epoch;
    int signal;
    uint32_t* signal_flags[NQ_MAX_TP];
    int m, n;  // job; m == 0: none
    uint32_t* flags;
    uint8_t* mc_partial;
    uint8_t* mc_out;
    uint32_t* mc_done;
    const uint8_t* peer_partial[NQ_MAX_TP];
    uint8_t* peer_out[NQ_MAX_TP];
    uint32_t* peer_done[NQ_MAX_TP];
    uint32_t* done;         // finish: non-NULL
    uint32_t done_target;   // finish: wait until *done reaches it (modulo 2^32)
    uint64_t peer_wait_ns;  // bound of a wait on another GPU's counts
};

// Per-chunk column operands of the epilogue: lane j holds column (col0 + j)'s
// scale and bias, or the exact identities 1.0 and -0.0 when absent
// (x * 1 == x and x + (-0) == x for every x, signed zeros included), so the
// element loop below runs without branches and its result is bit-identical to
// the conditional form.
struct ColOps {
    float cs, b;
};
__device__ __forceinline__ ColOps col_ops(const float* col_scale, const float* bias, int col0, int lane, int N) {
    const int c = min(col0 + lane, N - 1);
    ColOps o;
    o.cs = col_scale ? __ldg(col_scale + c) : 1.0f;
    o.b = bias ? __ldg(bias + c) : -0.0f;
    return o;
}
// ((acc * alpha) * rs) * cs[j] + b[j], one rounding per step; j's operands
// are broadcast from lane j.
__device__ __forceinline__ float epi_elem(float acc, float alpha, float rs, const ColOps& o, int j) {
    float v = __fmul_rn(__fmul_rn(acc, alpha), rs);
    v = __fmul_rn(v, __shfl_sync(0xffffffffu, o.cs, j));
    return __fadd_rn(v, __shfl_sync(0xffffffffu, o.b, j));
}

// v = ((acc * alpha) [* rs]) [* cs] [+ b]: one rounding per step, never fused.
__device__ __forceinline__ float epi_value(float acc, float alpha, float rs, const float* col_scale,
                                           const float* bias, int col) {
    float v = __fmul_rn(acc, alpha);
    if (rs != 1.0f) v = __fmul_rn(v, rs);
    if (col_scale) v = __fmul_rn(v, __ldg(col_scale + col));
    if (bias) v = __fadd_rn(v, __ldg(bias + col));
    return v;
}

// quantize_ops.hpp:75-77: clamp to [-127, 127], then std::round.
__device__ __forceinline__ int8_t requant_s8(float v) {
    v = fmaxf(-127.0f, fminf(127.0f, v));
    return static_cast<int8_t>(roundf(v));
}

// Called by all 32 lanes together (the column operands are shuffled across
// the warp); only lanes with row_ok store.
template <bool INT_ACC>
__device__ __forceinline__ void store_chunk(const Epi& ep, const uint32_t (&r)[32], int row, int col0, int N,
                                            float rs, bool row_ok) {
    if (INT_ACC && ep.out_dtype == NQ_S32) {
        if (!row_ok) return;
        int32_t* o = static_cast<int32_t*>(ep.out) + static_cast<size_t>(row) * ep.ldo + col0;
        if (col0 + 32 <= N) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
                *reinterpret_cast<int4*>(o + j) = make_int4(r[j], r[j + 1], r[j + 2], r[j + 3]);
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (col0 + j < N) o[j] = static_cast<int32_t>(r[j]);
        }
        return;
    }
    float v[32];
    // columns past N are computed (with column N-1's operands) but never stored
    const ColOps cop = col_ops(ep.col_scale, ep.bias, col0, static_cast<int>(lane_id()), N);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        const float acc = INT_ACC ? __int2float_rn(static_cast<int32_t>(r[j])) : __uint_as_float(r[j]);
        v[j] = epi_elem(acc, ep.alpha, rs, cop, j);
    }
    if (!row_ok) return;
    if (ep.out_dtype == NQ_S8) {
        int8_t* o = static_cast<int8_t*>(ep.out) + static_cast<size_t>(row) * ep.ldo + col0;
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (col0 + j < N) o[j] = requant_s8(v[j]);
    } else if (ep.out_dtype == NQ_BF16) {
        uint16_t* o = static_cast<uint16_t*>(ep.out) + static_cast<size_t>(row) * ep.ldo + col0;
        if (col0 + 32 <= N) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
                uint4 w;
                w.x = f32x2_to_bf16x2(v[j], v[j + 1]);
                w.y = f32x2_to_bf16x2(v[j + 2], v[j + 3]);
                w.z = f32x2_to_bf16x2(v[j + 4], v[j + 5]);
                w.w = f32x2_to_bf16x2(v[j + 6], v[j + 7]);
                *reinterpret_cast<uint4*>(o + j) = w;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (col0 + j < N) o[j] = static_cast<uint16_t>(f32x2_to_bf16x2(v[j], 0.0f));
        }
    } else {
        float* o = static_cast<float*>(ep.out) + static_cast<size_t>(row) * ep.ldo + col0;
        if (col0 + 32 <= N) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) *reinterpret_cast<float4*>(o + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (col0 + j < N) o[j] = v[j];
        }
    }
}

template <bool INT8_KIND, bool B_KN>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N, int K,
              uint32_t idesc, Epi ep, uint32_t* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * A_STAGE;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sB + STAGES * B_STAGE);
    uint64_t* full = bars;                // [STAGES] TMA -> MMA
    uint64_t* empty = bars + STAGES;      // [STAGES] MMA -> TMA
    uint64_t* tfull = bars + 2 * STAGES;  // [2] MMA -> epilogue
    uint64_t* tempty = tfull + 2;         // [2] epilogue -> MMA
    uint64_t* done = tempty + 2;          // MMA drain
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int m_tiles = (M + BM - 1) / BM;
    const int n_tiles = (N + BN - 1) / BN;
    const int num_tiles = m_tiles * n_tiles;
    const int kblocks = (K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 128);
        }
        mbar_init(done, 1);
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (elect_one()) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                const int mb = tile % m_tiles, nb = tile / m_tiles;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, err)) { ok = false; break; }
                    mbar_arrive_expect_tx(&full[stage], A_STAGE + B_STAGE);
                    tma_load_2d(sA + stage * A_STAGE, &tmA, &full[stage], kb * BK, mb * BM);
                    if (B_KN) {
                        tma_load_2d(sB + stage * B_STAGE, &tmB, &full[stage], nb * BN, kb * BK);
                        tma_load_2d(sB + stage * B_STAGE + B_STAGE / 2, &tmB, &full[stage], nb * BN + BN / 2, kb * BK);
                    } else {
                        tma_load_2d(sB + stage * B_STAGE, &tmB, &full[stage], kb * BK, nb * BN);
                    }
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
            }
            if (!ok) {
                // Let the copies already issued land before the CTA can exit.
                for (int s = 0; s < STAGES; ++s) {
                    int st = stage - 1 - s;
                    uint32_t ph = phase;
                    if (st < 0) { st += STAGES; ph ^= 1u; }
                    mbar_wait(&full[st], ph, nullptr);
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (elect_one()) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            int it = 0;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++it) {
                const int acc = it & 1;
                const uint32_t acc_phase = (static_cast<uint32_t>(it) >> 1) & 1u;
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, err)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&full[stage], phase, err)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sA + stage * A_STAGE);
                    const uint32_t b_addr = smem_u32(sB + stage * B_STAGE);
#pragma unroll
                    for (int kk = 0; kk < BK / 32; ++kk) {
                        // A: K-major, 128-byte rows, 8-row groups 1024 B apart;
                        //    the k-th 32-byte slice starts 32*kk bytes in.
                        const uint64_t adesc = smem_desc_sw128(a_addr + 32u * kk, 16u, 1024u);
                        // B (K x N): MN-major, two 128-column halves B_STAGE/2
                        //    apart (LBO), 8-row k groups 1024 B apart (SBO); the
                        //    k-th slice of 32 rows starts 32*128 bytes in.
                        // B (N x K): K-major like A.
                        const uint64_t bdesc = B_KN ? smem_desc_sw128(b_addr + 4096u * kk, B_STAGE / 2, 1024u)
                                                    : smem_desc_sw128(b_addr + 32u * kk, 16u, 1024u);
                        const uint32_t accum = (kb > 0 || kk > 0) ? 1u : 0u;
                        if (INT8_KIND) mma_i8(d_tmem, adesc, bdesc, idesc, accum);
                        else mma_f8f6f4(d_tmem, adesc, bdesc, idesc, accum);
                    }
                    tc_commit(&empty[stage]);
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
                if (ok) tc_commit(&tfull[acc]);
            }
            // Every MMA issued by this thread completes before TMEM is freed.
            tc_commit(done);
            mbar_wait(done, 0, err);
        }
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter+32)
        const int row_in_tile = quarter * 32 + lane;
        int it = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
            const int acc = it & 1;
            const uint32_t acc_phase = (static_cast<uint32_t>(it) >> 1) & 1u;
            bool ok = mbar_wait(&tfull[acc], acc_phase, err);
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            const int mb = tile % m_tiles, nb = tile / m_tiles;
            const int row = mb * BM + row_in_tile;
            const float rs = (ep.row_scale && row < M) ? __ldg(ep.row_scale + row) : 1.0f;
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(taddr + 32u * c, r);
                tmem_ld_wait();
                const int col0 = nb * BN + c * 32;
                if (col0 < N) store_chunk<INT8_KIND>(ep, r, row, col0, N, rs, row < M);
            }
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
        }
    }
    __syncwarp();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// ---------------- CTA-pair kernel (cta_group::2, 256 x 256 tiles) ----------------
// A cluster of two CTAs computes one 256 x 256 tile per step with
// tcgen05.mma.cta_group::2 (M=256, N=256, K=32).  Each CTA TMA-loads its own
// half of A (128 rows) and its own half of B (128 columns) into its shared
// memory, so per SM the tensor core reads 32 KB and TMA writes 32 KB per
// 128-deep k-block -- a third less shared-memory traffic per FLOP than the
// single-CTA 128 x 256 tile.  The leader CTA (rank 0) issues the MMAs; its
// `full` barriers count both CTAs' bytes (cta_group::2 loads signal the
// leader), `empty` and `tfull` are multicast commits to both CTAs, and both
// CTAs' epilogue warps arrive on the leader's `tempty`.  Each CTA's TMEM holds
// its 128 rows of the tile.  No TMA multicast.
constexpr int P_BM = 256, P_BN = 256;
constexpr int P_STAGES = 5;
// warp 0 TMA producer, warp 1 MMA issuer, warps 2..9 epilogue: two warps per
// TMEM lane quarter, each draining 128 of the tile's 256 columns
constexpr int P_THREADS = 320;
constexpr int P_EPI_WARPS = 8;
constexpr int P_A_STAGE = 128 * BK;  // 16 KB per CTA
constexpr int P_B_STAGE = 128 * BK;  // 16 KB per CTA
// Stream-K schedule.  Tiles [0, dp_tiles) are whole tiles dealt round-robin
// to the clusters; the k-blocks of the last sk_tiles tiles are cut into one
// equal contiguous range per cluster, so the last (1 + fraction) waves keep
// every cluster busy instead of leaving part of the machine idle.  A tile cut
// by range boundaries is finished by the cluster holding its first k-block,
// which reaches that part last (it ends that cluster's range); every later
// cluster touching the tile does its part first, parks the raw accumulators
// in its own workspace slot and counts its 16 epilogue warps in its flag.  The
// finishing cluster adds the parked parts in cluster order before its
// epilogue: deterministic, exact for int32.  A cluster parks at most once
// (only its first stream-K item can start inside a tile).
// Half tiles: when the last wave of whole tiles would fill at most half the
// clusters, each of its `half_tiles` tiles is computed as two 256 x 128
// halves (tcgen05.mma N = 128) on two clusters instead, so the tail takes
// half a tile's time and needs no cross-cluster fixup.  Excludes stream-K.
struct StreamK {
    int dp_tiles;     // whole tiles, round-robin
    int sk_tiles;     // tiles whose k-blocks are shared out (0: none)
    uint32_t* ws;     // [clusters][256 x 256] parked accumulators
    uint32_t* flags;  // [clusters] epilogue warps that parked
    int half_tiles;   // tiles [dp_tiles, dp_tiles + half_tiles) done as two 256 x 128 halves
};
struct Unit {
    int tile, kb0, kb1;
    int park;            // the accumulators go to this cluster's workspace slot
    int c_first, c_last; // the tile's later parts, parked by these clusters (none if c_first > c_last)
    int half;            // 0: the whole tile; 1 / 2: its columns [0, 128) / [128, 256)
};
__host__ __device__ __forceinline__ long long sk_begin(long long total, int c, int nclusters) {
    return total * c / nclusters;
}
// Work items of `cluster`: its whole tiles, then one item per tile its
// stream-K range touches.
__device__ __forceinline__ int sched_whole(const StreamK& sk, int cluster, int nclusters) {
    return sk.dp_tiles > cluster ? (sk.dp_tiles - cluster + nclusters - 1) / nclusters : 0;
}
__device__ __forceinline__ int sched_items(const StreamK& sk, int kblocks, int cluster, int nclusters) {
    int n = sched_whole(sk, cluster, nclusters);
    if (sk.half_tiles > 0 && cluster < 2 * sk.half_tiles) n += (2 * sk.half_tiles - cluster + nclusters - 1) / nclusters;
    if (sk.sk_tiles > 0) {
        const long long total = static_cast<long long>(sk.sk_tiles) * kblocks;
        const long long b0 = sk_begin(total, cluster, nclusters), b1 = sk_begin(total, cluster + 1, nclusters);
        if (b1 > b0) n += static_cast<int>((b1 - 1) / kblocks - b0 / kblocks + 1);
    }
    return n;
}
__device__ __forceinline__ Unit sched_unit(const StreamK& sk, int kblocks, int cluster, int nclusters, int n_whole,
                                           int j) {
    if (j < n_whole) return Unit{cluster + j * nclusters, 0, kblocks, 0, 1, 0, 0};
    if (sk.half_tiles > 0) {
        const int hu = cluster + (j - n_whole) * nclusters;
        return Unit{sk.dp_tiles + hu / 2, 0, kblocks, 0, 1, 0, 1 + (hu & 1)};
    }
    const long long total = static_cast<long long>(sk.sk_tiles) * kblocks;
    const long long b0 = sk_begin(total, cluster, nclusters), b1 = sk_begin(total, cluster + 1, nclusters);
    const long long lt = b0 / kblocks + (j - n_whole);
    const long long t0 = lt * kblocks, t1 = t0 + kblocks;
    Unit u;
    u.tile = sk.dp_tiles + static_cast<int>(lt);
    u.kb0 = static_cast<int>((b0 > t0 ? b0 : t0) - t0);
    u.kb1 = static_cast<int>((b1 < t1 ? b1 : t1) - t0);
    u.park = u.kb0 > 0;
    u.half = 0;
    u.c_first = cluster + 1;
    u.c_last = cluster;
    if (!u.park && b1 < t1) {
        // the tile runs past this range: the clusters whose ranges start inside it
        u.c_last = u.c_first;
        while (u.c_last + 1 < nclusters && sk_begin(total, u.c_last + 1, nclusters) < t1) ++u.c_last;
    }
    return u;
}
// Parked accumulators of one epilogue warp (w16 = its index among the pair's
// 16 epilogue warps): 4 chunks x 8 uint4 x 32 lanes, lane-fastest so that each
// warp-wide access is 512 contiguous bytes.
__device__ __forceinline__ uint4* park_slot(uint32_t* ws, int cluster, int w16) {
    return reinterpret_cast<uint4*>(ws + static_cast<size_t>(cluster) * (256 * 256)) + static_cast<size_t>(w16) * (4 * 8 * 32);
}
// acc[4q .. 4q+3] += parked values (int32 exact, fp32 one rounding each).
template <bool INT_ACC>
__device__ __forceinline__ void add_parked4(uint32_t (&acc)[32], int q, const uint4& v) {
    const uint32_t p[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const int e = 4 * q + t;
        if (INT_ACC) acc[e] = static_cast<uint32_t>(static_cast<int32_t>(acc[e]) + static_cast<int32_t>(p[t]));
        else acc[e] = __float_as_uint(__fadd_rn(__uint_as_float(acc[e]), __uint_as_float(p[t])));
    }
}
// acc += one parked 32-column chunk.
template <bool INT_ACC>
__device__ __forceinline__ void add_parked(uint32_t (&acc)[32], const uint4 (&v)[8]) {
#pragma unroll
    for (int q = 0; q < 8; ++q) add_parked4<INT_ACC>(acc, q, v[q]);
}
// Tile order of the persistent schedule: bands of P_BAND M-tiles; inside a
// band the tiles walk N, M fastest.  The clusters in flight at any moment
// then share at most P_BAND A panels and ~clusters/P_BAND B panels, a working
// set that stays in L2 when A alone (M x K) does not (M = 16384, K = 8192:
// 128 MiB), so each operand panel comes from HBM about once per band.
constexpr int P_BAND = 16;
__device__ __forceinline__ void tile_coords(int tile, int m_tiles, int n_tiles, int& mb, int& nb) {
    const int band = tile / (P_BAND * n_tiles);
    const int rows = min(P_BAND, m_tiles - band * P_BAND);
    const int local = tile - band * P_BAND * n_tiles;
    mb = band * P_BAND + local % rows;
    nb = local / rows;
}
// Spins (bounded) until *flag >= want, reading with acquire semantics.
__device__ __forceinline__ bool wait_flag_geq(const uint32_t* flag, uint32_t want, uint32_t* err) {
    const uint64_t t0 = globaltimer();
    while (true) {
        uint32_t v;
        asm volatile("ld.global.acquire.gpu.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
        if (v >= want) return true;
        if (globaltimer() - t0 > kWaitLimitNs) {
            if (err) atomicOr(err, kErrWaitTimeout);
            return false;
        }
        __nanosleep(64);
    }
}

// Spins (bounded by `limit` ns) until the system-scope counter at p has
// reached `want`.  The all-reduce counters only grow and are compared modulo
// 2^32 (the signed difference), so a counter and a target that both wrapped
// past 2^32 still compare right; a counter is never more than a forward's
// worth of counts (far below 2^31) away from its target.
__device__ __forceinline__ bool counter_reached(uint32_t v, uint32_t want) {
    return static_cast<int32_t>(v - want) >= 0;
}
__device__ __forceinline__ bool wait_sys_geq(const uint32_t* p, uint32_t want, uint32_t* err, uint64_t limit) {
    const uint64_t t0 = globaltimer();
    while (!counter_reached(ld_acquire_sys(p), want)) {
        if (globaltimer() - t0 > limit) {
            if (err) atomicOr(err, kErrWaitTimeout);
            return false;
        }
        __nanosleep(128);
    }
    return true;
}

// Epilogue staging: per epilogue warp two 4 KB slots, each one 32 x 32 output
// chunk (rows of 128 B for 4-byte outputs, 64 B for bf16), swizzled so that
// the row-per-lane writes are bank-conflict free; a TMA store per chunk.
constexpr int P_EPI_SLOT = 4096;
constexpr int P_EPI_BYTES = P_EPI_WARPS * 2 * P_EPI_SLOT;
constexpr int P_SMEM_BYTES = 1024 + P_STAGES * (P_A_STAGE + P_B_STAGE) + P_EPI_BYTES + 256;


// A operand quantized inside the GEMM (per-token dynamic quantization fused
// into the kernel): bf16 activations x (rows x cols), their E4M3 codes and
// per-row scales.  Rows [0, head) -- the first band of M-tiles, all the first
// waves of tiles need -- are quantized by every warp of the grid before the
// GEMM roles start (phase 1a); rows [head, rows) by the epilogue warps while
// the first tiles' MMAs run (phase 1b).  done[0] / done[1] count the rows of
// each part.
struct QuantA {
    const uint16_t* x;
    uint8_t* codes;
    float* scales;
    uint32_t* done;  // [2], zero before the launch
    int rows, cols;
    int head;        // rows of phase 1a
};
constexpr int QA_REG_VECS = 16;  // rows up to 16 * 32 * 8 = 4096 values fit in registers

__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ void red_add_release_gpu(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Codes of the 8-value vectors idx = lane + 32 i (i < n) of a row, from v[].
template <bool MUL, int NV>
__device__ __forceinline__ void encode_row_vecs(const uint4 (&v)[NV], int n, int lane, int nv, uint8_t* out,
                                                const RowScale& rs) {
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int idx = lane + 32 * i;
        if (i < n && idx < nv) encode_vec<kE4M3, uint16_t, MUL>(v[i], out + idx * 8, rs);
    }
}
// One row from global memory: in registers when it has at most 4096 values,
// else an amax pass and an encode pass (the second read hits L2).  Returns
// the row's scale; the codes are stored to `out`.  The arithmetic of
// nq_quantize_rows, bit for bit.
__device__ float quant_row_global(const uint16_t* row, uint8_t* out, int nv, int lane) {
    RowScale rs;
    if (nv <= QA_REG_VECS * 32) {
        uint4 v[QA_REG_VECS];
        float a = 0.0f;
#pragma unroll
        for (int i = 0; i < QA_REG_VECS; ++i) {
            const int idx = lane + 32 * i;
            if (idx < nv) v[i] = ld_stream_v4(row + idx * 8);
        }
#pragma unroll
        for (int i = 0; i < QA_REG_VECS; ++i)
            if (lane + 32 * i < nv)
#pragma unroll
                for (int e = 0; e < 8; ++e) a = fmaxf(a, fabsf(vec_elem<uint16_t>(v[i], e)));
        rs = row_scale<kE4M3>(warp_max_f(a));
        if (rs.mul) encode_row_vecs<true>(v, QA_REG_VECS, lane, nv, out, rs);
        else encode_row_vecs<false>(v, QA_REG_VECS, lane, nv, out, rs);
        return rs.s;
    }
    float a = 0.0f;
    for (int idx0 = 0; idx0 < nv; idx0 += 32 * 8) {
        uint4 v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int idx = idx0 + lane + 32 * i;
            if (idx < nv) v[i] = ld_stream_v4(row + idx * 8);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (idx0 + lane + 32 * i < nv)
#pragma unroll
                for (int e = 0; e < 8; ++e) a = fmaxf(a, fabsf(vec_elem<uint16_t>(v[i], e)));
    }
    rs = row_scale<kE4M3>(warp_max_f(a));
    for (int idx0 = 0; idx0 < nv; idx0 += 32 * 8) {
        uint4 v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int idx = idx0 + lane + 32 * i;
            if (idx < nv) v[i] = __ldcg(reinterpret_cast<const uint4*>(row) + idx);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int idx = idx0 + lane + 32 * i;
            if (idx >= nv) continue;
            if (rs.mul) encode_vec<kE4M3, uint16_t, true>(v[i], out + idx * 8, rs);
            else encode_vec<kE4M3, uint16_t, false>(v[i], out + idx * 8, rs);
        }
    }
    return rs.s;
}
// Counts `mine` finished rows on *done once the warp's codes and scales are
// written: a release after a proxy fence (TMA reads the codes back).
__device__ __forceinline__ void qa_publish(uint32_t* done, uint32_t mine, int lane) {
    fence_proxy_async_global();
    __syncwarp();
    if (lane == 0 && mine) red_add_release_gpu(done, mine);
}
// Phase 1a: rows [0, qa.head) over every warp of the grid.  Each warp's rows
// stream through its slice of the CTA's shared memory (still unused by the
// GEMM) with cp.async, `stages` rows in flight; every lane reads back only
// the 16-byte pieces it copied itself, so no barrier is needed between the
// copy and the use.  Rows that do not fit the slice take quant_row_global.
__device__ void quant_rows_head(const QuantA& qa, int warp, int lane, int warps_per_cta, uint8_t* smem,
                                uint32_t smem_bytes) {
    const int nv = qa.cols / 8;
    const uint32_t rb = static_cast<uint32_t>(qa.cols) * 2;
    const uint32_t slice = (smem_bytes / warps_per_cta) & ~15u;
    const int stages = static_cast<int>(min(4u, slice / rb));
    const long long nw = static_cast<long long>(gridDim.x) * warps_per_cta;
    const long long r0 = static_cast<long long>(blockIdx.x) * warps_per_cta + warp;
    uint32_t mine = 0;
    if (stages < 1) {
        for (long long r = r0; r < qa.head; r += nw, ++mine) {
            const float sc = quant_row_global(qa.x + r * qa.cols, qa.codes + r * qa.cols, nv, lane);
            if (lane == 0) qa.scales[r] = sc;
        }
        qa_publish(qa.done, mine, lane);
        return;
    }
    uint8_t* ring = smem + static_cast<size_t>(warp) * slice;
    auto issue = [&](long long r, int st) {
        if (r < qa.head) {
            const uint4* src = reinterpret_cast<const uint4*>(qa.x + r * qa.cols);
            uint4* dst = reinterpret_cast<uint4*>(ring + static_cast<size_t>(st) * rb);
            for (int idx = lane; idx < nv; idx += 32) cp_async_16(dst + idx, src + idx);
        }
        cp_async_commit();  // an empty group past the last row keeps the count uniform
    };
    for (int st = 0; st < stages; ++st) issue(r0 + st * nw, st);
    int st = 0;
    for (long long r = r0; r < qa.head; r += nw, ++mine) {
        // the oldest group (this row) has landed once at most stages-1 remain
        switch (stages) {
            case 1: cp_async_wait<0>(); break;
            case 2: cp_async_wait<1>(); break;
            case 3: cp_async_wait<2>(); break;
            default: cp_async_wait<3>(); break;
        }
        const uint4* buf = reinterpret_cast<const uint4*>(ring + static_cast<size_t>(st) * rb);
        float a = 0.0f;
        for (int idx = lane; idx < nv; idx += 32) {
            const uint4 q = buf[idx];
#pragma unroll
            for (int e = 0; e < 8; ++e) a = fmaxf(a, fabsf(vec_elem<uint16_t>(q, e)));
        }
        const RowScale rs = row_scale<kE4M3>(warp_max_f(a));
        uint8_t* out = qa.codes + r * qa.cols;
        if (rs.mul)
            for (int idx = lane; idx < nv; idx += 32) encode_vec<kE4M3, uint16_t, true>(buf[idx], out + idx * 8, rs);
        else
            for (int idx = lane; idx < nv; idx += 32) encode_vec<kE4M3, uint16_t, false>(buf[idx], out + idx * 8, rs);
        if (lane == 0) qa.scales[r] = rs.s;
        issue(r + static_cast<long long>(stages) * nw, st);  // this lane's pieces of buffer st are consumed
        if (++st == stages) st = 0;
    }
    cp_async_wait<0>();
    qa_publish(qa.done, mine, lane);
}
// Phase 1b: rows [qa.head, qa.rows) over the grid's epilogue warps (ew of
// new_w), from global memory.
__device__ void quant_rows_tail(const QuantA& qa, int ew, int new_w, int lane) {
    const int nv = qa.cols / 8;
    const long long nw = static_cast<long long>(gridDim.x) * new_w;
    uint32_t mine = 0;
    for (long long r = qa.head + static_cast<long long>(blockIdx.x) * new_w + ew; r < qa.rows; r += nw, ++mine) {
        const float sc = quant_row_global(qa.x + r * qa.cols, qa.codes + r * qa.cols, nv, lane);
        if (lane == 0) qa.scales[r] = sc;
    }
    qa_publish(qa.done + 1, mine, lane);
}
// Waits (bounded) until the rows of part `part` (0: [0, head), 1: the rest)
// are all quantized.  Called by lane 0 of a warp only (one poller per warp,
// 256 ns apart, so waiting warps do not crowd the counter's L2 slice while
// other CTAs still read their rows); the caller's __syncwarp orders the other
// lanes' reads after the acquire.  `tma`: also order this thread's later TMA
// reads (cross-proxy).
__device__ __forceinline__ bool qa_wait(const QuantA& qa, int part, uint32_t* err, bool tma) {
    const uint32_t want = static_cast<uint32_t>(part == 0 ? qa.head : qa.rows - qa.head);
    if (want) {
        const uint64_t t0 = globaltimer();
        while (true) {
            uint32_t v;
            asm volatile("ld.global.acquire.gpu.u32 %0, [%1];" : "=r"(v) : "l"(qa.done + part) : "memory");
            if (v >= want) break;
            if (globaltimer() - t0 > kWaitLimitNs) {
                if (err) atomicOr(err, kErrWaitTimeout);
                return false;
            }
            __nanosleep(256);
        }
    }
    if (tma) fence_proxy_async_global();
    return true;
}

// Reducer side of the fused all-reduce.  A group of AR_WARPS warps (warps 10
// and 11 of both CTAs of a GEMM pair plus the second CTA's idle warp 1, or
// one CTA of the finish kernel) takes the owned tiles i = group, group +
// ngroups, ... of the job (owned tile i is tile rank + tp * i in the producing
// GEMM's tile order); warp j of the group waits until all tp ranks have
// signalled the tile, then sums its rows j, j + nwarps,
// ... over the ranks (multicast: multimem.ld_reduce, fp32 accumulation in the
// switch; peer: fp32 sum in rank order) and writes the bf16 rows to every
// rank's output, then counts itself on every rank's completion counter.
// 32 lanes cover the 512 bytes of a tile row; 10 (multicast) or 4 (peer)
// rows in flight per warp.  Finally warp 0 of group 0 waits for done_target.
constexpr int AR_WARPS = 5;
constexpr int P_THREADS_AR = P_THREADS + 64;  // + warps 10, 11
constexpr int AR_SIGNALS_PER_TILE = 1;  // the signaller's one count per tile and rank
__device__ __forceinline__ void ar_job(const ArParams& ar, int j, int nwarps, int group, int ngroups, uint32_t* err) {
    const int lane = threadIdx.x & 31;
    bool ok = true;
    if (ar.m > 0) {
        const int m_tiles = (ar.m + P_BM - 1) / P_BM;
        const int n_tiles = ar.n / P_BN;
        const int num_tiles = m_tiles * n_tiles;
        const uint32_t want = ar.epoch * static_cast<uint32_t>(ar.tp) * AR_SIGNALS_PER_TILE;
        const size_t pitch = static_cast<size_t>(ar.n) * 2;
        for (int i = group;; i += ngroups) {
            const int t = ar.rank + ar.tp * i;
            if (t >= num_tiles) break;
            if (lane == 0) ok = wait_sys_geq(ar.flags + t, want, err, ar.peer_wait_ns);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            int mb, nb;
            tile_coords(t, m_tiles, n_tiles, mb, nb);
            const int r0 = mb * P_BM;
            const int rows = min(P_BM, ar.m - r0);
            const size_t base = static_cast<size_t>(r0) * pitch + static_cast<size_t>(nb) * P_BN * 2 + lane * 16;
            if (ar.mc_partial) {
                constexpr int U = 10;
                for (int r = j; r < rows; r += U * nwarps) {
                    uint4 v[U];
#pragma unroll
                    for (int u = 0; u < U; ++u)
                        if (r + u * nwarps < rows)
                            v[u] = multimem_ld_reduce_bf16x8(ar.mc_partial + base + (r + u * nwarps) * pitch);
#pragma unroll
                    for (int u = 0; u < U; ++u)
                        if (r + u * nwarps < rows) multimem_st_v4(ar.mc_out + base + (r + u * nwarps) * pitch, v[u]);
                }
            } else {
                constexpr int U = 4;
                for (int r = j; r < rows; r += U * nwarps) {
                    float acc[U][8];
#pragma unroll
                    for (int u = 0; u < U; ++u)
#pragma unroll
                        for (int e = 0; e < 8; ++e) acc[u][e] = 0.0f;
                    for (int p = 0; p < ar.tp; ++p) {
                        uint4 q[U];
#pragma unroll
                        for (int u = 0; u < U; ++u)
                            if (r + u * nwarps < rows)
                                q[u] = __ldcg(reinterpret_cast<const uint4*>(ar.peer_partial[p] + base +
                                                                             (r + u * nwarps) * pitch));
#pragma unroll
                        for (int u = 0; u < U; ++u) {
                            if (r + u * nwarps >= rows) continue;
                            const uint32_t w[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                acc[u][2 * e] = __fadd_rn(acc[u][2 * e], __uint_as_float(w[e] << 16));
                                acc[u][2 * e + 1] = __fadd_rn(acc[u][2 * e + 1], __uint_as_float(w[e] & 0xFFFF0000u));
                            }
                        }
                    }
#pragma unroll
                    for (int u = 0; u < U; ++u) {
                        if (r + u * nwarps >= rows) continue;
                        const uint4 o = make_uint4(f32x2_to_bf16x2(acc[u][0], acc[u][1]), f32x2_to_bf16x2(acc[u][2], acc[u][3]),
                                                   f32x2_to_bf16x2(acc[u][4], acc[u][5]), f32x2_to_bf16x2(acc[u][6], acc[u][7]));
                        for (int p = 0; p < ar.tp; ++p)
                            __stcg(reinterpret_cast<uint4*>(ar.peer_out[p] + base + (r + u * nwarps) * pitch), o);
                    }
                }
            }
            // this warp's rows are written everywhere: count them on every rank
            fence_acq_rel_sys();
            __syncwarp();
            if (lane == 0) {
                if (ar.mc_done) multimem_red_add_release(ar.mc_done, 1u);
                else
                    for (int p = 0; p < ar.tp; ++p) red_add_release_sys(ar.peer_done[p], 1u);
            }
        }
    }
    if (ar.done && group == 0 && j == 0 && lane == 0 && ok)
        wait_sys_geq(ar.done, ar.done_target, err, ar.peer_wait_ns);
}

// Job and / or finish without a GEMM: one CTA of AR_WARPS warps per group.
__global__ void __launch_bounds__(AR_WARPS * 32) k_ar_finish(const __grid_constant__ ArParams ar, uint32_t* err) {
    ar_job(ar, threadIdx.x >> 5, AR_WARPS, blockIdx.x, gridDim.x, err);
}

// Signaller of a GEMM whose output is a partial (ar.signal): one lane of the
// first CTA's warp 11 walks this cluster's tiles in order, waits (bounded)
// until both CTAs' 8 epilogue warps have counted the tile's stores complete on
// the cluster counter, and adds 1 to the tile's counter on its owner rank.  The
// system-scope release stays off the epilogue warps, which only do a
// cluster-scope add.
__device__ __forceinline__ void ar_signal_tiles(const ArParams& ar, uint32_t cnt_addr, int cluster, int nclusters,
                                                int num_tiles, uint32_t* err) {
    if ((threadIdx.x & 31) != 0) return;
    uint32_t want = 0;
    for (int t = cluster; t < num_tiles; t += nclusters) {
        want += 2 * P_EPI_WARPS;
        const uint64_t t0 = globaltimer();
        bool ok = true;
        while (ld_acquire_cluster(cnt_addr) < want) {
            if (globaltimer() - t0 > kWaitLimitNs) {
                atomicOr(err, kErrWaitTimeout);
                ok = false;
                break;
            }
            __nanosleep(64);
        }
        if (!ok) return;
        red_add_release_sys(ar.signal_flags[t % ar.tp] + t, 1u);
    }
}

// OUTK: 0 = 4-byte output (f32, or raw s32 for INT8) through TMA stores,
// 1 = bf16 through TMA stores, 2 = int8 requantized, direct stores.
// SWIGLU: columns [0,128) of each 256-wide tile are gate, [128,256) up; the
// tile writes 128 columns of silu(g) * u.
// AR: the kernel carries the reducer warps of the fused all-reduce (ar_job)
// and, with ar.signal, counts each bf16 output tile on its owner rank.
// QA: the A operand is quantized per row by the kernel itself (phase 1, all
// warps, before the GEMM roles start; QuantA).
template <bool INT8_KIND, bool B_KN, int OUTK, bool SWIGLU, bool AR, bool QA = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(AR ? P_THREADS_AR : P_THREADS, 1)
    k_gemm_tc2(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmBh, const __grid_constant__ CUtensorMap tmC, int M, int N, int K,
               uint32_t idesc, uint32_t idesc_h, Epi ep, StreamK sk, const __grid_constant__ ArParams ar,
               const __grid_constant__ QuantA qa, uint32_t* err) {
    static_assert(!AR || OUTK == 1, "the all-reduce signals bf16 tiles");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + P_STAGES * P_A_STAGE;
    uint8_t* sEpi = sB + P_STAGES * P_B_STAGE;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sEpi + P_EPI_BYTES);
    uint64_t* full = bars;                  // [P_STAGES] leader: both CTAs' TMA -> MMA
    uint64_t* empty = bars + P_STAGES;      // [P_STAGES] MMA -> each CTA's producer
    uint64_t* tfull = bars + 2 * P_STAGES;  // [2] MMA -> each CTA's epilogue
    uint64_t* tempty = tfull + 2;           // [2] leader: 16 epilogue warps -> MMA
    uint64_t* done = tempty + 2;            // leader: MMA drain
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    uint32_t* sig_cnt = tmem_slot + 1;      // AR: epilogue warps' completed tiles (first CTA)

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int cluster = blockIdx.x >> 1;
    const int nclusters = gridDim.x >> 1;
    const int m_tiles = (M + P_BM - 1) / P_BM;
    const int n_tiles = (N + P_BN - 1) / P_BN;
    const int num_tiles = m_tiles * n_tiles;
    const int kblocks = (K + BK - 1) / BK;
    const int n_whole = sched_whole(sk, cluster, nclusters);
    const int n_items = sched_items(sk, kblocks, cluster, nclusters);

    // With programmatic stream serialization the next kernel may start its
    // prologue as this grid's CTAs finish; up to pdl_wait() nothing here reads
    // or writes memory an earlier kernel may still write (the weight prefetch
    // only fills L2, which is coherent).
    pdl_launch_dependents();
    if (threadIdx.x == 0) {
        for (int s = 0; s < P_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 2 * P_EPI_WARPS);
        }
        mbar_init(done, 1);
        *sig_cnt = 0u;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        if (sk.half_tiles) tma_prefetch_desc(&tmBh);
        if (OUTK != 2) tma_prefetch_desc(&tmC);
        if (n_items > 0) {
            // this CTA's operand tiles of its first stages, into L2, while the
            // barriers and TMEM are set up (and, launched after a kernel that
            // triggers early, while that kernel finishes); A only when it is an
            // input of the launch
            const Unit u0 = sched_unit(sk, kblocks, cluster, nclusters, n_whole, 0);
            int mb0, nb0;
            tile_coords(u0.tile, m_tiles, n_tiles, mb0, nb0);
            for (int kb = u0.kb0; kb < u0.kb1 && kb < u0.kb0 + P_STAGES; ++kb) {
                if (!QA) tma_prefetch_l2_2d(&tmA, kb * BK, mb0 * P_BM + static_cast<int>(rank) * 128);
                if (u0.half) continue;
                if (B_KN) tma_prefetch_l2_2d(&tmB, nb0 * P_BN + rank * 128, kb * BK);
                else tma_prefetch_l2_2d(&tmB, kb * BK, nb0 * P_BN + rank * 128);
            }
        }
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();
    if constexpr (QA) {
        // phase 1a through the operand ring and staging slots, then hand them
        // to TMA: the generic reads of this shared memory come before the
        // producer's async-proxy writes
        quant_rows_head(qa, warp, lane, static_cast<int>(blockDim.x >> 5), smem,
                        static_cast<uint32_t>(P_STAGES * (P_A_STAGE + P_B_STAGE) + P_EPI_BYTES));
        fence_proxy_async_smem();
        __syncthreads();
    }

    if (warp == 0) {
        // ---------------- TMA producer (both CTAs) ----------------
        if (elect_one()) {
            const uint32_t full_leader = mapa_shared(smem_u32(full), 0);
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            int qa_part = -1;  // QA: the last part of A's rows seen complete
            for (int j = 0; j < n_items && ok; ++j) {
                const Unit un = sched_unit(sk, kblocks, cluster, nclusters, n_whole, j);
                int mb, nb;
                tile_coords(un.tile, m_tiles, n_tiles, mb, nb);
                if constexpr (QA) {
                    // rows of this tile (both CTAs') quantized: a wait and a fence per part
                    const int part = (mb + 1) * P_BM > qa.head ? 1 : 0;
                    if (part > qa_part) {
                        for (int q = qa_part + 1; q <= part && ok; ++q) ok = qa_wait(qa, q, err, true);
                        if (!ok) break;
                        qa_part = part;
                    }
                }
                // a half tile: this CTA's 64 of the half's 128 columns of B
                const int hcol = nb * P_BN + (un.half - 1) * 128 + static_cast<int>(rank) * 64;
                const uint32_t b_bytes = un.half ? P_B_STAGE / 2 : P_B_STAGE;
                for (int kb = un.kb0; kb < un.kb1; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, err)) { ok = false; break; }
                    if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * (P_A_STAGE + b_bytes));
                    const uint32_t fb = full_leader + 8u * stage;
                    tma_load_2d_pair(sA + stage * P_A_STAGE, &tmA, fb, kb * BK, mb * P_BM + rank * 128);
                    if (un.half) {
                        if (B_KN) tma_load_2d_pair(sB + stage * P_B_STAGE, &tmBh, fb, hcol, kb * BK);
                        else tma_load_2d_pair(sB + stage * P_B_STAGE, &tmBh, fb, kb * BK, hcol);
                    } else if (B_KN) {
                        tma_load_2d_pair(sB + stage * P_B_STAGE, &tmB, fb, nb * P_BN + rank * 128, kb * BK);
                    } else {
                        tma_load_2d_pair(sB + stage * P_B_STAGE, &tmB, fb, kb * BK, nb * P_BN + rank * 128);
                    }
                    if (++stage == P_STAGES) { stage = 0; phase ^= 1u; }
                }
            }
            if (!ok) {
                // let issued copies land: the free signal of every stage in flight
                for (int s = 0; s < P_STAGES; ++s) mbar_wait(&empty[s], phase ^ 1u, nullptr);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (leader CTA only) ----------------
        if constexpr (AR) {
            // the second CTA's warp 1 is one of the reducers
            if (rank == 1) ar_job(ar, ar.signal ? 1 : 2, ar.signal ? AR_WARPS - 1 : AR_WARPS, cluster, nclusters, err);
        }
        if (rank == 0 && elect_one()) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            int it = 0;
            for (int j = 0; j < n_items && ok; ++j, ++it) {
                const Unit un = sched_unit(sk, kblocks, cluster, nclusters, n_whole, j);
                const int acc = it & 1;
                const uint32_t acc_phase = (static_cast<uint32_t>(it) >> 1) & 1u;
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, err)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * P_BN);
                for (int kb = un.kb0; kb < un.kb1; ++kb) {
                    if (!mbar_wait(&full[stage], phase, err)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sA + stage * P_A_STAGE);
                    const uint32_t b_addr = smem_u32(sB + stage * P_B_STAGE);
                    const uint32_t id = un.half ? idesc_h : idesc;
#pragma unroll
                    for (int kk = 0; kk < BK / 32; ++kk) {
                        // per CTA: A is 128 K-major rows; B is 128 columns (64 for a
                        // half tile), MN-major (K x N source: 128- or 64-byte
                        // swizzled rows) or K-major (N x K source)
                        const uint64_t adesc = smem_desc_sw128(a_addr + 32u * kk, 16u, 1024u);
                        uint64_t bdesc;
                        if (!B_KN) bdesc = smem_desc_sw128(b_addr + 32u * kk, 16u, 1024u);
                        else if (un.half) bdesc = smem_desc_sw64(b_addr + 2048u * kk, P_B_STAGE, 512u);
                        else bdesc = smem_desc_sw128(b_addr + 4096u * kk, P_B_STAGE, 1024u);
                        const uint32_t accum = (kb > un.kb0 || kk > 0) ? 1u : 0u;
                        if (INT8_KIND) mma_i8_pair(d_tmem, adesc, bdesc, id, accum);
                        else mma_f8f6f4_pair(d_tmem, adesc, bdesc, id, accum);
                    }
                    tc_commit_pair_mc(&empty[stage], 0x3);
                    if (++stage == P_STAGES) { stage = 0; phase ^= 1u; }
                }
                if (ok) tc_commit_pair_mc(&tfull[acc], 0x3);
            }
            tc_commit_pair_mc(done, 0x1);
            mbar_wait(done, 0, err);
        }
    } else if (AR && warp >= 2 + P_EPI_WARPS) {
        // ---------------- all-reduce (warps 10, 11 of both CTAs) ----------------
        // with ar.signal the first CTA's warp 11 is the signaller and 4 warps reduce
        if (ar.signal && rank == 0 && warp == 3 + P_EPI_WARPS) {
            ar_signal_tiles(ar, mapa_shared(smem_u32(sig_cnt), 0), cluster, nclusters, num_tiles, err);
        } else {
            const int j = warp - 2 - P_EPI_WARPS + (rank == 0 ? 0 : (ar.signal ? 2 : 3));
            ar_job(ar, j, ar.signal ? AR_WARPS - 1 : AR_WARPS, cluster, nclusters, err);
        }
    } else {
        // ---------------- epilogue (warps 2..9 of both CTAs) ----------------
        const int quarter = warp & 3;            // TMEM lanes [32 * quarter, +32)
        const int colh = (warp - 2) >> 2;        // columns [128 * colh, +128)
        const int row_in_tile = static_cast<int>(rank) * 128 + quarter * 32 + lane;
        const uint32_t tempty_leader = mapa_shared(smem_u32(tempty), 0);
        uint8_t* slots = sEpi + (warp - 2) * 2 * P_EPI_SLOT;
        const bool raw_s32 = INT8_KIND && OUTK == 0 && ep.out_dtype == NQ_S32;
        int it = 0;
        int chunk_seq = 0;  // chunks stored by this warp so far (selects the staging slot)
        // AR signal: the previous tile, counted on its owner once its stores are
        // complete -- one tile later, so the epilogue never waits on its own stores
        int sig_pending = -1;
        const uint32_t sig_cnt_leader = mapa_shared(smem_u32(sig_cnt), 0);
        const int w16 = static_cast<int>(rank) * P_EPI_WARPS + (warp - 2);
        int qa_part = -1;  // QA: the last part of A's rows whose scales this warp acquired
        // QA: the rows past the head, before this warp's first epilogue (the MMAs of
        // the first tiles run meanwhile)
        if constexpr (QA) quant_rows_tail(qa, warp - 2, P_EPI_WARPS, lane);
        for (int j = 0; j < n_items; ++j, ++it) {
            const Unit un = sched_unit(sk, kblocks, cluster, nclusters, n_whole, j);
            const int tile = un.tile;
            const int acc = it & 1;
            const uint32_t acc_phase = (static_cast<uint32_t>(it) >> 1) & 1u;
            int mb, nb;
            tile_coords(tile, m_tiles, n_tiles, mb, nb);
            // This unit's column operands (and row scale), requested before its
            // accumulator is ready: while the SMs stream operands, a global load
            // issued at the chunk that needs it waits about a microsecond (B200).
            ColOps cops[4];
            if constexpr (SWIGLU) {
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    cops[c] = col_ops(ep.col_scale, ep.bias, nb * P_BN + colh * 64 + c * 32, lane, N);
                    cops[2 + c] = col_ops(ep.col_scale, ep.bias, nb * P_BN + colh * 64 + c * 32 + 128, lane, N);
                }
            } else {
                const int cw0 = un.half ? 64 : 128;
                const int cb0 = nb * P_BN + (un.half ? (un.half - 1) * 128 : 0) + colh * cw0;
#pragma unroll
                for (int c = 0; c < 4; ++c) cops[c] = col_ops(ep.col_scale, ep.bias, cb0 + c * 32, lane, N);
            }
            const int row_pre = mb * P_BM + row_in_tile;
            const float rs_pre = (!QA && ep.row_scale && row_pre < M) ? __ldg(ep.row_scale + row_pre) : 1.0f;
            const bool fixup = !un.park && un.c_first <= un.c_last;
            if (fixup) {
                // wait (bounded) until the later parts' 16 warps have parked
                if (lane == 0)
                    for (int cc = un.c_first; cc <= un.c_last; ++cc) wait_flag_geq(sk.flags + cc, 2u * P_EPI_WARPS, err);
                __syncwarp();
            }
            bool ok = mbar_wait(&tfull[acc], acc_phase, err);
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            if constexpr (QA) {
                // the row scales of this tile come from phase 1 of this launch
                const int part = (mb + 1) * P_BM > qa.head ? 1 : 0;
                if (part > qa_part) {
                    if (lane == 0)
                        for (int q = qa_part + 1; q <= part; ++q) qa_wait(qa, q, err, false);
                    __syncwarp();
                    qa_part = part;
                }
            }
            const int row = mb * P_BM + row_in_tile;
            // this warp's columns: 128 of a whole tile, 64 of a half tile
            const int cw = un.half ? 64 : 128;
            const int nchunks = cw / 32;
            const int col_base = nb * P_BN + (un.half ? (un.half - 1) * 128 : 0) + colh * cw;
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                   static_cast<uint32_t>(acc * P_BN + colh * cw);
            if (un.park) {
                // a later part of a tile another cluster finishes: park the raw accumulators
                uint4* mine = park_slot(sk.ws, cluster, w16);
#pragma unroll 1
                for (int c = 0; c < 4; ++c) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(taddr + 32u * c, r);
                    tmem_ld_wait();
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                        __stcg(mine + (c * 8 + q) * 32 + lane, make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]));
                }
                tc_fence_before();
                __threadfence();
                __syncwarp();
                if (lane == 0) {
                    if (rank == 0) mbar_arrive(&tempty[acc]);
                    else mbar_arrive_remote(tempty_leader + 8u * acc);
                    atomicAdd(sk.flags + cluster, 1u);
                }
                continue;
            }
            const int row0_warp = mb * P_BM + static_cast<int>(rank) * 128 + quarter * 32;
            float rs;
            if constexpr (QA) {
                // the row scales come from phase 1 of this launch (acquired at the top)
                rs = row < M ? __ldcg(qa.scales + row) : 1.0f;
            } else {
                rs = rs_pre;
            }
            if constexpr (SWIGLU) {
                // this warp's 64 output columns: gate TMEM columns colh*64 + [0,64),
                // up columns 128 + colh*64 + [0,64)
                const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * P_BN);
#pragma unroll 1
                for (int c = 0; c < 2; ++c) {
                    uint32_t g[32], u[32];
                    tmem_ld_32x32b_x32(tbase + colh * 64 + c * 32, g);
                    tmem_ld_32x32b_x32(tbase + 128 + colh * 64 + c * 32, u);
                    tmem_ld_wait();
                    if (c == 1) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) {
                            if (rank == 0) mbar_arrive(&tempty[acc]);
                            else mbar_arrive_remote(tempty_leader + 8u * acc);
                        }
                    }
                    const int gcol0 = nb * P_BN + colh * 64 + c * 32;
                    const int hcol0 = nb * (P_BN / 2) + colh * 64 + c * 32;
                    if (row0_warp >= M) continue;
                    const ColOps gop = c == 0 ? cops[0] : cops[1];
                    const ColOps uop = c == 0 ? cops[2] : cops[3];
                    (void)gcol0;
                    uint8_t* slot = slots + (chunk_seq & 1) * P_EPI_SLOT;
                    if (lane == 0) bulk_wait_group_read<1>();
                    __syncwarp();
                    float h[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const float gv = epi_elem(__uint_as_float(g[j]), ep.alpha, rs, gop, j);
                        const float uv = epi_elem(__uint_as_float(u[j]), ep.alpha, rs, uop, j);
                        h[j] = __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv))), uv);
                    }
                    if (OUTK == 1) {
                        uint8_t* rowp = slot + lane * 64;
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            uint4 q;
                            q.x = f32x2_to_bf16x2(h[8 * j], h[8 * j + 1]);
                            q.y = f32x2_to_bf16x2(h[8 * j + 2], h[8 * j + 3]);
                            q.z = f32x2_to_bf16x2(h[8 * j + 4], h[8 * j + 5]);
                            q.w = f32x2_to_bf16x2(h[8 * j + 6], h[8 * j + 7]);
                            *reinterpret_cast<uint4*>(rowp + 16 * (j ^ ((lane >> 1) & 3))) = q;
                        }
                    } else {
                        uint8_t* rowp = slot + lane * 128;
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            *reinterpret_cast<uint4*>(rowp + 16 * (j ^ (lane & 7))) =
                                make_uint4(__float_as_uint(h[4 * j]), __float_as_uint(h[4 * j + 1]),
                                           __float_as_uint(h[4 * j + 2]), __float_as_uint(h[4 * j + 3]));
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&tmC, slot, hcol0, row0_warp);
                        bulk_commit_group();
                    }
                    ++chunk_seq;
                }
                continue;
            }
            int tile_groups = 0;  // bulk store groups this warp commits for this tile
            // this warp's 128 columns, 32 per tcgen05.ld, the next 32 in flight
            uint32_t r[32];
            // A unit with a fixup is the last of this cluster's range: every MMA
            // (of both CTAs) is complete, so the operand ring is idle and takes
            // this warp's 16 KB of the first parked part in one burst of
            // cp.async, instead of a load latency per chunk.
            const uint4* sp0 = reinterpret_cast<const uint4*>(smem) + static_cast<size_t>(warp - 2) * (4 * 8 * 32);
            if (fixup) {
                const uint4* p0 = park_slot(sk.ws, un.c_first, w16);
#pragma unroll 4
                for (int i = 0; i < 4 * 8; ++i) cp_async_16(const_cast<uint4*>(sp0) + i * 32 + lane, p0 + i * 32 + lane);
                cp_async_commit();
            }
            tmem_ld_32x32b_x32(taddr, r);
            if (fixup) {
                cp_async_wait<0>();
                __syncwarp();
            }
#pragma unroll 1
            for (int c = 0; c < nchunks; ++c) {
                tmem_ld_wait();
                uint32_t cur[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) cur[j] = r[j];
                if (c + 1 < nchunks) {
                    tmem_ld_32x32b_x32(taddr + 32u * (c + 1), r);  // next chunk in flight
                } else {
                    // this warp's TMEM columns have all been read: hand them back
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        if (rank == 0) mbar_arrive(&tempty[acc]);
                        else mbar_arrive_remote(tempty_leader + 8u * acc);
                    }
                }
                if (fixup) {
                    // the parked parts, in cluster order
#pragma unroll
                    for (int q = 0; q < 8; ++q) add_parked4<INT8_KIND>(cur, q, sp0[(c * 8 + q) * 32 + lane]);
                    for (int cc = un.c_first + 1; cc <= un.c_last; ++cc) {
                        const uint4* pc = park_slot(sk.ws, cc, w16) + c * 8 * 32;
#pragma unroll
                        for (int q = 0; q < 8; ++q) add_parked4<INT8_KIND>(cur, q, __ldcg(pc + q * 32 + lane));
                    }
                }
                const int col0 = col_base + c * 32;
                if (col0 >= N || row0_warp >= M) continue;
                if (OUTK == 2) {
                    store_chunk<INT8_KIND>(ep, cur, row, col0, N, rs, row < M);
                    continue;
                }
                uint8_t* slot = slots + (chunk_seq & 1) * P_EPI_SLOT;
                if (lane == 0) bulk_wait_group_read<1>();  // the store issued two chunks ago has read this slot
                __syncwarp();
                const ColOps cop = c == 0 ? cops[0] : (c == 1 ? cops[1] : (c == 2 ? cops[2] : cops[3]));
                // without column scales and bias the per-column operands are
                // the identities, and skipping them (and their shuffles) gives
                // the same bits; the branch is warp-uniform
                const bool plain = !ep.col_scale && !ep.bias;
                if (OUTK == 1) {
                    // bf16: 64-byte rows, 16-byte chunk j at j ^ ((row >> 1) & 3)
                    uint8_t* rowp = slot + lane * 64;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        float v[8];
#pragma unroll
                        for (int t = 0; t < 8; ++t) {
                            const int e = 8 * j + t;
                            const float a = INT8_KIND ? __int2float_rn(static_cast<int32_t>(cur[e])) : __uint_as_float(cur[e]);
                            v[t] = plain ? __fmul_rn(__fmul_rn(a, ep.alpha), rs) : epi_elem(a, ep.alpha, rs, cop, e);
                        }
                        uint4 q;
                        q.x = f32x2_to_bf16x2(v[0], v[1]);
                        q.y = f32x2_to_bf16x2(v[2], v[3]);
                        q.z = f32x2_to_bf16x2(v[4], v[5]);
                        q.w = f32x2_to_bf16x2(v[6], v[7]);
                        *reinterpret_cast<uint4*>(rowp + 16 * (j ^ ((lane >> 1) & 3))) = q;
                    }
                } else {
                    // 4-byte values: 128-byte rows, 16-byte chunk j at j ^ (row & 7)
                    uint8_t* rowp = slot + lane * 128;
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        uint4 q;
                        if (raw_s32) {
                            q = make_uint4(cur[4 * j], cur[4 * j + 1], cur[4 * j + 2], cur[4 * j + 3]);
                        } else {
                            uint32_t o[4];
#pragma unroll
                            for (int t = 0; t < 4; ++t) {
                                const int e = 4 * j + t;
                                const float a = INT8_KIND ? __int2float_rn(static_cast<int32_t>(cur[e])) : __uint_as_float(cur[e]);
                                o[t] = __float_as_uint(plain ? __fmul_rn(__fmul_rn(a, ep.alpha), rs)
                                                             : epi_elem(a, ep.alpha, rs, cop, e));
                            }
                            q = make_uint4(o[0], o[1], o[2], o[3]);
                        }
                        *reinterpret_cast<uint4*>(rowp + 16 * (j ^ (lane & 7))) = q;
                    }
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d(&tmC, slot, col0, row0_warp);
                    bulk_commit_group();
                }
                ++chunk_seq;
                ++tile_groups;
            }
            if constexpr (AR) {
                if (ar.signal) {
                    // the previous tile's part of this warp is in memory (every bulk group
                    // but the chunks just issued for this tile has completed): count it
                    if (lane == 0 && sig_pending >= 0) {
                        switch (tile_groups) {
                            case 0: bulk_wait_group<0>(); break;
                            case 1: bulk_wait_group<1>(); break;
                            case 2: bulk_wait_group<2>(); break;
                            case 3: bulk_wait_group<3>(); break;
                            default: bulk_wait_group<4>(); break;
                        }
                        fence_proxy_async_global();
                        red_add_release_cluster(sig_cnt_leader, 1u);
                    }
                    __syncwarp();
                    sig_pending = tile;
                }
            }
        }
        if (lane == 0) bulk_wait_group_all();
        if constexpr (AR) {
            if (ar.signal && lane == 0 && sig_pending >= 0) {
                fence_proxy_async_global();
                red_add_release_cluster(sig_cnt_leader, 1u);
            }
        }
    }
    __syncwarp();  // reconverge the producer / MMA warps before the aligned cluster barrier
    tc_fence_before();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, TMEM_COLS);
    }
}

// ---------------- decode-shaped kernel (few tokens, many output channels) ----------------
// For M <= 64 tokens against a large weight the roles are swapped: 128 weight
// rows form the MMA's M side and the (padded) tokens its N side
// (tcgen05.mma M=128, N=BT), so one MMA tile covers all tokens.  The work --
// weight slices of 128 rows times k-blocks, in slice-major order -- is cut into
// equal contiguous ranges, one per CTA (stream-K), so every SM streams the same
// number of weight bytes.  A slice inside one range is finished directly.  A
// slice cut by range boundaries is finished by the CTA holding its first
// k-block (it reaches that part last): every later CTA touching the slice parks
// its raw accumulators in its own workspace row and raises its flag, and the
// owner adds them in CTA order before the epilogue -- no atomics, exact for
// int32 and deterministic for fp32.
//
// Stores leave through the TMA: while every SM streams weights at full rate,
// thread-level global loads and stores wait microseconds each (a 64-token
// slice written row by row took ~10 us on B200, longer than the weights it
// streamed).  So the epilogue warps write a slice's outputs (or a parked part)
// into shared memory and one thread sends it with one bulk store, and the
// producer warp, once its last weight load is issued, fetches the later CTA's
// parked part of this CTA's last slice with one bulk load.
template <int BT>
struct DecodeCfg {
    static constexpr int B_STAGE = BT * BK;
    static constexpr int OUT_BYTES = BT * 128 * 4;  // a slice of outputs (any type) or of raw accumulators
    // as many stages as fit beside the two epilogue buffers (up to 8: ~128 KB of
    // weights in flight per SM; measured on B200: 12 stages, or L2 prefetches
    // further ahead, stream no faster)
    static constexpr int BUDGET = 216 * 1024 - 2 * OUT_BYTES;
    static constexpr int STAGES = BUDGET / (A_STAGE + B_STAGE) < 8 ? BUDGET / (A_STAGE + B_STAGE) : 8;
    static constexpr int SMEM = 1024 + STAGES * (A_STAGE + B_STAGE) + 2 * OUT_BYTES + BT * 4 + 256;
    static constexpr uint32_t TMEM = BT <= 16 ? 32 : (BT <= 32 ? 64 : 128);
};

__device__ __forceinline__ long long range_begin(long long total, int c, int G) { return total * c / G; }

// The later CTAs [c_first, c_last] whose ranges hold the rest of a slice that
// ends at k-block slice_end, when this CTA's part of it ends at s1 (c_first >
// c_last when s1 == slice_end: the slice is this CTA's alone from there on).
__device__ __forceinline__ void decode_later_ctas(long long total, int G, long long s1, long long slice_end, int* c_first,
                                                  int* c_last) {
    *c_first = blockIdx.x + 1;
    *c_last = blockIdx.x;
    if (s1 < slice_end) {
        int c = blockIdx.x + 1;
        while (c + 1 < G && range_begin(total, c + 1, G) < slice_end) ++c;
        *c_last = c;
    }
}

template <bool INT8_KIND, bool W_KN, int BT>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    k_gemm_decode(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                  const __grid_constant__ CUtensorMap tmO, int M, int N, int K, uint32_t idesc, Epi ep,
                  uint32_t* ws, uint32_t* flags, uint32_t* err) {
    using Cfg = DecodeCfg<BT>;
    constexpr int D_STAGES = Cfg::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sW = smem;
    uint8_t* sX = smem + D_STAGES * A_STAGE;
    uint8_t* sOut = sX + D_STAGES * Cfg::B_STAGE;            // outputs or a part to park
    uint32_t* sPart = reinterpret_cast<uint32_t*>(sOut + Cfg::OUT_BYTES);  // a later CTA's parked part
    float* sRs = reinterpret_cast<float*>(sOut + 2 * Cfg::OUT_BYTES);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sRs + BT + ((BT & 1) ? 1 : 0));
    uint64_t* full = bars;
    uint64_t* empty = bars + D_STAGES;
    uint64_t* tfull = bars + 2 * D_STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* done = tempty + 2;
    uint64_t* pfull = done + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pfull + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int G = gridDim.x;
    const int kblocks = (K + BK - 1) / BK;
    const long long total = static_cast<long long>((N + 127) / 128) * kblocks;
    const long long b0 = range_begin(total, blockIdx.x, G);
    const long long b1 = range_begin(total, blockIdx.x + 1, G);
    // this CTA's last segment: does it own a slice that later CTAs finish?
    const int last_slice = static_cast<int>((b1 - 1) / kblocks);
    const long long last_s0 = max(b0, static_cast<long long>(last_slice) * kblocks);
    int lc_first, lc_last;
    decode_later_ctas(total, G, b1, static_cast<long long>(last_slice + 1) * kblocks, &lc_first, &lc_last);
    const bool last_fetch = (last_s0 % kblocks) == 0 && lc_last == lc_first;  // one later part: bulk-fetched

    // Launched with programmatic stream serialization: the next kernel of the
    // stream may start its prologue as this grid's CTAs finish.  Everything up
    // to pdl_wait() touches no memory an earlier kernel may still write (the
    // weight prefetch only fills L2, which is coherent).
    pdl_launch_dependents();
    if (threadIdx.x == 0) {
        for (int s = 0; s < D_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 128);
        }
        mbar_init(done, 1);
        mbar_init(pfull, 1);
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmW);
        tma_prefetch_desc(&tmX);
        tma_prefetch_desc(&tmO);
        // this CTA's first weight tiles, into L2 while an earlier kernel finishes
        for (long long kl = b0; kl < b1 && kl < b0 + D_STAGES; ++kl) {
            const int slice = static_cast<int>(kl / kblocks), kb = static_cast<int>(kl % kblocks);
            if (W_KN) tma_prefetch_l2_2d(&tmW, slice * 128, kb * BK);
            else tma_prefetch_l2_2d(&tmW, kb * BK, slice * 128);
        }
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, Cfg::TMEM);
        tmem_relinquish();
    }
    pdl_wait();
    if (threadIdx.x >= 64 && threadIdx.x < 64 + BT) {
        const int t = threadIdx.x - 64;
        sRs[t] = (ep.row_scale && t < M) ? __ldg(ep.row_scale + t) : 1.0f;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (elect_one()) {
            int stage = 0;
            uint32_t phase = 0;
            for (long long kl = b0; kl < b1; ++kl) {
                const int slice = static_cast<int>(kl / kblocks), kb = static_cast<int>(kl % kblocks);
                if (!mbar_wait(&empty[stage], phase ^ 1u, err)) break;
                mbar_arrive_expect_tx(&full[stage], A_STAGE + Cfg::B_STAGE);
                if (W_KN) tma_load_2d(sW + stage * A_STAGE, &tmW, &full[stage], slice * 128, kb * BK);
                else tma_load_2d(sW + stage * A_STAGE, &tmW, &full[stage], kb * BK, slice * 128);
                tma_load_2d(sX + stage * Cfg::B_STAGE, &tmX, &full[stage], kb * BK, 0);
                if (++stage == D_STAGES) { stage = 0; phase ^= 1u; }
            }
            if (last_fetch) {
                // the later CTA parked its part long ago (it was the start of its range)
                if (wait_flag_geq(flags + lc_first * 4, 1u, err)) {
                    fence_proxy_async_global();
                    mbar_arrive_expect_tx(pfull, Cfg::OUT_BYTES);
                    bulk_load_1d(sPart, ws + static_cast<size_t>(lc_first) * BT * 128, Cfg::OUT_BYTES, pfull);
                } else {
                    mbar_arrive(pfull);
                }
            }
        }
    } else if (warp == 1) {
        if (elect_one()) {
            int stage = 0;
            uint32_t phase = 0;
            int seg = 0;
            bool ok = true;
            for (long long s0 = b0; s0 < b1 && ok; ++seg) {
                const int slice = static_cast<int>(s0 / kblocks);
                const long long s1 = min(b1, static_cast<long long>(slice + 1) * kblocks);
                const int acc = seg & 1;
                if (!mbar_wait(&tempty[acc], ((static_cast<uint32_t>(seg) >> 1) & 1u) ^ 1u, err)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BT);
                for (long long kl = s0; kl < s1; ++kl) {
                    if (!mbar_wait(&full[stage], phase, err)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sW + stage * A_STAGE);
                    const uint32_t b_addr = smem_u32(sX + stage * Cfg::B_STAGE);
#pragma unroll
                    for (int kk = 0; kk < BK / 32; ++kk) {
                        // weights: K-major rows (N x K source) or one 128-wide MN-major chunk (K x N source)
                        const uint64_t adesc = W_KN ? smem_desc_sw128(a_addr + 4096u * kk, A_STAGE, 1024u)
                                                    : smem_desc_sw128(a_addr + 32u * kk, 16u, 1024u);
                        const uint64_t bdesc = smem_desc_sw128(b_addr + 32u * kk, 16u, 1024u);
                        const uint32_t accum = (kl > s0 || kk > 0) ? 1u : 0u;
                        if (INT8_KIND) mma_i8(d_tmem, adesc, bdesc, idesc, accum);
                        else mma_f8f6f4(d_tmem, adesc, bdesc, idesc, accum);
                    }
                    tc_commit(&empty[stage]);
                    if (++stage == D_STAGES) { stage = 0; phase ^= 1u; }
                }
                if (ok) tc_commit(&tfull[acc]);
                s0 = s1;
            }
            tc_commit(done);
            mbar_wait(done, 0, err);
        }
    } else {
        const int quarter = warp & 3;
        const int nl = quarter * 32 + lane;  // weight row within the slice
        const bool issuer = threadIdx.x == 64;
        const int odt = ep.out_dtype;
        const int esize = odt == NQ_BF16 ? 2 : (odt == NQ_S8 ? 1 : 4);
        // After a wait that ran out (error bit set) the warps still pass every
        // named barrier in the same order, with garbage data: none may leave
        // the protocol early while the others wait at a barrier.
        bool failed = false;
        int seg = 0;
        for (long long s0 = b0; s0 < b1; ++seg) {
            const int slice = static_cast<int>(s0 / kblocks);
            const long long slice_end = static_cast<long long>(slice + 1) * kblocks;
            const long long s1 = min(b1, slice_end);
            const bool head = (s0 % kblocks) == 0;  // this CTA holds the slice's first k-block
            const int acc = seg & 1;
            const uint32_t tpar = (static_cast<uint32_t>(seg) >> 1) & 1u;
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BT);
            uint32_t* sOut32 = reinterpret_cast<uint32_t*>(sOut);
            if (!head) {
                // a later part of a slice owned by an earlier CTA: park it with one
                // bulk store of [token][row] accumulators, then raise the flag
                if (!failed && !__all_sync(0xffffffffu, mbar_wait(&tfull[acc], tpar, err))) failed = true;
                tc_fence_after();
                named_bar_sync(1, 128);  // the previous bulk store has read sOut
#pragma unroll 1
                for (int c = 0; c < BT; c += 16) {
                    uint32_t r[16];
                    tmem_ld_32x32b_x16(taddr + c, r);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 16; ++j) sOut32[(c + j) * 128 + nl] = r[j];
                }
                tc_fence_before();
                mbar_arrive(&tempty[acc]);
                fence_proxy_async_smem();
                named_bar_sync(1, 128);
                if (issuer) {
                    bulk_store_1d(ws + static_cast<size_t>(blockIdx.x) * BT * 128, sOut, Cfg::OUT_BYTES);
                    bulk_commit_group();
                    bulk_wait_group<0>();  // the part is in global memory
                    fence_proxy_async_global();
                    __threadfence();
                    atomicAdd(flags + blockIdx.x * 4, 1u);
                }
                s0 = s1;
                continue;
            }
            // owner: later CTAs touching this slice (if the range ends inside it)
            int c_first, c_last;
            decode_later_ctas(total, G, s1, slice_end, &c_first, &c_last);
            const bool split = c_last >= c_first;
            const bool fetched = split && s1 == b1 && last_fetch;  // the producer bulk-loads the part
            if (split && !fetched) {
                if (lane == 0)
                    for (int c = c_first; c <= c_last; ++c) wait_flag_geq(flags + c * 4, 1u, err);
                __syncwarp();
            }
            const int n = slice * 128 + nl;
            const float cs = ep.col_scale && n < N ? __ldg(ep.col_scale + n) : 1.0f;
            const float bs = ep.bias && n < N ? __ldg(ep.bias + n) : -0.0f;
            if (fetched && !failed && !__all_sync(0xffffffffu, mbar_wait(pfull, 0, err))) failed = true;
            if (!failed && !__all_sync(0xffffffffu, mbar_wait(&tfull[acc], tpar, err))) failed = true;
            tc_fence_after();
            // the previous bulk store has read sOut, and every warp has passed its
            // flag wait (so the flags can be cleared below)
            named_bar_sync(1, 128);
#pragma unroll 1
            for (int c = 0; c < BT; c += 16) {
                uint32_t r[16];
                tmem_ld_32x32b_x16(taddr + c, r);
                tmem_ld_wait();
                if (fetched) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const uint32_t q = sPart[(c + j) * 128 + nl];
                        if (INT8_KIND) r[j] = static_cast<uint32_t>(static_cast<int32_t>(r[j]) + static_cast<int32_t>(q));
                        else r[j] = __float_as_uint(__fadd_rn(__uint_as_float(r[j]), __uint_as_float(q)));
                    }
                } else if (split) {
                    for (int cc = c_first; cc <= c_last; ++cc) {
                        const uint32_t* part = ws + static_cast<size_t>(cc) * BT * 128;
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const uint32_t q = __ldcg(part + (c + j) * 128 + nl);
                            if (INT8_KIND) r[j] = static_cast<uint32_t>(static_cast<int32_t>(r[j]) + static_cast<int32_t>(q));
                            else r[j] = __float_as_uint(__fadd_rn(__uint_as_float(r[j]), __uint_as_float(q)));
                        }
                    }
                }
                // values first, then stores (branches hoisted out of the row loops:
                // with a type switch per row the rows ran one after another,
                // ~80 ns each on B200)
                uint32_t bits[16];  // output elements, low esize bytes
                if (INT8_KIND && odt == NQ_S32) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) bits[j] = r[j];
                } else {
                    float v[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const float a = INT8_KIND ? __int2float_rn(static_cast<int32_t>(r[j])) : __uint_as_float(r[j]);
                        v[j] = __fadd_rn(__fmul_rn(__fmul_rn(__fmul_rn(a, ep.alpha), sRs[c + j]), cs), bs);
                    }
                    if (odt == NQ_BF16) {
#pragma unroll
                        for (int j = 0; j < 16; j += 2) {
                            const uint32_t p2 = f32x2_to_bf16x2(v[j], v[j + 1]);
                            bits[j] = p2 & 0xFFFFu;
                            bits[j + 1] = p2 >> 16;
                        }
                    } else if (odt == NQ_S8) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) bits[j] = static_cast<uint32_t>(static_cast<uint8_t>(requant_s8(v[j])));
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; ++j) bits[j] = __float_as_uint(v[j]);
                    }
                }
                {
                    // [token][row] in the output type; the bulk store clips t >= M, n >= N
                    if (esize == 2) {
                        uint16_t* o = reinterpret_cast<uint16_t*>(sOut) + c * 128 + nl;
#pragma unroll
                        for (int j = 0; j < 16; ++j) o[j * 128] = static_cast<uint16_t>(bits[j]);
                    } else if (esize == 1) {
                        uint8_t* o = sOut + c * 128 + nl;
#pragma unroll
                        for (int j = 0; j < 16; ++j) o[j * 128] = static_cast<uint8_t>(bits[j]);
                    } else {
                        uint32_t* o = sOut32 + c * 128 + nl;
#pragma unroll
                        for (int j = 0; j < 16; ++j) o[j * 128] = bits[j];
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
            fence_proxy_async_smem();
            named_bar_sync(1, 128);
            if (issuer) {
                tma_store_2d(&tmO, sOut, slice * 128, 0);
                bulk_commit_group();
                bulk_wait_group_read<0>();
            }
            // each parked part has exactly one reader (a CTA parks at most the
            // first segment of its range): clear its flag for the next launch
            if (issuer)
                for (int cc = c_first; cc <= c_last; ++cc) flags[cc * 4] = 0u;
            s0 = s1;
        }
        if (issuer) bulk_wait_group<0>();
    }
    __syncwarp();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, Cfg::TMEM);
    }
}

// ---------------- SIMT kernel (odd shapes) ----------------
template <bool INT8_KIND>
__global__ void __launch_bounds__(256) k_gemm_simt(const uint8_t* __restrict__ a, const uint8_t* __restrict__ b, int M,
                                                   int N, int K, int b_kn, int fa, int fb, Epi ep) {
    __shared__ float lut_a[256], lut_b[256];
    if (!INT8_KIND) {
        for (int i = threadIdx.x; i < 256; i += blockDim.x) {
            lut_a[i] = fa == kE5M2 ? ocp_decode2<kE5M2>(i).x : ocp_decode2<kE4M3>(i).x;
            lut_b[i] = fb == kE5M2 ? ocp_decode2<kE5M2>(i).x : ocp_decode2<kE4M3>(i).x;
        }
        __syncthreads();
    }
    const int col = blockIdx.x * 16 + (threadIdx.x & 15);
    const int row = blockIdx.y * 16 + (threadIdx.x >> 4);
    if (row >= M || col >= N) return;
    const uint8_t* ar = a + static_cast<size_t>(row) * K;
    uint32_t r[32];
    if (INT8_KIND) {
        int32_t s = 0;
        for (int k = 0; k < K; ++k) {
            const int32_t bv = static_cast<int8_t>(b_kn ? b[static_cast<size_t>(k) * N + col] : b[static_cast<size_t>(col) * K + k]);
            s += static_cast<int32_t>(static_cast<int8_t>(ar[k])) * bv;
        }
        r[0] = static_cast<uint32_t>(s);
    } else {
        float s = 0.0f;
        for (int k = 0; k < K; ++k) {
            const float bv = lut_b[b_kn ? b[static_cast<size_t>(k) * N + col] : b[static_cast<size_t>(col) * K + k]];
            s = __fmaf_rn(lut_a[ar[k]], bv, s);
        }
        r[0] = __float_as_uint(s);
    }
    const float rs = ep.row_scale ? __ldg(ep.row_scale + row) : 1.0f;
    if (INT8_KIND && ep.out_dtype == NQ_S32) {
        static_cast<int32_t*>(ep.out)[static_cast<size_t>(row) * ep.ldo + col] = static_cast<int32_t>(r[0]);
        return;
    }
    const float acc = INT8_KIND ? __int2float_rn(static_cast<int32_t>(r[0])) : __uint_as_float(r[0]);
    const float v = epi_value(acc, ep.alpha, rs, ep.col_scale, ep.bias, col);
    if (ep.out_dtype == NQ_S8)
        static_cast<int8_t*>(ep.out)[static_cast<size_t>(row) * ep.ldo + col] = requant_s8(v);
    else if (ep.out_dtype == NQ_BF16)
        static_cast<uint16_t*>(ep.out)[static_cast<size_t>(row) * ep.ldo + col] = static_cast<uint16_t>(f32x2_to_bf16x2(v, 0.0f));
    else
        static_cast<float*>(ep.out)[static_cast<size_t>(row) * ep.ldo + col] = v;
}

// ---------------- host side ----------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

nq_status_t get_encode_fn(EncodeTiledFn* fn) {
    static std::atomic<EncodeTiledFn> cached{nullptr};
    static std::mutex mu;
    EncodeTiledFn f = cached.load(std::memory_order_acquire);
    if (!f) {
        std::lock_guard<std::mutex> lk(mu);
        f = cached.load(std::memory_order_relaxed);
        if (!f) {
            void* p = nullptr;
            cudaDriverEntryPointQueryResult q;
            cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
            if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !p)
                return fail(NQ_ERROR_CUDA, "cuTensorMapEncodeTiled entry point not found");
            f = reinterpret_cast<EncodeTiledFn>(p);
            cached.store(f, std::memory_order_release);
        }
    }
    *fn = f;
    return NQ_SUCCESS;
}

// 2-D uint8 tensor map: inner extent `inner`, `outer` rows of `ld` bytes,
// box {box_inner, box_outer}, 128-byte swizzle, zero fill out of bounds.
nq_status_t make_map(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t ld,
                     uint32_t box_inner, uint32_t box_outer,
                     CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
    EncodeTiledFn fn;
    nq_status_t st = get_encode_fn(&fn);
    if (st != NQ_SUCCESS) return st;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {ld};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(NQ_ERROR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
    return NQ_SUCCESS;
}

// The shared-memory opt-in is a per-device function attribute.
template <class F>
nq_status_t ensure_smem_attr(F kern, int bytes, int device, std::atomic<uint64_t>* flags) {
    static std::mutex mu;
    return once_per_device(*flags, mu, device, [&]() -> nq_status_t {
        NQ_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes),
                      "cudaFuncSetAttribute(gemm)");
        return NQ_SUCCESS;
    });
}

uint32_t gemm_idesc(const nq_gemm_desc_t& d, bool i8, bool kn, uint32_t m, uint32_t n) {
    if (i8) return make_idesc(2u, 1u, 1u, kn ? 1u : 0u, m, n);
    return make_idesc(1u, d.a_format == NQ_E5M2 ? 1u : 0u, d.b_format == NQ_E5M2 ? 1u : 0u, kn ? 1u : 0u, m, n);
}

// Output map of the TMA-store epilogue: 32 x 32 boxes, swizzled to match
// the epilogue's staging layout (128-byte rows: SWIZZLE_128B, 64-byte bf16 rows:
// SWIZZLE_64B).
nq_status_t make_out_map(CUtensorMap* map, void* out, const nq_gemm_desc_t& d) {
    EncodeTiledFn fn;
    nq_status_t st = get_encode_fn(&fn);
    if (st != NQ_SUCCESS) return st;
    const bool bf = d.out_dtype == NQ_BF16;
    const uint64_t esize = bf ? 2 : 4;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(d.n), static_cast<cuuint64_t>(d.m)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(d.n) * esize};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt = bf ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                      : (d.out_dtype == NQ_S32 ? CU_TENSOR_MAP_DATA_TYPE_INT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32);
    CUresult r = fn(map, dt, 2, out, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    bf ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(NQ_ERROR_CUDA, "cuTensorMapEncodeTiled (output) failed (" + std::to_string(int(r)) + ")");
    return NQ_SUCCESS;
}

// Stream-K plan of the pair kernel for `tiles` tiles of `kblocks` k-blocks on
// `clusters` co-resident clusters.  Whole waves stay whole tiles; the last
// (1 + fraction) waves -- all tiles when there are fewer than two waves --
// are shared out by k-blocks only when the last wave would be at most half
// full and K is long (>= 48 k-blocks).  Measured on B200: for shorter K the
// parking, the flag clear and the in-order fixup waits of the epilogue warps
// (a short head part waits for its neighbour's long part while holding a
// TMEM accumulator) cost more than the idle half wave saves -- at 4096^3
// (3.46 waves, 32 k-blocks) whole tiles are 3-5 us faster.
StreamK plan_stream_k(int tiles, int kblocks, int clusters, bool allowed) {
    StreamK p{tiles, 0, nullptr, nullptr, 0};
    if (!allowed || clusters < 2 || kblocks < 48 || tiles % clusters == 0) return p;
    // (measured: also with fewer than two waves -- M = 256, N = 28672, K = 8192,
    // 112 tiles on 74 clusters -- whole tiles are 3-6 us faster)
    if (tiles % clusters > clusters / 2) return p;
    const int waves = tiles / clusters;
    const int dp = waves >= 2 ? (waves - 1) * clusters : 0;
    if (static_cast<long long>(tiles - dp) * kblocks < 4LL * clusters) return p;
    p.dp_tiles = dp;
    p.sk_tiles = tiles - dp;
    return p;
}

// qap (QA launches): the activations to quantize in phase 1; `a` is then the
// codes buffer the kernel fills and reads back.
template <bool I8, bool KN, int OUTK, bool SWIGLU = false, bool AR = false, bool QA = false>
nq_status_t launch_tc2(const nq_gemm_desc_t& d, const void* a, const void* b, void* out, const Epi& ep,
                       cudaStream_t s, const DeviceInfo& di, const ArParams* arp = nullptr,
                       const QuantA* qap = nullptr) {
    CUtensorMap ma, mb, mbh, mc;
    nq_status_t st = make_map(&ma, a, d.k, d.m, d.k, BK, 128);
    if (st != NQ_SUCCESS) return st;
    if (KN) st = make_map(&mb, b, d.n, d.k, d.n, 128, BK);
    else st = make_map(&mb, b, d.k, d.n, d.k, BK, 128);
    if (st != NQ_SUCCESS) return st;
    // half tiles: 64 columns of B per CTA (K x N: 64-byte swizzled rows)
    if (KN) st = make_map(&mbh, b, d.n, d.k, d.n, 64, BK, CU_TENSOR_MAP_SWIZZLE_64B);
    else st = make_map(&mbh, b, d.k, d.n, d.k, BK, 64);
    if (st != NQ_SUCCESS) return st;
    if (d.out_dtype != NQ_S8) {
        nq_gemm_desc_t od = d;
        if (SWIGLU) od.n = d.n / 2;
        st = make_out_map(&mc, out, od);
    } else {
        std::memset(&mc, 0, sizeof(mc));
    }
    if (st != NQ_SUCCESS) return st;
    const uint32_t idesc = gemm_idesc(d, I8, KN, P_BM, P_BN);
    const uint32_t idesc_h = gemm_idesc(d, I8, KN, P_BM, P_BN / 2);
    auto kern = k_gemm_tc2<I8, KN, OUTK, SWIGLU, AR, QA>;
    static std::atomic<uint64_t> attr_set{0};
    st = ensure_smem_attr(kern, P_SMEM_BYTES, di.device, &attr_set);
    if (st != NQ_SUCCESS) return st;
    // as many clusters as can be resident at once (an SM without a free partner
    // in its GPC cannot host half of a pair)
    static std::atomic<int> max_clusters[64];
    if (!max_clusters[di.device & 63].load(std::memory_order_relaxed)) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * (di.sm_count / 2));
        cfg.blockDim = dim3(AR ? P_THREADS_AR : P_THREADS);
        cfg.dynamicSmemBytes = P_SMEM_BYTES;
        int nc = 0;
        if (cudaOccupancyMaxActiveClusters(&nc, kern, &cfg) != cudaSuccess || nc <= 0) {
            cudaGetLastError();
            nc = di.sm_count / 2;
        }
        max_clusters[di.device & 63].store(nc, std::memory_order_relaxed);
    }
    const int tiles = ((d.m + P_BM - 1) / P_BM) * ((d.n + P_BN - 1) / P_BN);
    const int kblocks = (d.k + BK - 1) / BK;
    const int resident = std::max(1, max_clusters[di.device & 63].load(std::memory_order_relaxed));
    StreamK plan = plan_stream_k(tiles, kblocks, resident, !SWIGLU && !AR);
    if (!SWIGLU && !AR && plan.sk_tiles == 0) {
        // a last wave that fills at most half the clusters runs as half tiles
        const int rem = tiles % resident;
        if (rem > 0 && 2 * rem <= resident) {
            plan.dp_tiles = tiles - rem;
            plan.half_tiles = rem;
        }
    }
    // a QA or half-tile launch uses every resident cluster, whatever its tile count
    const int clusters = (plan.sk_tiles > 0 || plan.half_tiles > 0 || QA) ? resident
                                                                         : std::max(1, std::min(tiles, resident));
    constexpr int threads = AR ? P_THREADS_AR : P_THREADS;
    const int grid = 2 * clusters;
    StreamK sk = plan;
    void* scratch = nullptr;
    if (sk.sk_tiles > 0) {
        // one 256 x 256 accumulator slot and one flag per cluster
        const size_t ws_bytes = static_cast<size_t>(clusters) * P_BM * P_BN * 4;
        st = scratch_alloc(&scratch, ws_bytes + 256 * ((clusters * 4 + 255) / 256), s);
        if (st != NQ_SUCCESS) return st;
        sk.ws = static_cast<uint32_t*>(scratch);
        sk.flags = reinterpret_cast<uint32_t*>(static_cast<char*>(scratch) + ws_bytes);
        cudaError_t e = cudaMemsetAsync(sk.flags, 0, sizeof(uint32_t) * clusters, s);
        if (e != cudaSuccess) {
            scratch_free(scratch, s);
            return cuda_status(e, "nq_gemm: clear stream-K flags");
        }
    }
    QuantA qa;
    std::memset(&qa, 0, sizeof(qa));
    void* qa_flags = nullptr;
    if (QA) {
        // the count of quantized rows, zero before the launch
        qa = *qap;
        const size_t fb = 2 * sizeof(uint32_t);
        st = scratch_alloc(&qa_flags, 256, s);
        if (st != NQ_SUCCESS) {
            if (scratch) scratch_free(scratch, s);
            return st;
        }
        qa.done = static_cast<uint32_t*>(qa_flags);
        cudaError_t e = cudaMemsetAsync(qa.done, 0, fb, s);
        if (e != cudaSuccess) {
            scratch_free(qa_flags, s);
            if (scratch) scratch_free(scratch, s);
            return cuda_status(e, "nq_gemm: clear row-block flags");
        }
    }
    uint32_t* err = device_error_word();
    ArParams ar;
    if (arp) ar = *arp;
    else std::memset(&ar, 0, sizeof(ar));
    // the fused all-reduce launches keep plain stream order (their kernels wait
    // on other GPUs); the others overlap their prologue with the previous kernel
    cudaError_t e = cudaSuccess;
    if (AR) {
        kern<<<grid, threads, P_SMEM_BYTES, s>>>(ma, mb, mbh, mc, d.m, d.n, d.k, idesc, idesc_h, ep, sk, ar, qa, err);
        e = cudaGetLastError();
    } else {
        e = launch_pdl(kern, dim3(grid), dim3(threads), P_SMEM_BYTES, s, ma, mb, mbh, mc, d.m, d.n, d.k, idesc, idesc_h, ep,
                       sk, ar, qa, err);
    }
    if (scratch) scratch_free(scratch, s);
    if (qa_flags) scratch_free(qa_flags, s);
    return cuda_status(e, "nq_gemm (tcgen05, CTA pair)");
}

template <bool I8, bool KN, int BT>
nq_status_t launch_decode_bt(const nq_gemm_desc_t& d, const void* a, const void* b, const Epi& ep, cudaStream_t s,
                             const DeviceInfo& di) {
    using Cfg = DecodeCfg<BT>;
    CUtensorMap mw, mx, mo;
    // weights (the GEMM's B) are the MMA's A operand, tokens (the GEMM's A) its B operand
    nq_status_t st = KN ? make_map(&mw, b, d.n, d.k, d.n, 128, BK) : make_map(&mw, b, d.k, d.n, d.k, BK, 128);
    if (st != NQ_SUCCESS) return st;
    st = make_map(&mx, a, d.k, d.m, d.k, BK, BT);
    if (st != NQ_SUCCESS) return st;
    // outputs leave as one 128 x BT box per slice (nq_gemm takes this path only
    // with a 16-byte aligned output and N % 16 == 0, so the rows are addressable)
    const int esize = d.out_dtype == NQ_BF16 ? 2 : (d.out_dtype == NQ_S8 ? 1 : 4);
    if ((reinterpret_cast<uintptr_t>(ep.out) % 16) != 0 || (static_cast<size_t>(ep.ldo) * esize) % 16 != 0)
        return fail(NQ_ERROR_UNSUPPORTED, "nq_gemm (decode): the output must be 16-byte aligned with 16-byte rows");
    {
        EncodeTiledFn fn;
        st = get_encode_fn(&fn);
        if (st != NQ_SUCCESS) return st;
        cuuint64_t dims[2] = {static_cast<cuuint64_t>(d.n), static_cast<cuuint64_t>(d.m)};
        cuuint64_t strides[1] = {static_cast<cuuint64_t>(ep.ldo) * esize};
        cuuint32_t box[2] = {128, static_cast<cuuint32_t>(BT)};
        cuuint32_t estr[2] = {1, 1};
        const CUtensorMapDataType dt = esize == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16
                                     : esize == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                                  : CU_TENSOR_MAP_DATA_TYPE_UINT32;
        CUresult r = fn(&mo, dt, 2, ep.out, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS)
            return fail(NQ_ERROR_CUDA, "cuTensorMapEncodeTiled (decode output) failed (" + std::to_string(int(r)) + ")");
    }
    const uint32_t idesc = I8 ? make_idesc(2u, 1u, 1u, 0u, 128u, BT, KN ? 1u : 0u)
                              : make_idesc(1u, d.b_format == NQ_E5M2 ? 1u : 0u, d.a_format == NQ_E5M2 ? 1u : 0u, 0u,
                                           128u, BT, KN ? 1u : 0u);
    auto kern = k_gemm_decode<I8, KN, BT>;
    static std::atomic<uint64_t> attr_set{0};
    st = ensure_smem_attr(kern, Cfg::SMEM, di.device, &attr_set);
    if (st != NQ_SUCCESS) return st;
    const long long total = static_cast<long long>((d.n + 127) / 128) * ((d.k + BK - 1) / BK);
    const int grid = static_cast<int>(std::max<long long>(1, std::min<long long>(total, di.sm_count)));
    // per CTA one parked part (BT x 128 accumulators) and one flag (stride 4),
    // taken from the stream's flag words, which every launch leaves cleared: no
    // memset on the launch path
    const size_t ws_bytes = static_cast<size_t>(grid) * Cfg::OUT_BYTES;
    const size_t fl_bytes = static_cast<size_t>(grid) * 4 * 4;
    uint32_t* flags = nullptr;
    st = stream_flags(&flags, grid * 4, s);
    if (st != NQ_SUCCESS) return st;
    void* ws = nullptr;
    st = scratch_alloc(&ws, ws_bytes + (flags ? 0 : fl_bytes), s);
    if (st != NQ_SUCCESS) return st;
    cudaError_t e = cudaSuccess;
    if (!flags) {
        // inside a graph capture: flags of this launch, cleared by a memset node
        flags = reinterpret_cast<uint32_t*>(static_cast<char*>(ws) + ws_bytes);
        e = cudaMemsetAsync(flags, 0, fl_bytes, s);
    }
    if (e == cudaSuccess) {
        e = launch_pdl(kern, dim3(grid), dim3(GEMM_THREADS), Cfg::SMEM, s, mw, mx, mo, d.m, d.n, d.k, idesc, ep,
                       static_cast<uint32_t*>(ws), flags, device_error_word());
    }
    scratch_free(ws, s);
    return cuda_status(e, "nq_gemm (decode)");
}

template <bool I8, bool KN>
nq_status_t launch_decode(const nq_gemm_desc_t& d, const void* a, const void* b, const Epi& ep, cudaStream_t s,
                          const DeviceInfo& di) {
    if (d.m <= 16) return launch_decode_bt<I8, KN, 16>(d, a, b, ep, s, di);
    if (d.m <= 32) return launch_decode_bt<I8, KN, 32>(d, a, b, ep, s, di);
    return launch_decode_bt<I8, KN, 64>(d, a, b, ep, s, di);
}

// Few tokens against a large weight: too few output tiles to fill the SMs.
// Up to 64 tokens the swapped stream-K path streams the weights to all SMs.
bool use_decode(const nq_gemm_desc_t& d, int sm_count) {
    if (d.m > 64) return false;
    const long long tiles = static_cast<long long>((d.m + BM - 1) / BM) * ((d.n + BN - 1) / BN);
    return tiles < 2LL * sm_count && static_cast<long long>(d.n) * d.k >= (16LL << 20);
}

template <bool I8, bool KN>
nq_status_t launch_tc(const nq_gemm_desc_t& d, const void* a, const void* b, const Epi& ep, cudaStream_t s,
                      const DeviceInfo& di) {
    if (d.epilogue == NQ_EPI_SWIGLU) {
        if (I8) return fail(NQ_ERROR_UNSUPPORTED, "nq_gemm: SwiGLU epilogue is FP8-only");
        if (d.out_dtype == NQ_BF16) return launch_tc2<I8, KN, 1, true>(d, a, b, ep.out, ep, s, di);
        return launch_tc2<I8, KN, 0, true>(d, a, b, ep.out, ep, s, di);
    }
    if (use_decode(d, di.sm_count)) return launch_decode<I8, KN>(d, a, b, ep, s, di);
    if (d.m > BM) {
        if (d.out_dtype == NQ_BF16) return launch_tc2<I8, KN, 1>(d, a, b, ep.out, ep, s, di);
        if (d.out_dtype == NQ_S8) return launch_tc2<I8, KN, 2>(d, a, b, ep.out, ep, s, di);
        return launch_tc2<I8, KN, 0>(d, a, b, ep.out, ep, s, di);
    }
    CUtensorMap ma, mb;
    nq_status_t st = make_map(&ma, a, d.k, d.m, d.k, BK, BM);
    if (st != NQ_SUCCESS) return st;
    if (KN) st = make_map(&mb, b, d.n, d.k, d.n, BN / 2, BK);
    else st = make_map(&mb, b, d.k, d.n, d.k, BK, BN);
    if (st != NQ_SUCCESS) return st;
    const uint32_t idesc = gemm_idesc(d, I8, KN, BM, BN);
    auto kern = k_gemm_tc<I8, KN>;
    static std::atomic<uint64_t> attr_set{0};
    st = ensure_smem_attr(kern, SMEM_BYTES, di.device, &attr_set);
    if (st != NQ_SUCCESS) return st;
    const int tiles = ((d.m + BM - 1) / BM) * ((d.n + BN - 1) / BN);
    const int grid = std::max(1, std::min(tiles, di.sm_count));
    uint32_t* err = device_error_word();
    kern<<<grid, GEMM_THREADS, SMEM_BYTES, s>>>(ma, mb, d.m, d.n, d.k, idesc, ep, err);
    NQ_LAUNCH_CHECK("nq_gemm (tcgen05)");
    return NQ_SUCCESS;
}

// QuantizedMatmul::mixed_precision (quantize_ops.hpp:83-102).  Every output
// keeps the reference's order and roundings -- for p = 0 .. K-1:
// s = s + a[i,p] * (float(b[p,j]) * scale[p]), one rounding per multiply and add
// -- so the sum runs sequentially over K; the parallelism is across outputs.  A
// thread carries MP_ROWS rows of one column: each weight byte is read and
// scaled once per MP_ROWS outputs, and the block's activation rows are staged
// in shared memory ([k][row], two 16-byte reads per k).
constexpr int MP_ROWS = 8, MP_COLS = 128, MP_KC = 64;
__global__ void __launch_bounds__(MP_COLS) k_mixed_precision(const float* __restrict__ a, const int8_t* __restrict__ b,
                                                             const float* __restrict__ scale_b, float* __restrict__ out,
                                                             int M, int K, int N) {
    __shared__ __align__(16) float sa[MP_KC][MP_ROWS];
    const int col = blockIdx.x * MP_COLS + threadIdx.x;
    const int r0 = blockIdx.y * MP_ROWS;
    float acc[MP_ROWS];
#pragma unroll
    for (int r = 0; r < MP_ROWS; ++r) acc[r] = 0.0f;
    for (int p0 = 0; p0 < K; p0 += MP_KC) {
        const int kc = min(MP_KC, K - p0);
        __syncthreads();
        for (int i = threadIdx.x; i < MP_KC * MP_ROWS; i += MP_COLS) {
            const int r = i / MP_KC, p = i % MP_KC;  // consecutive threads: consecutive k of one row
            sa[p][r] = (r0 + r < M && p < kc) ? __ldg(a + static_cast<size_t>(r0 + r) * K + p0 + p) : 0.0f;
        }
        __syncthreads();
        if (col < N) {
            for (int p = 0; p < kc; ++p) {
                const float bv = __fmul_rn(static_cast<float>(b[static_cast<size_t>(p0 + p) * N + col]),
                                           __ldg(scale_b + p0 + p));
                const float4 x0 = *reinterpret_cast<const float4*>(&sa[p][0]);
                const float4 x1 = *reinterpret_cast<const float4*>(&sa[p][4]);
                const float xs[MP_ROWS] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
                for (int r = 0; r < MP_ROWS; ++r) acc[r] = __fadd_rn(acc[r], __fmul_rn(xs[r], bv));
            }
        }
    }
    if (col < N) {
#pragma unroll
        for (int r = 0; r < MP_ROWS; ++r)
            if (r0 + r < M) out[static_cast<size_t>(r0 + r) * N + col] = acc[r];
    }
}

// Byte transpose (rows x cols -> cols x rows) through 32 x 32 shared tiles,
// coalesced on both sides; used to give a GEMM a K-major copy of an operand.
__global__ void __launch_bounds__(256) k_transpose_u8(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                                      int rows, int cols) {
    __shared__ uint8_t tile[32][33];
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 8 rows of 32 per pass
    for (int y = ty; y < 32; y += 8) {
        const int r = r0 + y, c = c0 + tx;
        if (r < rows && c < cols) tile[y][tx] = src[static_cast<size_t>(r) * cols + c];
    }
    __syncthreads();
    for (int y = ty; y < 32; y += 8) {
        const int c = c0 + y, r = r0 + tx;
        if (c < cols && r < rows) dst[static_cast<size_t>(c) * rows + r] = tile[tx][y];
    }
}

}  // namespace

nq_status_t gemm_impl(const nq_gemm_desc_t* d, const void* a, const void* b, void* out, cudaStream_t s,
                      int force_simt) {
    if (!d) return fail(NQ_ERROR_INVALID_VALUE, "nq_gemm: null descriptor");
    if (d->m < 0 || d->n < 0 || d->k < 0) return fail(NQ_ERROR_INVALID_VALUE, "nq_gemm: negative size");
    if (d->m == 0 || d->n == 0) return NQ_SUCCESS;
    if (!a || !b || !out) {
        if (d->k > 0 || !out) return fail(NQ_ERROR_INVALID_VALUE, "nq_gemm: null operand");
    }
    const bool i8 = d->a_format == NQ_INT8;
    if (i8 != (d->b_format == NQ_INT8)) return fail(NQ_ERROR_INVALID_VALUE, "nq_gemm: INT8 needs both operands INT8");
    if (d->a_format < NQ_E4M3 || d->a_format > NQ_INT8 || d->b_format < NQ_E4M3 || d->b_format > NQ_INT8)
        return fail(NQ_ERROR_INVALID_VALUE, "nq_gemm: format");
    if (d->b_layout != NQ_B_KN && d->b_layout != NQ_B_NK) return fail(NQ_ERROR_INVALID_VALUE, "nq_gemm: b_layout");
    if (d->out_dtype != NQ_F32 && d->out_dtype != NQ_BF16 && d->out_dtype != NQ_S8 && !(i8 && d->out_dtype == NQ_S32))
        return fail(NQ_ERROR_INVALID_VALUE, "nq_gemm: out_dtype");
    if (d->epilogue != NQ_EPI_NONE && d->epilogue != NQ_EPI_SWIGLU)
        return fail(NQ_ERROR_INVALID_VALUE, "nq_gemm: epilogue");
    const bool swiglu = d->epilogue == NQ_EPI_SWIGLU;
    if (swiglu && (d->n % 256 != 0 || i8 || (d->out_dtype != NQ_BF16 && d->out_dtype != NQ_F32)))
        return fail(NQ_ERROR_UNSUPPORTED, "nq_gemm: SwiGLU needs FP8 operands, N % 256 == 0 and f32/bf16 output");
    DeviceInfo di;
    nq_status_t st = current_device(&di);
    if (st != NQ_SUCCESS) return st;
    Epi ep{out, swiglu ? d->n / 2 : d->n, d->out_dtype, d->alpha, d->row_scale, d->col_scale, d->bias};
    const bool kn = d->b_layout == NQ_B_KN;
    const bool tc_ok = !force_simt && d->k > 0 && d->k % 16 == 0 && d->n % 16 == 0 && aligned16(a) && aligned16(b) &&
                       aligned16(out);
    if (swiglu && !tc_ok) return fail(NQ_ERROR_UNSUPPORTED, "nq_gemm: SwiGLU needs the tensor-core path (aligned operands)");
    if (tc_ok) {
        if (i8) return kn ? launch_tc<true, true>(*d, a, b, ep, s, di) : launch_tc<true, false>(*d, a, b, ep, s, di);
        return kn ? launch_tc<false, true>(*d, a, b, ep, s, di) : launch_tc<false, false>(*d, a, b, ep, s, di);
    }
    dim3 grid((d->n + 15) / 16, (d->m + 15) / 16);
    if (grid.y > 65535) return fail(NQ_ERROR_UNSUPPORTED, "nq_gemm: M too large for the SIMT path");
    const uint8_t* a8 = static_cast<const uint8_t*>(a);
    const uint8_t* b8 = static_cast<const uint8_t*>(b);
    if (i8) k_gemm_simt<true><<<grid, 256, 0, s>>>(a8, b8, d->m, d->n, d->k, kn, 0, 0, ep);
    else k_gemm_simt<false><<<grid, 256, 0, s>>>(a8, b8, d->m, d->n, d->k, kn, d->a_format, d->b_format, ep);
    NQ_LAUNCH_CHECK("nq_gemm (simt)");
    return NQ_SUCCESS;
}

namespace {
nq_status_t fill_ar(const nq_allreduce_desc_t* r, ArParams* ar) {
    std::memset(ar, 0, sizeof(*ar));
    if (!r) return fail(NQ_ERROR_INVALID_VALUE, "all-reduce: null descriptor");
    if (r->tp < 1 || r->tp > NQ_MAX_TP || r->rank < 0 || r->rank >= r->tp)
        return fail(NQ_ERROR_INVALID_VALUE, "all-reduce: tp / rank");
    ar->peer_wait_ns = peer_wait_limit_ns();
    ar->tp = r->tp;
    ar->rank = r->rank;
    ar->epoch = r->epoch;
    ar->signal = r->signal ? 1 : 0;
    if (ar->signal)
        for (int p = 0; p < r->tp; ++p) {
            if (!r->signal_flags[p]) return fail(NQ_ERROR_INVALID_VALUE, "all-reduce: signal_flags");
            ar->signal_flags[p] = r->signal_flags[p];
        }
    if (r->m < 0) return fail(NQ_ERROR_INVALID_VALUE, "all-reduce: job rows");
    if (r->m > 0) {
        if (r->n <= 0 || r->n % P_BN != 0) return fail(NQ_ERROR_UNSUPPORTED, "all-reduce: job n must be a multiple of 256");
        if (!r->flags) return fail(NQ_ERROR_INVALID_VALUE, "all-reduce: job flags");
        const bool mc = r->mc_partial != nullptr;
        if (mc) {
            if (!r->mc_out || !r->mc_done || !aligned16(r->mc_partial) || !aligned16(r->mc_out))
                return fail(NQ_ERROR_INVALID_VALUE, "all-reduce: multicast addresses");
        } else {
            for (int p = 0; p < r->tp; ++p)
                if (!r->peer_partial[p] || !r->peer_out[p] || !r->peer_done[p] || !aligned16(r->peer_partial[p]) ||
                    !aligned16(r->peer_out[p]))
                    return fail(NQ_ERROR_INVALID_VALUE, "all-reduce: peer pointers");
        }
        ar->m = r->m;
        ar->n = r->n;
        ar->flags = r->flags;
        ar->mc_partial = static_cast<uint8_t*>(r->mc_partial);
        ar->mc_out = static_cast<uint8_t*>(r->mc_out);
        ar->mc_done = r->mc_done;
        for (int p = 0; p < r->tp; ++p) {
            ar->peer_partial[p] = static_cast<const uint8_t*>(r->peer_partial[p]);
            ar->peer_out[p] = static_cast<uint8_t*>(r->peer_out[p]);
            ar->peer_done[p] = r->peer_done[p];
        }
    }
    if (r->done) {
        ar->done = r->done;
        ar->done_target = r->done_target;
    }
    return NQ_SUCCESS;
}
}  // namespace

nq_status_t gemm_allreduce_impl(const nq_gemm_desc_t* d, const nq_allreduce_desc_t* r, const void* a, const void* b,
                                void* out, cudaStream_t s) {
    if (!d) return fail(NQ_ERROR_INVALID_VALUE, "nq_gemm_allreduce: null descriptor");
    if (d->m <= 0 || d->n <= 0 || d->k <= 0) return fail(NQ_ERROR_INVALID_VALUE, "nq_gemm_allreduce: sizes must be positive");
    if (!a || !b || !out) return fail(NQ_ERROR_INVALID_VALUE, "nq_gemm_allreduce: null operand");
    const bool i8 = d->a_format == NQ_INT8;
    if (i8 != (d->b_format == NQ_INT8)) return fail(NQ_ERROR_INVALID_VALUE, "nq_gemm_allreduce: INT8 needs both operands INT8");
    if (d->a_format < NQ_E4M3 || d->a_format > NQ_INT8 || d->b_format < NQ_E4M3 || d->b_format > NQ_INT8)
        return fail(NQ_ERROR_INVALID_VALUE, "nq_gemm_allreduce: format");
    if (d->b_layout != NQ_B_KN && d->b_layout != NQ_B_NK) return fail(NQ_ERROR_INVALID_VALUE, "nq_gemm_allreduce: b_layout");
    if (d->epilogue != NQ_EPI_NONE && d->epilogue != NQ_EPI_SWIGLU)
        return fail(NQ_ERROR_INVALID_VALUE, "nq_gemm_allreduce: epilogue");
    const bool swiglu = d->epilogue == NQ_EPI_SWIGLU;
    if (d->out_dtype != NQ_BF16) return fail(NQ_ERROR_UNSUPPORTED, "nq_gemm_allreduce: bf16 output only");
    if (d->k % 16 != 0 || d->n % 16 != 0 || !aligned16(a) || !aligned16(b) || !aligned16(out))
        return fail(NQ_ERROR_UNSUPPORTED, "nq_gemm_allreduce: needs k, n % 16 == 0 and 16-byte aligned operands");
    if (swiglu && (i8 || d->n % P_BN != 0))
        return fail(NQ_ERROR_UNSUPPORTED, "nq_gemm_allreduce: SwiGLU needs FP8 operands and n % 256 == 0");
    ArParams ar;
    nq_status_t st = fill_ar(r, &ar);
    if (st != NQ_SUCCESS) return st;
    if (ar.signal && (swiglu || d->n % P_BN != 0))
        return fail(NQ_ERROR_UNSUPPORTED, "nq_gemm_allreduce: a signalling GEMM needs n % 256 == 0 and no fused activation");
    DeviceInfo di;
    st = current_device(&di);
    if (st != NQ_SUCCESS) return st;
    Epi ep{out, swiglu ? d->n / 2 : d->n, NQ_BF16, d->alpha, d->row_scale, d->col_scale, d->bias};
    const bool kn = d->b_layout == NQ_B_KN;
    if (swiglu)
        return kn ? launch_tc2<false, true, 1, true, true>(*d, a, b, out, ep, s, di, &ar)
                  : launch_tc2<false, false, 1, true, true>(*d, a, b, out, ep, s, di, &ar);
    if (i8) return kn ? launch_tc2<true, true, 1, false, true>(*d, a, b, out, ep, s, di, &ar)
                      : launch_tc2<true, false, 1, false, true>(*d, a, b, out, ep, s, di, &ar);
    return kn ? launch_tc2<false, true, 1, false, true>(*d, a, b, out, ep, s, di, &ar)
              : launch_tc2<false, false, 1, false, true>(*d, a, b, out, ep, s, di, &ar);
}

// GEMM whose A operand is per-token quantized inside the kernel (QuantA).
nq_status_t gemm_quant_a_impl(const nq_gemm_desc_t* d, const void* x, uint8_t* a_codes, float* a_scales,
                              const void* b, void* out, cudaStream_t s) {
    if (!d) return fail(NQ_ERROR_INVALID_VALUE, "nq_gemm_quant_a: null descriptor");
    if (d->m < 0 || d->n < 0 || d->k < 0) return fail(NQ_ERROR_INVALID_VALUE, "nq_gemm_quant_a: negative size");
    if (d->m == 0 || d->n == 0) return NQ_SUCCESS;
    if (!x || !a_codes || !a_scales || !b || !out) return fail(NQ_ERROR_INVALID_VALUE, "nq_gemm_quant_a: null pointer");
    if (d->a_format != NQ_E4M3 || (d->b_format != NQ_E4M3 && d->b_format != NQ_E5M2))
        return fail(NQ_ERROR_UNSUPPORTED, "nq_gemm_quant_a: A is quantized to E4M3; B must be E4M3 or E5M2");
    if (d->b_layout != NQ_B_KN && d->b_layout != NQ_B_NK) return fail(NQ_ERROR_INVALID_VALUE, "nq_gemm_quant_a: b_layout");
    if (d->row_scale) return fail(NQ_ERROR_INVALID_VALUE, "nq_gemm_quant_a: row_scale must be NULL (the kernel's per-token scales are used)");
    if (d->out_dtype != NQ_BF16 && d->out_dtype != NQ_F32) return fail(NQ_ERROR_UNSUPPORTED, "nq_gemm_quant_a: f32 or bf16 output");
    if (d->epilogue != NQ_EPI_NONE && d->epilogue != NQ_EPI_SWIGLU) return fail(NQ_ERROR_INVALID_VALUE, "nq_gemm_quant_a: epilogue");
    const bool swiglu = d->epilogue == NQ_EPI_SWIGLU;
    if (swiglu && d->n % P_BN != 0) return fail(NQ_ERROR_UNSUPPORTED, "nq_gemm_quant_a: SwiGLU needs n % 256 == 0");
    if (d->k == 0 || d->k % 16 != 0 || d->n % 16 != 0 || !aligned16(x) || !aligned16(a_codes) || !aligned16(b) ||
        !aligned16(out))
        return fail(NQ_ERROR_UNSUPPORTED, "nq_gemm_quant_a: needs k, n % 16 == 0 and 16-byte aligned pointers");
    DeviceInfo di;
    nq_status_t st = current_device(&di);
    if (st != NQ_SUCCESS) return st;
    Epi ep{out, swiglu ? d->n / 2 : d->n, d->out_dtype, d->alpha, a_scales, d->col_scale, d->bias};
    // the first band of M-tiles (the rows the first waves of tiles need) is
    // quantized before the GEMM starts, the rest by the epilogue warps
    QuantA qa{static_cast<const uint16_t*>(x), a_codes, a_scales, nullptr, d->m, d->k, std::min(d->m, P_BAND * P_BM)};
    const bool kn = d->b_layout == NQ_B_KN;
    if (swiglu) {
        if (d->out_dtype == NQ_BF16)
            return kn ? launch_tc2<false, true, 1, true, false, true>(*d, a_codes, b, out, ep, s, di, nullptr, &qa)
                      : launch_tc2<false, false, 1, true, false, true>(*d, a_codes, b, out, ep, s, di, nullptr, &qa);
        return kn ? launch_tc2<false, true, 0, true, false, true>(*d, a_codes, b, out, ep, s, di, nullptr, &qa)
                  : launch_tc2<false, false, 0, true, false, true>(*d, a_codes, b, out, ep, s, di, nullptr, &qa);
    }
    if (d->out_dtype == NQ_BF16)
        return kn ? launch_tc2<false, true, 1, false, false, true>(*d, a_codes, b, out, ep, s, di, nullptr, &qa)
                  : launch_tc2<false, false, 1, false, false, true>(*d, a_codes, b, out, ep, s, di, nullptr, &qa);
    return kn ? launch_tc2<false, true, 0, false, false, true>(*d, a_codes, b, out, ep, s, di, nullptr, &qa)
              : launch_tc2<false, false, 0, false, false, true>(*d, a_codes, b, out, ep, s, di, nullptr, &qa);
}

nq_status_t allreduce_finish_impl(const nq_allreduce_desc_t* r, cudaStream_t s) {
    ArParams ar;
    nq_status_t st = fill_ar(r, &ar);
    if (st != NQ_SUCCESS) return st;
    if (ar.signal) return fail(NQ_ERROR_INVALID_VALUE, "nq_allreduce_finish: nothing to signal without a GEMM");
    if (ar.m == 0 && !ar.done) return NQ_SUCCESS;
    DeviceInfo di;
    st = current_device(&di);
    if (st != NQ_SUCCESS) return st;
    // owned tiles spread over one group per SM
    const int owned = ar.m > 0 ? (nq_gemm_allreduce_counters(ar.m, ar.n) + ar.tp - 1) / ar.tp : 1;
    const int grid = std::max(1, std::min(owned, di.sm_count));
    k_ar_finish<<<grid, AR_WARPS * 32, 0, s>>>(ar, device_error_word());
    NQ_LAUNCH_CHECK("nq_allreduce_finish");
    return NQ_SUCCESS;
}

}  // namespace nq

extern "C" {

nq_status_t nq_gemm(const nq_gemm_desc_t* desc, const void* a, const void* b, void* out, nq_stream_t s) {
    return nq::gemm_impl(desc, a, b, out, s, 0);
}

int nq_gemm_allreduce_counters(int m, int n) {
    if (m <= 0 || n <= 0) return 0;
    return ((m + nq::P_BM - 1) / nq::P_BM) * ((n + nq::P_BN - 1) / nq::P_BN);
}

int nq_allreduce_done_per_job(int m, int n, int in_signalling_kernel) {
    return nq_gemm_allreduce_counters(m, n) * (in_signalling_kernel ? nq::AR_WARPS - 1 : nq::AR_WARPS);
}

nq_status_t nq_gemm_allreduce(const nq_gemm_desc_t* d, const nq_allreduce_desc_t* a_r, const void* a, const void* b,
                              void* out, nq_stream_t s) {
    return nq::gemm_allreduce_impl(d, a_r, a, b, out, s);
}

nq_status_t nq_allreduce_finish(const nq_allreduce_desc_t* a_r, nq_stream_t s) {
    return nq::allreduce_finish_impl(a_r, s);
}

nq_status_t nq_gemm_quant_a(const nq_gemm_desc_t* desc, const void* x, uint8_t* a_codes, float* a_scales,
                            const void* b, void* out, nq_stream_t s) {
    return nq::gemm_quant_a_impl(desc, x, a_codes, a_scales, b, out, s);
}

// Test hook: the same GEMM forced onto the SIMT kernel (exact sequential-k).
nq_status_t nq_gemm_simt(const nq_gemm_desc_t* desc, const void* a, const void* b, void* out, nq_stream_t s) {
    return nq::gemm_impl(desc, a, b, out, s, 1);
}

static nq_status_t fp8_forward(const uint8_t* a, const uint8_t* b, float* out, int m, int k, int n, float sa, float sb,
                               float so, nq_format_t f, nq_stream_t s) {
    nq_gemm_desc_t d;
    std::memset(&d, 0, sizeof(d));
    d.m = m; d.n = n; d.k = k;
    d.a_format = f; d.b_format = f;
    d.b_layout = NQ_B_KN;
    d.out_dtype = NQ_F32;
    d.alpha = (sa * sb) * so;
    d.epilogue = NQ_EPI_NONE;
    return nq::gemm_impl(&d, a, b, out, s, 0);
}

nq_status_t nq_fp8_gemm_forward(const uint8_t* a, const uint8_t* b, float* out, int m, int k, int n, float scale_a,
                                float scale_b, float scale_out, nq_stream_t s) {
    return fp8_forward(a, b, out, m, k, n, scale_a, scale_b, scale_out, NQ_E4M3, s);
}

nq_status_t nq_fp8e5m2_gemm_forward(const uint8_t* a, const uint8_t* b, float* out, int m, int k, int n, float scale_a,
                                    float scale_b, float scale_out, nq_stream_t s) {
    return fp8_forward(a, b, out, m, k, n, scale_a, scale_b, scale_out, NQ_E5M2, s);
}

nq_status_t nq_fp8_gemm_backward(const uint8_t* grad_out, nq_format_t grad_format, const uint8_t* a, const uint8_t* b,
                                 float* grad_a, float* grad_b, int m, int k, int n, float scale_grad, float scale_a,
                                 float scale_b, nq_stream_t s) {
    if (m < 0 || k < 0 || n < 0) return nq::fail(NQ_ERROR_INVALID_VALUE, "nq_fp8_gemm_backward: negative size");
    if (grad_format != NQ_E4M3 && grad_format != NQ_E5M2)
        return nq::fail(NQ_ERROR_INVALID_VALUE, "nq_fp8_gemm_backward: grad_format must be E4M3 or E5M2");
    if (m == 0 || k == 0 || n == 0) return NQ_SUCCESS;
    if (!grad_out || (grad_a && !b) || (grad_b && !a))
        return nq::fail(NQ_ERROR_INVALID_VALUE, "nq_fp8_gemm_backward: null operand");
    if (m > 65535 * 32 || k > 65535 * 32) return nq::fail(NQ_ERROR_UNSUPPORTED, "nq_fp8_gemm_backward: M or K too large");
    nq_gemm_desc_t d;
    std::memset(&d, 0, sizeof(d));
    d.out_dtype = NQ_F32;
    d.epilogue = NQ_EPI_NONE;
    if (grad_a) {
        // grad_a (M x K) = grad_out (M x N) . B^T: B (K x N row-major) is the N-by-K
        // "packed" layout of the transposed operand
        d.m = m; d.n = k; d.k = n;
        d.a_format = grad_format; d.b_format = NQ_E4M3;
        d.b_layout = NQ_B_NK;
        d.alpha = scale_grad * scale_b;
        nq_status_t st = nq::gemm_impl(&d, grad_out, b, grad_a, s, 0);
        if (st != NQ_SUCCESS) return st;
    }
    if (grad_b) {
        // grad_b (K x N) = A^T (K x M) . grad_out (M x N): A transposed once into
        // pool scratch, grad_out read as a K x N (here M x N) row-major operand
        void* at = nullptr;
        nq_status_t st = nq::scratch_alloc(&at, static_cast<size_t>(m) * k, s);
        if (st != NQ_SUCCESS) return st;
        dim3 grid((k + 31) / 32, (m + 31) / 32);
        nq::k_transpose_u8<<<grid, 256, 0, s>>>(a, static_cast<uint8_t*>(at), m, k);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) {
            nq::scratch_free(at, s);
            return nq::cuda_status(e, "nq_fp8_gemm_backward: transpose");
        }
        d.m = k; d.n = n; d.k = m;
        d.a_format = NQ_E4M3; d.b_format = grad_format;
        d.b_layout = NQ_B_KN;
        d.alpha = scale_a * scale_grad;
        st = nq::gemm_impl(&d, at, grad_out, grad_b, s, 0);
        nq::scratch_free(at, s);
        if (st != NQ_SUCCESS) return st;
    }
    return NQ_SUCCESS;
}

nq_status_t nq_mixed_precision_matmul(const float* a, const int8_t* b, const float* scale_b, float* out, int m, int k,
                                      int n, nq_stream_t s) {
    if (m < 0 || k < 0 || n < 0) return nq::fail(NQ_ERROR_INVALID_VALUE, "nq_mixed_precision_matmul: negative size");
    if (m == 0 || n == 0) return NQ_SUCCESS;
    if (!out || (k > 0 && (!a || !b || !scale_b)))
        return nq::fail(NQ_ERROR_INVALID_VALUE, "nq_mixed_precision_matmul: null pointer");
    nq::DeviceInfo di;
    nq_status_t st = nq::current_device(&di);
    if (st != NQ_SUCCESS) return st;
    dim3 grid((n + nq::MP_COLS - 1) / nq::MP_COLS, (m + nq::MP_ROWS - 1) / nq::MP_ROWS);
    if (grid.y > 65535) return nq::fail(NQ_ERROR_UNSUPPORTED, "nq_mixed_precision_matmul: M too large");
    nq::k_mixed_precision<<<grid, nq::MP_COLS, 0, s>>>(a, b, scale_b, out, m, k, n);
    NQ_LAUNCH_CHECK("nq_mixed_precision_matmul");
    return NQ_SUCCESS;
}

size_t nq_fp8_gemm_workspace_size(int m, int k, int n) {
    auto al = [](size_t x) { return (x + 255) / 256 * 256; };
    return al(static_cast<size_t>(m) * k) + al(static_cast<size_t>(k) * n) + al(static_cast<size_t>(m) * n * sizeof(float));
}

}  // extern "C"

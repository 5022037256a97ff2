"""Tensor-parallel quantized layers and the SwiGLU MLP.

Mirror of pplmx/nova's cuda::neural tensor-parallel layers
(include/cuda/neural/tensor_parallel_layers.h:51 ColumnParallelLayer, :194
RowParallelLayer, :328 TensorParallelMLP; forward of the MLP at
src/cuda/neural/tensor_parallel_layers.cpp:561-579): gate and up are
column-parallel, down is row-parallel, one all-reduce sums the row-parallel
output.  Here the layers are W8A8 FP8 on the tcgen05 GEMMs of libnova_q:

  x (bf16, replicated)   -> per-token FP8 quantize          nq_quantize_rows
  [Wg|Wu] column shards  -> one GEMM, fused silu(g)*u       nq_gemm + NQ_EPI_SWIGLU
  h (bf16, this shard)   -> per-token FP8 quantize          nq_quantize_rows
  Wd row shard           -> partial output + all-reduce     nq_gemm_allreduce

The all-reduce runs inside the GEMM kernels over NVLink (allreduce "auto":
NVSwitch multicast when present, else peer memory): the down GEMM of a token
chunk writes this rank's partial tiles and signals their owners; the chunk's
reduction runs in the reducer warps of the next chunk's gate/up GEMM, and the
last down GEMM reduces its own chunk and waits for completion.  allreduce
"nccl" keeps a chunked torch.distributed all_reduce instead.

Weights are per-output-channel FP8 E4M3 (scale = column amax / 448, computed
on each rank's shard).  Shard layouts follow the reference set_weight
(column shard: columns [r*N/tp, (r+1)*N/tp) of a row-major K x N weight,
tensor_parallel_layers.cpp:111-136; row shard: rows [r*K/tp, ...), :344-368).
The reference takes an NcclContext; these classes take a torch.distributed
process group (NCCL on GPUs), whose size is the TP degree.  Rendezvous,
symmetric memory mappings, streams and device memory come from PyTorch; all
arithmetic and the all-reduce run in libnova_q.
"""
from __future__ import annotations

import numpy as np

BLOCK = 128  # gate/up packing granularity of the SwiGLU epilogue


# ---- pure host logic (tested on CPU) ------------------------------------------
def shard_columns(w, rank: int, tp: int):
    """Column shard of a row-major K x N weight (tensor_parallel_layers.cpp:111-136)."""
    n = w.shape[1]
    if n % tp:
        raise ValueError(f"out_features {n} is not divisible by tp={tp}")
    nl = n // tp
    return w[:, rank * nl:(rank + 1) * nl]


def shard_rows(w, rank: int, tp: int):
    """Row shard of a row-major K x N weight (tensor_parallel_layers.cpp:344-368)."""
    k = w.shape[0]
    if k % tp:
        raise ValueError(f"in_features {k} is not divisible by tp={tp}")
    kl = k // tp
    return w[rank * kl:(rank + 1) * kl]


def swiglu_pack_order(n_local: int) -> np.ndarray:
    """Column order of the packed [gate | up] weight: block j of 256 columns is
    gate columns 128j..128j+127 followed by up columns 128j..128j+127, indexed
    into the concatenation [gate (n_local) | up (n_local)]."""
    if n_local % BLOCK:
        raise ValueError(f"intermediate shard {n_local} must be a multiple of {BLOCK}")
    j = np.arange(n_local // BLOCK)[:, None]
    c = np.arange(BLOCK)[None, :]
    return np.concatenate([j * BLOCK + c, n_local + j * BLOCK + c], axis=1).reshape(-1)


def chunk_bounds(tokens: int, chunks: int, align: int = 256):
    """Token ranges of the overlapped GEMM / all-reduce pipeline, each a
    multiple of `align` rows except the last."""
    if tokens <= 0:
        return []
    chunks = max(1, min(chunks, (tokens + align - 1) // align))
    step = ((tokens + chunks - 1) // chunks + align - 1) // align * align
    return [(r0, min(tokens, r0 + step)) for r0 in range(0, tokens, step)]


def plan_chunks(tokens: int, n_gate_up: int, k_gate_up: int, n_down: int, k_down: int, tp: int,
                clusters: int = 74, max_chunks: int = 8, align: int = 256):
    """Token ranges of the fused TP pipeline (TensorParallelMLP._forward_fused),
    chosen with a model of it.  Unit of time: the MMAs of one 128-deep
    k-block of one 256 x 256 tile on one CTA pair (about 0.37 us on a B200).
      * a GEMM of r row tiles takes ceil(r * ceil(n / 256) / clusters) waves of
        ceil(k / 128) units: a nearly empty last wave costs a whole wave;
      * chunk c's all-reduce (its rows x n_down bf16 partial leaving each GPU
        once, at about 770 GB/s) runs under chunk c+1's GEMMs; the last chunk's
        is reduced inside its own down GEMM as its tiles complete, so at least
        one wave's share of it follows that GEMM;
      * every chunk costs a fixed 25 units of launches and per-token quantize.
    Candidates: equal splits into 1..max_chunks chunks, and chunks of r row
    tiles followed by a smaller remainder.  The cheapest plan wins (fewer
    chunks on ties).  tp == 1 has no all-reduce: one chunk."""
    if tokens <= 0:
        return []
    if tp <= 1:
        return [(0, tokens)]
    unit_s = 0.37e-6
    link_bytes_per_unit = 770e9 * unit_s
    nt_gu, nt_dn = -(-n_gate_up // 256), -(-n_down // 256)
    kb_gu, kb_dn = -(-k_gate_up // 128), -(-k_down // 128)

    def cost(bounds):
        t = ar_free = 0.0
        for c, (r0, r1) in enumerate(bounds):
            r = -(-(r1 - r0) // align)
            t += 25.0 + -(-(r * nt_gu) // clusters) * kb_gu
            dn_start = t
            waves_dn = -(-(r * nt_dn) // clusters)
            t += waves_dn * kb_dn
            ar = (r1 - r0) * n_down * 2 / link_bytes_per_unit
            if c < len(bounds) - 1:
                ar_free = max(ar_free, t) + ar
            else:
                ar_free = max(max(ar_free, dn_start) + ar, t + ar / waves_dn)
        return max(t, ar_free)

    cands = [chunk_bounds(tokens, c, align) for c in range(1, max_chunks + 1)]
    for r in range(1, -(-tokens // align) + 1):
        step = r * align
        b = [(r0, min(tokens, r0 + step)) for r0 in range(0, tokens, step)]
        if len(b) <= max_chunks:
            cands.append(b)
    best = min(cands, key=lambda b: (round(cost(b), 6), len(b)))
    return best


def reduce_pipeline(bounds, compute, group=None, tp: int = 1):
    """For each token range: compute(r0, r1) enqueues the partial rows and
    returns the tensor view holding them; with tp > 1 an asynchronous sum
    all-reduce of that view follows at once, so the next range's GEMM runs
    while this one is on the wire (RowParallelLayer::forward's all_reduce,
    tensor_parallel_layers.cpp:406, split into chunks).  Waits for every
    all-reduce before returning."""
    import torch.distributed as dist
    works = []
    for r0, r1 in bounds:
        view = compute(r0, r1)
        if tp > 1:
            works.append(dist.all_reduce(view, op=dist.ReduceOp.SUM, group=group, async_op=True))
    for w in works:
        w.wait()


def _group_info(group):
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group), dist.get_world_size(group)
    return 0, 1


def _as_tensor(w):
    import torch
    return w if isinstance(w, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(w, np.float32))


# ---- fused GEMM + all-reduce over peer memory -------------------------------------
class _ArState:
    """Symmetric buffers and counters of one m x n all-reduced output split
    into token chunks, and the epoch (forward count) of its counters."""

    def __init__(self, **kw):
        self.__dict__.update(kw)


class SymmetricAllReduce:
    """Symmetric buffers (torch.distributed._symmetric_memory: the same
    allocation mapped into every rank of `group`, plus an NVSwitch multicast
    mapping when the box has one) for the fused all-reduce of libnova_q
    (nq_gemm_allreduce / nq_allreduce_finish): per output shape and chunking
    a bf16 partial and a bf16 output buffer, the per-tile arrival counters of
    every chunk and one completion counter.  mode "nvls" reduces through
    multimem (needs multicast), "p2p" through peer loads and stores, "auto"
    picks nvls when multicast is present."""

    def __init__(self, group=None, mode: str = "auto"):
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm
        from . import capi
        self.torch, self.dist, self.symm, self.nq = torch, dist, symm, capi
        self.group = group if group is not None else dist.group.WORLD
        self.rank, self.tp = dist.get_rank(self.group), dist.get_world_size(self.group)
        if self.tp > capi.MAX_TP:
            raise ValueError(f"the fused all-reduce supports up to {capi.MAX_TP} ranks")
        if mode not in ("auto", "nvls", "p2p"):
            raise ValueError("mode must be 'auto', 'nvls' or 'p2p'")
        self.mode = mode
        self._states = {}

    def _map(self, t):
        """([peer pointers], multicast pointer or 0, handle) of a symmetric tensor."""
        h = self.symm.rendezvous(t, self.group.group_name)
        base = h.buffer_ptrs[self.rank]
        off = t.data_ptr() - base
        if off < 0 or off + t.numel() * t.element_size() > h.buffer_size:
            raise RuntimeError("symmetric tensor outside its allocation")
        mc = h.multicast_ptr + off if h.multicast_ptr else 0
        return [p + off for p in h.buffer_ptrs], mc, h

    def state(self, m, n, bounds):
        """Buffers for an m x n bf16 output reduced in the token chunks
        `bounds`, created (collectively: every rank calls in the same order)
        on first use.  Counters are zeroed on every rank before any rank can
        signal (a barrier follows the clear).  States live as long as the
        layer: peers may still be reading a buffer when this rank moves to
        another shape.  Each new token count therefore costs one collective
        allocation and 4 * m * n bytes of symmetric memory kept until the
        layer is dropped: callers with many distinct token counts should pad
        them to a few sizes."""
        key = (m, n, tuple(bounds))
        if key not in self._states:
            t, nq = self.torch, self.nq
            dev = t.device("cuda", t.cuda.current_device())
            offs, tiles = [], 0
            for r0, r1 in bounds:
                offs.append(tiles)
                tiles += nq.gemm_allreduce_counters(r1 - r0, n)
            flags = self.symm.empty(max(tiles, 1), dtype=t.int32, device=dev)
            done = self.symm.empty(16, dtype=t.int32, device=dev)
            partial = self.symm.empty(m, n, dtype=t.bfloat16, device=dev)
            out = self.symm.empty(m, n, dtype=t.bfloat16, device=dev)
            flags.zero_()
            done.zero_()
            t.cuda.synchronize()
            pf, _, hf = self._map(flags)
            pd, mcd, hd = self._map(done)
            pp, mcp, hp = self._map(partial)
            po, mco, ho = self._map(out)
            self.dist.barrier(group=self.group)
            have_mc = bool(mcp and mco and mcd)
            use_mc = self.mode == "nvls" or (self.mode == "auto" and have_mc)
            if use_mc and not have_mc:
                raise RuntimeError("NVSwitch multicast is not available for these buffers (mode 'nvls')")
            # chunk c < C-1 is reduced by a gate/up GEMM (5 reducer warps), the
            # last chunk by its own signalling down GEMM (4 reducer warps)
            per_forward = sum(nq.allreduce_done_per_job(r1 - r0, n, int(c == len(bounds) - 1))
                              for c, (r0, r1) in enumerate(bounds))
            self._states[key] = _ArState(m=m, n=n, bounds=list(bounds), offs=offs, flags=flags, done=done,
                                         partial=partial, out=out, pf=pf, pd=pd, pp=pp, po=po, mcp=mcp, mco=mco,
                                         mcd=mcd, use_mc=use_mc, per_forward=per_forward, epoch=0,
                                         handles=(hf, hd, hp, ho))
        return self._states[key]

    def begin(self, st):
        """Advances the state's epoch: call once per forward, before its descriptors."""
        st.epoch += 1

    def desc(self, st, signal=None, job=None, finish=False):
        """nq_allreduce_desc_t: `signal` = chunk whose partial the GEMM writes,
        `job` = chunk to reduce, `finish` = wait for every chunk of this epoch."""
        nq = self.nq
        d = nq.AllreduceDesc()
        # epochs and counter targets are taken modulo 2^32 (the kernels compare
        # counters by their signed difference, so wrapping is harmless)
        d.tp, d.rank, d.epoch = self.tp, self.rank, st.epoch & 0xFFFFFFFF
        if signal is not None:
            d.signal = 1
            for r in range(self.tp):
                d.signal_flags[r] = st.pf[r] + 4 * st.offs[signal]
        if job is not None:
            r0, r1 = st.bounds[job]
            row = 2 * r0 * st.n
            d.m, d.n = r1 - r0, st.n
            d.flags = st.flags.data_ptr() + 4 * st.offs[job]
            if st.use_mc:
                d.mc_partial, d.mc_out, d.mc_done = st.mcp + row, st.mco + row, st.mcd
            for r in range(self.tp):
                d.peer_partial[r], d.peer_out[r], d.peer_done[r] = st.pp[r] + row, st.po[r] + row, st.pd[r]
        if finish:
            d.done = st.done.data_ptr()
            d.done_target = (st.epoch * st.per_forward) & 0xFFFFFFFF
        return d

    def multicast(self):
        return any(v.use_mc for v in self._states.values())


# ---- layers ------------------------------------------------------------------------
class _FP8Linear:
    """Per-channel FP8 E4M3 weight (K x N, row-major) on the current device,
    applied to per-token FP8 activations with a bf16 output."""

    def __init__(self):
        import torch
        from . import capi
        self.nq, self.torch = capi, torch
        self.q = self.s = None
        self._ws = {}

    def load(self, w):
        t, nq = self.torch, self.nq
        dev = t.device("cuda", t.cuda.current_device())
        w = w.to(dev, t.float32).contiguous()
        k, n = w.shape
        self.k, self.n = k, n
        self.q = t.empty(k, n, dtype=t.uint8, device=dev)
        self.s = t.empty(n, dtype=t.float32, device=dev)
        nq.quantize_cols(w.data_ptr(), self.q.data_ptr(), self.s.data_ptr(), k, n, nq.E4M3,
                         t.cuda.current_stream().cuda_stream)

    def act(self, x, T, r0=0, r1=None):
        """Per-token FP8 quantize of rows [r0, r1) of a bf16 T x K activation
        into this layer's T-row code/scale buffers -> (codes, scales)."""
        t, nq = self.torch, self.nq
        r1 = T if r1 is None else r1
        if T not in self._ws:
            self._ws = {T: (t.empty(T, self.k, dtype=t.uint8, device=x.device),
                            t.empty(T, dtype=t.float32, device=x.device))}
        xq, sx = self._ws[T]
        if r1 > r0:
            nq.quantize_rows(x.data_ptr() + 2 * r0 * self.k, nq.BF16, xq.data_ptr() + r0 * self.k,
                             sx.data_ptr() + 4 * r0, r1 - r0, self.k, nq.E4M3, t.cuda.current_stream().cuda_stream)
        return xq, sx

    def gemm(self, xq, sx, out, r0, r1, epilogue=0):
        nq = self.nq
        n_out = self.n // 2 if epilogue else self.n
        d = nq.make_desc(r1 - r0, self.n, self.k, nq.E4M3, nq.E4M3, nq.B_KN, nq.BF16, 1.0,
                         sx.data_ptr() + 4 * r0, self.s.data_ptr(), 0, epilogue)
        nq.gemm(d, xq.data_ptr() + r0 * self.k, self.q.data_ptr(), out.data_ptr() + 2 * r0 * n_out,
                self.torch.cuda.current_stream().cuda_stream)


def _check_io(t, x, T, cols, name):
    if x.dtype != t.bfloat16 or not x.is_cuda or not x.is_contiguous() or x.numel() != T * cols:
        raise ValueError(f"{name} must be a contiguous bf16 CUDA tensor of {T} x {cols}")


class ColumnParallelLayer:
    """W8A8 FP8 column-parallel linear (tensor_parallel_layers.h:51): input
    [batch*seq x in_features] replicated, output [batch*seq x out_features/tp]
    this rank's column block, no communication."""

    def __init__(self, in_features: int, out_features: int, group=None):
        import torch
        self.torch, self.group = torch, group
        self.rank, self.tp = _group_info(group)
        if out_features % self.tp:
            raise ValueError("out_features must be divisible by the TP degree")
        self.in_features, self.out_features = in_features, out_features
        self.lin = _FP8Linear()

    def set_weight(self, weight):
        """Full weight [in_features x out_features], row-major (host or device)."""
        self.lin.load(shard_columns(_as_tensor(weight), self.rank, self.tp))
        self.torch.cuda.current_stream().synchronize()

    def forward(self, input, output, batch: int, seq: int):
        T = batch * seq
        if self.lin.q is None:
            raise RuntimeError("ColumnParallelLayer: set_weight has not been called")
        _check_io(self.torch, input, T, self.in_features, "input")
        _check_io(self.torch, output, T, self.out_features // self.tp, "output")
        if T == 0:
            return output
        xq, sx = self.lin.act(input, T)
        self.lin.gemm(xq, sx, output, 0, T)
        self.torch.cuda.current_stream().synchronize()
        return output


class RowParallelLayer:
    """W8A8 FP8 row-parallel linear (tensor_parallel_layers.h:194): input
    [batch*seq x in_features/tp] this rank's shard, output [batch*seq x
    out_features] replicated after the sum all-reduce (bf16, chunked)."""

    def __init__(self, in_features: int, out_features: int, group=None, chunks=None, allreduce: str = "auto"):
        import torch
        if allreduce not in ("auto", "nvls", "p2p", "nccl"):
            raise ValueError("allreduce must be 'auto', 'nvls', 'p2p' or 'nccl'")
        self.torch, self.group = torch, group
        self.rank, self.tp = _group_info(group)
        self.chunks = chunks if chunks is not None else (4 if self.tp > 1 else 1)
        # fused: one kernel does the GEMM and the all-reduce over peer memory
        # (nq_gemm_allreduce); nccl: GEMM chunks + torch.distributed all_reduce
        self.allreduce = allreduce if self.tp > 1 else "none"
        self.fused = SymmetricAllReduce(group, allreduce) if self.tp > 1 and allreduce != "nccl" else None
        if in_features % self.tp:
            raise ValueError("in_features must be divisible by the TP degree")
        self.in_features, self.out_features = in_features, out_features
        self.lin = _FP8Linear()

    def set_weight(self, weight):
        self.lin.load(shard_rows(_as_tensor(weight), self.rank, self.tp))
        self.torch.cuda.current_stream().synchronize()

    def forward(self, input, output, batch: int, seq: int, sync: bool = True):
        """output None (fused all-reduce only): returns the layer's symmetric
        output buffer, valid until the next forward of this shape."""
        T = batch * seq
        if self.lin.q is None:
            raise RuntimeError("RowParallelLayer: set_weight has not been called")
        _check_io(self.torch, input, T, self.in_features // self.tp, "input")
        if output is not None or self.fused is None:
            _check_io(self.torch, output, T, self.out_features, "output")
        if T == 0:
            return output
        xq, sx = self.lin.act(input, T)
        if self.fused is not None:
            # one kernel: the GEMM, its tiles' all-reduce and the completion wait
            ar = self.fused
            st = ar.state(T, self.out_features, [(0, T)])
            ar.begin(st)
            lin, nq = self.lin, self.lin.nq
            d = nq.make_desc(T, lin.n, lin.k, nq.E4M3, nq.E4M3, nq.B_KN, nq.BF16, 1.0, sx.data_ptr(),
                             lin.s.data_ptr(), 0)
            nq.gemm_allreduce(d, ar.desc(st, signal=0, job=0, finish=True), xq.data_ptr(), lin.q.data_ptr(),
                              st.partial.data_ptr(), self.torch.cuda.current_stream().cuda_stream)
            if output is None:
                output = st.out
            else:
                output.copy_(st.out)
            if sync:
                self.torch.cuda.current_stream().synchronize()
            return output

        def compute(r0, r1):
            self.lin.gemm(xq, sx, output, r0, r1)
            return output[r0:r1]

        reduce_pipeline(chunk_bounds(T, self.chunks), compute, self.group, self.tp)
        if sync:
            self.torch.cuda.current_stream().synchronize()
        return output


class TensorParallelMLP:
    """out = down( silu(gate(x)) * up(x) ) (tensor_parallel_layers.h:328).
    hidden_dim H, intermediate_size I, tp = size of `group`.  set_weight
    takes the FULL fp32 weights in the reference layout (gate, up: H x I;
    down: I x H, row-major); forward(input, output, batch, seq) reads and
    writes bf16 device tensors of [batch*seq x H] and synchronises the
    stream, as the reference's forward does.  Gate and up of this rank's
    shard are one packed FP8 weight (alternating 128-column blocks) so one
    GEMM with the SwiGLU epilogue produces silu(g) * u directly."""

    def __init__(self, hidden_dim: int, intermediate_size: int, group=None, chunks=None,
                 overlap: str = "full", allreduce: str = "auto", chunk_rows=None):
        import torch
        if overlap not in ("full", "down"):
            raise ValueError("overlap must be 'full' or 'down'")
        self.torch, self.group, self.overlap = torch, group, overlap
        self.rank, self.tp = _group_info(group)
        if intermediate_size % (self.tp * BLOCK):
            raise ValueError("intermediate_size must be a multiple of 128 * tp")
        if hidden_dim % 16:
            raise ValueError("hidden_dim must be a multiple of 16")
        self.H, self.I = hidden_dim, intermediate_size
        self.I_local = intermediate_size // self.tp
        # token chunks of the GEMM / all-reduce pipeline (an explicit value is
        # always honoured): 1 up to tp = 4, where the fused all-reduce hides
        # inside the single down GEMM; 3 from tp = 8, where the all-reduce
        # outgrows the down GEMM and chunk c's reduction runs inside chunk
        # c+1's gate/up GEMM.  Measured on B200, T = 16384, H = 8192,
        # I = 28672: tp = 4 2.16 ms with 1 chunk, 2.23 with 2, 2.27 with 3 or
        # 4; tp = 8 1.32 ms with 3 chunks, 1.36 with 2, 1.36-1.40 with 4.
        self.chunks = chunks if chunks is not None else (1 if self.tp <= 4 else 3)
        # chunk_rows: tokens per chunk (a multiple of 256; the last chunk takes
        # the remainder) instead of `chunks` equal chunks; "plan": plan_chunks'
        # model of the pipeline
        if chunk_rows is not None and chunk_rows != "plan" and (int(chunk_rows) <= 0 or int(chunk_rows) % 256):
            raise ValueError("chunk_rows must be a positive multiple of 256 or 'plan'")
        self.chunk_rows = chunk_rows
        self.gate_up = _FP8Linear()
        self.down = RowParallelLayer(intermediate_size, hidden_dim, group, self.chunks, allreduce)
        self._h = {}

    def _bounds(self, T):
        """Token ranges of the chunked pipeline for T tokens."""
        if self.chunk_rows == "plan":
            return plan_chunks(T, 2 * self.I_local, self.H, self.H, self.I_local, self.tp)
        if self.chunk_rows:
            step = int(self.chunk_rows)
            return [(r0, min(T, r0 + step)) for r0 in range(0, T, step)]
        return chunk_bounds(T, self.chunks)

    def set_weight(self, gate_weight, up_weight, down_weight):
        """Full weights (host or device, fp32): keeps this rank's shards."""
        t = self.torch
        dev = t.device("cuda", t.cuda.current_device())
        g = shard_columns(_as_tensor(gate_weight), self.rank, self.tp).to(dev, t.float32)
        u = shard_columns(_as_tensor(up_weight), self.rank, self.tp).to(dev, t.float32)
        order = t.from_numpy(swiglu_pack_order(self.I_local))
        # per-column scales do not depend on the column order, so quantizing
        # the packed matrix equals packing the separately quantized shards
        self.gate_up.load(t.cat([g, u], dim=1).index_select(1, order.to(g.device)))
        self.down.set_weight(down_weight)

    def forward(self, input, output, batch: int, seq: int, sync: bool = True):
        """overlap = "full": the token chunks run the whole MLP (gate/up GEMM,
        quantize, down GEMM) back to back, so chunk i's all-reduce overlaps
        chunk i+1's three kernels; "down": gate/up for all tokens first, then
        only the down-projection is chunked."""
        t = self.torch
        T = batch * seq
        if self.gate_up.q is None:
            raise RuntimeError("TensorParallelMLP: set_weight has not been called")
        _check_io(t, input, T, self.H, "input")
        if output is not None or self.down.fused is None:
            _check_io(t, output, T, self.H, "output")
        if T == 0:
            return output
        if T not in self._h:
            self._h = {T: t.empty(T, self.I_local, dtype=t.bfloat16, device=input.device)}
        h = self._h[T]
        epi = self.gate_up.nq.EPI_SWIGLU
        down = self.down.lin
        xq, sx = self.gate_up.act(input, T)
        if self.down.fused is not None:
            return self._forward_fused(xq, sx, h, output, T, sync)
        bounds = self._bounds(T)
        if self.overlap == "down" or len(bounds) == 1:
            self.gate_up.gemm(xq, sx, h, 0, T, epilogue=epi)

        def compute(r0, r1):
            if self.overlap != "down" and len(bounds) > 1:
                self.gate_up.gemm(xq, sx, h, r0, r1, epilogue=epi)
            hq, sh = down.act(h, T, r0, r1)
            down.gemm(hq, sh, output, r0, r1)
            return output[r0:r1]

        reduce_pipeline(bounds, compute, self.group, self.tp)
        if sync:
            t.cuda.current_stream().synchronize()
        return output

    def _forward_fused(self, xq, sx, h, output, T, sync):
        """Token chunks c = 0..C-1: gate/up GEMM of chunk c (its reducer warps
        all-reduce chunk c-1), quantize h, down GEMM of chunk c writing this
        rank's partial and signalling its tiles; the last down GEMM also
        reduces its own chunk and waits until every chunk is complete."""
        t, nq = self.torch, self.gate_up.nq
        s = t.cuda.current_stream().cuda_stream
        ar, down, gu = self.down.fused, self.down.lin, self.gate_up
        bounds = self._bounds(T)
        st = ar.state(T, self.H, bounds)
        ar.begin(st)
        C = len(bounds)
        for c, (r0, r1) in enumerate(bounds):
            d1 = nq.make_desc(r1 - r0, gu.n, gu.k, nq.E4M3, nq.E4M3, nq.B_KN, nq.BF16, 1.0, sx.data_ptr() + 4 * r0,
                              gu.s.data_ptr(), 0, nq.EPI_SWIGLU)
            if c == 0:
                nq.gemm(d1, xq.data_ptr() + r0 * gu.k, gu.q.data_ptr(), h.data_ptr() + 2 * r0 * self.I_local, s)
            else:
                nq.gemm_allreduce(d1, ar.desc(st, job=c - 1), xq.data_ptr() + r0 * gu.k, gu.q.data_ptr(),
                                  h.data_ptr() + 2 * r0 * self.I_local, s)
            hq, sh = down.act(h, T, r0, r1)
            d2 = nq.make_desc(r1 - r0, down.n, down.k, nq.E4M3, nq.E4M3, nq.B_KN, nq.BF16, 1.0,
                              sh.data_ptr() + 4 * r0, down.s.data_ptr(), 0)
            last = c == C - 1
            nq.gemm_allreduce(d2, ar.desc(st, signal=c, job=c if last else None, finish=last),
                              hq.data_ptr() + r0 * down.k, down.q.data_ptr(),
                              st.partial.data_ptr() + 2 * r0 * self.H, s)
        if output is None:
            output = st.out
        else:
            output.copy_(st.out)
        if sync:
            t.cuda.current_stream().synchronize()
        return output

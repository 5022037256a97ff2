"""Failure detection on the host, the form this path supports without a GPU
fault: a rank that leaves between steps.  Two gloo ranks (CPU) run a step of
the chunked all-reduce pipeline the TP layers use (nova_b200.tp.
reduce_pipeline); then rank 1 exits without taking part in step 2, and rank
0's next collective must end with an error within its process-group timeout
instead of waiting for ever -- the host-side counterpart of the reference's
deadline on a collective (safe_stream_wait, src/cuda/nccl/nccl_error.cpp:
13-83: a bounded wait that reports the failure).  No GPU is touched."""
import os
import socket
import time

import pytest


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, timeout_s, result_dir):
    import datetime

    import torch
    import torch.distributed as dist
    from nova_b200 import tp
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
    out = torch.zeros(600, 64)
    src = torch.full((600, 64), float(rank + 1))

    def compute(r0, r1):
        out[r0:r1] = src[r0:r1]
        return out[r0:r1]

    tp.reduce_pipeline(tp.chunk_bounds(600, 4), compute, None, world)   # step 1: every rank
    assert torch.all(out == 3.0)
    if rank == 1:
        os._exit(0)                                                       # leaves between steps
    t0 = time.monotonic()
    err = ""
    try:
        tp.reduce_pipeline(tp.chunk_bounds(600, 4), compute, None, world)  # step 2: the peer is gone
    except Exception as e:  # the failure the survivor must see
        err = f"{type(e).__name__}: {e}"
    dt = time.monotonic() - t0
    with open(os.path.join(result_dir, "rank0.txt"), "w") as f:
        f.write(f"{dt}\n{err}\n")
    os._exit(0)


def test_survivor_sees_a_departed_rank(tmp_path):
    import torch.multiprocessing as mp
    timeout_s = 5
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, timeout_s, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("a rank did not finish: the survivor's collective waited past its timeout")
    dt, err = open(tmp_path / "rank0.txt").read().split("\n", 1)
    assert err.strip(), "the survivor's collective succeeded without its peer"
    assert float(dt) <= 4 * timeout_s, dt

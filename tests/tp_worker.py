"""torchrun worker of the tp > 1 parity test (tests/test_tp_gpu.py): every
rank builds the same seeded full weights, keeps its shards, runs the FP8
SwiGLU MLP with the chunked NCCL all-reduce, and rank 0 checks every
rank's SwiGLU intermediate and the replicated output against the oracle
(tolerances as in tests/test_tp_gpu.py)."""
import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    from nova_b200.tp import TensorParallelMLP
    from test_tp_gpu import bits, check_mlp, to_dev_bf16, weights
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    ok = True
    modes = sys.argv[1:] or ["nccl", "p2p", "auto"]
    # (T, H, I, overlap, chunks): chunks None = the layer's default for this tp;
    # 3 exercises the chunked pipeline (jobs hosted by the gate/up GEMMs) at any tp
    cases = [(600, 256, 512, "full", None), (1024, 512, 1024, "down", None), (1000, 512, 2048, "full", 3),
             (600, 256, 512, "full", None)]
    for allreduce in modes:
        for T, H, I, overlap, chunks in cases:
            unit = 128 * world
            I = max(unit, (I + unit - 1) // unit * unit)   # each rank's shard a multiple of 128
            x, wg, wu, wd = weights(T, H, I)
            mlp = TensorParallelMLP(H, I, overlap=overlap, allreduce=allreduce, chunks=chunks)
            mlp.set_weight(wg, wu, wd)
            out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
            for _ in range(2):   # repeated calls: the fused path's counters must come back to zero
                out.zero_()
                mlp.forward(to_dev_bf16(x), out, 1, T)
            # every rank holds the same replicated output
            mx = out.float().clone()
            dist.all_reduce(mx, op=dist.ReduceOp.MAX)
            flag = torch.tensor([int(torch.equal(mx, out.float()))], device="cuda")
            dist.all_reduce(flag, op=dist.ReduceOp.MIN)
            hs = [torch.empty_like(mlp._h[T]) for _ in range(world)]
            dist.all_gather(hs, mlp._h[T])
            import nova_b200.capi as nq
            errs = torch.tensor([nq.device_error_flags()], device="cuda")
            dist.all_reduce(errs, op=dist.ReduceOp.MAX)
            if rank == 0:
                h_err, out_err, full_err = check_mlp(bits(out), [bits(h) for h in hs], x, wg, wu, wd, world)
                mc = mlp.down.fused.multicast() if mlp.down.fused is not None else False
                print(f"allreduce={allreduce} multicast={mc} T={T} H={H} I={I} tp={world} overlap={overlap} "
                      f"chunks={mlp.chunks} "
                      f"h_err={h_err:.3e} out_err={out_err:.3e} full_norm_err={full_err:.3e} "
                      f"replicated={bool(flag.item())} device_errors={int(errs.item())}", flush=True)
                ok = ok and h_err <= 1e-2 and out_err <= 1e-2 and full_err <= 1e-2 and bool(flag.item()) \
                    and int(errs.item()) == 0
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print("TP_WORKER_OK" if ok else "TP_WORKER_FAIL")
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())

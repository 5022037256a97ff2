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
    for T, H, I, overlap in [(600, 256, 512, "full"), (1024, 512, 1024, "down"), (1000, 512, 2048, "full")]:
        x, wg, wu, wd = weights(T, H, I)
        mlp = TensorParallelMLP(H, I, overlap=overlap)
        mlp.set_weight(wg, wu, wd)
        out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
        mlp.forward(to_dev_bf16(x), out, 1, T)
        # every rank holds the same replicated output
        mx = out.float().clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        flag = torch.tensor([int(torch.equal(mx, out.float()))], device="cuda")
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        hs = [torch.empty_like(mlp._h[T]) for _ in range(world)]
        dist.all_gather(hs, mlp._h[T])
        if rank == 0:
            h_err, out_err, full_err = check_mlp(bits(out), [bits(h) for h in hs], x, wg, wu, wd, world)
            print(f"T={T} H={H} I={I} tp={world} overlap={overlap} chunks={mlp.chunks} h_err={h_err:.3e} "
                  f"out_err={out_err:.3e} full_norm_err={full_err:.3e} replicated={bool(flag.item())}")
            ok = ok and h_err <= 1e-2 and out_err <= 1e-2 and full_err <= 1e-2 and bool(flag.item())
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print("TP_WORKER_OK" if ok else "TP_WORKER_FAIL")
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())

"""torchrun worker of the tp > 1 parity test (tests/test_tp_gpu.py): every
rank builds the same seeded full weights, keeps its shards, runs the FP8
SwiGLU MLP with the chunked NCCL all-reduce, and rank 0 compares the
replicated output with the sum of the oracle's per-rank partials."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    import oracle_lib as O
    from nova_b200.tp import TensorParallelMLP
    from test_tp_gpu import bits, rel_err, to_dev_bf16, weights
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    ok = True
    for T, H, I, overlap in [(600, 256, 512, "full"), (1024, 512, 1024, "down")]:
        x, wg, wu, wd = weights(T, H, I)
        mlp = TensorParallelMLP(H, I, overlap=overlap)
        mlp.set_weight(wg, wu, wd)
        out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
        mlp.forward(to_dev_bf16(x), out, 1, T)
        got = O.bf16_bits_to_f32(bits(out))
        # every rank holds the same replicated output
        g = torch.from_numpy(got).cuda()
        mx = g.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        same = bool(torch.equal(mx, g))
        flag = torch.tensor([int(same)], device="cuda")
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        if rank == 0:
            want = sum(O.bf16_bits_to_f32(O.tp_mlp_partial(x, wg, wu, wd, r, world)[1]).astype(np.float64)
                       for r in range(world))
            err = rel_err(got, want)
            print(f"T={T} H={H} I={I} tp={world} overlap={overlap} rel_err={err:.3e} replicated={bool(flag.item())}")
            ok = ok and err <= 2e-2 and bool(flag.item())
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print("TP_WORKER_OK" if ok else "TP_WORKER_FAIL")
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())

"""Multi-GPU parity of the expert-parallel layer (run under torchrun, one rank per GPU; driven by test_gpu_ep_multi.py).

Each rank routes its own tokens, exchanges rows with the other ranks -- over NCCL, and over peer memory (the library's
store kernels into the other GPUs' exchange buffers, ep.PeerExchange) -- and compares the result with the single-GPU
block it computes itself from the whole layer: top-k identical, x within 1e-5 relative L2. The peer exchange runs several
steps in a row with batches of different sizes (its regions and step signals are reused). Exits non-zero on a mismatch.
"""
import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import clutor_b200 as cb  # noqa: E402
from clutor_b200 import ep, synth  # noqa: E402


def main() -> int:
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    ctx = cb.Context(local)
    worst, ok = 0.0, True
    xchg = ep.PeerExchange(ctx, 256, 2048, 8)
    for gt in (synth.T_Q4_K, synth.T_Q8_0):
        L = synth.device_layer(E=2048, FF=768, NE=128, K=8, seed=31, gate_type=gt, router_scale=0.05)
        full = ctx.bind(L)
        sh = ep.shard_layer(L, rank, world)
        if gt == synth.T_Q8_0:   # the expert-parallel entry points take K-quant experts; Q8_0 must be refused
            try:
                ep.GpuCompute(ctx, full, ctx.bind(sh), L.E, L.K).route(torch.zeros((4, L.E), device="cuda"))
                ok = False
                print(f"rank {rank}: a Q8_0 layer was not refused", flush=True)
            except RuntimeError:
                pass
            continue
        comp = ep.GpuCompute(ctx, full, ctx.bind(sh), L.E, L.K)
        # (T >= 2: the single-GPU block the results are checked against takes its batched path, the same arithmetic as the
        # expert side; one token would take the one-token kernel's exact integer path)
        for T, via in ((256, None), (37, None), (256, xchg), (37, xchg), (2, xchg), (200, xchg), (256, xchg)):
            x0 = torch.from_numpy(synth.activations(T, L.E, seed=100 * rank + T)).cuda()
            x = x0.clone()
            sel, _ = ep.moe_layer(x, comp, L.NE // world, L.resid_scale, xchg=via)
            xb = x0.clone()
            selb = torch.zeros((T, L.K), dtype=torch.int32, device="cuda")
            ctx.moe_ffn_dev(full, xb, selb)
            ctx.status()
            err = float(torch.linalg.norm((x - xb).double()) / torch.linalg.norm((xb - x0).double()))
            worst = max(worst, err)
            if not torch.equal(sel, selb) or not err <= 1e-5:
                ok = False
                print(f"rank {rank} T={T} ({'peer' if via else 'nccl'}): top-k equal {torch.equal(sel, selb)}, relative L2 {err:.2e}",
                      flush=True)
    xchg.close()
    try:
        ctx.status()
    except Exception as e:   # a peer wait that ran out
        ok = False
        print(f"rank {rank}: {e}", flush=True)
    flag = torch.tensor([0 if ok else 1], device="cuda")
    dist.all_reduce(flag)
    if rank == 0:
        print(f"expert-parallel parity over {world} GPUs: {'ok' if flag.item() == 0 else 'FAILED'}, worst relative L2 {worst:.2e}", flush=True)
    dist.destroy_process_group()
    ctx.close()
    return int(flag.item() != 0)


if __name__ == "__main__":
    sys.exit(main())

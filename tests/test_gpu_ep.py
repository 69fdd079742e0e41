"""The expert-parallel halves (clb200_ep_route / clb200_ep_experts) on a B200, driven by clutor_b200.ep in one process.

Bar: with every expert on the one GPU the exchange is the identity and the result is the batched block's, bit for bit;
with the experts split into shards run one after another (as N GPUs would), the top-k is identical and x is within 1e-5
relative L2 of the block (only the order of the fp32 additions over a token's experts differs).
"""
import numpy as np
import pytest

from clutor_b200 import ep, synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    import clutor_b200 as cb
    c = cb.Context(0)
    yield c
    c.close()


def test_one_gpu_is_the_batched_block(ctx):
    import torch
    L = synth.device_layer(E=2048, FF=768, NE=128, K=8, seed=21, router_scale=0.05)
    full = ctx.bind(L)
    comp = ep.GpuCompute(ctx, full, full, L.E, L.K)
    x0 = torch.from_numpy(synth.activations(300, L.E, seed=3)).cuda()
    x = x0.clone()
    sel, wt = ep.moe_layer(x, comp, L.NE, L.resid_scale)
    xb = x0.clone()
    selb = torch.zeros((300, 8), dtype=torch.int32, device="cuda")
    ctx.moe_ffn_dev(full, xb, selb)
    ctx.status()
    assert torch.equal(sel, selb)
    assert torch.equal(x.view(torch.int32), xb.view(torch.int32))


@pytest.mark.parametrize("shards", [2, 4, 8])
def test_sharded_experts_match_the_block(ctx, shards):
    """The exchange of N ranks emulated in one process: every shard's expert side runs on the rows routed to it."""
    import torch
    L = synth.device_layer(E=2048, FF=768, NE=128, K=8, seed=22, router_scale=0.05)
    full = ctx.bind(L)
    parts = [ctx.bind(ep.shard_layer(L, r, shards)) for r in range(shards)]
    T = 200
    x0 = torch.from_numpy(synth.activations(T, L.E, seed=4)).cuda()
    comp = ep.GpuCompute(ctx, full, full, L.E, L.K)
    sel, wt, qs, d, bs = comp.route(x0.clone())
    idx, lsel = ep.dispatch_plan(sel, shards, L.NE // shards)
    msum = torch.zeros_like(x0)
    for r in range(shards):
        cr = ep.GpuCompute(ctx, full, parts[r], L.E, L.K)
        i = idx[r]
        msum[i] += cr.experts(qs[i].contiguous(), d[i].contiguous(), bs[i].contiguous(), lsel[r].contiguous(), wt[i].contiguous())
    x = x0 + L.resid_scale * msum
    xb = x0.clone()
    selb = torch.zeros((T, 8), dtype=torch.int32, device="cuda")
    ctx.moe_ffn_dev(full, xb, selb)
    ctx.status()
    assert torch.equal(sel, selb)
    dd, wd = (x - x0).double(), (xb - x0).double()
    err = float(torch.linalg.norm(dd - wd) / torch.linalg.norm(wd))
    assert err <= 1e-5, err


@pytest.mark.parametrize("n_ranks", [1, 2, 3, 8])
def test_device_exchange_equals_the_host_form(ctx, n_ranks):
    """clb200_ep_pack gives the torch form's rows byte for byte (destination order, tokens ascending) and clb200_ep_combine
    its bits; experts past the last rank (128 experts over 3 ranks of 42) go nowhere in both."""
    import torch
    T, E, K, NE = 300, 1024, 8, 128
    n_local = NE // n_ranks
    g = torch.Generator().manual_seed(n_ranks)
    sel = torch.stack([torch.randperm(NE, generator=g)[:K] for _ in range(T)]).to(torch.int32).cuda()
    wt = torch.rand((T, K), generator=g).cuda()
    qs = torch.randint(-127, 128, (T, E), dtype=torch.int8, generator=g).cuda()
    d = torch.rand((T, E // 256), generator=g).cuda()
    bs = torch.randint(-2000, 2000, (T, E // 16), dtype=torch.int16, generator=g).cuda()
    fmt = ep.RowFormat(E, K)
    host = ep.Compute()
    gpu = ep.GpuCompute(ctx, -1, -1, E, K)
    send_h, plan_h, counts_h = host.pack(fmt, sel, wt, qs, d, bs, n_ranks, n_local)
    send_d, plan_d, counts_d = gpu.pack(fmt, sel, wt, qs, d, bs, n_ranks, n_local)
    torch.cuda.synchronize()
    assert counts_d == counts_h
    assert torch.equal(send_d, send_h)
    S = sum(counts_h)
    back = torch.randn((S, E), generator=g).cuda()
    x0 = torch.randn((T, E), generator=g).cuda()
    xh, xd = x0.clone(), x0.clone()
    host.combine(xh, back, plan_h, counts_h, 0.75)
    gpu.combine(xd, back, plan_d, counts_d, 0.75)
    torch.cuda.synchronize()
    assert torch.equal(xd.view(torch.int32), xh.view(torch.int32))

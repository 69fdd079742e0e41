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


@pytest.mark.parametrize("n_ranks", [2, 3])
def test_peer_exchange_kernels_emulated(ctx, n_ranks):
    """The peer-memory exchange's kernels (clb200_ep_push / _wait / _push_back / _combine_regions) with N ranks emulated in
    one process on one GPU: every rank's exchange buffer is local here, and each wait runs after the pushes it waits for
    have finished (one stream), so no kernel waits on another that is still running. Two steps with different batches per
    rank reuse the regions and the step signals; each rank's x must match the single-GPU block on its tokens (top-k
    identical, 1e-5 relative L2)."""
    import ctypes as C

    import torch

    import clutor_b200 as cb
    L = synth.device_layer(E=2048, FF=768, NE=120, K=8, seed=23, router_scale=0.05)
    full = ctx.bind(L)
    n, n_local, t_max = n_ranks, L.NE // n_ranks, 256
    comps = [ep.GpuCompute(ctx, full, ctx.bind(ep.shard_layer(L, r, n)), L.E, L.K) for r in range(n)]
    lib = cb.lib()
    lib.clb200_ep_xbuf_layout.restype = None
    lib.clb200_ep_xbuf_layout.argtypes = [C.c_int] * 4 + [C.POINTER(C.c_size_t)] * 3
    lib.clb200_ep_xbuf_alloc.argtypes = [C.c_void_p] + [C.c_int] * 4 + [C.POINTER(C.c_void_p), C.c_char_p, C.c_char_p, C.c_size_t]
    lib.clb200_ep_xbuf_free.argtypes = [C.c_void_p, C.c_void_p, C.c_char_p, C.c_size_t]
    lib.clb200_ep_push.argtypes = [C.c_void_p] + [C.c_int] * 5 + [C.c_void_p] * 3 + [C.c_uint, C.c_void_p, C.c_char_p, C.c_size_t]
    lib.clb200_ep_push_back.argtypes = lib.clb200_ep_push.argtypes
    lib.clb200_ep_wait.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_uint, C.c_void_p, C.c_void_p, C.c_char_p, C.c_size_t]
    err = C.create_string_buffer(512)
    size, roff, boff = C.c_size_t(), C.c_size_t(), C.c_size_t()
    lib.clb200_ep_xbuf_layout(n, t_max, L.E, L.K, C.byref(size), C.byref(roff), C.byref(boff))
    fmt = ep.RowFormat(L.E, L.K)
    own, recv, back = [], [], []
    for r in range(n):
        p, h = C.c_void_p(), C.create_string_buffer(64)
        assert lib.clb200_ep_xbuf_alloc(ctx.handle, n, t_max, L.E, L.K, C.byref(p), h, err, 512) == 0, err.value.decode()
        own.append(p.value)
        whole = torch.as_tensor(ep._DeviceBytes(p.value, size.value), device="cuda")
        recv.append(whole[roff.value:roff.value + n * t_max * fmt.nbytes].view(n * t_max, fmt.nbytes))
        back.append(whole[boff.value:boff.value + n * t_max * L.E * 4].view(torch.float32).view(n * t_max, L.E))
    bufs = (C.c_void_p * n)(*own)
    st = C.c_void_p(cb._stream(None))
    try:
        for seq, Ts in ((1, (200, 37, 64)), (2, (5, 120, 256))):
            Ts = Ts[:n]
            x0 = [torch.from_numpy(synth.activations(T, L.E, seed=10 * seq + r)).cuda() for r, T in enumerate(Ts)]
            x = [v.clone() for v in x0]
            plans, sels = [], []
            for r in range(n):
                sel, wt, qs, d, bs = comps[r].route(x[r])
                sels.append(sel)
                plans.append(comps[r].pack_device(fmt, sel, wt, qs, d, bs, n, n_local))
            for r in range(n):
                send, _, counts = plans[r]
                assert lib.clb200_ep_push(ctx.handle, r, n, t_max, L.E, L.K, bufs, send.data_ptr(), counts.data_ptr(), seq, st,
                                          err, 512) == 0, err.value.decode()
            rcounts = [torch.zeros(n, dtype=torch.int32, device="cuda") for _ in range(n)]
            for r in range(n):
                assert lib.clb200_ep_wait(ctx.handle, own[r], n, 0, seq, rcounts[r].data_ptr(), st, err, 512) == 0
            partials = []
            for r in range(n):
                rows = fmt.unpack(recv[r])
                live = (torch.arange(t_max, device="cuda")[None, :] < rcounts[r][:, None].long()).reshape(-1, 1)
                partials.append(comps[r].experts(rows["qs"], rows["d"], rows["bs"], torch.where(live, rows["sel"], -1), rows["wt"]))
            for r in range(n):
                assert lib.clb200_ep_push_back(ctx.handle, r, n, t_max, L.E, L.K, bufs, partials[r].data_ptr(), rcounts[r].data_ptr(),
                                               seq, st, err, 512) == 0, err.value.decode()
            for r in range(n):
                assert lib.clb200_ep_wait(ctx.handle, own[r], n, 1, seq, None, st, err, 512) == 0
            for r in range(n):
                _, slot, counts = plans[r]
                comps[r].combine_regions(x[r], back[r], slot, counts, t_max, L.resid_scale)
            ctx.status()
            for r in range(n):
                # rows from sender q: its tokens with at least one expert on rank r
                want = torch.tensor([int(((sels[q] // n_local) == r).any(1).sum()) for q in range(n)], dtype=torch.int32)
                assert torch.equal(rcounts[r].cpu(), want), f"step {seq} rank {r}: rows received {rcounts[r].tolist()}"
                xb = x0[r].clone()
                selb = torch.zeros((Ts[r], L.K), dtype=torch.int32, device="cuda")
                ctx.moe_ffn_dev(full, xb, selb)
                ctx.status()
                assert torch.equal(sels[r], selb)
                e = float(torch.linalg.norm((x[r] - xb).double()) / torch.linalg.norm((xb - x0[r]).double()))
                assert e <= 1e-5, f"step {seq} rank {r}: relative L2 {e:.2e}"
    finally:
        torch.cuda.synchronize()
        for p in own:
            lib.clb200_ep_xbuf_free(ctx.handle, p, err, 512)

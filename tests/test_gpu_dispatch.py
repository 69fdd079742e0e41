"""Parity of the dispatch permutation and of the exact batched path with the reference engine (needs a B200).

The batched block's dispatch turns a batch's routing into per-expert work lists. The reference forms them inline in its
batched MoE block: todo[] holds the chosen experts in order of first appearance over the (token, rank) slots
(c/src/forward.c:1162-1163), and for each of them who[] / wgt[] hold the tokens that chose it, ascending, with their
routing weights (c/src/forward.c:1188-1189). clb200_moe_dispatch exposes the device's lists (dispatch_kernel); here they
are compared element for element, weights bit for bit, with the same loops of the reference harness
(oracle/ref_harness.c ref_dispatch, the code its batched block runs) on the same routing, and the routing itself is
compared with the reference's (top-k identical).

With clb200_set_exact(1) every batched expert product stays on the integer path; the MoE block's outputs must then equal
the reference engine's golden outputs bit for bit.
"""
import json

import numpy as np
import pytest

import oracle
from clutor_b200 import synth

pytestmark = pytest.mark.gpu

TOL_WT = 1e-6   # routing weights, relative (CUDA's exp against the C library's expf)


@pytest.fixture(scope="module")
def ctx():
    import clutor_b200 as cb
    c = cb.Context(0)
    yield c
    c.close()


def check_dispatch(ctx, sel_d, wt_d, n_expert):
    """The device's dispatch of (sel_d, wt_d) against the reference's lists of the same routing."""
    todo, offsets, pos_token, pos_wt = ctx.dispatch(sel_d, wt_d, n_expert)
    ctx.status()
    sel, wt = sel_d.cpu().numpy(), wt_d.cpu().numpy()
    want_todo, lists = oracle.ref_dispatch(sel, wt, n_expert)
    todo, off = todo.cpu().numpy(), offsets.cpu().numpy()
    pt, pw = pos_token.cpu().numpy(), pos_wt.cpu().numpy()
    n = int(todo[n_expert])
    assert n == len(want_todo), f"{n} experts dispatched, the reference has {len(want_todo)}"
    assert np.array_equal(todo[:n], want_todo), "todo order differs from the reference's order of first appearance"
    assert off[0] == 0 and np.all(np.diff(off) >= 0)
    assert off[n_expert] == sum(len(w) for w, _ in lists.values())
    for e in range(n_expert):
        who, wgt = pt[off[e]:off[e + 1]], pw[off[e]:off[e + 1]]
        if e not in lists:
            assert len(who) == 0, f"expert {e} has tokens on the device, none in the reference"
            continue
        assert np.array_equal(who, lists[e][0]), f"expert {e}: token list differs"
        assert np.array_equal(wgt.view(np.uint32), lists[e][1].view(np.uint32)), f"expert {e}: weights differ"
    return n


def routed(ctx, L, x0):
    """The device's routing of the tokens x0 through the whole block of a device layer: (sel, wt) device tensors."""
    import torch
    h = ctx.bind(L)
    T = x0.shape[0]
    x = torch.from_numpy(x0).cuda()
    sel = torch.zeros((T, L.K), dtype=torch.int32, device="cuda")
    wt = torch.zeros((T, L.K), dtype=torch.float32, device="cuda")
    ctx.moe_ffn_dev(h, x, sel, wt)
    ctx.status()
    ctx.release(h)
    return sel, wt


def check_routing(sel_d, wt_d, want_sel, want_wt):
    assert np.array_equal(sel_d.cpu().numpy(), want_sel), "top-k differs from the reference"
    assert np.allclose(wt_d.cpu().numpy(), want_wt, rtol=TOL_WT, atol=1e-9)


@pytest.mark.parametrize("T", [64, 512])
def test_dispatch_c2_shape(ctx, T):
    """The Qwen3-30B-A3B layer with Q8_0 experts (hidden 2048, 128 experts, top-8): T = 64 touches most experts, T = 512
    every one with long token lists."""
    L = synth.device_layer(gate_type=synth.T_Q8_0, seed=77 + T, router_scale=0.05)
    x0 = synth.activations(T, 2048, seed=3 + T)
    sel, wt = routed(ctx, L, x0)
    want_sel, want_wt = oracle.ref_route_batch(synth.to_host(L), x0)
    check_routing(sel, wt, want_sel, want_wt)
    n = check_dispatch(ctx, sel, wt, 128)
    print(f"T={T}: {n} experts dispatched, lists identical to the reference's")


def test_dispatch_c4_shape_2048_tokens(ctx):
    """The Qwen3-235B-A22B layer's routing (hidden 4096, 128 experts, top-8) of a 2048-token prefill, through the
    expert-parallel route kernel (the experts are never read, so they are left out), then the dispatch of all 2048 tokens."""
    import ctypes as C

    import torch

    import clutor_b200 as cb
    E, NE, K, T = 4096, 128, 8, 2048
    gen = torch.Generator(device="cuda")
    gen.manual_seed(2048)
    dummy = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    L = synth.DeviceLayer(E=E, FF=1536, NE=NE, K=K, gate_type=synth.T_Q4_K, up_type=synth.T_Q4_K, down_type=synth.T_Q4_K,
                          ffn_norm=(1.0 + 0.1 * torch.randn(E, device="cuda", generator=gen)).float(),
                          router=(0.02 * torch.randn(NE, E, device="cuda", generator=gen)).float(),
                          gate=dummy, up=dummy, down=dummy)
    h = ctx.bind(L)
    x0 = synth.activations(T, E, seed=41)
    x = torch.from_numpy(x0).cuda()
    sel = torch.empty((T, K), dtype=torch.int32, device="cuda")
    wt = torch.empty((T, K), dtype=torch.float32, device="cuda")
    qs = torch.empty((T, E), dtype=torch.int8, device="cuda")
    d = torch.empty((T, E // 256), dtype=torch.float32, device="cuda")
    bs = torch.empty((T, E // 16), dtype=torch.int16, device="cuda")
    lib = cb.lib()
    lib.clb200_ep_route.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int] + [C.c_void_p] * 6 + [C.c_char_p, C.c_size_t]
    err = C.create_string_buffer(512)
    assert lib.clb200_ep_route(ctx.handle, h, x.data_ptr(), T, sel.data_ptr(), wt.data_ptr(), qs.data_ptr(), d.data_ptr(),
                               bs.data_ptr(), C.c_void_p(cb._stream(None)), err, 512) == 0, err.value.decode()
    ctx.status()
    ctx.release(h)
    hl = synth.HostLayer(E=E, FF=1536, NE=NE, K=K, gate_type=synth.T_Q4_K, up_type=synth.T_Q4_K, down_type=synth.T_Q4_K,
                         ffn_norm=L.ffn_norm.cpu().numpy(), router=L.router.cpu().numpy(),
                         gate=dummy.cpu().numpy(), up=dummy.cpu().numpy(), down=dummy.cpu().numpy())
    want_sel, want_wt = oracle.ref_route_batch(hl, x0)
    check_routing(sel, wt, want_sel, want_wt)
    n = check_dispatch(ctx, sel, wt, NE)
    print(f"T={T}: {n} experts dispatched, lists identical to the reference's")


def ep_routed(ctx, E, NE, K, T, seed):
    """The routing of T tokens through the expert-parallel route entry point (clb200_ep_route, the batched block's first
    half; the experts are never read, so the layer carries placeholders): (sel, wt) device tensors, the layer's router and
    norm as host arrays, and the tokens."""
    import ctypes as C

    import torch

    import clutor_b200 as cb
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    dummy = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    L = synth.DeviceLayer(E=E, FF=1536, NE=NE, K=K, gate_type=synth.T_Q4_K, up_type=synth.T_Q4_K, down_type=synth.T_Q4_K,
                          ffn_norm=(1.0 + 0.1 * torch.randn(E, device="cuda", generator=gen)).float(),
                          router=(0.02 * torch.randn(NE, E, device="cuda", generator=gen)).float(),
                          gate=dummy, up=dummy, down=dummy)
    h = ctx.bind(L)
    x0 = synth.activations(T, E, seed=seed)
    x = torch.from_numpy(x0).cuda()
    sel = torch.empty((T, K), dtype=torch.int32, device="cuda")
    wt = torch.empty((T, K), dtype=torch.float32, device="cuda")
    qs = torch.empty((T, E), dtype=torch.int8, device="cuda")
    d = torch.empty((T, E // 256), dtype=torch.float32, device="cuda")
    bs = torch.empty((T, E // 16), dtype=torch.int16, device="cuda")
    lib = cb.lib()
    lib.clb200_ep_route.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int] + [C.c_void_p] * 6 + [C.c_char_p, C.c_size_t]
    err = C.create_string_buffer(512)
    assert lib.clb200_ep_route(ctx.handle, h, x.data_ptr(), T, sel.data_ptr(), wt.data_ptr(), qs.data_ptr(), d.data_ptr(),
                               bs.data_ptr(), C.c_void_p(cb._stream(None)), err, 512) == 0, err.value.decode()
    ctx.status()
    ctx.release(h)
    hl = synth.HostLayer(E=E, FF=1536, NE=NE, K=K, gate_type=synth.T_Q4_K, up_type=synth.T_Q4_K, down_type=synth.T_Q4_K,
                         ffn_norm=L.ffn_norm.cpu().numpy(), router=L.router.cpu().numpy(),
                         gate=dummy.cpu().numpy(), up=dummy.cpu().numpy(), down=dummy.cpu().numpy())
    return sel, wt, hl, x0


@pytest.mark.parametrize("T,E,NE,K", [(513, 2048, 128, 8), (600, 1280, 40, 6)])
def test_large_batch_router_chunks(ctx, T, E, NE, K):
    """Past 512 tokens (the expert-parallel route entry point takes any batch) the router takes 32 tokens a CTA and streams
    their rows through shared memory 512 elements at a time, each chain carrying across the chunks: T = 513 leaves one
    token in the last CTA; E = 1280 ends on a 256-element chunk; 40 experts leave a partial group of 32. The top-k equals
    the reference's, the weights within TOL_WT."""
    sel, wt, hl, x0 = ep_routed(ctx, E, NE, K, T, seed=T + E)
    want_sel, want_wt = oracle.ref_route_batch(hl, x0)
    check_routing(sel, wt, want_sel, want_wt)


@pytest.mark.parametrize("T,NE,K", [(300, 128, 8), (2048, 128, 8), (33, 16, 4)])
def test_dispatch_one_expert_takes_every_token(ctx, T, NE, K):
    """Expert 7 is in every token's choice (at a rank that moves with the token), the rest of each row is a seeded draw of
    distinct experts: expert 7's list is every token, and the order of first appearance starts from token 0's row."""
    import torch
    rng = np.random.default_rng(T)
    sel = np.zeros((T, K), np.int32)
    for t in range(T):
        others = rng.choice(np.setdiff1d(np.arange(NE), [7]), K - 1, replace=False)
        sel[t] = np.insert(others, t % K, 7)
    wt = rng.random((T, K), dtype=np.float32)
    n = check_dispatch(ctx, torch.from_numpy(sel).cuda(), torch.from_numpy(wt).cuda(), NE)
    assert n <= NE


def test_dispatch_one_token_and_every_expert(ctx):
    """One token (a list of one per chosen expert), and a batch in which every expert is chosen exactly once."""
    import torch
    sel = np.array([[5, 2, 9, 0]], np.int32)
    wt = np.array([[0.4, 0.3, 0.2, 0.1]], np.float32)
    check_dispatch(ctx, torch.from_numpy(sel).cuda(), torch.from_numpy(wt).cuda(), 16)
    sel = np.random.default_rng(1).permutation(32).astype(np.int32).reshape(8, 4)
    wt = np.full((8, 4), 0.25, np.float32)
    assert check_dispatch(ctx, torch.from_numpy(sel).cuda(), torch.from_numpy(wt).cuda(), 32) == 32


@pytest.mark.parametrize("name", ["small_q4k_t5", "c1_q4k_t17", "c2_q8_0_t64", "small_q6k_down_t3", "small_q8_0_t4",
                                  "small_no_renorm_t2", "ties_t2"])
def test_exact_path_equals_reference_bits(ctx, golden, name):
    """clb200_set_exact(1): the batched fixtures the reference engine produced (T = 2 to 64; Q4_K, Q6_K down, Q8_0; ties; no
    renormalisation) come out bit for bit: routing, weights and every output value."""
    from tests.golden.make_golden import make_layer
    p = json.loads(bytes(golden[f"{name}.params"]).decode())
    L = make_layer(p["layer"], p["special"])
    x = golden[f"{name}.x"]
    ctx.set_exact(True)
    try:
        xo, sel, wt = ctx.moe_ffn(L, x)
    finally:
        ctx.set_exact(False)
    assert np.array_equal(sel, golden[f"{name}.sel"])
    assert np.array_equal(wt.view(np.uint32), golden[f"{name}.wt"].view(np.uint32)), "routing weights differ in bits"
    diff = int(np.count_nonzero(xo.view(np.uint32) != golden[f"{name}.x_out"].view(np.uint32)))
    assert diff == 0, f"{name}: {diff} of {xo.size} output values differ from the reference's bits"

"""Parity of the CUDA MoE block with the oracle and the reference engine's golden outputs (needs a B200).

Bar: router top-k indices bit-exact; routing weights within 1e-6 relative (the softmax's exp is CUDA's, not glibc's);
outputs within 1e-3 relative L2 of the reference's (the bar this library states), and in practice far closer: the gate/up
and down dot products are bit-exact, only the SwiGLU exp can differ by an ulp.
"""
import json

import numpy as np
import pytest

import oracle
from clutor_b200 import synth

pytestmark = pytest.mark.gpu

TOL_REL_L2 = 1e-3     # the stated output tolerance
TOL_WT = 1e-6         # routing weights, relative


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def ctx():
    import clutor_b200 as cb
    c = cb.Context(0)
    yield c
    c.close()


def check(x_in, got, want, name=""):
    xo, sel, wt = got
    wxo, wsel, wwt = want
    assert np.array_equal(sel, wsel), f"{name}: top-k differs\n{sel}\n{wsel}"
    assert np.allclose(wt, wwt, rtol=TOL_WT, atol=1e-9), f"{name}: weights differ"
    # compare the MoE update (x_out - x_in): a tighter test than x_out itself
    d, wd = xo.astype(np.float64) - x_in, wxo.astype(np.float64) - x_in
    e = rel_l2(d, wd) if np.linalg.norm(wd) > 0 else float(np.abs(d).max())
    assert e <= TOL_REL_L2, f"{name}: relative L2 of the update {e:.3e}"
    return e


def test_golden_fixtures(ctx, golden):
    """Every fixture the reference engine produced (one token and batches; Q4_K, Q6_K down, Q8_0; ties; zeros)."""
    from tests.golden.make_golden import make_layer
    worst = 0.0
    for name in sorted({k.split(".")[0] for k in golden.files}):
        p = json.loads(bytes(golden[f"{name}.params"]).decode())
        L = make_layer(p["layer"], p["special"])
        x = golden[f"{name}.x"]
        got = ctx.moe_ffn(L, x)
        want = (golden[f"{name}.x_out"], golden[f"{name}.sel"], golden[f"{name}.wt"])
        worst = max(worst, check(x, got, want, name))
    print(f"worst relative L2 of the update over the fixtures: {worst:.3e}")


@pytest.mark.parametrize("gt,dt", [(synth.T_Q4_K, synth.T_Q4_K), (synth.T_Q4_K, synth.T_Q6_K), (synth.T_Q8_0, synth.T_Q8_0),
                                   (synth.T_Q6_K, synth.T_Q4_K)])
def test_decode_full_size_chain(ctx, gt, dt):
    """Qwen3-30B-A3B layer shape, one token through 4 layers (device layers, device entry point). Each layer is checked
    from the oracle's own input to it (top-k exact, weights 1e-6, update 1e-3), and the chain run on the GPU end to end is
    checked against the oracle's chain (top-k exact, final update 1e-3; Q8_0 layers take the tensor-core path, accurate to
    ~1e-7 rather than bit-exact, so chained inputs drift by that much)."""
    import torch
    layers = [synth.device_layer(gate_type=gt, down_type=dt, seed=100 + i) for i in range(4)]
    handles = [ctx.bind(L) for L in layers]
    host = [synth.to_host(L) for L in layers]
    x0 = synth.activations(1, 2048, seed=5)
    xr = x0.copy()
    worst = 0.0
    for i, h in enumerate(handles):           # layer by layer, from the oracle's input
        x = torch.from_numpy(xr).cuda()
        sel = torch.zeros((1, 8), dtype=torch.int32, device="cuda")
        wt = torch.zeros((1, 8), dtype=torch.float32, device="cuda")
        ctx.moe_ffn_dev(h, x, sel, wt)
        ctx.status()
        want = oracle.moe_ffn(host[i], xr, "oracle")
        worst = max(worst, check(xr, (x.cpu().numpy(), sel.cpu().numpy(), wt.cpu().numpy()), want, f"layer {i}"))
        xr = want[0]
    x = torch.from_numpy(x0).cuda()           # the chain on the GPU alone
    sel = torch.zeros((4, 8), dtype=torch.int32, device="cuda")
    for i, h in enumerate(handles):
        ctx.moe_ffn_dev(h, x, sel[i])
    ctx.status()
    xc = x0.copy()
    for i in range(4):
        xc, s, _ = oracle.moe_ffn(host[i], xc, "oracle")
        assert np.array_equal(sel[i].cpu().numpy(), s[0]), f"chained layer {i} top-k"
    e = rel_l2(x.cpu().numpy() - x0, xc - x0)
    assert e <= TOL_REL_L2
    print(f"{gt}/{dt}: worst per-layer relative L2 {worst:.3e}, chain of 4 {e:.3e}")


@pytest.mark.parametrize("T", [1, 3])
def test_zero_activations(ctx, T):
    """x = 0: every router logit is 0, so all experts tie and the lowest ids win; every Q8_K block has amax 0 (scale 0,
    quants 0), and the update is exactly 0, as in the reference."""
    L = synth.host_layer(E=1024, FF=512, NE=64, K=6, seed=5)
    x = np.zeros((T, 1024), np.float32)
    got, want = ctx.moe_ffn(L, x), oracle.moe_ffn(L, x, "oracle")
    check(x, got, want, f"zero x, T={T}")
    assert np.array_equal(got[1], np.tile(np.arange(6, dtype=got[1].dtype), (T, 1)))
    assert not np.any(got[0])


@pytest.mark.parametrize("T", [1, 5])
def test_tied_router_rows(ctx, T):
    """Experts 9 and 3 (and 40 and 12) have identical router rows, scaled up so they lead: their logits and probabilities
    tie exactly, and the lower id must come first (the reference's repeated arg-max)."""
    L = synth.host_layer(E=1024, FF=512, NE=64, K=6, seed=8)
    L.router[3] = L.router[9] = 4.0 * L.router[0]
    L.router[12] = L.router[40] = 3.0 * L.router[1]
    x = synth.activations(T, 1024, seed=77)
    got, want = ctx.moe_ffn(L, x), oracle.moe_ffn(L, x, "oracle")
    check(x, got, want, f"tied rows, T={T}")


@pytest.mark.parametrize("T", [1, 3])
def test_smallest_shapes_every_expert_no_renorm(ctx, T):
    """The smallest widths (one 256-block per row, one or two rows per CTA), every expert chosen (K = NE = 8), no
    renormalisation of the weights and a residual scale of 0.5."""
    L = synth.host_layer(E=256, FF=256, NE=8, K=8, seed=31, norm_topk=0, resid_scale=0.5)
    x = synth.activations(T, 256, seed=32)
    check(x, ctx.moe_ffn(L, x), oracle.moe_ffn(L, x, "oracle"), f"smallest, T={T}")


def test_repeated_calls_reset_their_counters(ctx):
    """The one-token kernel's cross-CTA counters are reset by its last CTA: many calls in a row stay correct."""
    L = synth.host_layer(E=1024, FF=512, NE=64, K=6, seed=9)
    for i in range(6):
        x = synth.activations(1, 1024, seed=40 + i)
        check(x, ctx.moe_ffn(L, x), oracle.moe_ffn(L, x, "oracle"), f"call {i}")


@pytest.mark.parametrize("T", [2, 7, 64, 130])
def test_batched_against_oracle(ctx, T):
    L = synth.host_layer(E=1024, FF=768, NE=32, K=4, seed=T, gate_type=synth.T_Q4_K, down_type=synth.T_Q6_K)
    x = synth.activations(T, 1024, seed=T + 1)
    check(x, ctx.moe_ffn(L, x), oracle.moe_ffn(L, x, "oracle"), f"T={T}")


def test_batched_q8_0_t64_full_size(ctx, golden):
    """The T=64 Q8_0 configuration (float path) at full size is among the fixtures; here the device entry point and the
    host entry point agree bit for bit on it."""
    import torch
    L = synth.device_layer(gate_type=synth.T_Q8_0, seed=77, router_scale=0.05)
    h = ctx.bind(L)
    x0 = synth.activations(64, 2048, seed=3)
    x = torch.from_numpy(x0).cuda()
    ctx.moe_ffn_dev(h, x)
    ctx.status()
    HL = synth.to_host(L)
    got = ctx.moe_ffn(HL, x0)
    assert np.array_equal(x.cpu().numpy().view(np.uint32), got[0].view(np.uint32))
    want = oracle.moe_ffn(HL, x0, "oracle")
    check(x0, got, want, "q8_0 T=64")


def test_bad_arguments_are_errors(ctx):
    import clutor_b200 as cb
    L = synth.host_layer(E=512, FF=256, NE=16, K=4, seed=2)
    with pytest.raises(cb.ClutorError, match="tokens"):
        ctx.moe_ffn(L, np.zeros((0, 512), np.float32))
    bad = synth.host_layer(E=512, FF=256, NE=16, K=4, seed=2)
    bad.K = 40
    with pytest.raises(cb.ClutorError, match="expert counts"):
        ctx.moe_ffn(bad, np.zeros((1, 512), np.float32))


@pytest.mark.parametrize("T,dt", [(130, synth.T_Q4_K), (512, synth.T_Q4_K), (300, synth.T_Q6_K)])
def test_batched_k_quant_tensor_core(ctx, T, dt):
    """Q4_K gate/up (and Q4_K down) as tensor-core grouped GEMMs of the dequantized weights and the value of the Q8_K
    activations, up to 128 tokens an expert (tiles of 64): top-k exact, update within 1e-3 of the oracle's integer dots."""
    L = synth.host_layer(E=1024, FF=768, NE=16, K=4, seed=T + 7, gate_type=synth.T_Q4_K, down_type=dt, router_scale=0.05)
    x = synth.activations(T, 1024, seed=T + 8)
    e = check(x, ctx.moe_ffn(L, x), oracle.moe_ffn(L, x, "oracle"), f"T={T}")
    print(f"T={T} down {dt}: relative L2 of the update {e:.2e}")

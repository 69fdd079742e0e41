"""The expert-group one-token kernel (group.cu) against the grid-wide one (decode.cu) and the oracle (needs a B200).

Both kernels compute the reference's arithmetic in the reference's order, so their results must agree bit for bit: routing,
weights and every output value. The expert-group kernel also ranks experts by logit to issue its copies before the softmax
is done, as the grid-wide kernel does too; the test hook CLB200_OPT_TEST_SPECULATION_MISS makes that first choice wrong at
rank K - 1 on every call, so the correction path (wait for the wrong copies, fetch the right expert) runs, and the results
must still be the same bits.
"""
import numpy as np
import pytest

import oracle
from clutor_b200 import synth

pytestmark = pytest.mark.gpu

TOL_REL_L2 = 1e-3


@pytest.fixture(scope="module")
def ctx():
    import clutor_b200 as cb
    c = cb.Context(0)
    yield c
    c.close()


def run(ctx, L, x, kernel, miss=0):
    ctx.set_option(ctx.OPT_DECODE_KERNEL, kernel)
    ctx.set_option(ctx.OPT_TEST_SPECULATION_MISS, miss)
    try:
        return ctx.moe_ffn(L, x)
    finally:
        ctx.set_option(ctx.OPT_DECODE_KERNEL, 0)
        ctx.set_option(ctx.OPT_TEST_SPECULATION_MISS, 0)


def same_bits(a, b, what):
    for u, v, name in zip(a, b, ("x", "sel", "wt")):
        assert np.array_equal(np.asarray(u).view(np.uint32), np.asarray(v).view(np.uint32)), f"{what}: {name} differs"


SHAPES = [
    # E, FF, NE, K, gate, down: the Qwen3-30B-A3B layer in both K-quant mixes, the smallest widths, more experts than SMs
    # (two logits per CTA), every expert used, one expert, sixteen experts, the widest rows
    (2048, 768, 128, 8, synth.T_Q4_K, synth.T_Q4_K),
    (2048, 768, 128, 8, synth.T_Q4_K, synth.T_Q6_K),
    (2048, 768, 128, 8, synth.T_Q6_K, synth.T_Q4_K),
    (256, 256, 8, 8, synth.T_Q4_K, synth.T_Q6_K),
    (768, 512, 256, 4, synth.T_Q6_K, synth.T_Q6_K),
    (1024, 512, 64, 1, synth.T_Q4_K, synth.T_Q4_K),
    (512, 1024, 32, 16, synth.T_Q4_K, synth.T_Q4_K),
    (4096, 256, 16, 2, synth.T_Q4_K, synth.T_Q6_K),
]


@pytest.mark.parametrize("E,FF,NE,K,gt,dt", SHAPES)
def test_group_kernel_equals_grid_kernel(ctx, E, FF, NE, K, gt, dt):
    L = synth.host_layer(E=E, FF=FF, NE=NE, K=K, gate_type=gt, down_type=dt, seed=E + FF + NE + K)
    for s in range(2):
        x = synth.activations(1, E, seed=900 + s)
        got = run(ctx, L, x, 0)
        want = run(ctx, L, x, 1)
        same_bits(got, want, f"E={E} FF={FF} NE={NE} K={K}")
        rx, rsel, _ = oracle.moe_ffn(L, x, "oracle")
        assert np.array_equal(got[1], rsel)
        d, rd = got[0].astype(np.float64) - x, rx.astype(np.float64) - x
        assert np.linalg.norm(d - rd) <= TOL_REL_L2 * max(np.linalg.norm(rd), 1e-30)


@pytest.mark.parametrize("kernel", [0, 1])
@pytest.mark.parametrize("E,FF,NE,K,gt,dt", [SHAPES[0], SHAPES[1], SHAPES[4], SHAPES[5], SHAPES[6]])
def test_speculation_correction_path(ctx, kernel, E, FF, NE, K, gt, dt):
    """The copies of rank K - 1 first go out for the expert ranked K + 1; the group (kernel 0) or the slot (kernel 1, the
    grid-wide kernel) that holds it must fetch the right expert and the result must not change by a bit."""
    L = synth.host_layer(E=E, FF=FF, NE=NE, K=K, gate_type=gt, down_type=dt, seed=7 * E + K)
    for s in range(3):
        x = synth.activations(1, E, seed=300 + s)
        same_bits(run(ctx, L, x, kernel, miss=1), run(ctx, L, x, kernel), f"correction kernel {kernel} E={E} K={K}")
        if kernel == 1:
            _, rsel, _ = oracle.moe_ffn(L, x, "oracle")
            assert np.array_equal(run(ctx, L, x, 1, miss=1)[1], rsel)


def test_many_calls_and_shared_scratch(ctx):
    """Launch tags advance over many calls; batched calls on the same context (which reuse its scratch) in between leave
    nothing the one-token kernel could mistake for its own words."""
    L = synth.host_layer(E=1024, FF=512, NE=64, K=6, seed=12)
    for i in range(40):
        x = synth.activations(1, 1024, seed=2000 + i)
        if i % 7 == 3:
            xb = synth.activations(5, 1024, seed=i)
            got_b, want_b = ctx.moe_ffn(L, xb), oracle.moe_ffn(L, xb, "oracle")
            assert np.array_equal(got_b[1], want_b[1])
        got, want = ctx.moe_ffn(L, x), oracle.moe_ffn(L, x, "oracle")
        assert np.array_equal(got[1], want[1]), f"call {i}"
        assert np.array_equal(got[0].view(np.uint32), want[0].view(np.uint32)), f"call {i}: output differs from the oracle"


def test_chain_in_a_graph_matches_eager(ctx):
    """Twelve full-size layers chained and replayed from a CUDA graph (programmatic dependent launches back to back) give
    the eager chain's bits on every replay."""
    import torch
    layers = [synth.device_layer(seed=500 + i) for i in range(12)]
    handles = [ctx.bind(L) for L in layers]
    x0 = torch.from_numpy(synth.activations(1, 2048, seed=8)).cuda()
    x = x0.clone()
    sel = torch.zeros((12, 1, 8), dtype=torch.int32, device="cuda")
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for i, h in enumerate(handles):
            ctx.moe_ffn_dev(h, x, sel[i], stream=stream)
    torch.cuda.synchronize()
    ctx.status()
    want_x, want_sel = x.clone(), sel.clone()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i, h in enumerate(handles):
            ctx.moe_ffn_dev(h, x, sel[i], stream=stream)
    for _ in range(5):
        x.copy_(x0)
        sel.zero_()
        g.replay()
        torch.cuda.synchronize()
        ctx.status()
        assert torch.equal(sel, want_sel)
        assert torch.equal(x.view(torch.int32), want_x.view(torch.int32))
    del g

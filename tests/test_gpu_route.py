"""SMART-ROUTE on a B200: clb200_route / clb200_route_dev against the oracle's restatement of cl_route (pinned to the
reference's own in tests/test_route_cpu.py), and the store's decode step with SMART-ROUTE on against the oracle given the
store's resident set.

Bar: the chosen experts identical (order included); the substitution count identical; the probability moved and the
largest move within 1e-12 (double arithmetic; CUDA's double exp is within an ulp of the C library's); in the store's step,
the weights are each chosen expert's own float router probability, renormalised, bit for bit.
"""
import numpy as np
import pytest

import oracle
from clutor_b200 import synth
from tests.test_route_cpu import random_case

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    import clutor_b200 as cb
    c = cb.Context(0)
    yield c
    c.close()


def same(got, want):
    assert got["selected"] == want["selected"]
    assert got["substituted"] == want["substituted"]
    assert abs(got["dropped_mass"] - want["dropped_mass"]) <= 1e-12
    assert abs(got["max_delta"] - want["max_delta"]) <= 1e-12


def test_known_answers(ctx):
    lg = np.array([-0.12 * i for i in range(64)], np.float32)
    res = np.zeros(64, np.uint8)
    res[8:14] = 1
    for smart in [(2, 12, 0.015), (2, 12, 1e9), (2, 12, 0.0), (2, 8, 1e9), (0, 64, 1e9), (8, 64, 1e9)]:
        same(ctx.route(lg, 8, smart, res), oracle.smart_route(lg, 8, smart, res))
    same(ctx.route(lg, 8), oracle.smart_route(lg, 8, None, None))
    assert ctx.route(lg[:8], 9) is None and ctx.route(lg, 0) is None and ctx.route(lg, 33) is None


@pytest.mark.parametrize("E,K", [(8, 8), (64, 8), (128, 8), (128, 32), (1024, 32), (300, 7)])
def test_route_random(ctx, E, K):
    rng = np.random.default_rng(7 * E + K)
    for i in range(40 if E == 1024 else 120):
        lg, smart, res = random_case(rng, E, K)
        same(ctx.route(lg, K, smart, res), oracle.smart_route(lg, K, smart, res))
        same(ctx.route(lg, K), oracle.smart_route(lg, K, None, None))


def test_route_dev_batch(ctx):
    """T tokens on device pointers, one residency set per token (stride E)."""
    import torch
    T, E, K = 96, 128, 8
    rng = np.random.default_rng(3)
    cases = [random_case(rng, E, K) for _ in range(T)]
    smart = (2, 24, 0.02)
    lg = torch.from_numpy(np.stack([c[0] for c in cases])).cuda()
    res = torch.from_numpy(np.stack([c[2] for c in cases])).cuda()
    out = torch.zeros(T * 152, dtype=torch.uint8, device="cuda")
    assert ctx.route_dev(lg, K, smart, res, out, resident_stride=E) == 0
    torch.cuda.synchronize()
    import clutor_b200 as cb
    raw = out.cpu().numpy().tobytes()
    for t in range(T):
        r = cb.RouteResult.from_buffer_copy(raw[152 * t:152 * (t + 1)])
        same(r.as_dict(), oracle.smart_route(cases[t][0], K, smart, cases[t][2]))
    assert ctx.route_dev(lg, 33, smart, res, out) == -1


NL, E_, FF, NE, K_ = 3, 1024, 512, 32, 4


def test_store_decode_with_smart_route(ctx):
    """The store's decode step routes on the device against its resident set: the choice is the oracle's cl_route on the
    layer's logits (computed by the oracle from the same x), each chosen expert weighted by its own float probability and
    renormalised; the counters add up as the reference's do."""
    import torch

    import clutor_b200 as cb
    layers = [synth.host_layer(E=E_, FF=FF, NE=NE, K=K_, seed=500 + i, gate_type=synth.T_Q4_K, down_type=synth.T_Q6_K,
                               router_scale=0.02) for i in range(NL)]
    st = cb.Store(ctx, layers[0], NL, cache_bytes=8 * (layers[0].expert_bytes + 256), stage_slots=0, policy=cb.WTINYLFU)
    for i, L in enumerate(layers):
        st.load_layer(i, L)
    st.set_prefetch(False)   # no fill lands between the residency the test reads and the one the step reads
    smart = (1, 12, 0.05)
    st.set_smart(smart)
    rng = np.random.default_rng(11)
    subs = 0
    dropped = 0.0
    maxd = 0.0
    for t in range(16):
        x = torch.from_numpy(synth.activations(1, E_, seed=int(rng.integers(1 << 30)))).cuda()[0]
        for l in range(NL):
            torch.cuda.synchronize()
            res = np.array([st.resident(l, e) for e in range(NE)], np.uint8)
            logits, probs = oracle.router_probs(layers[l], x.cpu().numpy())
            want = oracle.smart_route(logits, K_, smart, res)
            sel, wt = st.moe_ffn(l, x)
            assert list(sel) == want["selected"], f"token {t} layer {l}"
            w = probs[np.array(want["selected"])].astype(np.float32)
            z = np.float32(0)
            for v in w:
                z = np.float32(z + v)
            w = (w / z).astype(np.float32) if layers[l].norm_topk and z > 0 else w
            assert np.array_equal(wt.view(np.uint32), w.view(np.uint32)), f"token {t} layer {l}: weights"
            subs += want["substituted"]
            dropped += want["dropped_mass"]
            maxd = max(maxd, want["max_delta"])
        ctx.status()
    s = st.smart_stats()
    assert s["expert_slots"] == 16 * NL * K_
    assert s["substituted"] == subs and subs > 0
    assert abs(s["dropped_mass"] - dropped) <= 1e-9 and abs(s["max_delta"] - maxd) <= 1e-12
    # the harness-driven form: host logits, the store's residency
    lg = np.random.default_rng(5).standard_normal(NE).astype(np.float32)
    res = np.array([st.resident(0, e) for e in range(NE)], np.uint8)
    same(st.route(0, lg), oracle.smart_route(lg, K_, smart, res))
    with pytest.raises(cb.ClutorError, match="tau"):
        st.set_smart((1, 12, -1.0))
    before = st.smart_stats()["substituted"]
    st.set_smart(None)   # plain routing again: the float top-k of the reference's default path (forward.c:970-976)
    _, probs = oracle.router_probs(layers[0], x.cpu().numpy())
    sel, _ = st.moe_ffn(0, x)
    assert list(sel) == sorted(range(NE), key=lambda e: (-probs[e], e))[:K_]
    assert st.smart_stats()["substituted"] == before
    st.close()

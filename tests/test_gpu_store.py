"""The HBM expert store (clb200_store_*) on a B200.

Bar: a decode through the store gives the same bits as the block with every expert resident (the same kernel arithmetic;
only where the weights sit differs), top-k included; the store drives the cache policy exactly as the reference's
c/src/cache.c would (its recorded operations, replayed on the reference, give the same answers); its counters agree.
"""
import numpy as np
import pytest

import oracle
from clutor_b200 import synth

pytestmark = pytest.mark.gpu

NL, E, FF, NE, K = 4, 1024, 512, 32, 4


@pytest.fixture(scope="module")
def ctx():
    import clutor_b200 as cb
    c = cb.Context(0)
    yield c
    c.close()


@pytest.fixture(scope="module")
def layers():
    return [synth.host_layer(E=E, FF=FF, NE=NE, K=K, seed=300 + i, gate_type=synth.T_Q4_K, down_type=synth.T_Q6_K) for i in range(NL)]


def _store(ctx, layers, slots, stage, policy=1):
    import clutor_b200 as cb
    st = cb.Store(ctx, layers[0], NL, cache_bytes=slots * (layers[0].expert_bytes + 256), stage_slots=stage, policy=policy)
    for i, L in enumerate(layers):
        st.load_layer(i, L)
    return st


def _replay(log, cache_slots, stage_slots, universe, policy):
    """Replays the store's recorded cache operations on the reference's own policy; returns the mismatches."""
    ref = oracle.RefCache(cache_slots, stage_slots, universe, policy)
    bad = []
    for op, a, r in log:
        if op == 1:
            code, slot = ref.access(int(a))
            got = code * 65536 + slot if code >= 0 else -1
        elif op == 2:
            got = ref.stage(int(a))
        else:
            ref.unpin(int(a))
            got = 0
        if got != r:
            bad.append((int(op), int(a), int(r), got))
    ref.close()
    return bad


@pytest.mark.parametrize("slots,stage,policy", [(10, 8, 1), (4, 0, 0), (6, 4, 2)])
def test_stored_decode_is_bit_identical(ctx, layers, slots, stage, policy):
    import torch
    st = _store(ctx, layers, slots, stage, policy)
    st.log(True)
    rng = np.random.default_rng(slots)
    for t in range(12):
        x0 = synth.activations(1, E, seed=int(rng.integers(1 << 30)))
        want = x0.copy()
        xs = torch.from_numpy(x0.copy()).cuda()
        for l in range(NL):
            want, wsel, wwt = ctx.moe_ffn(layers[l], want)
            sel, wt = st.moe_ffn(l, xs[0])
            assert np.array_equal(sel, wsel[0]), f"token {t} layer {l}: top-k"
            assert np.array_equal(wt.view(np.uint32), wwt[0].view(np.uint32)), f"token {t} layer {l}: weights"
        ctx.status()
        got = xs.cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"token {t}: x differs"
    s = st.stats()
    assert s["accesses"] == 12 * NL * K
    assert s["hits"] + s["misses"] == s["accesses"]
    assert s["demand_bytes"] == s["misses"] * layers[0].expert_bytes
    assert s["misses"] > 0
    if slots >= 2 * K:
        assert s["hits"] > 0
    bad = _replay(st.read_log(), st.cache_slots() - stage - 1, stage, NL * NE, policy)
    assert not bad, bad[:5]
    st.close()


def test_given_routing_through_the_store(ctx, layers):
    """clb200_moe_experts_stored with the routing the block chose equals the block (resident weights)."""
    import torch
    st = _store(ctx, layers, 5, 4)
    x0 = synth.activations(1, E, seed=9)
    want, wsel, wwt = ctx.moe_ffn(layers[0], x0.copy())
    xs = torch.from_numpy(x0.copy()).cuda()
    st.experts(0, xs[0], wsel[0], wwt[0], next_pred=wsel[0])
    ctx.status()
    assert np.array_equal(xs.cpu().numpy().view(np.uint32), want.view(np.uint32))
    assert st.stats()["prefetch_issued"] == K
    st.close()


@pytest.mark.parametrize("mode,pn", [(0, 0), (1, 0), (2, 0), (2, 2)])
def test_prefetch_modes_stage_what_the_reference_stages(ctx, layers, mode, pn):
    """The forward pass's prefetch modes through clb200_moe_ffn_stored (c/src/forward.c:888-894, :937-946, :978-983).

    The staged keys, in order, are what the reference's forward pass would stage: layer 0 and (prev) layer l + 1 from the
    previous token's choice; (ahead) layer l + 1's top prefetch_n by its router on the x entering layer l, by the oracle.
    Layer 2's router rows are all equal, so its logits tie everywhere and router-ahead must pick the lowest ids. x stays
    the resident block's bits; the prediction counters match; the cache operations replay on the reference's cache.c."""
    import dataclasses

    import torch
    lay = list(layers)
    r = np.ascontiguousarray(lay[2].router, np.float32).reshape(NE, E).copy()
    r[:] = r[0]
    lay[2] = dataclasses.replace(lay[2], router=r.reshape(lay[2].router.shape))
    st = _store(ctx, lay, 10, 8)
    st.set_prefetch(mode, pn)
    st.log(True)
    n_pred = pn if 0 < pn < K else K
    prev = -np.ones((NL, K), np.int64)
    want_keys, pred_total, pred_hit = [], 0, 0
    rng = np.random.default_rng(40 + mode + pn)
    for t in range(10):
        x0 = synth.activations(1, E, seed=int(rng.integers(1 << 30)))
        want = x0.copy()
        xs = torch.from_numpy(x0.copy()).cuda()
        pred = -np.ones((NL, K), np.int64)
        if mode:
            pred[0, :n_pred] = prev[0, :n_pred]
            want_keys += [e for e in prev[0, :n_pred] if e >= 0]
        for l in range(NL):
            if mode == 1 and l + 1 < NL:
                pred[l + 1, :n_pred] = prev[l + 1, :n_pred]
                want_keys += [(l + 1) * NE + e for e in prev[l + 1, :n_pred] if e >= 0]
            if mode == 2 and l + 1 < NL:
                picks = oracle.router_ahead(lay[l + 1], want[0], n_pred)
                if l + 1 == 2:
                    assert picks.tolist() == list(range(n_pred))
                pred[l + 1, :n_pred] = picks
                want_keys += [(l + 1) * NE + int(e) for e in picks]
            want, wsel, wwt = ctx.moe_ffn(lay[l], want)
            sel, wt = st.moe_ffn(l, xs[0])
            assert np.array_equal(sel, wsel[0]), f"token {t} layer {l}: top-k"
            assert np.array_equal(wt.view(np.uint32), wwt[0].view(np.uint32))
            for e in pred[l, :n_pred]:
                if e >= 0:
                    pred_total += 1
                    pred_hit += int(e in sel)
            prev[l] = sel
        ctx.status()
        assert np.array_equal(xs.cpu().numpy().view(np.uint32), want.view(np.uint32)), f"token {t}: x differs"
    log = st.read_log()
    got_keys = [int(k) for op, k, _ in log if op == 2]
    assert got_keys == want_keys
    s = st.stats()
    assert (s["pred_total"], s["pred_hit"]) == (pred_total, pred_hit)
    assert s["prefetch_issued"] <= len(want_keys)
    if mode == 2:
        assert pred_hit > 0
    bad = _replay(log, st.cache_slots() - 8 - 1, 8, NL * NE, 1)
    assert not bad, bad[:5]
    st.close()


def test_demand_fills_go_before_waiting_prefetches(ctx, layers):
    """With a prefetch depth of 1, staged fills beyond the first wait on the host; a demand for one of them sends it at
    once (it is counted late), and the experts still give the resident block's bits."""
    import torch
    st = _store(ctx, layers, 10, 8)
    st.set_prefetch(0, depth=1)
    x0 = synth.activations(1, E, seed=77)
    want, wsel, wwt = ctx.moe_ffn(layers[1], x0.copy())
    for e in wsel[0]:
        st.prefetch(1, int(e))   # one goes on the copy stream, K - 1 wait on the host
    xs = torch.from_numpy(x0.copy()).cuda()
    st.experts(1, xs[0], wsel[0], wwt[0])
    ctx.status()
    s = st.stats()
    assert s["prefetch_issued"] == K and s["stage_hits"] == K and s["misses"] == 0
    assert s["prefetch_late"] >= 1
    assert np.array_equal(xs.cpu().numpy().view(np.uint32), want.view(np.uint32))
    st.close()

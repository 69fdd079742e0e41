"""The expert-cache policy (clb200_cache_*) against the reference's own c/src/cache.c, call by call (no GPU needed).

Bar: every return value and every slot number identical, the same key->slot map and segment of every slot, the same
statistics -- for random operation streams under all three policies and for the key stream of the reference's own stress
harness (c/src/stream.c:240-336: access the chosen experts, stage the predicted ones of the next layer, unpin after use).
"""
import ctypes as C

import numpy as np
import pytest

import oracle
from clutor_b200 import synth

pytestmark = pytest.mark.skipif(not oracle.ref_available(), reason="the reference library is not built")


def _pair(cache_slots, stage_slots, universe, policy, window_pct=0):
    import clutor_b200 as cb
    return (cb.ExpertCache(cache_slots, stage_slots, universe, policy, window_pct),
            oracle.RefCache(cache_slots, stage_slots, universe, policy, window_pct))


def _same_state(a, b, universe):
    assert a.stats() == b.stats()
    assert a.count() == b.count()
    assert a.total_slots() == b.total_slots()
    for k in range(universe):
        assert a.find(k) == b.find(k), f"key {k}"
        assert a.freq(k) == b.freq(k), f"freq of key {k}"
    for s in range(a.total_slots()):
        assert a.segment(s) == b.segment(s), f"slot {s}"


def test_stream_generator_matches_reference():
    """synth.ExpertStream is the reference harness's router, value for value (c/src/stream.c:116-140)."""
    L = oracle.ref_lib()
    L.ref_stream_new.restype = C.c_void_p
    L.ref_stream_new.argtypes = [C.c_int, C.c_int, C.c_double, C.c_ulonglong, C.c_double]
    L.ref_stream_logits.argtypes = [C.c_void_p, C.c_long, C.c_int, C.c_int, C.c_int, C.c_void_p]
    L.ref_stream_free.argtypes = [C.c_void_p]
    for (nl, E, loc, seed) in [(6, 128, 1.78, 1), (3, 64, 1.0, 12345)]:
        mine = synth.ExpertStream(nl, E, locality=loc, seed=seed, rho=0.8)
        ref = L.ref_stream_new(nl, E, loc, seed, 0.8)
        out = np.zeros(E, np.float32)
        try:
            for t in (0, 1, 15, 16, 17, 100, 4095):
                for l in range(nl):
                    for pred in (0, 1):
                        L.ref_stream_logits(ref, t, l, pred, 0, out.ctypes.data)
                        got = mine.logits(t, l, predicted=bool(pred))[0]
                        assert np.array_equal(got.view(np.uint32), out.view(np.uint32)), (t, l, pred)
        finally:
            L.ref_stream_free(ref)


@pytest.mark.parametrize("policy,cache_slots,stage_slots,universe,window_pct", [
    (0, 8, 0, 64, 0), (0, 5, 3, 40, 0), (1, 16, 4, 200, 0), (1, 1, 0, 10, 0), (1, 3, 2, 30, 0),
    (1, 40, 8, 6144, 20), (2, 32, 8, 500, 0), (2, 2, 1, 50, 0)])
def test_random_operations_match_reference(policy, cache_slots, stage_slots, universe, window_pct):
    a, b = _pair(cache_slots, stage_slots, universe, policy, window_pct)
    rng = np.random.default_rng(policy * 1000 + cache_slots)
    pinned: list[int] = []
    zipf = np.minimum(rng.zipf(1.3, size=30000) - 1, universe - 1)
    for i in range(30000):
        op = rng.random()
        key = int(zipf[i]) if rng.random() < 0.8 else int(rng.integers(universe))
        if op < 0.6:
            ra, rb = a.access(key), b.access(key)
            assert ra == rb, f"op {i}: access({key}) {ra} vs {rb}"
            if ra[0] >= 0:
                pinned.append(ra[1])
        elif op < 0.75:
            ra, rb = a.stage(key), b.stage(key)
            assert ra == rb, f"op {i}: stage({key})"
            if ra >= 0 and rng.random() < 0.7:
                a.unpin(ra), b.unpin(rb)       # the fill completed
            elif ra >= 0:
                pinned.append(ra)
        elif op < 0.95 and pinned:
            s = pinned.pop(int(rng.integers(len(pinned))))
            a.unpin(s), b.unpin(s)
        elif op < 0.97 and pinned:
            s = pinned.pop(int(rng.integers(len(pinned))))   # a fill that failed
            a.abandon(s), b.abandon(s)
            pinned = [p for p in pinned if p != s]
        elif pinned:
            s = pinned[int(rng.integers(len(pinned)))]
            a.pin(s), b.pin(s)
            pinned.append(s)
        if i % 5000 == 0:
            _same_state(a, b, universe)
    _same_state(a, b, universe)
    a.close(), b.close()


def test_stress_stream_replay_matches_reference():
    """The cache stress workload's key stream (48 layers x 128 experts, top-8, a cache of 40% of the experts, 16 staging
    slots, the next layer's predicted experts staged every step): identical hits, misses and slots."""
    nl, E, K = 48, 128, 8
    a, b = _pair(int(0.4 * nl * E), 2 * K, nl * E, 1)
    st = synth.ExpertStream(nl, E, locality=1.78, seed=1, rho=0.8)
    toks = np.arange(96)
    sel = {l: synth.route_topk(st.logits(toks, l), K)[0] for l in range(nl)}
    pred = {l: synth.route_topk(st.logits(toks, l, predicted=True), K)[0] for l in range(nl)}
    codes = []
    for t in toks:
        for l in range(nl):
            used = []
            for e in sel[l][t]:
                ra, rb = a.access(l * E + int(e)), b.access(l * E + int(e))
                assert ra == rb
                codes.append(ra[0])
                if ra[0] >= 0:
                    used.append(ra[1])
            if l + 1 < nl:
                for e in pred[l + 1][t]:
                    sa, sb = a.stage((l + 1) * E + int(e)), b.stage((l + 1) * E + int(e))
                    assert sa == sb
                    if sa >= 0:
                        a.unpin(sa), b.unpin(sb)
            for s in used:
                a.unpin(s), b.unpin(s)
    _same_state(a, b, nl * E)
    codes = np.array(codes)
    hit_rate = float(np.mean(codes >= 1))
    assert 0.2 < hit_rate < 1.0
    print(f"hit rate {hit_rate:.3f}, staged hits {np.mean(codes == 2):.3f}")
    a.close(), b.close()

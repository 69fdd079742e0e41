"""SMART-ROUTE (c/src/route.c:13-52) without a GPU: the oracle's restatement (orc_smart_route) against the reference's own
cl_route compiled into oracle/_ref, on the known-answer cases of c/test/test_engine.c:115-150 and on seeded random cases
(ties, tau 0 and unbounded, J and M at and beyond their clamps, nothing or everything resident, E up to 1024, K up to 32)."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.skipif(not oracle.ref_available(), reason="the reference engine is not built")


def both(lg, K, smart, res):
    a = oracle.smart_route(lg, K, smart, res, which="oracle")
    b = oracle.smart_route(lg, K, smart, res, which="ref")
    return a, b


def test_known_answers():
    """The cases of test_route (c/test/test_engine.c:115-150): 64 experts, logits -0.12 i, K = 8."""
    lg = np.array([-0.12 * i for i in range(64)], np.float32)
    plain = oracle.smart_route(lg, 8, None, None)
    assert plain["selected"] == list(range(8)) and plain["substituted"] == 0
    assert oracle.smart_route(lg[:8], 9, None, None) is None and oracle.smart_route(lg, 0, None, None) is None
    res = np.zeros(64, np.uint8)
    res[8:14] = 1                                   # only experts just outside the top-8 are in memory
    r = oracle.smart_route(lg, 8, (2, 12, 0.015), res)
    assert r["selected"][:2] == [0, 1]              # the true top-J stay
    assert r["max_delta"] <= 0.015 + 1e-12
    assert len(set(r["selected"])) == 8
    r2 = oracle.smart_route(lg, 8, (2, 12, 1e9), res)
    assert r2["substituted"] == 4 and r2["dropped_mass"] >= r["dropped_mass"]
    assert oracle.smart_route(lg, 8, (2, 12, 0.0), res)["substituted"] == 0
    assert oracle.smart_route(lg, 8, (2, 8, 1e9), res)["substituted"] == 0
    res[:8] = 1
    assert oracle.smart_route(lg, 8, (2, 12, 0.015), res)["substituted"] == 0
    for smart in [(2, 12, 0.015), (2, 12, 1e9)]:
        rs = np.zeros(64, np.uint8)
        rs[8:14] = 1
        a, b = both(lg, 8, smart, rs)
        assert a == b


def random_case(rng, E, K):
    kind = rng.integers(4)
    if kind == 0:
        lg = rng.standard_normal(E).astype(np.float32)
    elif kind == 1:                                  # many exact ties
        lg = rng.integers(-3, 3, E).astype(np.float32)
    elif kind == 2:                                  # a skewed router, as the stress harness draws it
        lg = (-3.0 * np.log(rng.permutation(E) + 1.0) / np.log(E) + rng.standard_normal(E)).astype(np.float32)
    else:                                            # large logits: exp underflows for most experts
        lg = (rng.standard_normal(E) * 40).astype(np.float32)
    J = int(rng.integers(-1, K + 2))
    M = int(rng.integers(0, E + 3))
    tau = float([0.0, 1e-3, 0.015, 0.1, 1e9][rng.integers(5)])
    p_res = [0.0, 0.2, 0.5, 0.9, 1.0][rng.integers(5)]
    res = (rng.random(E) < p_res).astype(np.uint8)
    return lg, (J, M, tau), res


@pytest.mark.parametrize("E,K", [(8, 8), (16, 4), (64, 8), (128, 8), (128, 32), (1024, 32), (300, 7)])
def test_oracle_equals_reference_random(E, K):
    rng = np.random.default_rng(E * 100 + K)
    n = 60 if E == 1024 else 300
    for i in range(n):
        lg, smart, res = random_case(rng, E, K)
        a, b = both(lg, K, smart, res)
        assert a == b, (i, smart)
        a, b = both(lg, K, None, None)
        assert a == b, i


def test_refused_arguments_match():
    lg = np.zeros(2048, np.float32)
    for E, K in [(1025, 8), (64, 33), (8, 9), (64, 0)]:
        a, b = both(lg[:E], K, None, None)
        assert a is None and b is None

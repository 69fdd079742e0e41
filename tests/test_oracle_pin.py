"""Pins the oracle (this repository's C restatement of the MoE block) before anything is checked against it:

* against the known-answer tests the reference's own unit tests hold for this path (c/test/test_engine.c), restated here;
* against the reference's independent Python restatement (c/test/tiny_olmoe.py) through tests/golden/dequant_golden.npz;
* against the reference engine compiled from its sources, through tests/golden/moe_golden.npz, and live when oracle/_ref is
  built.
"""
import json
import struct

import numpy as np
import pytest

import oracle
from clutor_b200 import synth


def test_f16_all_65536_values():
    """c/test/test_engine.c:199-241: the half to single conversion on every bit pattern (NaNs only need to be NaNs)."""
    lib = oracle.oracle_lib()
    vals = np.array([lib.orc_f16_to_f32(h) for h in range(65536)], np.float32)
    want = np.arange(65536, dtype=np.uint16).view(np.float16).astype(np.float32)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(vals), nan)
    assert np.array_equal(vals[~nan].view(np.uint32), want[~nan].view(np.uint32))
    assert lib.orc_f16_to_f32(0x3C00) == 1.0 and lib.orc_f16_to_f32(0xC000) == -2.0
    assert lib.orc_f16_to_f32(0x0001) == 2.0 ** -24 and np.isinf(lib.orc_f16_to_f32(0x7C00))
    if oracle.ref_available():
        ref = oracle.ref_lib()
        rv = np.array([ref.cl_f16_to_f32_soft(h) for h in range(0, 65536, 7)], np.float32)
        ov = vals[::7]
        assert np.array_equal(np.isnan(rv), np.isnan(ov))
        assert np.array_equal(rv[~np.isnan(rv)].view(np.uint32), ov[~np.isnan(ov)].view(np.uint32))


def test_dequant_kats():
    """c/test/test_engine.c:306-326: hand-made Q8_0, Q4_K and Q6_K blocks."""
    b8 = np.zeros(34, np.uint8)
    b8[1] = 0x3C
    b8[2:] = (np.arange(32) - 16).astype(np.int8).view(np.uint8)
    y = oracle.dequant_row(synth.T_Q8_0, b8, 32)
    assert y[0] == -16.0 and y[31] == 15.0
    q4 = np.zeros(144, np.uint8)
    q4[1] = 0x3C
    q4[4:8] = 1
    q4[12:16] = 1      # scales 0..3 (low 6 bits of bytes 0..3); mins stay 0
    q4[12:16] = 1
    q4[4 + 8:4 + 12] = 1   # scales 4..7: low nibble of bytes 8..11
    q4[16:] = 0x21
    y = oracle.dequant_row(synth.T_Q4_K, q4, 256)
    assert y[0] == 1.0 and y[31] == 1.0 and y[32] == 2.0 and y[63] == 2.0 and y[64] == 1.0 and y[255] == 2.0
    q6 = np.zeros(210, np.uint8)
    q6[192:208] = 1
    q6[209] = 0x3C
    y = oracle.dequant_row(synth.T_Q6_K, q6, 256)
    assert y[0] == -32.0 and y[255] == -32.0


def test_dequant_matches_reference_python(request):
    """Random blocks against the reference's pure-Python deq_q4k / deq_q6k (double precision): the float results must be
    the double results rounded (one rounding per multiply/subtract, so within a few float ulps)."""
    g = np.load(request.config.rootpath / "tests" / "golden" / "dequant_golden.npz")
    for name, type_, bb in (("q4k", synth.T_Q4_K, 144), ("q6k", synth.T_Q6_K, 210), ("q8_0", synth.T_Q8_0, 34)):
        raw = g[f"{name}.raw"]
        want = g[f"{name}.values"]
        n = want.size
        got = oracle.dequant_row(type_, raw, n)
        assert np.allclose(got, want, rtol=1e-6, atol=1e-6 * np.abs(want).max()), name
        if oracle.ref_available():
            assert np.array_equal(got.view(np.uint32), oracle.dequant_row(type_, raw, n, "ref").view(np.uint32)), name


def test_integer_dot_vs_dequantized():
    """c/test/test_engine.c:361-397: the K-quant integer dot equals dequantize-then-multiply in double within 1e-4*sum|w*x|."""
    rng = np.random.default_rng(777)
    cols = 768
    x = (rng.random(cols, np.float32) - 0.5) * np.where(np.arange(cols) % 97 == 0, 8.0, 1.0).astype(np.float32)
    xq = oracle.q8k_quantize(x)
    xd = np.concatenate([b["d"] * b["qs"].astype(np.float32) for b in xq])
    for type_, bb in ((synth.T_Q4_K, 144), (synth.T_Q6_K, 210)):
        w = rng.integers(0, 256, 40 * 3 * bb, dtype=np.uint8).reshape(40 * 3, bb)
        for b in range(40 * 3):
            d = 0x2400 + (b % 16) * 8
            dm = 0x2000 + (b % 7) * 8
            if type_ == synth.T_Q4_K:
                w[b, 0:2] = np.frombuffer(struct.pack("<H", d), np.uint8)
                w[b, 2:4] = np.frombuffer(struct.pack("<H", dm), np.uint8)
            else:
                w[b, 208:210] = np.frombuffer(struct.pack("<H", d), np.uint8)
        w = w.reshape(40, -1)
        for r in range(40):
            got = oracle.dot_row(type_, w[r], cols, xq, None)
            row = oracle.dequant_row(type_, w[r], cols).astype(np.float64)
            ref = float(np.dot(row, xd))
            mag = float(np.abs(row * xd).sum())
            assert abs(ref - got) <= 1e-4 * mag + 1e-6


def test_route_order_and_ties():
    """c/test/test_engine.c:115-120 and the tie rule of c/src/forward.c:971-976 (ties go to the lower expert id)."""
    logits = (-0.12 * np.arange(64)).astype(np.float32)
    sel, wt = oracle.route(logits, 8, 1)
    assert sel.tolist() == list(range(8))
    assert abs(float(wt.sum()) - 1.0) < 1e-6
    tied = np.zeros(16, np.float32)
    tied[[3, 7, 11]] = 1.0
    sel, _ = oracle.route(tied, 4, 1)
    assert sel.tolist() == [3, 7, 11, 0]


def _golden_cases(golden):
    return sorted({k.split(".")[0] for k in golden.files})


def _golden_layer(golden, name):
    from tests.golden.make_golden import make_layer
    p = json.loads(bytes(golden[f"{name}.params"]).decode())
    return make_layer(p["layer"], p["special"]), p


def test_oracle_matches_golden(golden):
    """The oracle reproduces every fixture the reference engine produced, bit for bit."""
    for name in _golden_cases(golden):
        L, p = _golden_layer(golden, name)
        x = golden[f"{name}.x"]
        xo, sel, wt = oracle.moe_ffn(L, x, "oracle")
        assert np.array_equal(sel, golden[f"{name}.sel"]), name
        assert np.array_equal(wt.view(np.uint32), golden[f"{name}.wt"].view(np.uint32)), name
        assert np.array_equal(xo.view(np.uint32), golden[f"{name}.x_out"].view(np.uint32)), name


def test_inputs_regenerate_bit_exactly(golden):
    """The seeded generator gives the fixture's inputs on this machine (bit-reproducible numpy arithmetic)."""
    from tests.golden.make_golden import make_x
    for name in _golden_cases(golden):
        p = json.loads(bytes(golden[f"{name}.params"]).decode())
        E = p["layer"].get("E", 2048)
        assert np.array_equal(make_x(p["T"], E, p["x_seed"], p["special"]).view(np.uint32), golden[f"{name}.x"].view(np.uint32)), name


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built (needs the reference sources)")
@pytest.mark.parametrize("gt,dt,T", [(synth.T_Q4_K, synth.T_Q4_K, 1), (synth.T_Q4_K, synth.T_Q6_K, 9),
                                      (synth.T_Q8_0, synth.T_Q8_0, 3), (synth.T_Q6_K, synth.T_Q8_0, 2)])
def test_oracle_matches_reference_live(gt, dt, T):
    L = synth.host_layer(E=768, FF=512, NE=24, K=6, gate_type=gt, down_type=dt, seed=31 + T)
    x = synth.activations(T, 768, seed=T)
    a = oracle.moe_ffn(L, x, "oracle")
    b = oracle.moe_ffn(L, x, "ref")
    for u, v in zip(a, b):
        assert np.array_equal(np.asarray(u).view(np.uint32), np.asarray(v).view(np.uint32))

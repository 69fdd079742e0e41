"""Generates the golden fixtures in this folder from the reference itself (run in a checkout that has the reference).

* ``moe_golden.npz`` -- MoE-layer outputs of the reference engine compiled from its own sources (oracle/_ref/libclref.so:
  c/src/quant.c, kernel.c, forward.c's rmsnorm/dotf and the block order of c/src/forward.c:949-1033 / :1132-1210) on seeded
  synthetic layers (clutor_b200.synth, bit-reproducible numpy). Each case stores its parameters, the input x, the routing
  (sel, wt) and the output x; the weights are regenerated from the seed.
* ``dequant_golden.npz`` -- random Q4_K / Q6_K / Q8_0 blocks dequantized by the reference's independent pure-Python
  restatement (c/test/tiny_olmoe.py: deq_q4k, deq_q6k; Q8_0 by its one-line definition), in float64.

Usage:  python tests/golden/make_golden.py [--ref-dir /root/reference]
"""
from __future__ import annotations

import argparse
import json
import os
import struct
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from clutor_b200 import synth  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))

# (name, layer kwargs, T, x seed, special)
CASES = [
    ("small_q4k_t1", dict(E=512, FF=256, NE=32, K=4, gate_type=synth.T_Q4_K, seed=11), 1, 1, None),
    ("small_q4k_t5", dict(E=512, FF=256, NE=32, K=4, gate_type=synth.T_Q4_K, seed=11), 5, 2, None),
    ("small_q6k_down_t3", dict(E=512, FF=512, NE=16, K=2, gate_type=synth.T_Q4_K, down_type=synth.T_Q6_K, seed=12), 3, 3, None),
    ("small_q8_0_t4", dict(E=512, FF=256, NE=32, K=4, gate_type=synth.T_Q8_0, seed=13), 4, 4, None),
    ("small_no_renorm_t2", dict(E=256, FF=256, NE=8, K=2, gate_type=synth.T_Q4_K, seed=14, norm_topk=0, resid_scale=0.5), 2, 5, None),
    ("ties_t2", dict(E=256, FF=256, NE=16, K=4, gate_type=synth.T_Q4_K, seed=15), 2, 6, "ties"),
    ("zeros_t1", dict(E=256, FF=256, NE=16, K=4, gate_type=synth.T_Q4_K, seed=16), 1, 7, "zeros"),
    ("c1_q4k_t1_a", dict(seed=1), 1, 21, None),
    ("c1_q4k_t1_b", dict(seed=1), 1, 22, None),
    ("c1_q4k_t1_c", dict(seed=2), 1, 23, None),
    ("c3mix_q6k_down_t1", dict(seed=3, down_type=synth.T_Q6_K), 1, 24, None),
    ("c2_q8_0_t64", dict(seed=4, gate_type=synth.T_Q8_0, router_scale=0.05), 64, 25, None),
    ("c1_q4k_t17", dict(seed=5), 17, 26, None),
]


def make_layer(kw: dict, special: str | None):
    L = synth.host_layer(**kw)
    if special == "ties":   # experts 1, 5 and 9 share expert 3's router row: equal logits, so ranks must fall to the lower id
        for e in (1, 5, 9):
            L.router[e] = L.router[3]
    return L


def make_x(T: int, E: int, seed: int, special: str | None) -> np.ndarray:
    return np.zeros((T, E), np.float32) if special == "zeros" else synth.activations(T, E, seed=seed)


def moe_cases() -> dict:
    out = {}
    for name, kw, T, xs, special in CASES:
        L = make_layer(kw, special)
        x = make_x(T, L.E, xs, special)
        xo, sel, wt = oracle.moe_ffn(L, x, "ref")
        out[f"{name}.params"] = np.frombuffer(json.dumps({"layer": kw, "T": T, "x_seed": xs, "special": special}).encode(), np.uint8)
        out[f"{name}.x"] = x
        out[f"{name}.sel"] = sel
        out[f"{name}.wt"] = wt
        out[f"{name}.x_out"] = xo
        print(f"{name}: T={T} sel[0]={sel[0].tolist()}", flush=True)
    return out


def dequant_cases(ref_dir: str) -> dict:
    sys.path.insert(0, os.path.join(ref_dir, "c", "test"))
    import tiny_olmoe as t  # the reference's independent Python restatement
    out = {}
    for type_, name, bb in ((synth.T_Q4_K, "q4k", 144), (synth.T_Q6_K, "q6k", 210), (synth.T_Q8_0, "q8_0", 34)):
        elems = synth.BLOCK_ELEMS[type_]
        raw = synth.quant_tensor(type_, 16 * 256, seed=77, stream=type_).reshape(-1, bb)
        vals = []
        for b in raw:
            bb_ = bytes(b)
            if type_ == synth.T_Q4_K:
                vals += t.deq_q4k(bb_)
            elif type_ == synth.T_Q6_K:
                vals += t.deq_q6k(bb_)
            else:
                d = struct.unpack("<e", bb_[:2])[0]
                vals += [d * v for v in struct.unpack("<32b", bb_[2:34])]
        assert len(vals) == raw.shape[0] * elems
        out[f"{name}.raw"] = raw.reshape(-1)
        out[f"{name}.values"] = np.array(vals, np.float64)
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-dir", default="/root/reference")
    a = ap.parse_args()
    oracle.build(os.path.join(a.ref_dir, "c", "src"))
    np.savez_compressed(os.path.join(HERE, "moe_golden.npz"), **moe_cases())
    np.savez_compressed(os.path.join(HERE, "dequant_golden.npz"), **dequant_cases(a.ref_dir))


if __name__ == "__main__":
    main()

"""The synthetic-model writer against the reference's own reader and forward pass (CPU): the files this library writes are
models the reference opens and runs, with the shapes, types and metadata the device loader expects."""
import os

import numpy as np
import pytest

import oracle
from clutor_b200 import gguf
from clutor_b200 import synth_model as sm


def test_gguf_round_trip(tmp_path):
    spec = sm.tiny()
    img = sm.image(spec, seed=2)
    path = os.path.join(tmp_path, "a.gguf")
    n = sm.write(path, spec, seed=2)
    assert n == img.nbytes
    assert open(path, "rb").read() == img.tobytes()   # the image and the file are the same bytes
    meta, tens = gguf.read(img.tobytes())
    assert meta["general.architecture"] == "qwen3moe"
    assert meta["qwen3moe.block_count"] == spec.n_layer
    t = tens["blk.0.ffn_down_exps.weight"]
    assert t.dims == [spec.FF, spec.E, spec.NE] and t.type == sm.T_Q6_K
    assert t.offset % gguf.ALIGN == 0


@pytest.mark.skipif(not oracle.ref_available(), reason="the reference engine is not built")
@pytest.mark.parametrize("arch", ["qwen3moe", "olmoe", "granitemoe"])
def test_reference_runs_synthetic_model(tmp_path, arch):
    spec = sm.tiny(arch=arch, n_kv=2 if arch == "olmoe" else 1)
    path = os.path.join(tmp_path, "m.gguf")
    sm.write(path, spec, seed=4)
    ref = oracle.RefModel(path, 32)
    assert (ref.n_layer, ref.n_embd, ref.n_vocab, ref.n_expert, ref.n_used, ref.head_dim) == (
        spec.n_layer, spec.E, spec.vocab, spec.NE, spec.K, spec.hd)
    logits, sel, wt = ref.step(3)
    assert np.isfinite(logits).all()
    assert sel.shape == (spec.n_layer, spec.K) and ((0 <= sel) & (sel < spec.NE)).all()
    if arch != "olmoe":   # qwen3moe and granitemoe renormalise the chosen weights
        assert np.allclose(wt.sum(axis=1), 1.0, atol=1e-6)
    toks = ref.greedy(5, 6)
    assert all(0 <= t < spec.vocab for t in toks)
    ref.close()


def test_model_bytes_qwen3_30b():
    b = sm.model_bytes(sm.QWEN3_30B_A3B)
    # per token: experts 48 * 8 * (2 * 884,736 + 1,290,240); the output matrix 151,936 rows of 1,680 bytes
    assert b["experts"] == 48 * 8 * (2 * 884736 + 1290240)
    assert b["output"] == 151936 * 1680
    assert 1.9e9 < b["total"] < 2.1e9

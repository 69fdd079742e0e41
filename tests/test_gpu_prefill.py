"""Parity of the batched prompt path (clb200_model_prefill) with the reference's own cl_fwd_prefill (run_std,
c/src/forward.c:1078-1225, compiled unmodified into oracle/_ref/libclref.so) on seeded synthetic GGUF models (needs a B200).

Bar, with the expert products on the integer path (clb200_set_exact): the logits after the prompt within 1e-3 relative L2
of the reference's and the same arg-max; then greedy steps from the state the prompt left (the key/value cache written by
the batched path): every token equal and the logits within 1e-3. With the expert products on the tensor cores (the
default; fp16 hi/lo operands, ~2e-5 from the integer products, and an 8-bit activation rounding downstream can turn that
into ~1e-4 per layer): the logits within 1e-2 relative L2, before and after the prompt.
The batch size is the reference's CLUTOR_PS_B (set in the environment for the reference, clb200_model_set_batch here), so
both cross the same batch boundaries.
"""
import os

import numpy as np
import pytest

import oracle
from clutor_b200 import synth_model as sm
from tests.test_gpu_model import SHAPES, TOL_REL_L2, rel_l2

TOL_TC = 1e-2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    import clutor_b200 as cb
    c = cb.Context(0)
    yield c
    c.close()


def run(ctx, tmp_path, spec, prompt, batch, steps=6, seed=5, n_ctx=512, exact=True):
    from clutor_b200.model import Model
    tol = TOL_REL_L2 if exact else TOL_TC
    path = os.path.join(tmp_path, "m.gguf")
    sm.write(path, spec, seed=seed)
    old = os.environ.get("CLUTOR_PS_B")
    if batch < 64:
        os.environ["CLUTOR_PS_B"] = str(batch)
    else:
        os.environ.pop("CLUTOR_PS_B", None)
    try:
        ref = oracle.RefModel(path, n_ctx)
        want = ref.prefill(prompt)
    finally:
        if old is None:
            os.environ.pop("CLUTOR_PS_B", None)
        else:
            os.environ["CLUTOR_PS_B"] = old
    dev = Model(ctx, path, n_ctx)
    ctx.set_exact(exact)
    try:
        dev.set_batch(batch)
        got = dev.prefill(prompt)
        assert dev.pos == len(prompt)
        e = rel_l2(got, want)
        assert e <= tol, f"prompt logits rel L2 {e:.3g}"
        if exact:
            assert int(np.argmax(got)) == int(np.argmax(want))
        tok = int(np.argmax(want))
        worst = e
        for t in range(steps):   # decoding on from the cache the prompt filled, the same tokens in both
            w, _, _ = ref.step(tok)
            g, nxt, _ = dev.step(tok)
            worst = max(worst, rel_l2(g, w))
            assert rel_l2(g, w) <= tol, f"step {t} after the prompt"
            if exact:
                assert nxt == int(np.argmax(w)), f"step {t}: greedy token"
            tok = int(np.argmax(w))
        return worst
    finally:
        ctx.set_exact(False)
        dev.close()
        ref.close()


@pytest.mark.parametrize("exact", [True, False], ids=["integer", "tensor-core"])
@pytest.mark.parametrize("name", sorted(SHAPES))
def test_prefill_parity(ctx, tmp_path, name, exact):
    rng = np.random.default_rng(len(name))
    prompt = rng.integers(0, SHAPES[name].vocab, 37).tolist()
    worst = run(ctx, tmp_path, SHAPES[name], prompt, batch=64, exact=exact)
    print(f"{name}: worst logits rel L2 {worst:.3g}")


def test_prefill_large_batch_tensor_cores(ctx, tmp_path):
    """300 tokens in one batch: the Q4_K dense products (256 tokens and more) run on the tensor cores too."""
    name = "qwen3moe_gqa8_q4k_down"
    rng = np.random.default_rng(17)
    prompt = rng.integers(0, SHAPES[name].vocab, 300).tolist()
    worst = run(ctx, tmp_path, SHAPES[name], prompt, batch=512, exact=False, steps=4)
    print(f"{name}, one batch of 300: worst logits rel L2 {worst:.3g}")


@pytest.mark.parametrize("n,batch", [(100, 16), (65, 64), (130, 64), (9, 1), (2, 512)])
def test_prefill_batch_boundaries(ctx, tmp_path, n, batch):
    """Batches of the reference's CLUTOR_PS_B sizes: several full batches and a short last one, a last batch of one token
    (a step, in both), every token a step (batch 1), and a batch larger than the prompt."""
    rng = np.random.default_rng(n * 7 + batch)
    spec = sm.tiny()
    prompt = rng.integers(0, spec.vocab, n).tolist()
    run(ctx, tmp_path, spec, prompt, batch=batch, steps=4)


def test_prefill_then_more_prompt(ctx, tmp_path):
    """Two prompts in a row (the second batch starts at a position past 0) and a single-token prefill (a step)."""
    from clutor_b200.model import Model
    spec = sm.tiny()
    path = os.path.join(tmp_path, "p.gguf")
    sm.write(path, spec, seed=3)
    rng = np.random.default_rng(1)
    a, b = rng.integers(0, spec.vocab, 40).tolist(), rng.integers(0, spec.vocab, 23).tolist()
    ref = oracle.RefModel(path, 256)
    ref.prefill(a, logits=False)
    want = ref.prefill(b)
    want1 = ref.prefill([7])
    ref.close()
    dev = Model(ctx, path, 256)
    ctx.set_exact(True)
    try:
        assert dev.prefill(a, logits=False) is None
        assert rel_l2(dev.prefill(b), want) <= TOL_REL_L2
        assert rel_l2(dev.prefill([7]), want1) <= TOL_REL_L2
        assert dev.pos == 64
    finally:
        ctx.set_exact(False)
        dev.close()


def test_prefill_errors(ctx, tmp_path):
    from clutor_b200 import ClutorError
    from clutor_b200.model import Model
    path = os.path.join(tmp_path, "e.gguf")
    sm.write(path, sm.tiny(), seed=1)
    dev = Model(ctx, path, 16)
    with pytest.raises(ClutorError, match="outside the vocabulary"):
        dev.prefill([1, 2, 10 ** 6])
    with pytest.raises(ClutorError, match="context is full"):
        dev.prefill(list(range(17)))
    with pytest.raises(ClutorError, match="nothing"):
        dev.prefill([])
    with pytest.raises(ClutorError):
        dev.set_batch(513)
    assert dev.pos == 0
    dev.prefill(list(range(16)), logits=False)
    assert dev.pos == 16
    dev.close()

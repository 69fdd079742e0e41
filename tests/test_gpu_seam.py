"""The reference engine driving clutor-b200 through its own C surfaces (needs a B200).

tests/seam/ builds two binaries from the reference's own sources with its Makefile's flags (tests/seam/Makefile): seam_ref
(the engine unmodified) and seam_hook (forward.c with INTEGRATION.md's MoE hook pasted in, the text taken from the
document). Each runs the reference's greedy loop (cl_fwd_open / cl_fwd_step, c/src/forward.h:113-117) on a synthetic GGUF.

* The plugin seam (c/src/backend.h:9-19, c/src/quant.c:977-1004): seam_ref registers clb200_backend() with
  cl_backend_register and selects "b200"; every Q4_K / Q6_K / Q8_0 product of the forward pass then runs on the GPU. The
  logits must be the CPU backend's bit for bit.
* The MoE hook: seam_hook with CLUTOR_B200=1 runs every layer's MoE block through
  clb200_moe_ffn; the greedy tokens and the logits must be the unmodified engine's, bit for bit (the block returns the
  reference's bits).
"""
import os
import subprocess

import numpy as np
import pytest

import oracle
from clutor_b200 import synth_model as sm

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SEAM = os.path.join(ROOT, "tests", "seam")
BINS = {k: os.path.join(SEAM, "_build", k) for k in ("seam_ref", "seam_hook")}
STEPS = 12
MODELS = {
    "qwen3moe": sm.tiny(),
    "qwen3moe_gqa8_q4k_down": sm.tiny(n_layer=3, E=512, n_head=8, n_kv=1, hd=128, FF=512, NE=16, K=4, down_type=sm.T_Q4_K),
    "olmoe": sm.tiny(arch="olmoe", n_head=2, n_kv=2, hd=128),
    "granitemoe": sm.tiny(arch="granitemoe", n_head=2, n_kv=1, hd=128),
}


@pytest.fixture(scope="module")
def binaries():
    if not all(os.path.exists(b) for b in BINS.values()):
        if not oracle.ref_dir():
            pytest.skip("tests/seam binaries are not built and the reference sources are absent (CLUTOR_REF_DIR)")
        subprocess.run(["make", "-C", SEAM, f"REF_DIR={oracle.ref_dir()}"], check=True, capture_output=True)
    return BINS


def run(binary, model, mode, out, env_extra=None):
    env = {k: v for k, v in os.environ.items() if k not in ("CLUTOR_B200", "CLUTOR_BACKEND")}
    env.update(env_extra or {})
    r = subprocess.run([binary, model, str(STEPS), mode, out], capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    raw = np.fromfile(out, np.uint8)
    toks = raw[-4 * STEPS:].view(np.int32)
    logits = raw[:-4 * STEPS].view(np.float32).reshape(STEPS, -1)
    return logits, toks


@pytest.mark.parametrize("name", sorted(MODELS))
def test_reference_engine_through_the_seams(binaries, tmp_path, name):
    model = str(tmp_path / f"{name}.gguf")
    sm.write(model, MODELS[name], seed=5)
    cpu_lg, cpu_tok = run(binaries["seam_ref"], model, "cpu", str(tmp_path / "cpu.bin"))
    be_lg, be_tok = run(binaries["seam_ref"], model, "b200", str(tmp_path / "b200.bin"))
    assert np.array_equal(be_tok, cpu_tok), "greedy tokens through the b200 backend"
    assert np.array_equal(be_lg.view(np.uint32), cpu_lg.view(np.uint32)), "the b200 backend's logits are not the CPU's bits"
    hk_lg, hk_tok = run(binaries["seam_hook"], model, "cpu", str(tmp_path / "hook.bin"), {"CLUTOR_B200": "1"})
    assert np.array_equal(hk_tok, cpu_tok), "greedy tokens through the MoE hook"
    assert np.array_equal(hk_lg.view(np.uint32), cpu_lg.view(np.uint32)), "the MoE hook's logits are not the CPU's bits"
    off_lg, off_tok = run(binaries["seam_hook"], model, "cpu", str(tmp_path / "off.bin"))   # the hooked engine, switch off
    assert np.array_equal(off_lg.view(np.uint32), cpu_lg.view(np.uint32))
    print(f"{name}: backend seam and MoE hook bit-identical to the CPU engine, tokens {cpu_tok[:6].tolist()}")

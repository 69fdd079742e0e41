"""The MoE hook the seam test compiles is INTEGRATION.md's own text, and it applies to the reference's forward.c (no GPU)."""
import importlib.util
import os

import pytest

import oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def patcher():
    spec = importlib.util.spec_from_file_location("patch_forward", os.path.join(ROOT, "tests", "seam", "patch_forward.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_hook_text_comes_from_the_document():
    static, hook = patcher().hook_text()
    assert static.startswith("static clb200_ctx *g_b200;")
    assert hook.startswith("if (g_b200 && !f->xs && !f->smart.enabled) {")
    assert "clb200_moe_ffn(g_b200, &L, f->x, 1, sel, wt, err, errlen)" in hook and hook.rstrip().endswith("}")


@pytest.mark.skipif(not (oracle.ref_dir() and os.path.isdir(oracle.ref_dir())), reason="needs the reference sources (CLUTOR_REF_DIR)")
def test_hook_applies_once_to_the_reference_forward_pass():
    src = open(os.path.join(oracle.ref_dir(), "forward.c")).read()
    out = patcher().patch(src)
    assert out.count("clb200_moe_ffn(g_b200") == 1 and out.count('getenv("CLUTOR_B200")') == 1
    assert len(out) > len(src)

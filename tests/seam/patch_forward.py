"""Writes a copy of the reference's forward.c carrying INTEGRATION.md's MoE hook (test infrastructure: the copy goes to
tests/seam/_build/, never into the repository). The hook's C text is read from INTEGRATION.md's section 1 code block, so
the test compiles exactly what the document tells an integrator to paste.

    python tests/seam/patch_forward.py <reference c/src dir> <out.c>
"""
import os
import re
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def hook_text() -> tuple[str, str]:
    """(the static declaration line, the hook block) from INTEGRATION.md's first C code block."""
    doc = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    block = re.search(r"```c\n(.*?)```", doc, re.S).group(1)
    lines = block.splitlines()
    static = next(l for l in lines if l.startswith("static clb200_ctx"))
    start = next(i for i, l in enumerate(lines) if l.startswith("if (g_b200"))
    return static, "\n".join(lines[start:])


def patch(src: str) -> str:
    static, hook = hook_text()
    anchor_step = "    /* mixture of experts */\n    rmsnorm(f->xn, f->x, y->ffn_norm_f, E, f->rms_eps);"
    if src.count(anchor_step) != 1:
        raise SystemExit("the one-token MoE block's first line was not found once in forward.c")
    body = "\n".join("    " + l if l else l for l in hook.splitlines())
    src = src.replace(anchor_step, body + "\n" + anchor_step)
    anchor_open = "int cl_fwd_open(cl_fwd *f, const char *path, int n_ctx, const cl_fwd_opts *opts, char *err, size_t errlen) {"
    if src.count(anchor_open) != 1:
        raise SystemExit("cl_fwd_open was not found once in forward.c")
    src = src.replace(anchor_open, anchor_open + '\n  if (!g_b200 && getenv("CLUTOR_B200")) { g_b200 = clb200_open(-1, err, errlen); if (!g_b200) return 1; }')
    first_include = src.index("#include")
    return src[:first_include] + '#include "clb200.h"\n' + static + "\n" + src[first_include:]


if __name__ == "__main__":
    ref_dir, out = sys.argv[1], sys.argv[2]
    os.makedirs(os.path.dirname(out), exist_ok=True)
    open(out, "w").write(patch(open(os.path.join(ref_dir, "forward.c")).read()))

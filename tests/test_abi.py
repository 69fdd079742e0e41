"""The C ABI without a GPU: the library loads, exports every function include/clb200.h declares, and its structs have the
reference's layouts (checked by compiling both headers with gcc)."""
import os
import subprocess
import tempfile

import pytest

import clutor_b200 as cb
import oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def built():
    from clutor_b200 import build
    build.build()
    return cb.lib()


def test_library_exports_every_declared_function(built):
    names = cb.header_functions()
    assert {"clb200_open", "clb200_moe_ffn", "clb200_backend", "clb200_layer_bind", "clb200_moe_ffn_dev"} <= set(names)
    missing = [n for n in names if not hasattr(built, n)]
    assert not missing, missing


def test_ctypes_mirror_matches_header():
    import ctypes as C
    assert C.sizeof(cb.Q8K) == 292
    assert C.sizeof(cb.CLW) == 24
    assert C.sizeof(cb.MV) == 72


@pytest.mark.skipif(not (oracle.ref_dir() and os.path.isdir(oracle.ref_dir())), reason="needs the reference headers (CLUTOR_REF_DIR)")
def test_struct_layouts_equal_the_reference():
    """clb200_w / clb200_q8k / clb200_xq / clb200_mv / clb200_backend_t / clb200_smart / clb200_route_result have the layout of
    the reference's cl_w (forward.h:18), cl_q8k / cl_xq / cl_mv (quant.h:22-34), cl_backend (backend.h:9-13), cl_smart and
    cl_route_result (route.h:14-22), so the reference can pass its own structs."""
    src = r"""
#include <stddef.h>
#include <stdio.h>
#include "clb200.h"
#include "backend.h"
#include "forward.h"
#include "route.h"
#define S(a, b) printf("%s %zu %zu\n", #a, sizeof(a), sizeof(b))
#define O(a, b, f) printf("%s.%s %zu %zu\n", #a, #f, offsetof(a, f), offsetof(b, f))
int main(void) {
  S(clb200_w, cl_w); O(clb200_w, cl_w, p); O(clb200_w, cl_w, type); O(clb200_w, cl_w, rows); O(clb200_w, cl_w, cols);
  S(clb200_q8k, cl_q8k); O(clb200_q8k, cl_q8k, qs); O(clb200_q8k, cl_q8k, bsums);
  S(clb200_xq, cl_xq); O(clb200_xq, cl_xq, n);
  S(clb200_mv, cl_mv); O(clb200_mv, cl_mv, w); O(clb200_mv, cl_mv, xf); O(clb200_mv, cl_mv, xq); O(clb200_mv, cl_mv, out);
  O(clb200_mv, cl_mv, nb); O(clb200_mv, cl_mv, xf_stride); O(clb200_mv, cl_mv, out_stride);
  S(clb200_backend_t, cl_backend); O(clb200_backend_t, cl_backend, supports); O(clb200_backend_t, cl_backend, matvec_batch);
  S(clb200_smart, cl_smart); O(clb200_smart, cl_smart, J); O(clb200_smart, cl_smart, M); O(clb200_smart, cl_smart, tau);
  S(clb200_route_result, cl_route_result); O(clb200_route_result, cl_route_result, k);
  O(clb200_route_result, cl_route_result, substituted); O(clb200_route_result, cl_route_result, dropped_mass);
  O(clb200_route_result, cl_route_result, max_delta);
  return 0;
}
"""
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "layout.c")
        exe = os.path.join(d, "layout")
        open(c, "w").write(src)
        subprocess.run(["gcc", "-std=c11", f"-I{ROOT}/include", f"-I{oracle.ref_dir()}", c, "-o", exe], check=True)
        out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout
    for line in out.strip().splitlines():
        name, a, b = line.split()
        assert a == b, line


def test_no_entry_point_without_library(monkeypatch):
    """Without the built library every entry point raises; nothing falls back to the CPU."""
    monkeypatch.setattr(cb, "LIB_PATH", "/nonexistent/libclutor_b200.so")
    monkeypatch.setattr(cb, "_lib", None)
    with pytest.raises(RuntimeError, match="not built"):
        cb.lib()

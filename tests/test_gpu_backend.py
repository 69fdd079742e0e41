"""The "b200" cl_backend against the reference's CPU backend: the same cl_mv jobs give the same numbers, bit for bit
(the reference's c/test/test_engine.c:408-437 asks a backend for "the CPU's numbers within the tolerance it documents";
this one documents zero). Needs a B200."""
import numpy as np
import pytest

import oracle
from clutor_b200 import synth

pytestmark = pytest.mark.gpu


def cpu_matvec(type_, w, rows, cols, xf, xq):
    """The oracle's row dots (pinned to the reference engine): one row at a time."""
    rb = synth.row_bytes(type_, cols)
    nb = xf.shape[0]
    out = np.zeros((nb, rows), np.float32)
    for b in range(nb):
        for r in range(rows):
            out[b, r] = oracle.dot_row(type_, w[r * rb:(r + 1) * rb], cols, xq[b] if xq is not None else None, xf[b])
    return out


@pytest.mark.parametrize("type_,rows,cols,nb", [(synth.T_Q4_K, 200, 2048, 1), (synth.T_Q4_K, 64, 768, 5),
                                                (synth.T_Q6_K, 100, 1536, 3), (synth.T_Q8_0, 130, 2048, 1),
                                                (synth.T_Q8_0, 40, 768, 9)])
def test_backend_matches_cpu(type_, rows, cols, nb):
    import clutor_b200 as cb
    be = cb.backend()
    assert be.name == b"b200"
    assert be.supports(synth.T_Q4_K) and be.supports(synth.T_Q6_K) and be.supports(synth.T_Q8_0)
    assert not be.supports(synth.T_F32) and not be.supports(synth.T_F16)
    w = synth.quant_tensor(type_, rows * cols, seed=rows, stream=cols)
    xf = synth.activations(nb, cols, seed=nb)
    xq = None
    if type_ != synth.T_Q8_0:
        xq = np.stack([oracle.q8k_quantize(xf[b]) for b in range(nb)])
    got = cb.matvec(type_, w, rows, cols, xf=xf, xq=xq)
    want = cpu_matvec(type_, w, rows, cols, xf, xq)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    if oracle.ref_available() and nb == 1:
        ref = oracle.ref_matvec(type_, w, rows, cols, xf[0], xq[0] if xq is not None else None)
        assert np.array_equal(got[0].view(np.uint32), ref.view(np.uint32))

"""The allocation-free entry point (clb200_moe_ffn_decode_noalloc), for hosts that cannot call cudaMalloc once they run.

It is checked against the context entry point (clb200_moe_ffn_dev) through the C ABI on the Qwen3-30B-A3B layer shape, on
two calls in a row (its fixed scratch array keeps the first call's contents, so the second call shows that whatever must
start at zero is cleared). This file is named to be collected last, so that a run which stops at the first failure has
run every other test before it; it also passes alone in a fresh process. Needs a B200.
"""
import ctypes as C

import numpy as np
import pytest

from clutor_b200 import synth

pytestmark = pytest.mark.gpu

TOL_REL_L2 = 1e-3   # the library's stated output tolerance (the two paths run the same kernel, so in practice 0)


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_noalloc_matches_context_path_on_two_calls():
    import torch

    import clutor_b200 as cb
    lib = cb.lib()
    err = C.create_string_buffer(512)
    ctx = cb.Context(0)
    layer = synth.device_layer(seed=321, down_type=synth.T_Q6_K)
    handle = ctx.bind(layer)
    s = cb.layer_struct(layer)          # device pointers
    free_before = None
    for call in range(2):
        x0 = synth.activations(1, layer.E, seed=500 + call)
        xa = torch.from_numpy(x0).cuda()
        sa = torch.zeros(layer.K, dtype=torch.int32, device="cuda")
        wa = torch.zeros(layer.K, dtype=torch.float32, device="cuda")
        ctx.moe_ffn_dev(handle, xa, sa, wa)
        ctx.status()
        xb = torch.from_numpy(x0).cuda()
        sb = torch.full((layer.K,), -1, dtype=torch.int32, device="cuda")
        wb = torch.zeros(layer.K, dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        if call == 1:
            free_before = torch.cuda.mem_get_info()[0]
        rc = lib.clb200_moe_ffn_decode_noalloc(C.byref(s), xb.data_ptr(), sb.data_ptr(), wb.data_ptr(), None, err, 512)
        assert rc == 0, err.value.decode()
        if call == 1:
            assert torch.cuda.mem_get_info()[0] == free_before, "the entry point changed the device's free memory"
        assert np.array_equal(sb.cpu().numpy(), sa.cpu().numpy())
        assert np.allclose(wb.cpu().numpy(), wa.cpu().numpy(), rtol=1e-6)
        ua, ub = xa.cpu().numpy() - x0, xb.cpu().numpy() - x0
        assert rel_l2(ub, ua) <= TOL_REL_L2
    ctx.close()


def test_noalloc_refuses_layers_beyond_its_scratch():
    import clutor_b200 as cb
    lib = cb.lib()
    err = C.create_string_buffer(512)
    layer = synth.device_layer(E=256, FF=4096, NE=8, K=8, seed=5)   # n_used * n_ff_exp = 32768 > 16384
    s = cb.layer_struct(layer)
    import torch
    x = torch.zeros((1, 256), device="cuda")
    rc = lib.clb200_moe_ffn_decode_noalloc(C.byref(s), x.data_ptr(), None, None, None, err, 512)
    assert rc == 1 and b"n_used * n_ff_exp" in err.value


def _refused(s, x):
    import clutor_b200 as cb
    err = C.create_string_buffer(512)
    before = x.clone()
    rc = cb.lib().clb200_moe_ffn_decode_noalloc(C.byref(s), x.data_ptr(), None, None, None, err, 512)
    import torch
    torch.cuda.synchronize()
    assert rc == 1, "the entry point accepted a layer it cannot run"
    assert torch.equal(x, before), "the kernel ran on a refused layer"
    return err.value.decode()


def test_noalloc_refuses_what_the_context_path_refuses():
    """Widths beyond the kernel's 4096, gate and up of different types, and slab sizes that do not match rows x row bytes
    are refused before anything is launched, with the context path's messages."""
    import torch

    import clutor_b200 as cb
    layer = synth.device_layer(E=512, FF=256, NE=16, K=4, seed=6)
    x = torch.ones((1, 512), device="cuda")
    s = cb.layer_struct(layer)                       # E = 8192 with K = 1: fits the scratch, not the kernel
    s.n_embd, s.n_used = 8192, 1
    s.gate.cols = s.up.cols = s.down.rows = 8192
    assert "between 256 and 4096" in _refused(s, x)
    s = cb.layer_struct(layer)                       # FF = 8192 with K = 1
    s.n_ff_exp, s.n_used = 8192, 1
    s.gate.rows = s.up.rows = s.down.cols = 8192
    assert "between 256 and 4096" in _refused(s, x)
    s = cb.layer_struct(layer)                       # a Q4_K gate with a Q6_K up
    s.up.type = synth.T_Q6_K
    assert "share a type" in _refused(s, x)
    s = cb.layer_struct(layer)                       # a gate slab one row short
    s.gate_slab -= 144 * 2
    assert "slab sizes" in _refused(s, x)

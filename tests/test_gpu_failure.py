"""Failure paths, made on purpose without a GPU fault (needs a B200).

* A device wait that runs out: CLB200_OPT_TEST_STALL_WAIT points the one-token kernel's wait for the router logits at a
  count that no CTA reaches, with a limit of about a millisecond. Every CTA takes its error path; the host call, or
  clb200_status after a device call, reports the wait's error code; the next call, with the hook off, gives the oracle's
  result (the counters were reset).
* A store fill that fails (a host-side injection, clb200_store_inject_fill_failure): the stored block returns 1 with a
  message, every handle of the layer goes back (as the reference's forward pass releases them, c/src/forward.c:1000-1001),
  and the store stays failed (the reference's sticky flag, c/src/xs.c:79-80).
"""
import numpy as np
import pytest

import oracle
from clutor_b200 import synth

pytestmark = pytest.mark.gpu

STALL_POLLS = 1 << 14   # about a millisecond of polling


@pytest.fixture(scope="module")
def ctx():
    import clutor_b200 as cb
    c = cb.Context(0)
    yield c
    c.close()


def same_as_oracle(got, L, x):
    want = oracle.moe_ffn(L, x, "oracle")
    assert np.array_equal(got[1], want[1])
    assert np.array_equal(got[0].view(np.uint32), want[0].view(np.uint32))


def test_stalled_wait_on_a_host_call(ctx):
    import clutor_b200 as cb
    L = synth.host_layer(E=1024, FF=512, NE=64, K=6, seed=21)
    x = synth.activations(1, 1024, seed=22)
    same_as_oracle(ctx.moe_ffn(L, x), L, x)
    ctx.set_option(ctx.OPT_TEST_STALL_WAIT, STALL_POLLS)
    try:
        with pytest.raises(cb.ClutorError, match="router logits"):
            ctx.moe_ffn(L, x)
        with pytest.raises(cb.ClutorError, match="router logits"):   # twice: the graph of the host call takes the hook too
            ctx.moe_ffn(L, x)
    finally:
        ctx.set_option(ctx.OPT_TEST_STALL_WAIT, 0)
    for s in range(3):   # the counters the failed launches left are cleared: calls are correct again
        x = synth.activations(1, 1024, seed=30 + s)
        same_as_oracle(ctx.moe_ffn(L, x), L, x)


def test_stalled_wait_on_device_calls(ctx):
    import torch

    import clutor_b200 as cb
    L = synth.device_layer(E=1024, FF=512, NE=64, K=6, seed=23)
    h = ctx.bind(L)
    HL = synth.to_host(L)
    x0 = synth.activations(1, 1024, seed=24)
    ctx.set_option(ctx.OPT_TEST_STALL_WAIT, STALL_POLLS)
    try:
        x = torch.from_numpy(x0).cuda()
        ctx.moe_ffn_dev(h, x)
        ctx.moe_ffn_dev(h, x)                          # a second failing launch queued behind the first
        with pytest.raises(cb.ClutorError, match="device error 1"):
            ctx.status()
        assert torch.equal(x.cpu(), torch.from_numpy(x0)), "a failed launch changed x"
    finally:
        ctx.set_option(ctx.OPT_TEST_STALL_WAIT, 0)
    ctx.status()                                       # the error word was cleared with the report
    x = torch.from_numpy(x0).cuda()
    sel = torch.zeros((1, 6), dtype=torch.int32, device="cuda")
    ctx.moe_ffn_dev(h, x, sel)
    ctx.status()
    want = oracle.moe_ffn(HL, x0, "oracle")
    assert np.array_equal(sel.cpu().numpy(), want[1])
    assert np.array_equal(x.cpu().numpy().view(np.uint32), want[0].view(np.uint32))


def test_failed_fill_releases_every_handle(ctx):
    import torch

    import clutor_b200 as cb
    NL, E, FF, NE, K = 3, 512, 256, 16, 4
    layers = [synth.host_layer(E=E, FF=FF, NE=NE, K=K, seed=700 + i) for i in range(NL)]
    st = cb.Store(ctx, layers[0], NL, cache_bytes=8 * (layers[0].expert_bytes + 256), stage_slots=0, policy=cb.WTINYLFU)
    for i, L in enumerate(layers):
        st.load_layer(i, L)
    x = torch.from_numpy(synth.activations(1, E, seed=5)).cuda()[0]
    wt = np.full(K, 0.25, np.float32)
    st.experts(0, x, np.arange(K, dtype=np.int32), wt)     # a healthy step
    torch.cuda.synchronize()
    assert not st.failed()
    st.log(True)
    st.inject_fill_failure(2)                              # the second miss of the next step fails
    with pytest.raises(cb.ClutorError, match="reading expert"):
        st.experts(1, x, np.arange(4, 4 + K, dtype=np.int32), wt)
    log = st.read_log()
    st.log(False)
    in_cache = [int(r) & 0xffff for op, _, r in log if op == 1 and r >= 0]
    unpinned = [int(a) for op, a, _ in log if op == 3]
    assert sorted(in_cache) == sorted(unpinned), (in_cache, unpinned)   # every requested slot went back
    assert st.failed()
    with pytest.raises(cb.ClutorError, match="reading expert"):       # the failure is sticky, as the reference's
        st.experts(2, x, np.arange(K, dtype=np.int32), wt)
    torch.cuda.synchronize()
    st.close()
    ctx.status()

"""The phase-trace summary (clutor_b200/trace.py) names boundaries that the one-token kernels stamp, in the order thread 0
passes them (checked against decode.cu's and group.cu's sources; no GPU)."""
import os
import re

from clutor_b200 import trace

CSRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "clutor_b200", "csrc")
SOURCES = {"grid": os.path.join(CSRC, "decode.cu"), "group": os.path.join(CSRC, "group.cu")}


def stamps_in_order(kernel):
    text = open(SOURCES[kernel]).read()
    return [int(m.group(1)) for m in re.finditer(r"trace_stamp\(a\.trace, (\d+)\)", text)]


def test_phases_follow_thread0_order():
    for kernel, (_, phases, _) in trace.KERNELS.items():
        order = stamps_in_order(kernel)
        assert order[0] == 0 and len(order) == len(set(order)), (kernel, order)
        want = [b for b, _ in phases]
        assert set(want) <= set(order), kernel
        assert [b for b in order if b in set(want)] == want, kernel   # the summary walks the boundaries in source order


def test_entry_exit_and_router_stamps_exist():
    for kernel, (_, _, (_, rb1)) in trace.KERNELS.items():
        text = open(SOURCES[kernel]).read()
        assert "trace_time(a.trace, 30)" in text and "trace_time(a.trace, 31)" in text
        assert f"trace_stamp_here(a.trace, {rb1})" in text

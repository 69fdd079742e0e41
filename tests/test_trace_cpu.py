"""The phase-trace summary (clutor_b200/trace.py) names boundaries that the one-token kernel stamps, in the order thread 0
passes them (checked against decode.cu's source; no GPU)."""
import os
import re

from clutor_b200 import trace

SRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "clutor_b200", "csrc", "decode.cu")


def stamps_in_order():
    text = open(SRC).read()
    return [int(m.group(1)) for m in re.finditer(r"trace_stamp\(a\.trace, (\d+)\)", text)]


def test_phases_follow_thread0_order():
    order = stamps_in_order()
    assert order[0] == 0 and len(order) == len(set(order)), order
    want = [b for b, _ in trace.PHASES]
    assert set(want) <= set(order)
    assert [b for b in order if b in set(want)] == want   # the summary walks the boundaries in source order


def test_entry_exit_and_router_stamps_exist():
    text = open(SRC).read()
    assert "trace_time(a.trace, 30)" in text and "trace_time(a.trace, 31)" in text
    assert "trace_stamp_here(a.trace, 5)" in text

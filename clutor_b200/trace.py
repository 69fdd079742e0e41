"""Phase trace of the one-token MoE kernels (clb200_set_trace) over a chain of layers replayed from a CUDA graph.

    python -m clutor_b200.trace [--layers 48] [--down q4_k] [--kernel group|grid]

--kernel group (the default) traces the expert-group kernel (group.cu), grid the grid-wide one (decode.cu). Each layer's
launch gets its own trace buffer (32 entries per CTA): thread 0 of every CTA writes its SM's cycle counter at each phase
boundary and the global nanosecond timer at entry and exit. The summary gives, per phase, the
median over CTAs 0-127 and over the layers after the first eight of the cycles between consecutive boundaries, in
microseconds at the SM clock the trace itself gives (cycles over global-timer nanoseconds from entry to exit); and,
from the global timer, the launch span and the gap between launches.
"""
from __future__ import annotations

import argparse

import numpy as np

# thread 0's boundaries in the order it passes them (group.cu), and the boundary the scoring warp stamps after its logits
GROUP_PHASES = [
    (1, "dependency wait"), (2, "x, sum of squares, norm weights landed"), (3, "rmsnorm"), (5, "all logits gathered"),
    (6, "ranking by logit"), (7, "copies issued"), (8, "softmax, probability order, weights"), (9, "gate/up rows (warp 0)"),
    (10, "the group's hg gathered"), (11, "Q8_K of hg, down rows landed"), (12, "down rows"), (13, "weighted rows published"),
    (19, "chunk combine, exit"),
]
GROUP_ROUTER = (3, 4)
# finer points inside the group kernel's phases: (name, from boundary, to boundary); 28 is the softmax warp's lane 0
GROUP_DETAIL = [("thread 0's logit polls", 3, 21), ("gather barrier", 21, 5), ("rank loop", 5, 22), ("rank barrier", 22, 23),
                ("copy issue (thread 0)", 6, 24), ("first row group landed, from the copies", 24, 25),
                ("named barrier wait (warp 0)", 25, 26), ("gate/up loop end (warp 0)", 25, 27),
                ("round barrier", 27, 8), ("softmax warp: copies issued to verdict", 7, 28)]
# the same for the grid-wide kernel (decode.cu)
PHASES = [
    (1, "dependency wait"), (2, "x, sum of squares"), (3, "router rows landed"), (4, "rmsnorm, router products"),
    (6, "Q8_K of xn"), (7, "all logits visible"), (8, "logits staged, max"), (21, "rank by logit"),
    (23, "gate/up copies issued"), (11, "barrier"), (12, "down copies issued"), (9, "exponentials, double sum"), (10, "probabilities"),
    (20, "barrier"), (22, "probability order checked, weights"), (25, "first expert slot landed"), (26, "first gate/up block"), (13, "gate/up rows"), (14, "hg rows released"),
    (15, "all hg visible"), (16, "Q8_K of hg"), (17, "down rows landed"), (18, "down rows"), (19, "combine, residual"),
]
GRID_ROUTER = (4, 5)
KERNELS = {"group": (0, GROUP_PHASES, GROUP_ROUTER), "grid": (1, PHASES, GRID_ROUTER)}
# the whole-model step (fwd.cu), one layer: thread 0's boundaries in order; the attention CTAs' own steps (query heads
# c, c + G, ...); the step's last boundary (12: after the last layer's closing grid barrier)
MODEL_PHASES = [
    (14, "rmsnorm, Q8_K, dense rows landed"), (1, "QKV rows"), (2, "grid barrier"), (4, "attention (32 CTAs), grid barrier"),
    (5, "Q8_K of att, O rows, residual"), (6, "grid barrier"), (7, "ffn rmsnorm, router products, Q8_K of xn"),
    (20, "all logits visible"), (21, "rank by logit, copies issued"), (22, "softmax"), (8, "probability order, weights"),
    (9, "gate/up rows"),
    (10, "grid barrier"), (23, "Q8_K of hg"), (24, "down rows landed"), (25, "down rows"), (11, "combine, residual"),
    (12, "grid barrier"),
]
ASSUMED_MHZ = 1950.0
MODEL_DETAIL = [("(MoE) probability check", 22, 27), ("(MoE) renormalisation", 27, 8)]
MODEL_ATTENTION = [("(attention CTAs) q, k, v, scores", 2, 15), ("(attention CTAs) softmax", 15, 16),
                   ("(attention CTAs) values", 16, 17), ("(attention CTAs) to the barrier's end", 17, 4)]


def run(n_layers: int = 48, down: str = "q4_k", replays: int = 20, kernel: str = "group", cooperative: bool = True) -> dict:
    import torch

    import clutor_b200 as cb
    from clutor_b200 import synth

    option, phases, (rb0, rb1) = KERNELS[kernel]
    ctx = cb.Context(0)
    ctx.set_option(ctx.OPT_DECODE_KERNEL, option)
    ctx.set_option(ctx.OPT_COOPERATIVE, int(cooperative))
    try:
        layers = [synth.device_layer(E=2048, FF=768, NE=128, K=8, gate_type=synth.T_Q4_K, down_type=synth.TYPE_NAMES[down],
                                     seed=i + 1, router_scale=0.02) for i in range(n_layers)]
        handles = [ctx.bind(L) for L in layers]
        x0 = torch.from_numpy(synth.activations(1, 2048, seed=11)).cuda()
        x = x0.clone()
        sel = torch.zeros((n_layers, 1, 8), dtype=torch.int32, device="cuda")
        wt = torch.zeros((n_layers, 1, 8), dtype=torch.float32, device="cuda")
        G = torch.cuda.get_device_properties(0).multi_processor_count
        tr = torch.zeros((n_layers, G, 32), dtype=torch.int64, device="cuda")
        st = torch.cuda.Stream()

        def step():
            for i, h in enumerate(handles):
                ctx.set_trace(tr[i])
                ctx.moe_ffn_dev(h, x, sel[i], wt[i], stream=st)
            ctx.set_trace(None)

        with torch.cuda.stream(st):
            step()
        ctx.status()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            step()
        for _ in range(5):
            g.replay()
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(st):
            ev0.record(st)
            for _ in range(replays):
                g.replay()
            ev1.record(st)
        torch.cuda.synchronize()
        ctx.status()
        us_per_layer = ev0.elapsed_time(ev1) * 1000.0 / replays / n_layers
        t = tr.cpu().numpy().astype(np.int64)
        del g
    finally:
        ctx.close()
    lay = slice(min(8, n_layers - 1), n_layers - 1)
    cta = slice(0, min(128, t.shape[1]))
    # the SM clock from the trace itself: cycles between the first and last boundary over nanoseconds between entry and exit
    mhz = float(np.median((t[lay, cta, 19] - t[lay, cta, 0]) / (t[lay, cta, 31] - t[lay, cta, 30]))) * 1000.0
    to_us = 1.0 / mhz   # cycles -> us
    rows, prev = [], 0
    for b, name in phases:
        d = (t[lay, cta, b] - t[lay, cta, prev]) * to_us
        rows.append((name, float(np.median(d)), float(np.percentile(d, 90))))
        prev = b
    router = float(np.median((t[lay, cta, rb1] - t[lay, cta, rb0]) * to_us))
    detail = []
    if kernel == "group":
        for name, b0, b1 in GROUP_DETAIL:
            d = (t[lay, cta, b1] - t[lay, cta, b0]) * to_us
            detail.append((name, float(np.median(d)), float(np.percentile(d, 90))))
    ent, ex = t[:, :, 30], t[:, :, 31]
    span = float(np.median(((ex.max(1) - ent.min(1)) / 1000.0)[lay]))
    gap = float(np.median(((ent[1:].min(1) - ex[:-1].max(1)) / 1000.0)[lay]))
    return {"us_per_layer": us_per_layer, "sm_mhz": mhz, "phases": rows, "router_warp_us": router, "launch_span_us": span,
            "gap_to_next_launch_us": gap, "detail": detail}


def run_model(n_layers: int = 48, warm: int = 60, steps: int = 12) -> dict:
    """The whole-model step (fwd.cu) at positions warm .. warm + steps - 1: each step launched alone with the trace on;
    the stamps of its last layer (every layer overwrites them), medians over CTAs 0-127 and the steps."""
    import dataclasses

    import torch

    import clutor_b200 as cb
    from clutor_b200 import synth_model as sm
    from clutor_b200.model import Model

    spec = dataclasses.replace(sm.QWEN3_30B_A3B, n_layer=n_layers)
    image = sm.image(spec, seed=1)
    ctx = cb.Context(0)
    try:
        model = Model(ctx, image, warm + steps + 8)
        tok = model.generate(1, warm)[-1]
        G = torch.cuda.get_device_properties(0).multi_processor_count
        tr = torch.zeros((steps, G, 32), dtype=torch.int64, device="cuda")
        for i in range(steps):
            ctx.set_trace(tr[i])
            _, tok, _ = model.step(tok, logits=False)
        ctx.set_trace(None)
        torch.cuda.synchronize()
        t = tr.cpu().numpy().astype(np.int64)
        n_head = spec.n_head
        model.close()
    finally:
        ctx.close()
    cta = slice(0, min(128, t.shape[1]))
    # the boundaries are SM cycles and only the step's entry and exit are global time, so the cycles are read at the
    # clock these B200s hold under this load (1,945-1,965 MHz in every bench's clock record)
    ns = (t[:, cta, 31] - t[:, cta, 30]).astype(np.float64)
    to_us = 1.0 / ASSUMED_MHZ
    rows, prev = [], 0
    for b, name in MODEL_PHASES:
        d = (t[:, cta, b] - t[:, cta, prev]) * to_us
        rows.append((name, float(np.median(d)), float(np.percentile(d, 90))))
        prev = b
    att = slice(0, min(n_head, t.shape[1]))
    detail = []
    for name, b0, b1 in MODEL_ATTENTION:
        d = (t[:, att, b1] - t[:, att, b0]) * to_us
        detail.append((name, float(np.median(d)), float(np.percentile(d, 90))))
    layer = float(np.median((t[:, cta, 12] - t[:, cta, 0]) * to_us))
    for name, b0, b1 in MODEL_DETAIL:
        d = (t[:, cta, b1] - t[:, cta, b0]) * to_us
        detail.append((name, float(np.median(d)), float(np.percentile(d, 90))))
    reranked = float(np.mean(t[:, cta, 26] != 0))
    return {"step_us": float(np.median(ns)) / 1000.0, "layer_us": layer, "phases": rows, "attention": detail,
            "reranked": reranked}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--down", default="q4_k", choices=["q4_k", "q6_k"])
    ap.add_argument("--kernel", default="group", choices=sorted(KERNELS) + ["model"])
    ap.add_argument("--plain-launch", action="store_true", help="launch without the cooperative attribute")
    a = ap.parse_args()
    if a.kernel == "model":
        r = run_model(a.layers)
        print(f"whole step {r['step_us']:.1f} us (global timer, entry to exit, traced); last layer {r['layer_us']:.2f} us at an "
              "assumed 1950 MHz SM clock")
        print("| phase (thread 0 of each CTA, last layer) | median us | p90 us |")
        print("|---|---|---|")
        for name, med, p90 in r["phases"]:
            print(f"| {name} | {med:.3f} | {p90:.3f} |")
        for name, med, p90 in r["attention"]:
            print(f"| (detail) {name} | {med:.3f} | {p90:.3f} |")
        print(f"last layers ranked again by probability (a tie on the logit order): {100 * r['reranked']:.1f} %")
        return
    r = run(a.layers, a.down, kernel=a.kernel, cooperative=not a.plain_launch)
    print(f"{r['us_per_layer']:.2f} us per layer (CUDA events, traced graph), SM clock {r['sm_mhz']:.0f} MHz (from the trace)")
    print("| phase (thread 0 of each CTA) | median us | p90 us |")
    print("|---|---|---|")
    for name, med, p90 in r["phases"]:
        print(f"| {name} | {med:.3f} | {p90:.3f} |")
    for name, med, p90 in r.get("detail", []):
        print(f"| (detail) {name} | {med:.3f} | {p90:.3f} |")
    print(f"scoring warp (from the boundary before its products to its logits stored): {r['router_warp_us']:.3f} us; launch span {r['launch_span_us']:.3f} us, "
          f"gap to the next launch {r['gap_to_next_launch_us']:.3f} us")


if __name__ == "__main__":
    main()

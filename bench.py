"""Benchmark of the MoE feed-forward hot path on B200.

Default workload (N=1 per GPU): the Qwen3-30B-A3B MoE layer at decode, one token (hidden 2048, 128 experts, top-8,
intermediate 768, Q4_K experts, fp32 router). A step is one token through a pool of `--layers` distinct layers (48, about
16 GB of expert weights, far larger than the 126 MB L2), chained: each layer's output is the next one's input, replayed
from a CUDA graph. The metric is MoE-layer tokens per second (layer-token = one token through one layer).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload decode|prefill64|cache] [--impl ours|reference]

Under torchrun with N > 1 every rank runs the same workload on its own GPU (the decode layer does not shard: replicas),
value = all ranks' layer-tokens / the slowest rank's time. --impl reference times the reference engine's own CPU code
(oracle/_ref, built from its sources) on the host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
METRIC = "MoE-layer tokens/s (decode, Qwen3-30B-A3B layer, Q4_K)"

WORKLOADS = {
    # name: (T, gate type, down type, E, FF, NE, K, layers)
    "decode": dict(T=1, gate="q4_k", down="q4_k", E=2048, FF=768, NE=128, K=8, layers=48,
                   desc="Qwen3-30B-A3B MoE layer, decode T=1, Q4_K experts"),
    "prefill64": dict(T=64, gate="q8_0", down="q8_0", E=2048, FF=768, NE=128, K=8, layers=8,
                      desc="Qwen3-30B-A3B MoE layer, T=64, Q8_0 experts"),
    "ep235b": dict(T=2048, gate="q4_k", down="q4_k", E=4096, FF=1536, NE=128, K=8, layers=2,
                   desc="Qwen3-235B-A22B MoE layer, prefill 2048 tokens per GPU, Q4_K experts, expert-parallel over the GPUs "
                        "(rows and partial sums over peer memory from this library's kernels)"),
    "model": dict(T=1, gate="q4_k", down="q6_k", E=2048, FF=768, NE=128, K=8, layers=48,
                  desc="Qwen3-30B-A3B whole model, greedy decode at batch 1 from a 1-token prompt: 48 layers, GQA 32/4 heads "
                       "x 128, QK-norm, NEOX rotary (base 1e6), fp16 key/value cache, Q4_K_M mix (Q4_K embedding, attn_q/k/o and "
                       "gate/up experts; Q6_K attn_v, down experts and the 151,936-row output matrix)"),
    "prompt": dict(T=64, gate="q4_k", down="q6_k", E=2048, FF=768, NE=128, K=8, layers=48, P=512,
                   desc="Qwen3-30B-A3B whole model, a 512-token prompt fed through the batched prompt path (the reference's "
                        "cl_fwd_prefill / run_std) in batches of 64 tokens (its batch for a model in memory), logits after "
                        "the last token; same model as 'model'"),
    "cache": dict(T=1, gate="q4_k", down="q4_k", E=2048, FF=768, NE=128, K=8, layers=48, budget=0.4, locality=1.78,
                  desc="expert-cache stress: 48 Qwen3-30B-A3B MoE layers (Q4_K), HBM cache of 40% of expert bytes, the rest "
                       "in pinned host memory, Zipf(1.1)-skewed routing with topics drifting every 16 tokens"),
}


def peaks() -> tuple[dict, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return json.load(open(p)), "measured"
    return PEAKS_FALLBACK, "fallback"


def layer_bytes(wl: dict, distinct: float) -> float:
    """Algorithmic bytes of one call: the distinct experts' gate/up/down slabs, the fp32 router, the norm weights, and x in
    and out."""
    from clutor_b200 import synth
    g = synth.TYPE_NAMES[wl["gate"]]
    d = synth.TYPE_NAMES[wl["down"]]
    E, FF, NE, T = wl["E"], wl["FF"], wl["NE"], wl["T"]
    expert = 2 * FF * synth.row_bytes(g, E) + E * synth.row_bytes(d, FF)
    return distinct * expert + NE * E * 4 + E * 4 + 2 * T * E * 4


class Clocks:
    """Samples the SM clock and the clock-event (throttle) reasons every millisecond through NVML during the timed region
    (nvidia-smi cannot sample a region this short)."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap",
               0x80: "hw_power_brake_slowdown"}

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.rows: list[tuple[int, int, int]] = []
        self.stop = threading.Event()
        self.t = None
        self.error = None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)

            def poll():
                while not self.stop.is_set():
                    try:
                        self.rows.append((pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM), self.max_mhz,
                                          pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)))
                    except Exception as e:  # keep the timing run alive; report what failed
                        self.error = str(e)
                        return
                    time.sleep(0.001)
            self.t = threading.Thread(target=poll, daemon=True)
            self.t.start()
        except Exception as e:
            self.error = f"NVML unavailable: {e}"
        return self

    def __exit__(self, *exc):
        self.stop.set()
        if self.t:
            self.t.join()

    def summary(self) -> dict:
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.error or "not sampled"]}
        reasons = sorted({name for _, _, r in self.rows for bit, name in self.REASONS.items() if r & bit})
        return {"sm_mhz": statistics.median(r[0] for r in self.rows), "sm_max_mhz": self.rows[0][1], "reasons": reasons,
                "samples": len(self.rows), "source": "NVML, 1 ms polling"}


def read_traffic(kernel: str) -> float | None:
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary (profiles/), if there is one."""
    p = os.path.join(ROOT, "profiles", f"{kernel}.md")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


def cpu_reference(wl: dict, seconds: float, threads: int | None = None) -> dict:
    """The reference engine's CPU path (oracle/_ref) on a bounded sample of the workload: one layer, fresh activations per
    call, all host threads (the reference caps its pool at 16)."""
    import numpy as np

    import oracle
    from clutor_b200 import synth
    if not oracle.ref_available():
        oracle.build(need_ref=True)
    nthreads = threads or min(os.cpu_count() or 1, 16)
    oracle.set_ref_threads(nthreads)
    L = synth.host_layer(E=wl["E"], FF=wl["FF"], NE=wl["NE"], K=wl["K"], gate_type=synth.TYPE_NAMES[wl["gate"]],
                         down_type=synth.TYPE_NAMES[wl["down"]], seed=1, router_scale=0.05 if wl["T"] > 1 else 0.02)
    xs = [synth.activations(wl["T"], wl["E"], seed=1000 + i) for i in range(8)]
    for i in range(2):
        oracle.moe_ffn(L, xs[i], "ref")
    n = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        oracle.moe_ffn(L, xs[n % len(xs)], "ref")
        n += 1
    dt = time.perf_counter() - t0
    path = oracle.ref_lib().cl_quant_path().decode()
    return {"value": n * wl["T"] / dt, "unit": "layer-tokens/s", "cores": nthreads, "kind": "reference",
            "sample": f"{n} calls of one layer ({wl['T']} token(s) each) in {dt:.1f} s on {nthreads} threads, ISA path {path}; "
                      f"reference built from its sources (oracle/_ref)", "ms_per_call": 1000 * dt / n}


MODEL_METRIC = "full-model decode tokens/s (Qwen3-30B-A3B, Q4_K_M mix, batch 1)"
SHM_MODEL = "/dev/shm/clutor_b200_qwen3_30b_a3b.gguf"


def model_reference(image, n_ctx: int, seconds: float, threads: int | None = None) -> dict:
    """The reference engine's own forward pass (cl_fwd_open / cl_fwd_step, oracle/_ref) on the same synthetic model, from a
    GGUF file in shared memory (the reference opens models by path): greedy steps from a 1-token prompt for about
    `seconds`, all host threads (the reference caps its pool at 16)."""
    import numpy as np

    import oracle
    if not oracle.ref_available():
        oracle.build(need_ref=True)
    nthreads = threads or min(os.cpu_count() or 1, 16)
    oracle.set_ref_threads(nthreads)
    image.tofile(SHM_MODEL)
    try:
        ref = oracle.RefModel(SHM_MODEL, n_ctx)
        tok, n = 1, 0
        logits, _, _ = ref.step(tok)        # the first step pages the weights in
        tok = int(np.argmax(logits))
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < seconds and n < n_ctx - 2:
            logits, _, _ = ref.step(tok)
            tok = int(np.argmax(logits))
            n += 1
        dt = time.perf_counter() - t0
        ref.close()
    finally:
        os.unlink(SHM_MODEL)
    path = oracle.ref_lib().cl_quant_path().decode()
    return {"value": n / dt, "unit": "tokens/s", "cores": nthreads, "kind": "reference",
            "sample": f"{n} greedy decode steps (positions 1..{n}) of the whole model in {dt:.1f} s on {nthreads} threads, ISA "
                      f"path {path}; the reference's cl_fwd_step built from its sources (oracle/_ref), model mapped from "
                      f"/dev/shm", "ms_per_token": 1000 * dt / max(n, 1)}


PROMPT_METRIC = "prompt tokens/s (Qwen3-30B-A3B, Q4_K_M mix, 512-token prompt)"


def prompt_reference(image, P: int, threads: int | None = None) -> dict:
    """The reference's cl_fwd_prefill of the same P-token prompt (run_std in batches of 64), all host threads (up to 16)."""
    import numpy as np

    import oracle
    if not oracle.ref_available():
        oracle.build(need_ref=True)
    nthreads = threads or min(os.cpu_count() or 1, 16)
    oracle.set_ref_threads(nthreads)
    image.tofile(SHM_MODEL)
    try:
        prompt = np.random.default_rng(3).integers(0, 151936, P).astype(np.int32)
        ref = oracle.RefModel(SHM_MODEL, P + 16)
        ref.prefill(prompt[:8], logits=False)   # pages the weights in
        ref.close()
        ref = oracle.RefModel(SHM_MODEL, P + 16)
        t0 = time.perf_counter()
        ref.prefill(prompt)
        dt = time.perf_counter() - t0
        ref.close()
    finally:
        os.unlink(SHM_MODEL)
    return {"value": P / dt, "unit": "tokens/s", "cores": nthreads, "kind": "reference",
            "sample": f"one {P}-token prompt through the reference's cl_fwd_prefill (run_std, batches of 64) in {dt:.1f} s on "
                      f"{nthreads} threads; built from its sources (oracle/_ref), model mapped from /dev/shm"}


def run_prompt(a, wl: dict) -> dict:
    """The batched prompt path of the whole model: a step is one P-token prompt from position 0 (clb200_model_prefill, batches
    of wl["T"] tokens), logits of the last token copied out. The call is synchronous (one synchronization per batch), so it is
    timed on the host clock around the call, after a device synchronize; there are no inputs but the token ids."""
    import numpy as np
    import torch

    import clutor_b200 as cb
    from clutor_b200 import synth_model as sm
    from clutor_b200.model import Model

    torch.cuda.set_device(0)
    spec = sm.QWEN3_30B_A3B
    if a.layers:
        spec = dataclasses.replace(spec, n_layer=a.layers)
    image = sm.image(spec, seed=1)
    ctx = cb.Context(0)
    P, B = wl["P"], (a.batch or wl["T"])
    model = Model(ctx, image, P + 16)
    model.set_batch(B)
    prompt = np.random.default_rng(3).integers(0, spec.vocab, P).astype(np.int32)

    def timed(exact: bool, n: int) -> float:
        ctx.set_exact(exact)
        for _ in range(a.warmup):
            model.reset()
            model.prefill(prompt)
        ts = []
        for _ in range(n):
            model.reset()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            model.prefill(prompt)
            ts.append(time.perf_counter() - t0)
        return max(ts)

    with Clocks(0) as clk:
        dt = timed(False, a.steps)
    dt_exact = timed(True, max(1, a.steps // 4))
    ctx.set_exact(False)
    cpu = None
    if not a.no_cpu_baseline:
        cpu = prompt_reference(image, P)
    mb = sm.model_bytes(spec)
    line = {"metric": PROMPT_METRIC, "value": round(P / dt, 2), "unit": "tokens/s", "n_gpus": 1, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(1000 * dt, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8 dot (Q8_K x K-quant) for dense products; Q4_K experts on tcgen05 from fp16 "
            "hi/lo operands (fp32 accumulate); fp32 attention, fp16 key/value cache",
            "data": "synthetic (seeded random GGUF weights with the model's shapes and types; seeded random prompt)",
            "config": {"workload": wl["desc"], "layers": spec.n_layer, "prompt_tokens": P, "batch": B,
                       "timing": "host clock around the synchronous call (slowest of the timed steps)",
                       "model_bytes": mb["total"], "parallelism": "single GPU"},
            "integer_path_value": round(P / dt_exact, 2),
            "roofline": None, "cpu_baseline": cpu,
            "e2e": {"value": round(P / dt, 2), "unit": "tokens/s", "h2d_bytes_per_step": 4 * P, "d2h_bytes_per_step": 4 * spec.vocab,
                    "api": "clb200_model_prefill (host token ids in, host logits out)"},
            "gpu_launches": None, "clocks": clk.summary()}
    model.close()
    ctx.close()
    return line


def run_reference_arm(a, wl, rank: int) -> None:
    if rank != 0:
        return
    if a.workload == "prompt":
        from clutor_b200 import synth_model as sm
        cb = prompt_reference(sm.image(sm.QWEN3_30B_A3B, seed=1), wl["P"])
        line = {"impl": "reference", "metric": PROMPT_METRIC, "value": round(cb["value"], 3), "unit": "tokens/s",
                "n_gpus": a.gpus, "steps": 1, "warmup": 0, "ms_per_step": round(1000 * wl["P"] / cb["value"], 1),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8 dot (Q8_K x K-quant), fp32",
                "data": "synthetic (seeded random GGUF)", "config": {"workload": wl["desc"]},
                "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": round(cb["value"], 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        line["cpu_baseline"]["value"] = line["value"]   # the line's own value, as rounded
        print(json.dumps(line), flush=True)
        return
    if a.workload == "model":
        from clutor_b200 import synth_model as sm
        image = sm.image(sm.QWEN3_30B_A3B, seed=1)
        secs = max(5.0, min(60.0, 2.0 * a.steps))
        cb = model_reference(image, a.warmup + a.steps + 8, secs)
        line = {"impl": "reference", "metric": MODEL_METRIC, "value": round(cb["value"], 4), "unit": "tokens/s",
                "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(cb["ms_per_token"], 3),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "int8 dot (Q8_K x K-quant), fp32 accumulate; fp32 attention", "data": "synthetic (seeded random GGUF)",
                "config": {"workload": wl["desc"]},
                "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": round(cb["value"], 4), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        line["cpu_baseline"]["value"] = line["value"]   # the line's own value, as rounded
        print(json.dumps(line), flush=True)
        return
    secs = max(5.0, min(60.0, 2.0 * a.steps))
    cb = cpu_reference(wl, secs)
    line = {"impl": "reference", "metric": METRIC if a.workload == "decode" else METRIC.replace("decode", "T=64").replace("Q4_K", "Q8_0"),
            "value": round(cb["value"], 3), "unit": "layer-tokens/s", "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": round(cb["ms_per_call"], 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8 dot (Q8_K x K-quant), fp32 accumulate" if wl["gate"] != "q8_0" else "f32",
            "data": "synthetic (seeded)", "config": layers_config(wl, int(os.environ.get("WORLD_SIZE", "1"))),
            "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": round(cb["value"], 3), "unit": "layer-tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    line["cpu_baseline"]["value"] = line["value"]
    print(json.dumps(line), flush=True)


def run_cache(a, wl: dict) -> dict:
    """The expert-cache stress workload through the HBM expert store. A step is one decode token through every layer; the
    routing of each (token, layer) comes from the reference stress harness's synthetic router (c/src/stream.c:114-140,
    restated in clutor_b200.synth.ExpertStream), top-8 of its logits, and the predictor's logits (correlation 0.8) choose
    what is staged for the next layer, as that harness does. Single GPU (a store is one device's HBM)."""
    import numpy as np
    import torch

    import clutor_b200 as cb
    import oracle
    from clutor_b200 import synth

    torch.cuda.set_device(0)
    NL, NE, K, E = wl["layers"], wl["NE"], wl["K"], wl["E"]
    ctx = cb.Context(0)
    mk = lambda i: synth.device_layer(E=E, FF=wl["FF"], NE=NE, K=K, gate_type=synth.TYPE_NAMES[wl["gate"]],
                                      down_type=synth.TYPE_NAMES[wl["down"]], seed=i + 1, router_scale=0.02)
    first = mk(0)
    expert_bytes = first.expert_bytes
    budget = int(wl["budget"] * NL * NE * expert_bytes)
    store = cb.Store(ctx, first, NL, cache_bytes=budget, stage_slots=2 * K, policy=cb.WTINYLFU)
    store.set_prefetch_depth(a.prefetch_depth)
    store.load_layer(0, first)
    del first
    for i in range(1, NL):
        L = mk(i)
        store.load_layer(i, L)
        del L
    torch.cuda.empty_cache()
    # routing of every (token, layer): the harness's logits, top-K, weights renormalised over the K
    ntok = a.warmup + a.steps
    gen = synth.ExpertStream(NL, NE, locality=wl["locality"], seed=1, rho=0.8)
    toks = np.arange(ntok)
    sel = np.zeros((NL, ntok, K), np.int32)
    wt = np.zeros((NL, ntok, K), np.float32)
    pred = np.zeros((NL, ntok, K), np.int32)
    lg_all = np.zeros((NL, ntok, NE), np.float32)
    for l in range(NL):
        lg_all[l] = gen.logits(toks, l)
        sel[l], p = synth.route_topk(lg_all[l], K)
        wt[l] = p / p.sum(axis=1, keepdims=True, dtype=np.float32)
        pred[l] = synth.route_topk(gen.logits(toks, l, predicted=True), K)[0]
    smart = tuple(t(v) for t, v in zip((int, int, float), a.smart.split(","))) if a.smart else None
    if smart:   # SMART-ROUTE (c/src/stream.c:288-291): each (token, layer) routed on the device against the resident set
        store.set_smart(smart)
        pz = np.exp(lg_all.astype(np.float64) - lg_all.max(axis=2, keepdims=True))
        probs = (pz / pz.sum(axis=2, keepdims=True)).astype(np.float32)
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream
    x = torch.from_numpy(synth.activations(1, E, seed=11)).cuda()[0]
    store.log(True)

    # the store's C entry point called as a C host calls it: argument values prepared once, the routing arrays addressed
    # in place (sel / wt / pred are C-contiguous [layer, token, K])
    import ctypes as C
    fn, errb = cb.lib().clb200_moe_experts_stored, C.create_string_buffer(512)
    sel, wt, pred = (np.ascontiguousarray(v) for v in (sel, wt, pred))
    if 0 < a.prefetch_n < K:   # stage only the predictor's top prefetch_n (the reference's --prefetch-n); -1 stages nothing
        pred[:, :, a.prefetch_n:] = -1
    row = K * 4
    ctx_h, store_h, xp = C.c_void_p(ctx.handle), C.c_void_p(store.h), C.c_void_p(x.data_ptr())
    sel0, wt0, pred0 = sel.ctypes.data, wt.ctypes.data, pred.ctypes.data

    def token(t):
        for l in range(NL):
            nxt = pred[l + 1, t] if l + 1 < NL else None
            if smart:
                s = np.array(store.route(l, lg_all[l, t])["selected"], np.int32)
                w = probs[l, t, s]
                store.experts(l, x, s, (w / w.sum(dtype=np.float32)).astype(np.float32), nxt, stream=sp)
            else:
                o = (l * ntok + t) * row
                if fn(ctx_h, store_h, l, xp, sel0 + o, wt0 + o, pred0 + ((l + 1) * ntok + t) * row if l + 1 < NL else None, sp, errb, 512):
                    raise cb.ClutorError(errb.value.decode())

    for t in range(a.warmup):
        token(t)
    torch.cuda.synchronize()
    ctx.status()
    store.reset_stats()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(0) as clk:
        ev0.record(stream)
        for t in range(a.warmup, ntok):
            token(t)
        ev1.record(stream)
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    ctx.status()
    st = store.stats()
    # the policy decisions, replayed on the reference's own cache.c
    log = store.read_log()
    ref = oracle.RefCache(store.cache_slots() - 2 * K - 1, 2 * K, NL * NE, cb.WTINYLFU)
    mism = 0
    for op, k, r in log:
        if op == 1:
            code, slot = ref.access(int(k))
            mism += (code * 65536 + slot if code >= 0 else -1) != r
        elif op == 2:
            mism += ref.stage(int(k)) != r
        else:
            ref.unpin(int(k))
    ref.close()
    # the host-to-device link: one 1 GiB copy from pinned memory
    hb = torch.empty(1 << 30, dtype=torch.uint8).pin_memory()
    db = torch.empty(1 << 30, dtype=torch.uint8, device="cuda")
    db.copy_(hb, non_blocking=True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    db.copy_(hb, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    link = (1 << 30) / (e0.elapsed_time(e1) / 1000.0) / 1e9
    del hb, db
    h2d = (st["demand_bytes"] + st["prefetch_bytes"]) / (ms / 1000.0) / 1e9
    hit = st["hits"] / max(st["accesses"], 1)
    value = a.steps / (ms / 1000.0)
    cpu = None
    if not a.no_cpu_baseline:
        dec = dict(WORKLOADS["decode"])
        cpu = cpu_reference(dec, a.cpu_seconds)
        cpu.pop("ms_per_call", None)
        cpu["value"] = round(cpu["value"] / NL, 3)
        cpu["unit"] = "tokens/s"
        cpu["sample"] = cpu.get("sample", "") + f"; tokens/s = layer-tokens/s / {NL} layers, every expert in RAM"
    line = {"metric": "decode tokens/s through the HBM expert cache (48 Qwen3-30B-A3B MoE layers, Q4_K)",
            "value": round(value, 3), "unit": "tokens/s", "n_gpus": 1, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": round(ms / a.steps, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8 dot (Q8_K x K-quant), fp32 accumulate", "data": "synthetic (seeded GGUF blocks; routing from the reference harness's synthetic router)",
            "config": {"workload": wl["desc"], "layers": NL, "experts": NE, "top_k": K, "hidden": E, "ff": wl["FF"],
                       "expert_bytes": expert_bytes, "hbm_cache_bytes": budget, "cache_slots": store.cache_slots(),
                       "stage_slots": 2 * K, "prefetch_depth": a.prefetch_depth, "prefetch_n": a.prefetch_n or K, "policy": "W-TinyLFU", "locality": wl["locality"], "predict_corr": 0.8,
                       "parallelism": "single GPU", "l2": "expert bytes 16 GB, far beyond L2"},
            "cache": {"hit_rate": round(hit, 4), "stage_hits": st["stage_hits"], "misses": st["misses"],
                      "prefetch_issued": st["prefetch_issued"], "prefetch_late": st["prefetch_late"],
                      "prefetch_wasted": st["prefetch_wasted"], "evictions": st["evictions"],
                      "prefetch_overlap": round(1.0 - st["wait_ns"] / max(st["copy_ns"], 1), 4),
                      "copy_ms": round(st["copy_ns"] / 1e6, 3), "wait_ms": round(st["wait_ns"] / 1e6, 3),
                      "policy_replay_on_reference": f"{len(log)} operations, {mism} mismatches",
                      "smart_route": None if not smart else dict(J=smart[0], M=smart[1], tau=smart[2], **store.smart_stats())},
            "roofline": {"bound": "h2d", "achieved": round(h2d, 2), "peak": round(link, 2), "unit": "GB/s",
                         "frac": round(h2d / link, 4), "traffic": None, "peak_kind": "measured here: one 1 GiB pinned copy"},
            "cpu_baseline": cpu,
            "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0,
                    "note": "the step is host-driven already: routing on the host, the public C entry point per layer"},
            "gpu_launches": NL * a.steps, "clocks": clk.summary()}
    store.close()
    ctx.close()
    del store, ctx
    torch.cuda.empty_cache()
    return line


EP_METRIC = "MoE-layer tokens/s (Qwen3-235B-A22B layer, prefill 2048 tokens/GPU, Q4_K, expert-parallel)"


def ep_measure(steps: int, warmup: int, rank: int, world: int, local: int, dist=None, layers: int | None = None, exchange: str = "peer",
               clocks: bool = False) -> dict | None:
    """Expert-parallel MoE layers of the Qwen3-235B-A22B shape on the `world` ranks of the process
    group, one per GPU: each rank holds the router and 128/N experts of every layer. A step is one pass of the tokens through
    `layers` layers, one all-to-all each way per layer (NCCL over NVLink). Two runs: weak scaling (2048 tokens routed by
    every rank) and strong scaling (the config's one 2048-token prefill split over the ranks). Rank 0 also times the phases
    of one step, counts the bytes it sends to the other ranks, and checks its tokens of layer 0 against the single-GPU
    block on the whole layer (top-k identical, relative L2 <= 1e-5). Every rank takes the same collective steps; rank 0
    returns the summary, the others None."""
    import numpy as np
    import torch

    import clutor_b200 as cb
    from clutor_b200 import ep, synth

    wl = WORKLOADS["ep235b"]
    T, NL, K, E, FF, NE = wl["T"], layers or wl["layers"], wl["K"], wl["E"], wl["FF"], wl["NE"]
    n_local = NE // world
    ctx = cb.Context(local)
    comps, keep, full0 = [], [], None
    for i in range(NL):
        L = synth.device_layer(E=E, FF=FF, NE=NE, K=K, gate_type=synth.TYPE_NAMES[wl["gate"]],
                               down_type=synth.TYPE_NAMES[wl["down"]], seed=i + 1, router_scale=0.02)
        sh = ep.shard_layer(L, rank, world)
        g, u, d = sh.gate.clone(), sh.up.clone(), sh.down.clone()
        mk = lambda ne, router: synth.DeviceLayer(E=E, FF=FF, NE=ne, K=K, gate_type=L.gate_type, up_type=L.up_type,
                                                  down_type=L.down_type, ffn_norm=L.ffn_norm, router=router, gate=g, up=u, down=d)
        route_layer = mk(NE, L.router)              # norm + router; routing never reads the expert pointers
        shard_layer = mk(n_local, sh.router.clone())
        keep.append((route_layer, shard_layer))
        comps.append(ep.GpuCompute(ctx, ctx.bind(route_layer), ctx.bind(shard_layer), E, K))
        if i == 0 and rank == 0:
            full0 = (L, ctx.bind(L))                # rank 0 keeps layer 0 whole for the parity check
        del L, sh
        torch.cuda.empty_cache()

    # the exchange: stores into the other GPUs' memory from the library's kernels (default), or NCCL all-to-alls
    xchg = None
    if dist and exchange == "peer":
        try:
            xchg = ep.PeerExchange(ctx, T, E, K)
        except RuntimeError as e:   # every rank gives up together (the constructor agrees on it): NCCL instead
            exchange = f"nccl ({e})"

    def timed_run(Tr: int, seed: int):
        x0 = torch.from_numpy(synth.activations(Tr, E, seed=seed + rank)).cuda()
        x = x0.clone()

        def step(timed=None):
            x.copy_(x0)
            for c in comps:
                ep.moe_layer(x, c, n_local, 1.0, timings=timed, xchg=xchg)

        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        ctx.status()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        ev0.record()
        for _ in range(steps):
            step()
        ev1.record()
        torch.cuda.synchronize()
        ms = ev0.elapsed_time(ev1)
        ctx.status()
        phases: dict = {}
        step(phases)   # one more step with the phase events (not timed above)
        torch.cuda.synchronize()
        if dist:
            t = torch.tensor([ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms, phases

    with Clocks(local) if clocks else _NoClocks() as clk:
        ms_w, ph_w = timed_run(T, 11)
        ms_s, ph_s = timed_run(T // world, 31)
    parity = None
    if dist:
        dist.barrier()
    # the parity step is a collective (every rank runs layer 0 on 256 tokens of its own); rank 0 checks its tokens against
    # the whole layer on its own GPU
    xr = torch.from_numpy(synth.activations(256, E, seed=77 + rank)).cuda()
    xe = xr.clone()
    sel_e, _ = ep.moe_layer(xe, comps[0], n_local, 1.0, xchg=xchg)
    torch.cuda.synchronize()
    if full0 is not None:
        L, h = full0
        xb = xr.clone()
        selb = torch.zeros((256, K), dtype=torch.int32, device="cuda")
        ctx.moe_ffn_dev(h, xb, selb)
        ctx.status()
        err = float(torch.linalg.norm((xe - xb).double()) / torch.linalg.norm((xb - xr).double()))
        parity = {"tokens": 256, "layer": 0, "topk_identical": bool(torch.equal(sel_e, selb)), "rel_l2": err,
                  "bar": 1e-5, "ok": bool(torch.equal(sel_e, selb) and err <= 1e-5),
                  "against": "the single-GPU block on the whole layer (clb200_moe_ffn_dev)"}
    if xchg is not None:
        xchg.close()
    del comps, keep, full0
    ctx.close()
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    pk, pk_kind = peaks()

    def summary(ms: float, Tr: int, ph: dict, scaling: str) -> dict:
        value = NL * Tr * steps * world / (ms / 1000.0)
        flop = Tr * K * 3 * 2 * E * FF * NL * steps * world   # algorithmic expert FLOPs of all ranks
        achieved = flop / (ms / 1000.0) / 1e12 / world      # per GPU
        per = {k: round(sum(ev[0].elapsed_time(ev[1]) for ev in v) / NL, 4) for k, v in ph.items() if k not in ("rows", "xbytes")}
        xb = float(np.mean(ph.get("xbytes", [0])))
        xms = per.get("dispatch", 0.0) + per.get("combine", 0.0)
        return {"value": round(value, 3), "unit": "layer-tokens/s", "ms_per_step": round(ms / steps, 4), "scaling": scaling,
                "tokens_per_gpu": Tr, "tokens_total": Tr * world, "phases_ms_per_layer_rank0": per,
                "rows_received_rank0": int(np.mean(ph.get("rows", [0]))),
                "exchange_rank0": {"bytes_per_layer": int(xb), "exchange_ms_per_layer": round(xms, 4),
                                   "gbs": round(xb / (xms * 1e-3) / 1e9, 2) if xms > 0 else None,
                                   "note": "bytes rank 0 sends to the other ranks per layer (dispatched Q8_K rows out, "
                                           "partial sums back) over the dispatch + combine all-to-all time"},
                "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": pk.get("bf16_tflops"),
                             "unit": "TFLOP/s per GPU", "frac": round(achieved / pk.get("bf16_tflops", 1.0), 4),
                             "peak_kind": pk_kind}}

    return {"workload": wl["desc"], "metric": EP_METRIC, "n_gpus": world, "layers_per_step": NL, "steps": steps,
            "warmup": warmup, "hidden": E, "experts": NE, "experts_per_gpu": n_local, "top_k": K, "ff": FF,
            "parallelism": f"ep{world}",
            "exchange": ("stores into the other GPUs' memory from the library's kernels (CUDA IPC mappings), arrival signals "
                         "waited on in a kernel; no host synchronisation" if exchange == "peer" else
                         "NCCL all_to_all_single (counts, rows, partial sums)" + (exchange[4:] if exchange.startswith("nccl (") else ""))
                        if world > 1 else "none (one GPU)",
            "weak": summary(ms_w, T, ph_w, "weak"), "strong": summary(ms_s, T // world, ph_s, "strong"),
            "parity_rank0": parity, "clocks": clk.summary() if clocks else None,
            # this library's kernels a layer step launches: route 3, pack 2, experts 7, combine 1, and with the peer exchange
            # its push, wait, push-back and wait
            "gpu_launches_per_layer": 16 if (world > 1 and exchange == "peer") else 13, "dtype": "int8 dot (Q8_K x Q4_K) exact router; Q4_K experts on tcgen05 from fp16 hi/lo "
            "operands, fp32 accumulate"}


class _NoClocks:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


def run_ep(a, wl: dict) -> None:
    """The expert-parallel workload alone (--workload ep235b, under torchrun for N > 1): its weak-scaling figures as the
    line's value."""
    import datetime

    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    r = ep_measure(a.steps, a.warmup, rank, world, local, dist if world > 1 else None, layers=a.layers, clocks=True,
                   exchange=a.ep_exchange)
    if rank == 0:
        w = r["weak"]
        line = {"metric": EP_METRIC, "value": w["value"], "unit": "layer-tokens/s", "n_gpus": world, "steps": a.steps,
                "warmup": a.warmup, "ms_per_step": w["ms_per_step"], "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": r["dtype"], "data": "synthetic (seeded random GGUF blocks)",
                "config": {"workload": wl["desc"], "tokens_per_gpu": wl["T"], "layers_per_step": r["layers_per_step"],
                           "hidden": wl["E"], "experts": wl["NE"], "experts_per_gpu": r["experts_per_gpu"], "top_k": wl["K"],
                           "ff": wl["FF"], "parallelism": f"ep{world}",
                           "l2": f"inputs larger than L2: {r['layers_per_step']} layers, "
                                 f"{wl['NE'] * wl['E'] * wl['FF'] * 3 * 144 / 256 / 1e9 * r['layers_per_step'] / world:.2f} GB of experts per GPU"},
                "roofline": w["roofline"], "ep": r, "cpu_baseline": None, "e2e": None,
                "gpu_launches": r["layers_per_step"] * a.steps * r["gpu_launches_per_layer"], "clocks": r["clocks"]}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_model(a, wl: dict, own_group: bool = True) -> dict | None:
    """The whole model, one token per step: the persistent one-step kernel (fwd.cu) replayed from a graph, each step
    feeding the previous step's greedy choice. Every rank runs its own replica (the model does not shard)."""
    import numpy as np
    import torch

    import clutor_b200 as cb
    from clutor_b200 import synth_model as sm
    from clutor_b200.model import Model

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        if own_group:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    spec = sm.QWEN3_30B_A3B
    if a.layers:   # a shorter stack of the same layers (small ncu captures); the default is the whole model
        spec = dataclasses.replace(spec, n_layer=a.layers)
    t_img = time.perf_counter()
    image = sm.image(spec, seed=1)
    t_img = time.perf_counter() - t_img
    ctx = cb.Context(local)
    n_ctx = a.warmup + 2 * a.steps + 16
    model = Model(ctx, image, n_ctx)
    W, K = a.warmup, a.steps
    first = 1
    warm = model.generate(first, W)          # positions 0..W-1; captures the one-step graph
    stream = torch.cuda.Stream()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        with torch.cuda.stream(stream):
            ev0.record(stream)
            model.generate_async(warm[-1], K, stream.cuda_stream)   # positions W..W+K-1
            ev1.record(stream)
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    toks = model.tokens(W, K)
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = K * world / (ms / 1000.0)
    ms_per_step = ms / K
    mb = sm.model_bytes(spec)
    avg_pos = W + (K - 1) / 2.0
    kv_bytes = 2 * 2 * spec.n_kvw * spec.n_layer * (avg_pos + 1)      # keys and values read per token, half precision
    bytes_per_token = mb["total"] + mb["embedding_row"] + kv_bytes
    pk, pk_kind = peaks()
    achieved = bytes_per_token / (ms_per_step * 1e-3) / 1e9
    roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
            "frac": round(achieved / pk["hbm_gbs"], 4), "traffic": read_traffic("fwd_kernel_model"), "peak_kind": pk_kind,
            "kernel": "fwd_kernel", "bytes_per_launch": int(bytes_per_token), "launch_us": round(1000 * ms_per_step, 2),
            "note": "one launch per token: experts 1.175 GB + attention 0.523 GB + routers 50 MB + output 255 MB + "
                    "key/value reads at the mean position"}
    # end to end through the public API with host buffers: clb200_model_generate (state up, tokens down, synchronous)
    e2e = None
    if not a.no_e2e:
        model.reset()
        model.generate(first, W)
        t0 = time.perf_counter()
        out = model.generate(warm[-1], K)
        dt = time.perf_counter() - t0
        if dist:
            tt = torch.tensor([dt], device="cuda")
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            dt = float(tt.item())
        same = out == toks
        e2e = {"value": round(K * world / dt, 3), "unit": "tokens/s", "h2d_bytes_per_step": round(24 / K, 3),
               "d2h_bytes_per_step": round(4 + 24 / K, 3), "api": "clb200_model_generate (host token buffer, synchronous)",
               "same_tokens_as_timed_run": same}
    cpu = None
    if rank == 0 and not a.no_cpu_baseline:
        cpu = model_reference(image, W + K + 8, a.cpu_seconds)
        cpu.pop("ms_per_token", None)
    if rank == 0:
        line = {"metric": MODEL_METRIC, "value": round(value, 3), "unit": "tokens/s", "n_gpus": world, "steps": K,
                "warmup": W, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "int8 dot (Q8_K x K-quant), fp32 accumulate; fp32 attention, fp16 key/value cache",
                "data": "synthetic (seeded random GGUF weights with the model's shapes and types)",
                "config": {"workload": wl["desc"], "layers": spec.n_layer, "model_bytes": mb["total"], "positions": [W, W + K - 1],
                           "parallelism": f"replicas x{world}", "l2": "inputs larger than L2: 2.0 GB of weights per token",
                           "image_seconds": round(t_img, 1)},
                "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": K, "clocks": clk.summary(),
                "tokens": toks[:16]}
    model.close()
    ctx.close()
    del model, ctx, image
    torch.cuda.empty_cache()
    if dist and own_group:
        dist.destroy_process_group()
    return line if rank == 0 else None


def layers_config(wl: dict, world: int) -> dict:
    """The config object of the layer-pool workloads (decode, prefill64), shared by both arms of the bench."""
    from clutor_b200 import synth
    g, d = synth.TYPE_NAMES[wl["gate"]], synth.TYPE_NAMES[wl["down"]]
    expert = 2 * wl["FF"] * synth.row_bytes(g, wl["E"]) + wl["E"] * synth.row_bytes(d, wl["FF"])
    return {"workload": wl["desc"], "tokens_per_call": wl["T"], "layers_per_step": wl["layers"], "hidden": wl["E"],
            "experts": wl["NE"], "top_k": wl["K"], "ff": wl["FF"], "parallelism": f"replicas x{world}",
            "l2": f"inputs larger than L2: {wl['layers']} distinct layers, {wl['layers'] * wl['NE'] * expert / 1e9:.1f} GB of experts"}


def run_layers(a, wl: dict, rank: int, world: int, local: int, dist) -> dict | None:
    """The layer-pool workloads (decode: BASELINE config 1; prefill64: config 2): a step is the tokens through `layers`
    distinct layers, chained, replayed from a CUDA graph; every rank runs its own replica (the layer does not shard)."""
    import numpy as np
    import torch

    import clutor_b200 as cb
    from clutor_b200 import synth

    T, NL, K = wl["T"], wl["layers"], wl["K"]
    ctx = cb.Context(local)
    layers = [synth.device_layer(E=wl["E"], FF=wl["FF"], NE=wl["NE"], K=K, gate_type=synth.TYPE_NAMES[wl["gate"]],
                                 down_type=synth.TYPE_NAMES[wl["down"]], seed=1000 * rank + i + 1,
                                 router_scale=0.05 if T > 1 else 0.02) for i in range(NL)]
    handles = [ctx.bind(L) for L in layers]
    x0 = torch.from_numpy(synth.activations(T, wl["E"], seed=11 + rank)).cuda()
    x = x0.clone()
    sel = torch.zeros((NL, T, K), dtype=torch.int32, device="cuda")
    wt = torch.zeros((NL, T, K), dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()

    def step():
        for i, h in enumerate(handles):
            ctx.moe_ffn_dev(h, x, sel[i], wt[i], stream=stream)

    # warm up eagerly once (sizes the scratch), then capture one step into a graph
    with torch.cuda.stream(stream):
        step()
    ctx.status()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    for _ in range(a.warmup):
        x.copy_(x0)
        graph.replay()
    torch.cuda.synchronize()
    ctx.status()
    launches_per_step = NL * (1 if T == 1 else 7)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for _ in range(a.steps):
                graph.replay()
            ev1.record(stream)
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    ctx.status()
    if dist:
        dist.barrier()
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    units = NL * T * a.steps * world
    value = units / (ms / 1000.0)
    ms_per_step = ms / a.steps
    # roofline of the dominant kernel (the whole step is its launches)
    distinct = float(np.mean([len(np.unique(sel[i].cpu().numpy())) for i in range(NL)]))
    bytes_per_launch = layer_bytes(wl, distinct)
    launch_us = 1000.0 * ms_per_step / NL
    pk, pk_kind = peaks()
    achieved = bytes_per_launch / (launch_us * 1e-6) / 1e9
    kernel = "moe_decode_kernel" if T == 1 else "moe_batched"
    roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
            "frac": round(achieved / pk["hbm_gbs"], 4), "traffic": read_traffic(f"{kernel}_{a.workload}"),
            "peak_kind": pk_kind, "kernel": kernel, "bytes_per_launch": int(bytes_per_launch), "launch_us": round(launch_us, 3)}

    # end to end through the host-pointer entry point (clb200_moe_ffn): x from pinned host memory in, x/sel/wt back out
    e2e = None
    if not a.no_e2e:
        ne = min(NL, 16)
        host_layers = [synth.to_host(L) for L in layers[:ne]]
        structs = [cb.layer_struct(L) for L in host_layers]
        xh = torch.from_numpy(synth.activations(T, wl["E"], seed=21 + rank)).pin_memory()
        selh = torch.zeros((T, K), dtype=torch.int32).pin_memory()
        wth = torch.zeros((T, K), dtype=torch.float32).pin_memory()
        xn, sn, wn = xh.numpy(), selh.numpy(), wth.numpy()
        for s in structs:                # the first call of each layer uploads its weights
            ctx.moe_ffn_inplace(s, xn, sn, wn)
        # the calls as a C host makes them: the argument values prepared once (ctypes converts nothing per call)
        import ctypes as C
        fn, errb = cb.lib().clb200_moe_ffn, C.create_string_buffer(512)
        calls = [(C.c_void_p(ctx.handle), C.byref(s), C.c_void_p(xn.ctypes.data), T, C.c_void_p(sn.ctypes.data),
                  C.c_void_p(wn.ctypes.data), errb, 512) for s in structs]
        if dist:
            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(a.steps):
            for args in calls:
                if fn(*args):
                    raise cb.ClutorError(errb.value.decode())
        dt = time.perf_counter() - t0
        if dist:
            tt = torch.tensor([dt], device="cuda")
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            dt = float(tt.item())
        e2e = {"value": round(ne * T * a.steps * world / dt, 3), "unit": "layer-tokens/s",
               "h2d_bytes_per_step": ne * T * wl["E"] * 4, "d2h_bytes_per_step": ne * T * (wl["E"] * 4 + 2 * K * 4),
               "calls_per_step": ne, "api": "clb200_moe_ffn (host pointers, synchronous)"}
    cpu = None
    if rank == 0 and not a.no_cpu_baseline:
        cpu = cpu_reference(wl, a.cpu_seconds)
        cpu.pop("ms_per_call", None)
    line = None
    if rank == 0:
        line = {"metric": METRIC if a.workload == "decode" else METRIC.replace("decode", "T=64").replace("Q4_K", "Q8_0"),
                "value": round(value, 3), "unit": "layer-tokens/s", "n_gpus": world, "steps": a.steps,
                "warmup": a.warmup, "ms_per_step": round(ms_per_step, 5), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "int8 dot (Q8_K x K-quant), fp32 accumulate" if wl["gate"] != "q8_0" else "f32",
                "data": "synthetic (seeded random GGUF blocks)", "config": layers_config(wl, world),
                "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches_per_step * a.steps,
                "clocks": clk.summary()}
    del graph, layers, handles
    ctx.close()
    torch.cuda.empty_cache()
    return line


def secondary(a) -> list:
    """The other configurations on one GPU, each as its own line (value, roofline, the reference's CPU figure, clocks) with
    shorter runs: T = 64 with Q8_0 experts, the whole model's decode (config 3) and the expert-cache
    stress (config 5, its 4096 decode steps)."""
    out = []
    for name, steps, warmup in (("prefill64", 20, 3), ("model", 32, 3), ("cache", 4096, 16)):
        b = argparse.Namespace(**vars(a))
        b.workload, b.steps, b.warmup, b.layers, b.cpu_seconds, b.smart = name, steps, warmup, None, 5.0, None
        wl = dict(WORKLOADS[name])
        t0 = time.perf_counter()
        try:
            line = {"prefill64": lambda: run_layers(b, wl, 0, 1, 0, None), "model": lambda: run_model(b, wl, own_group=False),
                    "cache": lambda: run_cache(b, wl)}[name]()
            line["workload"] = name
            line["wall_s"] = round(time.perf_counter() - t0, 1)
        except Exception as e:   # one configuration failing must not lose the headline line
            line = {"workload": name, "error": f"{type(e).__name__}: {e}"}
        out.append(line)
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="decode")
    ap.add_argument("--layers", type=int, default=None, help="distinct layers in the pool (default: the workload's)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--prefetch-depth", type=int, default=2, help="cache workload: prefetch fills in flight at once")
    ap.add_argument("--prefetch-n", type=int, default=4,
                    help="cache workload: experts a prediction stages (the reference's --prefetch-n; 0: n_used). 4 is the "
                         "fastest measured: on a link-bound workload every wrong prediction costs a 2.65 MB copy")
    ap.add_argument("--smart", default=None, help="cache workload: SMART-ROUTE J,M,TAU (for example 2,12,0.015)")
    ap.add_argument("--batch", type=int, default=None, help="prompt workload: tokens per batch (the reference's CLUTOR_PS_B, 1..512)")
    ap.add_argument("--no-ep", action="store_true", help="decode workload: leave out the expert-parallel figures")
    ap.add_argument("--ep-exchange", choices=["peer", "nccl"], default="peer",
                    help="expert parallelism over N > 1 GPUs: stores into peer memory from the library's kernels, or NCCL")
    ap.add_argument("--no-secondary", action="store_true", help="decode workload at N=1: leave out the other configurations")
    a = ap.parse_args()
    wl = dict(WORKLOADS[a.workload])
    if a.layers:
        wl["layers"] = a.layers
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if a.impl == "reference":
        run_reference_arm(a, wl, rank)
        return
    if a.workload == "cache":
        print(json.dumps(run_cache(a, wl)), flush=True)
        return
    if a.workload == "prompt":
        print(json.dumps(run_prompt(a, wl)), flush=True)
        return
    if a.workload == "ep235b":
        run_ep(a, wl)
        return
    if a.workload == "model":
        line = run_model(a, wl)
        if line:
            print(json.dumps(line), flush=True)
        return

    import torch
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    line = run_layers(a, wl, rank, world, local, dist)
    if a.workload == "decode" and not a.no_ep:   # the sharded configuration (config 4) at this N, every rank taking part
        ep = ep_measure(5, 2, rank, world, local, dist, exchange=a.ep_exchange)
        if rank == 0:
            line["ep"] = ep
    if a.workload == "decode" and world == 1 and not a.no_secondary:
        line["secondary"] = secondary(a)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()



if __name__ == "__main__":
    main()

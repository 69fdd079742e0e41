"""The expert-parallel exchange (clutor_b200.ep) on CPU ranks over gloo: routing, dispatch plan, row packing, the two
all-to-alls and the rank-ordered combine, with the oracle standing in for the CUDA kernels on both sides.

Bar: each rank's tokens come out as the single-process block (oracle.moe_ffn) computes them: top-k identical, x within
1e-5 relative L2 (only the order of the fp32 additions over a token's experts differs).
"""
import os
import socket

import numpy as np
import pytest
import torch

import oracle
from clutor_b200 import ep, synth

E, FF, NE, K, T = 256, 256, 8, 2, 12


class OracleCompute(ep.Compute):
    """Both halves of the block from the oracle's scalar functions (c/src restated), on numpy."""

    def __init__(self, full, shard):
        self.full, self.shard = full, shard

    def route(self, x):
        L = self.full
        xs = x.numpy()
        sel = np.zeros((len(xs), K), np.int32)
        wt = np.zeros((len(xs), K), np.float32)
        qs = np.zeros((len(xs), E), np.int8)
        d = np.zeros((len(xs), E // 256), np.float32)
        bs = np.zeros((len(xs), E // 16), np.int16)
        for t, row in enumerate(xs):
            xn = oracle.rmsnorm(row, L.ffn_norm, L.rms_eps)
            q = oracle.q8k_quantize(xn)
            logits = np.array([oracle.dotf(L.router[e], xn) for e in range(L.NE)], np.float32)
            sel[t], wt[t] = oracle.route(logits, K, L.norm_topk)
            qs[t], d[t], bs[t] = q["qs"].reshape(-1), q["d"], q["bsums"].reshape(-1)
        return tuple(torch.from_numpy(a) for a in (sel, wt, qs, d, bs))

    def _expert(self, e, q8):
        L = self.shard
        grb, drb = synth.row_bytes(L.gate_type, E), synth.row_bytes(L.down_type, FF)
        g = np.array([oracle.dot_row(L.gate_type, L.gate[e * L.gate_slab + j * grb:][:grb], E, q8, None) for j in range(FF)], np.float32)
        u = np.array([oracle.dot_row(L.up_type, L.up[e * L.up_slab + j * grb:][:grb], E, q8, None) for j in range(FF)], np.float32)
        h = (g / (np.float32(1) + np.exp(-g)) * u).astype(np.float32)
        hq = oracle.q8k_quantize(h)
        return np.array([oracle.dot_row(L.down_type, L.down[e * L.down_slab + i * drb:][:drb], FF, hq, None) for i in range(E)], np.float32)

    def experts(self, qs, d, bs, sel_local, wt):
        R = qs.shape[0]
        out = np.zeros((R, E), np.float32)
        sl, w = sel_local.numpy(), wt.numpy()
        first = {}
        for s, e in enumerate(sl.reshape(-1)):   # each expert's first appearance over the (row, k) slots
            if e >= 0 and e not in first:
                first[int(e)] = s
        for t in range(R):
            q8 = np.zeros(E // 256, oracle.Q8K_DTYPE)
            q8["qs"] = qs[t].numpy().reshape(-1, 256)
            q8["d"] = d[t].numpy()
            q8["bsums"] = bs[t].numpy().reshape(-1, 16)
            m = np.zeros(E, np.float32)
            for k in sorted((k for k in range(K) if sl[t, k] >= 0), key=lambda k: first[int(sl[t, k])]):
                m = (m + w[t, k] * self._expert(int(sl[t, k]), q8)).astype(np.float32)
            out[t] = m
        return torch.from_numpy(out)


def _rank(rank, world, port):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = synth.host_layer(E=E, FF=FF, NE=NE, K=K, seed=5, gate_type=synth.T_Q4_K, down_type=synth.T_Q6_K, router_scale=0.3)
        shard = ep.shard_layer(full, rank, world)
        x0 = synth.activations(T, E, seed=40 + rank)
        x = torch.from_numpy(x0.copy())
        sel, wt = ep.moe_layer(x, OracleCompute(full, shard), NE // world, full.resid_scale)
        want, wsel, wwt = oracle.moe_ffn(full, x0)
        assert np.array_equal(sel.numpy(), wsel), f"rank {rank}: top-k"
        assert np.array_equal(wt.numpy(), wwt), f"rank {rank}: weights"
        d, wd = x.numpy().astype(np.float64) - x0, want.astype(np.float64) - x0
        err = np.linalg.norm(d - wd) / np.linalg.norm(wd)
        assert err <= 1e-5, f"rank {rank}: relative L2 of the update {err:.2e}"
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [1, 2, 4])
def test_expert_parallel_exchange_matches_the_block(world):
    import torch.multiprocessing as mp
    mp.start_processes(_rank, args=(world, _free_port()), nprocs=world, join=True, start_method="spawn")


def test_dispatch_plan_covers_every_slot_once():
    sel = torch.tensor([[0, 5], [7, 1], [2, 3], [6, 4]], dtype=torch.int32)
    idx, lsel = ep.dispatch_plan(sel, 4, 2)
    seen = set()
    for r in range(4):
        for i, t in enumerate(idx[r].tolist()):
            for k in range(2):
                if lsel[r][i, k] >= 0:
                    seen.add((t, int(lsel[r][i, k]) + 2 * r, k))
                    assert sel[t, k] == lsel[r][i, k] + 2 * r
    assert len(seen) == sel.numel()
    fmt = ep.RowFormat(256, 2)
    cols = dict(qs=torch.randint(-127, 128, (3, 256), dtype=torch.int8), d=torch.rand(3, 1), bs=torch.randint(-99, 99, (3, 16), dtype=torch.int16),
                sel=torch.tensor([[0, -1], [1, 0], [-1, 1]], dtype=torch.int32), wt=torch.rand(3, 2))
    back = fmt.unpack(fmt.pack(**cols))
    for k, v in cols.items():
        assert torch.equal(back[k], v)


class StubCompute(ep.Compute):
    """Cheap halves for the exchange-only tests: a fixed routing per token, experts that return zeros."""

    def __init__(self, n_experts):
        self.NE = n_experts

    def route(self, x):
        T = x.shape[0]
        sel = torch.stack([torch.arange(T) % self.NE, (torch.arange(T) + 1) % self.NE], 1).to(torch.int32)
        wt = torch.full((T, K), 0.5)
        return sel, wt, torch.zeros((T, E), dtype=torch.int8), torch.ones((T, E // 256)), torch.zeros((T, E // 16), dtype=torch.int16)

    def experts(self, qs, d, bs, sel_local, wt):
        return torch.zeros((qs.shape[0], E))


def _leaving_rank(rank, world, port, outdir):
    """Every rank takes one exchange step; rank 1 then leaves (its process ends without another collective). The others'
    next step must end in an error within the process group's timeout, not hang."""
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    comp = StubCompute(NE)
    x = torch.from_numpy(synth.activations(T, E, seed=rank))
    ep.moe_layer(x, comp, NE // world, 1.0)
    import time
    if rank == 1:
        # leaves between steps, with no step of its own in flight -- once every other rank has its first step's data
        # (otherwise rows still on their way from this process could be lost with it, and the FIRST step would fail);
        # the others say so through files, not through another collective
        t_end = time.monotonic() + 60.0
        while time.monotonic() < t_end and not all(os.path.exists(os.path.join(outdir, f"step1.{r}")) for r in range(world) if r != 1):
            time.sleep(0.05)
        return
    open(os.path.join(outdir, f"step1.{rank}"), "w").close()
    t0 = time.monotonic()
    try:
        ep.moe_layer(x, comp, NE // world, 1.0)
        outcome = "completed"
    except Exception as e:   # the exchange with the departed rank fails
        outcome = f"error after {time.monotonic() - t0:.1f} s: {type(e).__name__}"
    with open(os.path.join(outdir, f"rank{rank}"), "w") as f:
        f.write(outcome)


@pytest.mark.parametrize("world", [2, 3])
def test_a_rank_that_leaves_ends_the_next_exchange_with_an_error(world, tmp_path):
    import torch.multiprocessing as mp
    mp.start_processes(_leaving_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True, start_method="spawn")
    for r in range(world):
        if r == 1:
            continue
        outcome = (tmp_path / f"rank{r}").read_text()
        assert outcome.startswith("error"), f"rank {r}: {outcome}"
        assert float(outcome.split()[2]) < 60.0, f"rank {r}: {outcome}"

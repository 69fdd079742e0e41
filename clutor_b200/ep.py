"""Expert parallelism for the batched MoE block: the experts of a layer spread over the GPUs of one node, one process per
GPU, with one exchange each way over NCCL (NVLink / NVSwitch).

Every rank holds the router (replicated) and experts [r * n_local, (r + 1) * n_local). A layer step for a rank's own T
tokens:

1. route (source side, clb200_ep_route): rmsnorm, the Q8_K row of xn, router, softmax, top-k, renormalisation -- exactly
   the single-GPU arithmetic, so the routing is bit-identical;
2. dispatch: each token goes once to every rank that holds at least one of its experts: its Q8_K row (the input every
   K-quant expert reads), its K expert ids made local (-1 where the expert is elsewhere) and its K weights, packed as one
   byte row per (token, destination), in ascending token order per destination; one all-to-all of the counts, one of the
   rows;
3. expert side (clb200_ep_experts): the received rows of all sources as one batch through the local experts; per row the
   weighted sum of its present experts (no residual);
4. combine: one all-to-all back of those partial sums; the source adds them per token in rank order and applies the
   residual, x += resid_scale * sum.

Compared with the single-GPU block only the order of the fp32 additions over a token's experts differs (per-rank partial
sums, then ranks in order), so outputs agree to about 1e-7 relative and the top-k is identical.

The exchange logic is generic over a `Compute` (the CUDA kernels here; an oracle stand-in on the CPU in the tests) and
any torch.distributed process group (NCCL on GPUs, gloo on the CPU).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch


@dataclass
class RowFormat:
    """Byte layout of one dispatched row: Q8_K qs [E] int8, d [E/256] fp32, bsums [E/16] int16, sel [K] int32, wt [K] fp32."""
    E: int
    K: int

    @property
    def parts(self):
        E, K = self.E, self.K
        return [("qs", torch.int8, E), ("d", torch.float32, E // 256), ("bs", torch.int16, E // 16),
                ("sel", torch.int32, K), ("wt", torch.float32, K)]

    @property
    def nbytes(self) -> int:
        return sum(n * torch.tensor([], dtype=dt).element_size() for _, dt, n in self.parts)

    def pack(self, **cols) -> torch.Tensor:
        """cols: name -> [n, width] tensors; returns [n, nbytes] uint8."""
        return torch.cat([cols[name].contiguous().view(torch.uint8).reshape(cols[name].shape[0], -1) for name, _, _ in self.parts], dim=1)

    def unpack(self, rows: torch.Tensor) -> dict:
        out, o = {}, 0
        for name, dt, n in self.parts:
            w = n * torch.tensor([], dtype=dt).element_size()
            out[name] = rows[:, o:o + w].contiguous().view(dt).reshape(rows.shape[0], n)
            o += w
        return out


class Compute:
    """The two local halves of the block; see GpuCompute."""

    def route(self, x: torch.Tensor):
        """-> (sel [T,K] int32, wt [T,K] f32, qs [T,E] int8, d [T,E/256] f32, bs [T,E/16] int16)"""
        raise NotImplementedError

    def experts(self, qs, d, bs, sel_local, wt) -> torch.Tensor:
        """-> partial [R,E] f32: per row, the weighted sum of its present local experts."""
        raise NotImplementedError

    def pack(self, fmt: "RowFormat", sel, wt, qs, d, bs, n_ranks: int, n_local: int):
        """The rows each token sends: -> (send [S, nbytes] uint8 in destination order, tokens ascending within one;
        plan, an opaque value for combine; counts per destination as a list)."""
        t_idx, _, lsel, counts = flat_plan(sel, n_ranks, n_local)
        return fmt.pack(qs=qs[t_idx], d=d[t_idx], bs=bs[t_idx], sel=lsel, wt=wt[t_idx]), t_idx, counts

    def combine(self, x, back, plan, counts, resid_scale: float) -> None:
        """x += resid_scale * (each token's returned partial sums added in rank order)."""
        t_idx = plan
        msum = torch.zeros_like(x)
        o = 0
        for c in counts:   # ranks in order; a token appears at most once per rank, so each addition is one per token
            if c:
                msum[t_idx[o:o + c]] += back[o:o + c]
            o += c
        x += resid_scale * msum


class GpuCompute(Compute):
    """The CUDA kernels: a context, the full layer bound for routing and this rank's expert shard bound for the experts."""

    def __init__(self, ctx, route_handle: int, shard_handle: int, E: int, K: int, stream=None):
        from . import lib
        self.ctx, self.L, self.rh, self.sh, self.E, self.K = ctx, lib(), route_handle, shard_handle, E, K
        self.stream = stream
        self._err = C.create_string_buffer(512)
        L = self.L
        L.clb200_ep_route.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int] + [C.c_void_p] * 6 + [C.c_char_p, C.c_size_t]
        L.clb200_ep_experts.argtypes = [C.c_void_p, C.c_int, C.c_int] + [C.c_void_p] * 7 + [C.c_char_p, C.c_size_t]
        L.clb200_ep_pack.argtypes = [C.c_void_p] + [C.c_int] * 5 + [C.c_void_p] * 9 + [C.c_char_p, C.c_size_t]
        L.clb200_ep_combine.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_float,
                                        C.c_void_p, C.c_char_p, C.c_size_t]

    def _s(self):   # ordered with the torch work around each call
        from . import _stream
        return _stream(self.stream)

    def route(self, x):
        T, E, K = x.shape[0], self.E, self.K
        dev = x.device
        sel = torch.empty((T, K), dtype=torch.int32, device=dev)
        wt = torch.empty((T, K), dtype=torch.float32, device=dev)
        qs = torch.empty((T, E), dtype=torch.int8, device=dev)
        d = torch.empty((T, E // 256), dtype=torch.float32, device=dev)
        bs = torch.empty((T, E // 16), dtype=torch.int16, device=dev)
        if self.L.clb200_ep_route(self.ctx.handle, self.rh, x.data_ptr(), T, sel.data_ptr(), wt.data_ptr(), qs.data_ptr(),
                                  d.data_ptr(), bs.data_ptr(), self._s(), self._err, 512):
            raise RuntimeError(self._err.value.decode())
        return sel, wt, qs, d, bs

    def experts(self, qs, d, bs, sel_local, wt):
        R = qs.shape[0]
        out = torch.empty((R, self.E), dtype=torch.float32, device=qs.device)
        if R == 0:
            return out
        if self.L.clb200_ep_experts(self.ctx.handle, self.sh, R, qs.data_ptr(), d.data_ptr(), bs.data_ptr(), sel_local.data_ptr(),
                                    wt.data_ptr(), out.data_ptr(), self._s(), self._err, 512):
            raise RuntimeError(self._err.value.decode())
        return out

    def pack(self, fmt, sel, wt, qs, d, bs, n_ranks, n_local):
        """The plan and the rows in two launches (clb200_ep_pack); one host synchronisation for the counts."""
        T, K = sel.shape
        dev = sel.device
        send = torch.empty((T * n_ranks, fmt.nbytes), dtype=torch.uint8, device=dev)
        slot = torch.empty((T, n_ranks), dtype=torch.int32, device=dev)
        counts = torch.zeros(n_ranks, dtype=torch.int32, device=dev)
        if self.L.clb200_ep_pack(self.ctx.handle, T, self.E, K, n_ranks, n_local, sel.data_ptr(), wt.data_ptr(), qs.data_ptr(),
                                 d.data_ptr(), bs.data_ptr(), send.data_ptr(), slot.data_ptr(), counts.data_ptr(), self._s(),
                                 self._err, 512):
            raise RuntimeError(self._err.value.decode())
        cl = counts.tolist()
        return send[:sum(cl)], slot, cl

    def combine(self, x, back, plan, counts, resid_scale):
        slot = plan
        if self.L.clb200_ep_combine(self.ctx.handle, x.shape[0], self.E, slot.shape[1], slot.data_ptr(), back.data_ptr(), x.data_ptr(),
                                    resid_scale, self._s(), self._err, 512):
            raise RuntimeError(self._err.value.decode())


def flat_plan(sel: torch.Tensor, n_ranks: int, n_local: int):
    """The dispatch on the device with one host synchronisation (the counts, which the exchange needs on the host anyway):
    (t_idx [S], r_idx [S], lsel [S, K], counts [n_ranks] as a list), the (token, destination) pairs a token goes to --
    once per rank that holds at least one of its experts -- in destination order, tokens ascending within a destination;
    lsel the token's expert ids made local to the destination, -1 where the expert is elsewhere."""
    T = sel.shape[0]
    dev = sel.device
    owner = torch.div(sel, n_local, rounding_mode="floor").long()
    hit = torch.zeros((T, n_ranks + 1), dtype=torch.bool, device=dev)   # the last column: experts no rank holds
    if T:
        hit.scatter_(1, owner.clamp(0, n_ranks), True)
    hit = hit[:, :n_ranks]
    counts = hit.sum(0).tolist()
    key = torch.where(hit, torch.arange(n_ranks, device=dev)[None, :] * T + torch.arange(T, device=dev)[:, None], n_ranks * T)
    order = torch.argsort(key.reshape(-1), stable=True)[:sum(counts)]
    t_idx, r_idx = order // n_ranks, order % n_ranks
    lsel = torch.where(owner[t_idx] == r_idx[:, None], sel[t_idx] - (r_idx[:, None] * n_local).to(sel.dtype),
                       torch.full_like(sel[t_idx], -1))
    return t_idx, r_idx, lsel, counts


def dispatch_plan(sel: torch.Tensor, n_ranks: int, n_local: int):
    """Per destination rank: the ascending indices of the tokens that go there and their local sel (-1 elsewhere)."""
    t_idx, _, lsel, counts = flat_plan(sel, n_ranks, n_local)
    return list(torch.split(t_idx, counts)), list(torch.split(lsel, counts))


def moe_layer(x: torch.Tensor, comp: Compute, n_local: int, resid_scale: float, group=None, timings: dict | None = None):
    """One expert-parallel MoE layer step on this rank's tokens x [T, E] (updated in place); returns (sel, wt)."""
    import torch.distributed as dist
    n = dist.get_world_size(group) if dist.is_initialized() else 1
    T, E = x.shape
    cuda = x.is_cuda and timings is not None

    def mark(name):
        if cuda:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            timings.setdefault("_open", {})[name] = ev

    def close(name):
        if cuda:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            timings.setdefault(name, []).append((timings["_open"].pop(name), ev))

    mark("route")
    sel, wt, qs, d, bs = comp.route(x)
    close("route")
    mark("dispatch")
    K = sel.shape[1]
    fmt = RowFormat(E, K)
    send, plan, sc = comp.pack(fmt, sel, wt, qs, d, bs, n, n_local)
    me = dist.get_rank(group) if n > 1 else 0
    if n > 1:
        scount = torch.tensor(sc, dtype=torch.int64, device=x.device)
        rcount = torch.empty_like(scount)
        dist.all_to_all_single(rcount, scount, group=group)
        rc = rcount.tolist()
        recv = torch.empty((sum(rc), fmt.nbytes), dtype=torch.uint8, device=x.device)
        dist.all_to_all_single(recv, send, rc, sc, group=group)
    else:
        rc = sc
        recv = send
    close("dispatch")
    r = fmt.unpack(recv)
    mark("experts")
    partial = comp.experts(r["qs"], r["d"], r["bs"], r["sel"], r["wt"])
    close("experts")
    if timings is not None:
        timings.setdefault("rows", []).append(int(recv.shape[0]))
        # bytes this rank sends to the other ranks: its dispatched rows, then the partial sums of the rows it received
        timings.setdefault("xbytes", []).append(sum(c for d, c in enumerate(sc) if d != me) * fmt.nbytes +
                                                sum(c for d, c in enumerate(rc) if d != me) * E * 4)
    mark("combine")
    if n > 1:
        back = torch.empty((sum(sc), E), dtype=torch.float32, device=x.device)
        dist.all_to_all_single(back, partial, sc, rc, group=group)
    else:
        back = partial
    comp.combine(x, back, plan, sc, resid_scale)
    close("combine")
    if timings is not None:
        timings.pop("_open", None)
    return sel, wt


def shard_layer(layer, rank: int, n_ranks: int):
    """The expert shard [rank * n_local, (rank + 1) * n_local) of a synth layer (the same kind of object, n_local experts,
    views of the layer's tensors). n_used stays the layer's K: the expert side's sel rows have K entries."""
    import copy
    n_local = layer.NE // n_ranks
    if n_local * n_ranks != layer.NE or n_local < layer.K:
        raise ValueError(f"{layer.NE} experts do not split into {n_ranks} shards of at least {layer.K}")
    s = copy.copy(layer)
    e0, e1 = rank * n_local, (rank + 1) * n_local
    s.gate = layer.gate[e0 * layer.gate_slab:e1 * layer.gate_slab]
    s.up = layer.up[e0 * layer.up_slab:e1 * layer.up_slab]
    s.down = layer.down[e0 * layer.down_slab:e1 * layer.down_slab]
    s.router = layer.router[e0:e1]   # unused on the expert side; consistent with n_expert
    s.NE = n_local
    return s

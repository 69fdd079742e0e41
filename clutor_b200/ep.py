"""Expert parallelism for the batched MoE block: the experts of a layer spread over the GPUs of one node, one process per
GPU, with one exchange each way over NVLink / NVSwitch: by default stores straight into the other GPUs' memory from the
library's own kernels (PeerExchange: no library collective and no host synchronisation), or NCCL all-to-alls.

Every rank holds the router (replicated) and experts [r * n_local, (r + 1) * n_local). A layer step for a rank's own T
tokens:

1. route (source side, clb200_ep_route): rmsnorm, the Q8_K row of xn, router, softmax, top-k, renormalisation -- exactly
   the single-GPU arithmetic, so the routing is bit-identical;
2. dispatch: each token goes once to every rank that holds at least one of its experts: its Q8_K row (the input every
   K-quant expert reads), its K expert ids made local (-1 where the expert is elsewhere) and its K weights, packed as one
   byte row per (token, destination), in ascending token order per destination; PeerExchange: a kernel stores each
   destination's rows into that GPU's receive area and signals it with their count (the receiver waits on the signal in a
   kernel); NCCL: one all-to-all of the counts, one of the rows;
3. expert side (clb200_ep_experts): the received rows of all sources as one batch through the local experts; per row the
   weighted sum of its present experts (no residual);
4. combine: the partial sums go back the same way (a store kernel and a signal, or one all-to-all); the source adds them
   per token in rank order and applies the residual, x += resid_scale * sum.

Compared with the single-GPU block only the order of the fp32 additions over a token's experts differs (per-rank partial
sums, then ranks in order), so outputs agree to about 1e-7 relative and the top-k is identical.

The exchange logic is generic over a `Compute` (the CUDA kernels here; an oracle stand-in on the CPU in the tests) and
any torch.distributed process group (NCCL on GPUs, gloo on the CPU).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional

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
        L.clb200_ep_combine_regions.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                                C.c_void_p, C.c_float, C.c_void_p, C.c_char_p, C.c_size_t]

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

    def pack_device(self, fmt, sel, wt, qs, d, bs, n_ranks, n_local):
        """The plan and the rows (clb200_ep_pack) with the counts left on the device: (send [T * n_ranks, nbytes], slot,
        counts [n_ranks] int32 device tensor)."""
        T, K = sel.shape
        dev = sel.device
        send = torch.empty((max(T, 1) * n_ranks, fmt.nbytes), dtype=torch.uint8, device=dev)
        slot = torch.empty((T, n_ranks), dtype=torch.int32, device=dev)
        counts = torch.zeros(n_ranks, dtype=torch.int32, device=dev)
        if T and self.L.clb200_ep_pack(self.ctx.handle, T, self.E, K, n_ranks, n_local, sel.data_ptr(), wt.data_ptr(), qs.data_ptr(),
                                       d.data_ptr(), bs.data_ptr(), send.data_ptr(), slot.data_ptr(), counts.data_ptr(), self._s(),
                                       self._err, 512):
            raise RuntimeError(self._err.value.decode())
        return send, slot, counts

    def combine_regions(self, x, back, slot, counts, t_max, resid_scale):
        """x += resid_scale * (each token's partial sums from the exchange's back area, ranks in order)."""
        if x.shape[0] and self.L.clb200_ep_combine_regions(self.ctx.handle, x.shape[0], self.E, slot.shape[1], t_max, slot.data_ptr(),
                                                           counts.data_ptr(), back.data_ptr(), x.data_ptr(), resid_scale, self._s(),
                                                           self._err, 512):
            raise RuntimeError(self._err.value.decode())

    def combine(self, x, back, plan, counts, resid_scale):
        slot = plan
        if self.L.clb200_ep_combine(self.ctx.handle, x.shape[0], self.E, slot.shape[1], slot.data_ptr(), back.data_ptr(), x.data_ptr(),
                                    resid_scale, self._s(), self._err, 512):
            raise RuntimeError(self._err.value.decode())


class _DeviceBytes:
    """A view of `nbytes` of device memory at `ptr` that torch can wrap without copying (__cuda_array_interface__)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3, "strides": None}


class PeerExchange:
    """The exchange over peer memory for one process group: this rank's exchange buffer (clb200_ep_xbuf_alloc) and every
    other rank's, mapped here through CUDA IPC; rows and partial sums go out by the library's store kernels
    (clb200_ep_push / clb200_ep_push_back) and arrive behind (step, rows) signals that a kernel waits on
    (clb200_ep_wait), so a layer step needs no host synchronisation. t_max bounds the tokens any rank sends in one step.
    Every rank of the group constructs it (a collective) and closes it (a collective)."""

    def __init__(self, ctx, t_max: int, E: int, K: int, group=None):
        import torch.distributed as dist
        from . import lib
        self.ctx, self.L, self.t_max, self.E, self.K, self.group = ctx, lib(), t_max, E, K, group
        self.n, self.me = dist.get_world_size(group), dist.get_rank(group)
        self.fmt = RowFormat(E, K)
        self.seq = 0
        self._err = C.create_string_buffer(512)
        L = self.L
        L.clb200_ep_xbuf_layout.restype = None
        L.clb200_ep_xbuf_layout.argtypes = [C.c_int] * 4 + [C.POINTER(C.c_size_t)] * 3
        L.clb200_ep_xbuf_alloc.argtypes = [C.c_void_p] + [C.c_int] * 4 + [C.POINTER(C.c_void_p), C.c_char_p, C.c_char_p, C.c_size_t]
        L.clb200_ep_xbuf_open.argtypes = [C.c_void_p, C.c_char_p, C.POINTER(C.c_void_p), C.c_char_p, C.c_size_t]
        L.clb200_ep_xbuf_close.argtypes = [C.c_void_p, C.c_void_p, C.c_char_p, C.c_size_t]
        L.clb200_ep_xbuf_free.argtypes = [C.c_void_p, C.c_void_p, C.c_char_p, C.c_size_t]
        L.clb200_ep_push.argtypes = [C.c_void_p] + [C.c_int] * 5 + [C.c_void_p] * 3 + [C.c_uint, C.c_void_p, C.c_char_p, C.c_size_t]
        L.clb200_ep_wait.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_uint, C.c_void_p, C.c_void_p, C.c_char_p, C.c_size_t]
        L.clb200_ep_push_back.argtypes = L.clb200_ep_push.argtypes
        size, roff, boff = C.c_size_t(), C.c_size_t(), C.c_size_t()
        L.clb200_ep_xbuf_layout(self.n, t_max, E, K, C.byref(size), C.byref(roff), C.byref(boff))
        self.size, self.recv_off, self.back_off = size.value, roff.value, boff.value
        own, handle, failure = C.c_void_p(), C.create_string_buffer(64), None
        if L.clb200_ep_xbuf_alloc(ctx.handle, self.n, t_max, E, K, C.byref(own), handle, self._err, 512):
            failure = self._err.value.decode()
        self.own = own.value if not failure else None
        handles = [None] * self.n
        dist.all_gather_object(handles, None if failure else bytes(handle.raw), group=group)
        self.mapped, bases = [], []
        for r in range(self.n):
            if failure:
                break
            if r == self.me:
                bases.append(self.own)
                continue
            if handles[r] is None:
                failure = f"rank {r} could not allocate its exchange buffer"
                break
            p = C.c_void_p()
            if L.clb200_ep_xbuf_open(ctx.handle, handles[r], C.byref(p), self._err, 512):
                failure = self._err.value.decode()
                break
            self.mapped.append(p.value)
            bases.append(p.value)
        # every rank learns whether every rank mapped every buffer (a collective every rank reaches, failed or not), so
        # that all give up together and a caller can fall back to another exchange on all ranks
        ok = torch.tensor([0 if failure else 1], dtype=torch.int32, device=f"cuda:{torch.cuda.current_device()}")
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        if int(ok.item()) == 0:
            for p in self.mapped:
                L.clb200_ep_xbuf_close(ctx.handle, p, self._err, 512)
            if self.own:
                L.clb200_ep_xbuf_free(ctx.handle, self.own, self._err, 512)
            self.own, self.mapped = None, []
            raise RuntimeError(f"peer-memory exchange unavailable: {failure or 'another rank could not map the buffers'}")
        self.bases = (C.c_void_p * self.n)(*bases)
        whole = torch.as_tensor(_DeviceBytes(self.own, self.size), device=f"cuda:{torch.cuda.current_device()}")
        R = self.n * t_max
        self.recv = whole[self.recv_off:self.recv_off + R * self.fmt.nbytes].view(R, self.fmt.nbytes)
        self.back = whole[self.back_off:self.back_off + R * E * 4].view(torch.float32).view(R, E)
        self.rcounts = torch.zeros(self.n, dtype=torch.int32, device=whole.device)
        self._whole = whole   # (every rank mapped every buffer before anyone pushes: the all_reduce above)

    def _check(self, rc):
        if rc:
            raise RuntimeError(self._err.value.decode())

    def next_step(self) -> None:
        self.seq = self.seq % 0xFFFFFFFE + 1   # 1, 2, ...: a zeroed header carries step 0, which no step uses

    def push(self, send, counts, stream) -> None:
        self._check(self.L.clb200_ep_push(self.ctx.handle, self.me, self.n, self.t_max, self.E, self.K, self.bases, send.data_ptr(),
                                          counts.data_ptr(), self.seq, stream, self._err, 512))

    def wait_rows(self, stream) -> torch.Tensor:
        self._check(self.L.clb200_ep_wait(self.ctx.handle, self.own, self.n, 0, self.seq, self.rcounts.data_ptr(), stream,
                                          self._err, 512))
        return self.rcounts

    def push_back(self, partial, stream) -> None:
        self._check(self.L.clb200_ep_push_back(self.ctx.handle, self.me, self.n, self.t_max, self.E, self.K, self.bases,
                                               partial.data_ptr(), self.rcounts.data_ptr(), self.seq, stream, self._err, 512))

    def wait_back(self, stream) -> None:
        self._check(self.L.clb200_ep_wait(self.ctx.handle, self.own, self.n, 1, self.seq, None, stream, self._err, 512))

    def close(self) -> None:
        """A collective: every rank stops using the mapped buffers, unmaps them, and frees its own once every rank has."""
        import torch.distributed as dist
        if self.own is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for p in self.mapped:
            self.L.clb200_ep_xbuf_close(self.ctx.handle, p, self._err, 512)
        self.mapped = []
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        self.recv = self.back = self._whole = None
        self.L.clb200_ep_xbuf_free(self.ctx.handle, self.own, self._err, 512)
        self.own = None


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


def moe_layer(x: torch.Tensor, comp: Compute, n_local: int, resid_scale: float, group=None, timings: dict | None = None,
              xchg: Optional[PeerExchange] = None):
    """One expert-parallel MoE layer step on this rank's tokens x [T, E] (updated in place); returns (sel, wt). With
    xchg (a PeerExchange of the same group) the rows and partial sums move over peer memory, else by NCCL all-to-alls."""
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
    if xchg is not None and n > 1:
        return _moe_layer_peer(x, comp, n_local, resid_scale, xchg, fmt, sel, wt, qs, d, bs, mark, close, timings)
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


def _moe_layer_peer(x, comp, n_local, resid_scale, xchg: PeerExchange, fmt, sel, wt, qs, d, bs, mark, close, timings):
    """The rest of moe_layer over peer memory: pack, push, wait for every sender's rows, the local experts over the whole
    receive area (rows past a sender's count are left from earlier steps and get no expert), push the partial sums
    back, wait for every rank's, combine."""
    n, T = xchg.n, x.shape[0]
    if T > xchg.t_max:
        raise ValueError(f"{T} tokens: the exchange was set up for at most {xchg.t_max}")
    st = comp._s()
    send, slot, counts = comp.pack_device(fmt, sel, wt, qs, d, bs, n, n_local)
    xchg.next_step()
    xchg.push(send, counts, st)
    rcounts = xchg.wait_rows(st)
    close("dispatch")
    r = fmt.unpack(xchg.recv)
    live = (torch.arange(xchg.t_max, device=x.device)[None, :] < rcounts[:, None].to(torch.int64)).reshape(-1, 1)
    mark("experts")
    partial = comp.experts(r["qs"], r["d"], r["bs"], torch.where(live, r["sel"], -1), r["wt"])
    close("experts")
    mark("combine")
    xchg.push_back(partial, st)
    xchg.wait_back(st)
    comp.combine_regions(x, xchg.back, slot, counts, xchg.t_max, resid_scale)
    close("combine")
    if timings is not None:   # a measured step: the counts are read on the host here (the timed steps never do)
        sc, rc = counts.tolist(), rcounts.tolist()
        me = xchg.me
        timings.setdefault("rows", []).append(int(sum(rc)))
        timings.setdefault("xbytes", []).append(sum(c for dd, c in enumerate(sc) if dd != me) * fmt.nbytes +
                                                sum(c for dd, c in enumerate(rc) if dd != me) * x.shape[1] * 4)
        timings.pop("_open", None)
    return sel, wt

"""clutor-b200: the Clutor engine's MoE feed-forward block on B200 (sm_100a), through the C ABI of include/clb200.h.

This module is the Python view of that ABI (ctypes), used by the tests and bench.py; C host code (the reference engine)
calls the same entry points directly. There is no CPU path: importing works anywhere, but every entry point needs the
built library (python -m clutor_b200.build) and a CUDA device, and fails loudly without them.
"""
from __future__ import annotations

import ctypes as C
import os
import re

import numpy as np

from . import synth

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libclutor_b200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "clb200.h")

T_F32, T_F16, T_Q8_0, T_Q4_K, T_Q6_K = 0, 1, 8, 12, 14


class CLW(C.Structure):
    """clb200_w == the reference's cl_w (c/src/forward.h:18)."""
    _fields_ = [("p", C.c_void_p), ("type", C.c_uint32), ("rows", C.c_int), ("cols", C.c_int)]


class MoELayer(C.Structure):
    """clb200_moe_layer (include/clb200.h)."""
    _fields_ = [("ffn_norm_f", C.c_void_p), ("router_f", C.c_void_p), ("gate", CLW), ("up", CLW), ("down", CLW),
                ("gate_slab", C.c_uint64), ("up_slab", C.c_uint64), ("down_slab", C.c_uint64),
                ("n_embd", C.c_int), ("n_ff_exp", C.c_int), ("n_expert", C.c_int), ("n_used", C.c_int),
                ("norm_topk", C.c_int), ("resid_scale", C.c_float), ("rms_eps", C.c_float)]


class Q8K(C.Structure):
    _fields_ = [("d", C.c_float), ("qs", C.c_int8 * 256), ("bsums", C.c_int16 * 16)]


class XQ(C.Structure):
    _fields_ = [("b", C.c_void_p), ("n", C.c_int)]


class MV(C.Structure):
    """clb200_mv == the reference's cl_mv (c/src/quant.h:31-34)."""
    _fields_ = [("type", C.c_uint32), ("w", C.c_void_p), ("rows", C.c_int), ("cols", C.c_int), ("xf", C.c_void_p),
                ("xq", C.c_void_p), ("out", C.c_void_p), ("nb", C.c_int), ("xf_stride", C.c_size_t),
                ("out_stride", C.c_size_t)]


SUPPORTS = C.CFUNCTYPE(C.c_int, C.c_uint32)
MATVEC = C.CFUNCTYPE(None, C.POINTER(MV), C.c_int)


class Backend(C.Structure):
    """clb200_backend_t == the reference's cl_backend (c/src/backend.h:9-13)."""
    _fields_ = [("name", C.c_char_p), ("supports", SUPPORTS), ("matvec_batch", MATVEC)]


class CacheStats(C.Structure):
    """clb200_cache_stats == the reference's cl_cache_stats (c/src/cache.h:14-17)."""
    _fields_ = [(n, C.c_uint64) for n in ("hits", "misses", "stage_hits", "inserts", "evictions", "admit_rejects",
                                         "stage_inserts", "stage_wasted", "aging_resets")] + [("window_slots", C.c_uint32)]

    def as_dict(self) -> dict:
        return {n: getattr(self, n) for n, _ in self._fields_}


LRU, WTINYLFU, ADAPTIVE = 0, 1, 2


class StoreStats(C.Structure):
    """clb200_store_stats (the reference's cl_xs_stats, c/src/xs.h:14-17, with copy_ns for read_ns)."""
    _fields_ = [(n, C.c_uint64) for n in ("accesses", "hits", "stage_hits", "misses", "bypass", "prefetch_issued",
                                         "prefetch_late", "prefetch_wasted", "admit_rejects", "evictions", "demand_bytes",
                                         "prefetch_bytes", "copy_ns", "wait_ns", "pred_total", "pred_hit")]

    def as_dict(self) -> dict:
        return {n: getattr(self, n) for n, _ in self._fields_}


_lib: C.CDLL | None = None


class Smart(C.Structure):
    """clb200_smart (the layout of the reference's cl_smart, c/src/route.h:14)."""
    _fields_ = [("enabled", C.c_int), ("J", C.c_int), ("M", C.c_int), ("tau", C.c_double)]


class RouteResult(C.Structure):
    """clb200_route_result (the layout of cl_route_result, c/src/route.h:16-22)."""
    _fields_ = [("selected", C.c_int * 32), ("k", C.c_int), ("substituted", C.c_int), ("dropped_mass", C.c_double),
                ("max_delta", C.c_double)]

    def as_dict(self) -> dict:
        return {"selected": list(self.selected[:self.k]), "substituted": self.substituted,
                "dropped_mass": self.dropped_mass, "max_delta": self.max_delta}


class SmartStats(C.Structure):
    _fields_ = [("substituted", C.c_uint64), ("expert_slots", C.c_uint64), ("dropped_mass", C.c_double),
                ("max_delta", C.c_double)]

    def as_dict(self) -> dict:
        return {f: getattr(self, f) for f, _ in self._fields_}


def header_functions() -> list[str]:
    """Names of the functions include/clb200.h declares."""
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(clb200_\w+)\s*\(", text, re.M)))


def lib() -> C.CDLL:
    """The CUDA library; raises if it is not built (there is no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is not built: run `python -m clutor_b200.build` (no CPU fallback exists)")
        L = C.CDLL(LIB_PATH)
        L.clb200_open.restype = C.c_void_p
        L.clb200_open.argtypes = [C.c_int, C.c_char_p, C.c_size_t]
        L.clb200_close.argtypes = [C.c_void_p]
        L.clb200_moe_ffn.argtypes = [C.c_void_p, C.POINTER(MoELayer), C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_char_p, C.c_size_t]
        L.clb200_layer_bind.argtypes = [C.c_void_p, C.POINTER(MoELayer), C.c_int, C.c_char_p, C.c_size_t]
        L.clb200_moe_ffn_dev.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_char_p, C.c_size_t]
        L.clb200_status.argtypes = [C.c_void_p, C.c_char_p, C.c_size_t]
        L.clb200_layer_release.argtypes = [C.c_void_p, C.c_int]
        L.clb200_moe_ffn_decode_noalloc.argtypes = [C.POINTER(MoELayer), C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                                    C.c_char_p, C.c_size_t]
        L.clb200_moe_dispatch.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                          C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_char_p, C.c_size_t]
        L.clb200_device_bytes.restype = C.c_uint64
        L.clb200_device_bytes.argtypes = [C.c_void_p]
        L.clb200_set_trace.argtypes = [C.c_void_p, C.c_void_p]
        L.clb200_set_exact.argtypes = [C.c_void_p, C.c_int]
        L.clb200_set_option.argtypes = [C.c_void_p, C.c_int, C.c_int]
        L.clb200_backend.restype = C.POINTER(Backend)
        L.clb200_cache_new.restype = C.c_void_p
        L.clb200_cache_new.argtypes = [C.c_uint32, C.c_uint32, C.c_uint32, C.c_int, C.c_uint32]
        L.clb200_cache_free.argtypes = [C.c_void_p]
        L.clb200_cache_access.argtypes = [C.c_void_p, C.c_uint32, C.POINTER(C.c_int)]
        L.clb200_cache_stage.argtypes = [C.c_void_p, C.c_uint32]
        for f in ("pin", "unpin", "abandon"):
            getattr(L, f"clb200_cache_{f}").argtypes = [C.c_void_p, C.c_int]
        L.clb200_cache_find.argtypes = [C.c_void_p, C.c_uint32]
        L.clb200_cache_freq.argtypes = [C.c_void_p, C.c_uint32]
        L.clb200_cache_freq.restype = C.c_uint32
        L.clb200_cache_count.argtypes = [C.c_void_p]
        L.clb200_cache_count.restype = C.c_uint32
        L.clb200_cache_total_slots.argtypes = [C.c_void_p]
        L.clb200_cache_total_slots.restype = C.c_uint32
        L.clb200_cache_segment.argtypes = [C.c_void_p, C.c_int]
        L.clb200_cache_slot_key.argtypes = [C.c_void_p, C.c_int]
        L.clb200_cache_slot_key.restype = C.c_uint32
        L.clb200_cache_get_stats.argtypes = [C.c_void_p]
        L.clb200_cache_get_stats.restype = CacheStats
        L.clb200_store_open.restype = C.c_void_p
        L.clb200_store_open.argtypes = [C.c_void_p, C.POINTER(MoELayer), C.c_int, C.c_uint64, C.c_int, C.c_int, C.c_char_p, C.c_size_t]
        L.clb200_store_close.argtypes = [C.c_void_p]
        L.clb200_store_load_layer.argtypes = [C.c_void_p, C.c_int, C.POINTER(MoELayer), C.c_char_p, C.c_size_t]
        L.clb200_store_cache_slots.argtypes = [C.c_void_p]
        L.clb200_store_cache_slots.restype = C.c_uint32
        L.clb200_store_slot_bytes.argtypes = [C.c_void_p]
        L.clb200_store_slot_bytes.restype = C.c_uint64
        L.clb200_store_get_stats.argtypes = [C.c_void_p]
        L.clb200_store_get_stats.restype = StoreStats
        L.clb200_store_reset_stats.argtypes = [C.c_void_p]
        L.clb200_store_set_prefetch.argtypes = [C.c_void_p, C.c_int]
        L.clb200_store_set_prefetch_n.argtypes = [C.c_void_p, C.c_int]
        L.clb200_store_set_prefetch_depth.argtypes = [C.c_void_p, C.c_int]
        L.clb200_store_log.argtypes = [C.c_void_p, C.c_int]
        L.clb200_store_read_log.argtypes = [C.c_void_p, C.c_void_p, C.c_int64]
        L.clb200_store_read_log.restype = C.c_int64
        L.clb200_store_request.argtypes = [C.c_void_p, C.c_int, C.c_int]
        L.clb200_store_wait.argtypes = [C.c_void_p, C.c_int]
        L.clb200_store_wait.restype = C.c_void_p
        L.clb200_store_release.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
        L.clb200_store_resident.argtypes = [C.c_void_p, C.c_int, C.c_int]
        L.clb200_store_prefetch.argtypes = [C.c_void_p, C.c_int, C.c_int]
        L.clb200_moe_ffn_stored.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                            C.c_char_p, C.c_size_t]
        L.clb200_moe_experts_stored.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                                C.c_void_p, C.c_char_p, C.c_size_t]
        L.clb200_route.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_char_p,
                                   C.c_size_t]
        L.clb200_route_dev.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_int,
                                       C.c_void_p, C.c_void_p]
        L.clb200_store_set_smart.argtypes = [C.c_void_p, C.c_void_p, C.c_char_p, C.c_size_t]
        L.clb200_store_smart_stats.argtypes = [C.c_void_p]
        L.clb200_store_smart_stats.restype = SmartStats
        L.clb200_store_route.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_char_p, C.c_size_t]
        L.clb200_store_failed.argtypes = [C.c_void_p]
        L.clb200_store_inject_fill_failure.argtypes = [C.c_void_p, C.c_int]
        _lib = L
    return _lib


class ClutorError(RuntimeError):
    pass


def _ptr(a) -> int:
    if a is None:
        return 0
    if isinstance(a, np.ndarray):
        assert a.flags["C_CONTIGUOUS"]
        return a.ctypes.data
    return a.data_ptr()   # torch tensor


def _stream(stream) -> int:
    """The cudaStream_t for a call on torch tensors: the given torch stream, else torch's current stream (so the call is
    ordered with the torch work that made its inputs and will read its outputs)."""
    import torch
    st = (stream if stream is not None else torch.cuda.current_stream()).cuda_stream
    return st or CUDA_STREAM_LEGACY   # torch's default stream is the legacy stream; 0 would mean the context's own stream


CUDA_STREAM_LEGACY = 1   # cudaStreamLegacy


def layer_struct(layer) -> MoELayer:
    """A clb200_moe_layer over a synth.HostLayer (numpy, host pointers) or synth.DeviceLayer (torch, device pointers)."""
    s = MoELayer()
    s.ffn_norm_f, s.router_f = _ptr(layer.ffn_norm), _ptr(layer.router)
    E, FF = layer.E, layer.FF
    s.gate = CLW(_ptr(layer.gate), layer.gate_type, FF, E)
    s.up = CLW(_ptr(layer.up), layer.up_type, FF, E)
    s.down = CLW(_ptr(layer.down), layer.down_type, E, FF)
    s.gate_slab, s.up_slab, s.down_slab = layer.gate_slab, layer.up_slab, layer.down_slab
    s.n_embd, s.n_ff_exp, s.n_expert, s.n_used = E, FF, layer.NE, layer.K
    s.norm_topk, s.resid_scale, s.rms_eps = layer.norm_topk, layer.resid_scale, layer.rms_eps
    return s


class Context:
    """A clb200 context on one CUDA device (clb200_open)."""

    def __init__(self, device: int = 0):
        self._err = C.create_string_buffer(512)
        self.handle = lib().clb200_open(device, self._err, 512)
        if not self.handle:
            raise ClutorError(self._err.value.decode())
        self.device = device
        self._keep: list = []

    def close(self) -> None:
        if self.handle:
            lib().clb200_close(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc: int) -> None:
        if rc:
            raise ClutorError(self._err.value.decode())

    def moe_ffn(self, layer: "synth.HostLayer", x: np.ndarray):
        """The host-pointer entry point (clb200_moe_ffn): returns (x_out, sel, wt); x is not modified."""
        x = np.ascontiguousarray(x, dtype=np.float32).copy()
        T = x.shape[0]
        sel = np.zeros((T, layer.K), np.int32)
        wt = np.zeros((T, layer.K), np.float32)
        s = layer_struct(layer)
        self._check(lib().clb200_moe_ffn(self.handle, C.byref(s), _ptr(x), T, _ptr(sel), _ptr(wt), self._err, 512))
        return x, sel, wt

    def moe_ffn_inplace(self, s: MoELayer, x: np.ndarray, sel: np.ndarray, wt: np.ndarray) -> None:
        """clb200_moe_ffn on caller buffers (x updated in place), with a prebuilt layer struct: no copies on the Python side
        (for timing the host entry point from pinned memory)."""
        self._check(lib().clb200_moe_ffn(self.handle, C.byref(s), _ptr(x), x.shape[0], _ptr(sel), _ptr(wt), self._err, 512))

    def bind(self, layer, on_device: bool | None = None) -> int:
        """Registers a layer (clb200_layer_bind); device tensors are used in place, host arrays are uploaded."""
        if on_device is None:
            on_device = not isinstance(layer.gate, np.ndarray)
        s = layer_struct(layer)
        h = lib().clb200_layer_bind(self.handle, C.byref(s), 1 if on_device else 0, self._err, 512)
        if h < 0:
            raise ClutorError(self._err.value.decode())
        self._keep.append(layer)
        return h

    def release(self, handle: int) -> None:
        """Frees a bound layer's device copy (clb200_layer_release)."""
        if lib().clb200_layer_release(self.handle, handle):
            raise ClutorError(f"no layer {handle}")

    def moe_ffn_dev(self, handle: int, x, sel=None, wt=None, stream=None) -> None:
        """The device entry point (clb200_moe_ffn_dev) on torch CUDA tensors; asynchronous on `stream` (a torch stream)."""
        T = x.shape[0]
        st = _stream(stream)
        self._check(lib().clb200_moe_ffn_dev(self.handle, handle, _ptr(x), T, _ptr(sel), _ptr(wt), C.c_void_p(st), self._err, 512))

    def status(self) -> None:
        self._check(lib().clb200_status(self.handle, self._err, 512))

    def dispatch(self, sel, wt, n_expert: int, stream=None):
        """clb200_moe_dispatch on torch CUDA tensors sel [T, K] int32 and wt [T, K] float32. Returns device tensors
        (todo [n_expert + 1], offsets [n_expert + 1], pos_token [T * K], pos_wt [T * K]); asynchronous."""
        import torch
        T, K = sel.shape
        todo = torch.full((n_expert + 1,), -1, dtype=torch.int32, device=sel.device)
        offsets = torch.full((n_expert + 1,), -1, dtype=torch.int32, device=sel.device)
        pos_token = torch.full((T * K,), -1, dtype=torch.int32, device=sel.device)
        pos_wt = torch.zeros((T * K,), dtype=torch.float32, device=sel.device)
        self._check(lib().clb200_moe_dispatch(self.handle, T, n_expert, K, _ptr(sel), _ptr(wt), _ptr(todo), _ptr(offsets),
                                              _ptr(pos_token), _ptr(pos_wt), C.c_void_p(_stream(stream)), self._err, 512))
        return todo, offsets, pos_token, pos_wt

    def device_bytes(self) -> int:
        return int(lib().clb200_device_bytes(self.handle))

    def set_exact(self, on: bool) -> None:
        """clb200_set_exact: batched expert products on the integer path only (bit-exact), or on the tensor cores."""
        lib().clb200_set_exact(self.handle, int(on))

    OPT_DECODE_KERNEL, OPT_TEST_SPECULATION_MISS, OPT_TEST_STALL_WAIT, OPT_COOPERATIVE = 1, 2, 3, 4

    def set_option(self, option: int, value: int) -> None:
        """clb200_set_option: OPT_DECODE_KERNEL (0 expert-group kernel where it fits, 1 grid-wide kernel, the default) or
        the OPT_TEST_SPECULATION_MISS test hook."""
        if lib().clb200_set_option(self.handle, option, int(value)):
            raise ClutorError(f"option {option} = {value} refused")

    def set_trace(self, buf=None) -> None:
        """Phase trace of the one-token kernel (clb200_set_trace): buf is a torch uint64/int64 CUDA tensor of 32 entries per
        SM, or None to stop."""
        lib().clb200_set_trace(self.handle, _ptr(buf))


    def route(self, logits: np.ndarray, K: int, smart: tuple | None = None, resident: np.ndarray | None = None) -> dict | None:
        """cl_route on the GPU (clb200_route): logits [E] float32 (host); smart = (J, M, tau) or None; resident [E] bytes
        or None. Returns the result as a dict, or None when the arguments are out of range (as cl_route's -1)."""
        lg = np.ascontiguousarray(logits, np.float32)
        res = None if resident is None else np.ascontiguousarray(resident, np.uint8)
        sm = Smart(1, *smart) if smart else None
        out = RouteResult()
        rc = lib().clb200_route(self.handle, lg.ctypes.data, lg.shape[0], K, C.addressof(sm) if sm else None,
                                None if res is None else res.ctypes.data, C.addressof(out), self._err, 512)
        if rc < 0:
            return None
        self._check(rc)
        return out.as_dict()

    def route_dev(self, logits, K: int, smart: tuple | None, resident, out, resident_stride: int = 0, stream=None) -> int:
        """clb200_route_dev on torch CUDA tensors: logits [T, E] float32, resident uint8 or None, out a uint8 tensor of
        T * 152 bytes (clb200_route_result each). Returns the C return code."""
        sm = Smart(1, *smart) if smart else None
        T, E = logits.shape
        return lib().clb200_route_dev(self.handle, _ptr(logits), T, E, K, C.addressof(sm) if sm else None,
                                      None if resident is None else _ptr(resident), resident_stride, _ptr(out),
                                      C.c_void_p(_stream(stream)))


def backend() -> Backend:
    """The "b200" cl_backend struct (clb200_backend)."""
    return lib().clb200_backend().contents


def matvec(type_: int, w: np.ndarray, rows: int, cols: int, xf: np.ndarray | None = None, xq: np.ndarray | None = None):
    """One cl_mv job through the backend's matvec_batch (host pointers, like the reference's seam). xf [nb, cols] float32;
    xq: numpy array of Q8K structured dtype [nb, cols/256]. Returns out [nb, rows]."""
    nb = (xf.shape[0] if xf is not None and xf.ndim == 2 else (xq.shape[0] if xq is not None and xq.ndim == 2 else 1))
    out = np.zeros((nb, rows), np.float32)
    xqs = None
    if xq is not None:
        xq = np.ascontiguousarray(xq.reshape(nb, -1))
        xqs = (XQ * nb)(*[XQ(xq[b].ctypes.data, cols) for b in range(nb)])
    xf_c = None if xf is None else np.ascontiguousarray(xf.reshape(nb, cols), dtype=np.float32)
    job = MV(type_, _ptr(np.ascontiguousarray(w)), rows, cols, _ptr(xf_c), C.addressof(xqs) if xqs is not None else 0,
             _ptr(out), nb, cols, rows)
    be = backend()
    be.matvec_batch(C.byref(job), 1)
    return out


class ExpertCache:
    """The expert-cache policy (clb200_cache_*): which expert holds which HBM slot. Host code; needs no GPU."""

    def __init__(self, cache_slots: int, stage_slots: int, universe: int, policy: int = WTINYLFU, window_pct: int = 0):
        self.L = lib()
        self.h = self.L.clb200_cache_new(cache_slots, stage_slots, universe, policy, window_pct)
        if not self.h:
            raise ValueError("clb200_cache_new refused the sizes")

    def close(self) -> None:
        if self.h:
            self.L.clb200_cache_free(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def access(self, key: int) -> tuple[int, int]:
        slot = C.c_int(-1)
        r = self.L.clb200_cache_access(self.h, key, C.byref(slot))
        return r, slot.value

    def stage(self, key: int) -> int:
        return self.L.clb200_cache_stage(self.h, key)

    def pin(self, slot: int) -> None:
        self.L.clb200_cache_pin(self.h, slot)

    def unpin(self, slot: int) -> None:
        self.L.clb200_cache_unpin(self.h, slot)

    def abandon(self, slot: int) -> None:
        self.L.clb200_cache_abandon(self.h, slot)

    def find(self, key: int) -> int:
        return self.L.clb200_cache_find(self.h, key)

    def freq(self, key: int) -> int:
        return self.L.clb200_cache_freq(self.h, key)

    def count(self) -> int:
        return self.L.clb200_cache_count(self.h)

    def total_slots(self) -> int:
        return self.L.clb200_cache_total_slots(self.h)

    def segment(self, slot: int) -> int:
        return self.L.clb200_cache_segment(self.h, slot)

    def stats(self) -> dict:
        return self.L.clb200_cache_get_stats(self.h).as_dict()


class Store:
    """The HBM expert store (clb200_store_*): every layer's experts in pinned host memory, a cache budget of them in HBM."""

    def __init__(self, ctx: "Context", shape, n_layer: int, cache_bytes: int, stage_slots: int, policy: int = WTINYLFU):
        self.ctx, self.L = ctx, lib()
        self._err = C.create_string_buffer(512)
        self._shape = layer_struct(shape)
        self.h = self.L.clb200_store_open(ctx.handle, C.byref(self._shape), n_layer, cache_bytes, stage_slots, policy, self._err, 512)
        if not self.h:
            raise ClutorError(self._err.value.decode())
        self.K = shape.K

    def close(self) -> None:
        if self.h:
            self.L.clb200_store_close(self.h)
            self.h = None

    def load_layer(self, i: int, layer) -> None:
        s = layer_struct(layer)
        if self.L.clb200_store_load_layer(self.h, i, C.byref(s), self._err, 512):
            raise ClutorError(self._err.value.decode())

    def cache_slots(self) -> int:
        return self.L.clb200_store_cache_slots(self.h)

    def slot_bytes(self) -> int:
        return self.L.clb200_store_slot_bytes(self.h)

    def stats(self) -> dict:
        return self.L.clb200_store_get_stats(self.h).as_dict()

    def reset_stats(self) -> None:
        self.L.clb200_store_reset_stats(self.h)

    PREFETCH_OFF, PREFETCH_PREV, PREFETCH_AHEAD = 0, 1, 2

    def set_prefetch_depth(self, depth: int) -> None:
        self.L.clb200_store_set_prefetch_depth(self.h, int(depth))

    def prefetch(self, layer: int, expert: int) -> None:
        """Stages one expert (clb200_store_prefetch, the reference's cl_xs_prefetch)."""
        self.L.clb200_store_prefetch(self.h, int(layer), int(expert))

    def set_prefetch(self, mode: int, n: int = 0, depth: int | None = None) -> None:
        """mode 0 off, 1 prev (the previous token's choice), 2 ahead (the next layer's router on this x); n experts staged per
        prediction (0: n_used); depth: prefetch fills in flight at once."""
        self.L.clb200_store_set_prefetch(self.h, int(mode))
        self.L.clb200_store_set_prefetch_n(self.h, int(n))
        if depth is not None:
            self.L.clb200_store_set_prefetch_depth(self.h, int(depth))

    def log(self, on: bool) -> None:
        self.L.clb200_store_log(self.h, int(on))

    def read_log(self) -> np.ndarray:
        n = self.L.clb200_store_read_log(self.h, None, 0)
        out = np.zeros(n, np.int64)
        self.L.clb200_store_read_log(self.h, out.ctypes.data, n)
        return out.reshape(-1, 3)

    def moe_ffn(self, layer: int, x, stream=None):
        """One token of `layer` through the store; x a device tensor [n_embd], updated in place. Returns (sel, wt)."""
        sel = np.zeros(self.K, np.int32)
        wt = np.zeros(self.K, np.float32)
        if self.L.clb200_moe_ffn_stored(self.ctx.handle, self.h, layer, _ptr(x), sel.ctypes.data, wt.ctypes.data,
                                        stream if isinstance(stream, int) else _stream(stream), self._err, 512):
            raise ClutorError(self._err.value.decode())
        return sel, wt

    def set_smart(self, smart: tuple | None) -> None:
        """SMART-ROUTE in moe_ffn / route (clb200_store_set_smart): (J, M, tau), or None for plain routing."""
        sm = Smart(1, *smart) if smart else None
        if self.L.clb200_store_set_smart(self.h, C.addressof(sm) if sm else None, self._err, 512):
            raise ClutorError(self._err.value.decode())

    def smart_stats(self) -> dict:
        return self.L.clb200_store_smart_stats(self.h).as_dict()

    def route(self, layer: int, logits: np.ndarray) -> dict:
        """Routing of `layer` from host logits against the store's resident set (clb200_store_route)."""
        lg = np.ascontiguousarray(logits, np.float32)
        out = RouteResult()
        if self.L.clb200_store_route(self.ctx.handle, self.h, layer, lg.ctypes.data, C.addressof(out), self._err, 512):
            raise ClutorError(self._err.value.decode())
        return out.as_dict()

    def failed(self) -> bool:
        return bool(self.L.clb200_store_failed(self.h))

    def inject_fill_failure(self, n: int) -> None:
        """Test hook: the n-th fill from now copies nothing and fails (clb200_store_inject_fill_failure)."""
        self.L.clb200_store_inject_fill_failure(self.h, n)

    def resident(self, layer: int, expert: int) -> bool:
        return bool(self.L.clb200_store_resident(self.h, layer, expert))

    def experts(self, layer: int, x, sel: np.ndarray, wt: np.ndarray, next_pred: np.ndarray | None = None, stream=None):
        """The experts of a given routing (host arrays) through the store; x a device tensor, updated in place."""
        sel = np.ascontiguousarray(sel, np.int32)
        wt = np.ascontiguousarray(wt, np.float32)
        nxt = None if next_pred is None else np.ascontiguousarray(next_pred, np.int32)
        if self.L.clb200_moe_experts_stored(self.ctx.handle, self.h, layer, _ptr(x), sel.ctypes.data, wt.ctypes.data,
                                            None if nxt is None else nxt.ctypes.data,
                                            stream if isinstance(stream, int) else _stream(stream), self._err, 512):
            raise ClutorError(self._err.value.decode())

"""TEST INFRASTRUCTURE ONLY -- the oracle.

Python bindings (ctypes) for the two CPU checkers that oracle/Makefile builds:

* ``liboracle.so`` -- this repository's plain-C restatement of the Clutor MoE feed-forward block (moe_oracle.c);
* ``_ref/libclref.so`` -- the reference engine's own C sources (c/src/{quant,kernel,iq,cache,xs,route,gguf,meta}.c and,
  through ref_harness.c, c/src/forward.c), compiled unmodified.

Only tests/, ``__graft_entry__.smoke()`` and the CPU-baseline leg of bench.py import this package, and only as the
checker: the product (clutor_b200) never calls into it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libclref.so")

def ref_dir() -> str | None:
    """The reference engine's c/src directory, from the CLUTOR_REF_DIR environment variable (None when it is unset)."""
    d = os.environ.get("CLUTOR_REF_DIR")
    return d or None

T_F32, T_F16, T_Q8_0, T_Q4_K, T_Q6_K = 0, 1, 8, 12, 14


class Layer(C.Structure):
    """Mirror of ``orc_layer`` / ``ref_layer`` (both laid out like the fields the reference binds, c/src/forward.h:18-29)."""
    _fields_ = [
        ("ffn_norm", C.c_void_p), ("router", C.c_void_p),
        ("gate_type", C.c_uint32), ("up_type", C.c_uint32), ("down_type", C.c_uint32),
        ("gate", C.c_void_p), ("up", C.c_void_p), ("down", C.c_void_p),
        ("gate_slab", C.c_uint64), ("up_slab", C.c_uint64), ("down_slab", C.c_uint64),
        ("E", C.c_int), ("FF", C.c_int), ("NE", C.c_int), ("K", C.c_int), ("norm_topk", C.c_int),
        ("resid_scale", C.c_float), ("rms_eps", C.c_float),
    ]


def build(src: str | None = None, quiet: bool = True, need_ref: bool = False) -> None:
    """Compiles liboracle.so, and _ref/libclref.so from the reference's c/src directory `src` (default: CLUTOR_REF_DIR).
    Without a directory only liboracle.so is built; with need_ref that is an error."""
    src = src or ref_dir()
    out = subprocess.DEVNULL if quiet else None
    subprocess.run(["make", "-C", HERE, "liboracle.so"], check=True, stdout=out)
    if src and os.path.isdir(src):
        subprocess.run(["make", "-C", HERE, "ref", f"REF_DIR={src}"], check=True, stdout=out)
    elif need_ref and not ref_available():
        raise RuntimeError("oracle/_ref is not built and no reference sources are given: set CLUTOR_REF_DIR to the "
                           "reference engine's c/src directory")


_libs: dict[str, C.CDLL] = {}


def _load(path: str) -> C.CDLL:
    if path not in _libs:
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} is not built (run `make -C oracle`)")
        _libs[path] = C.CDLL(path)
    return _libs[path]


def oracle_lib() -> C.CDLL:
    lib = _load(ORACLE_SO)
    lib.orc_f16_to_f32.restype = C.c_float
    lib.orc_f16_to_f32.argtypes = [C.c_uint16]
    lib.orc_dot_row.restype = C.c_float
    lib.orc_dotf.restype = C.c_float
    lib.orc_row_bytes.restype = C.c_uint64
    return lib


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref_lib() -> C.CDLL:
    lib = _load(REF_SO)
    lib.cl_f16_to_f32_soft.restype = C.c_float
    lib.cl_f16_to_f32_soft.argtypes = [C.c_uint16]
    lib.ref_dotf.restype = C.c_float
    lib.cl_quant_path.restype = C.c_char_p
    lib.cl_cache_new.restype = C.c_void_p
    lib.cl_cache_new.argtypes = [C.c_uint32, C.c_uint32, C.c_uint32, C.c_int, C.c_uint32]
    lib.cl_cache_access.argtypes = [C.c_void_p, C.c_uint32, C.POINTER(C.c_int)]
    lib.cl_cache_stage.argtypes = [C.c_void_p, C.c_uint32]
    lib.cl_cache_unpin.argtypes = [C.c_void_p, C.c_int]
    lib.cl_cache_pin.argtypes = [C.c_void_p, C.c_int]
    lib.cl_cache_find.argtypes = [C.c_void_p, C.c_uint32]
    lib.cl_cache_free.argtypes = [C.c_void_p]
    lib.cl_cache_freq.argtypes = [C.c_void_p, C.c_uint32]
    lib.cl_cache_freq.restype = C.c_uint32
    lib.cl_cache_count.argtypes = [C.c_void_p]
    lib.cl_cache_count.restype = C.c_uint32
    lib.cl_cache_abandon.argtypes = [C.c_void_p, C.c_int]
    lib.cl_cache_total_slots.argtypes = [C.c_void_p]
    lib.cl_cache_total_slots.restype = C.c_uint32
    lib.cl_cache_list.argtypes = [C.c_void_p, C.c_int]
    lib.cl_cache_get_stats.argtypes = [C.c_void_p]
    lib.cl_cache_get_stats.restype = CacheStats
    return lib


class CacheStats(C.Structure):
    """cl_cache_stats (c/src/cache.h:14-17)."""
    _fields_ = [(n, C.c_uint64) for n in ("hits", "misses", "stage_hits", "inserts", "evictions", "admit_rejects",
                                         "stage_inserts", "stage_wasted", "aging_resets")] + [("window_slots", C.c_uint32)]

    def as_dict(self) -> dict:
        return {n: getattr(self, n) for n, _ in self._fields_}


class RefCache:
    """The reference's own expert-cache policy (c/src/cache.c, compiled into _ref/libclref.so), driven call by call."""

    def __init__(self, cache_slots: int, stage_slots: int, universe: int, policy: int, window_pct: int = 0):
        self.L = ref_lib()
        self.h = self.L.cl_cache_new(cache_slots, stage_slots, universe, policy, window_pct)
        if not self.h:
            raise ValueError("cl_cache_new refused the sizes")

    def close(self) -> None:
        if self.h:
            self.L.cl_cache_free(self.h)
            self.h = None

    def access(self, key: int) -> tuple[int, int]:
        slot = C.c_int(-1)
        r = self.L.cl_cache_access(self.h, key, C.byref(slot))
        return r, slot.value

    def stage(self, key: int) -> int:
        return self.L.cl_cache_stage(self.h, key)

    def pin(self, slot: int) -> None:
        self.L.cl_cache_pin(self.h, slot)

    def unpin(self, slot: int) -> None:
        self.L.cl_cache_unpin(self.h, slot)

    def abandon(self, slot: int) -> None:
        self.L.cl_cache_abandon(self.h, slot)

    def find(self, key: int) -> int:
        return self.L.cl_cache_find(self.h, key)

    def freq(self, key: int) -> int:
        return self.L.cl_cache_freq(self.h, key)

    def count(self) -> int:
        return self.L.cl_cache_count(self.h)

    def total_slots(self) -> int:
        return self.L.cl_cache_total_slots(self.h)

    def segment(self, slot: int) -> int:
        return self.L.cl_cache_list(self.h, slot)

    def stats(self) -> dict:
        return self.L.cl_cache_get_stats(self.h).as_dict()


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def make_struct(layer) -> Layer:
    """A Layer struct pointing into the numpy arrays of a clutor_b200.synth.HostLayer (kept alive by the caller)."""
    s = Layer()
    s.ffn_norm, s.router = _ptr(layer.ffn_norm), _ptr(layer.router)
    s.gate_type, s.up_type, s.down_type = layer.gate_type, layer.up_type, layer.down_type
    s.gate, s.up, s.down = _ptr(layer.gate), _ptr(layer.up), _ptr(layer.down)
    s.gate_slab, s.up_slab, s.down_slab = layer.gate_slab, layer.up_slab, layer.down_slab
    s.E, s.FF, s.NE, s.K, s.norm_topk = layer.E, layer.FF, layer.NE, layer.K, layer.norm_topk
    s.resid_scale, s.rms_eps = layer.resid_scale, layer.rms_eps
    return s


def moe_ffn(layer, x: np.ndarray, which: str = "oracle"):
    """Runs one MoE layer on the CPU. ``which`` is "oracle" (the restatement) or "ref" (the reference engine).

    Returns (x_out [T, E] float32, sel [T, K] int32, wt [T, K] float32); x is not modified."""
    x = np.ascontiguousarray(x, dtype=np.float32).copy()
    T = x.shape[0]
    sel = np.zeros((T, layer.K), np.int32)
    wt = np.zeros((T, layer.K), np.float32)
    s = make_struct(layer)
    if which == "oracle":
        rc = oracle_lib().orc_moe_ffn(C.byref(s), C.c_void_p(_ptr(x)), T, C.c_void_p(_ptr(sel)), C.c_void_p(_ptr(wt)))
    else:
        rc = ref_lib().ref_moe_ffn(C.byref(s), C.c_void_p(_ptr(x)), T, C.c_void_p(_ptr(sel)), C.c_void_p(_ptr(wt)))
    if rc:
        raise RuntimeError(f"{which} moe_ffn failed")
    return x, sel, wt


def ref_route_batch(layer, x: np.ndarray):
    """The reference's routing of T tokens alone (rmsnorm, dotf, softmax, top-k, renormalisation; c/src/forward.c:1065-1072,
    1135-1157): (sel [T, K] int32, wt [T, K] float32)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    T = x.shape[0]
    sel = np.zeros((T, layer.K), np.int32)
    wt = np.zeros((T, layer.K), np.float32)
    s = make_struct(layer)
    if ref_lib().ref_route_batch(C.byref(s), C.c_void_p(_ptr(x)), T, C.c_void_p(_ptr(sel)), C.c_void_p(_ptr(wt))):
        raise RuntimeError("ref_route_batch failed")
    return sel, wt


def ref_dispatch(sel: np.ndarray, wt: np.ndarray, n_expert: int):
    """The batched block's dispatch as the reference forms it (c/src/forward.c:1162-1163, 1188-1189): returns (todo, lists)
    with todo the experts in order of first appearance and lists[e] = (who, wgt) for each of them: its tokens ascending and
    their weights."""
    sel = np.ascontiguousarray(sel, dtype=np.int32)
    wt = np.ascontiguousarray(wt, dtype=np.float32)
    T, K = sel.shape
    todo = np.zeros(n_expert, np.int32)
    woff = np.zeros(n_expert + 1, np.int32)
    who = np.zeros(T * K, np.int32)
    wgt = np.zeros(T * K, np.float32)
    n = ref_lib().ref_dispatch(C.c_void_p(_ptr(sel)), C.c_void_p(_ptr(wt)), T, K, n_expert, C.c_void_p(_ptr(todo)),
                               C.c_void_p(_ptr(woff)), C.c_void_p(_ptr(who)), C.c_void_p(_ptr(wgt)))
    if n < 0:
        raise RuntimeError("ref_dispatch failed")
    lists = {int(todo[i]): (who[woff[i]:woff[i + 1]].copy(), wgt[woff[i]:woff[i + 1]].copy()) for i in range(n)}
    return todo[:n].copy(), lists


def set_ref_threads(n: int) -> None:
    ref_lib().cl_set_threads(int(n))


def dequant_row(type_: int, row: np.ndarray, n: int, which: str = "oracle") -> np.ndarray:
    out = np.zeros(n, np.float32)
    row = np.ascontiguousarray(row, dtype=np.uint8)
    if which == "oracle":
        oracle_lib().orc_dequant_row(C.c_uint32(type_), C.c_void_p(_ptr(row)), C.c_void_p(_ptr(out)), n)
    else:
        ref_lib().cl_dequant_row(C.c_uint32(type_), C.c_void_p(_ptr(row)), C.c_void_p(_ptr(out)), n)
    return out


Q8K_DTYPE = np.dtype([("d", "<f4"), ("qs", "i1", 256), ("bsums", "<i2", 16)])   # cl_q8k (c/src/quant.h:22), 292 bytes
assert Q8K_DTYPE.itemsize == 292


def q8k_quantize(x: np.ndarray, which: str = "oracle") -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.size
    out = np.zeros(n // 256, Q8K_DTYPE)
    if which == "oracle":
        oracle_lib().orc_q8k_quantize(C.c_void_p(_ptr(x)), n, C.c_void_p(out.ctypes.data))
    else:
        class XQ(C.Structure):
            _fields_ = [("b", C.c_void_p), ("n", C.c_int)]
        xq = XQ(out.ctypes.data, n)
        ref_lib().cl_xq_quantize(C.byref(xq), C.c_void_p(_ptr(x)))
    return out


def dot_row(type_: int, row: np.ndarray, cols: int, xq: np.ndarray | None, xf: np.ndarray | None) -> float:
    row = np.ascontiguousarray(row, dtype=np.uint8)
    xq_p = C.c_void_p(xq.ctypes.data) if xq is not None else C.c_void_p(0)
    xf_p = C.c_void_p(_ptr(np.ascontiguousarray(xf, dtype=np.float32))) if xf is not None else C.c_void_p(0)
    return oracle_lib().orc_dot_row(C.c_uint32(type_), C.c_void_p(_ptr(row)), cols, xq_p, xf_p)


def ref_matvec(type_: int, w: np.ndarray, rows: int, cols: int, xf: np.ndarray, xq: np.ndarray | None) -> np.ndarray:
    """The reference's cl_matvec_batch on one job (c/src/quant.c:995-1004)."""
    class XQ(C.Structure):
        _fields_ = [("b", C.c_void_p), ("n", C.c_int)]

    class MV(C.Structure):
        _fields_ = [("type", C.c_uint32), ("w", C.c_void_p), ("rows", C.c_int), ("cols", C.c_int), ("xf", C.c_void_p),
                    ("xq", C.c_void_p), ("out", C.c_void_p), ("nb", C.c_int), ("xf_stride", C.c_size_t),
                    ("out_stride", C.c_size_t)]
    w = np.ascontiguousarray(w, dtype=np.uint8)
    xf = np.ascontiguousarray(xf, dtype=np.float32)
    out = np.zeros(rows, np.float32)
    xqs = XQ(xq.ctypes.data, cols) if xq is not None else None
    job = MV(type_, _ptr(w), rows, cols, _ptr(xf), C.addressof(xqs) if xqs is not None else 0, _ptr(out), 1, 0, 0)
    ref_lib().cl_matvec_batch(C.byref(job), 1)
    return out


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float, which: str = "oracle") -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.zeros_like(x)
    fn = oracle_lib().orc_rmsnorm if which == "oracle" else ref_lib().ref_rmsnorm
    fn(C.c_void_p(_ptr(out)), C.c_void_p(_ptr(x)), C.c_void_p(_ptr(w)), x.size, C.c_float(eps))
    return out


def dotf(a: np.ndarray, b: np.ndarray, which: str = "oracle") -> float:
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    fn = oracle_lib().orc_dotf if which == "oracle" else ref_lib().ref_dotf
    fn.restype = C.c_float
    return fn(C.c_void_p(_ptr(a)), C.c_void_p(_ptr(b)), a.size)


def route(logits: np.ndarray, K: int, norm_topk: int = 1, which: str = "oracle"):
    rl = np.ascontiguousarray(logits, dtype=np.float32).copy()
    sel = np.zeros(K, np.int32)
    wt = np.zeros(K, np.float32)
    fn = oracle_lib().orc_route if which == "oracle" else ref_lib().ref_route
    fn(C.c_void_p(_ptr(rl)), rl.size, K, norm_topk, C.c_void_p(_ptr(sel)), C.c_void_p(_ptr(wt)))
    return sel, wt


class RefModel:
    """The reference's whole forward pass (cl_fwd_open / cl_fwd_step, c/src/forward.h:114-118, compiled into
    _ref/libclref.so) on a GGUF file: the checker for the device step."""

    def __init__(self, path: str, n_ctx: int):
        L = ref_lib()
        L.ref_fwd_open.restype = C.c_void_p
        L.ref_fwd_open.argtypes = [C.c_char_p, C.c_int, C.c_char_p, C.c_size_t]
        L.ref_fwd_info.argtypes = [C.c_void_p, C.c_void_p]
        L.ref_fwd_step.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_char_p, C.c_size_t]
        L.ref_fwd_close.argtypes = [C.c_void_p]
        L.ref_fwd_prefill.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_char_p, C.c_size_t]
        self.L = L
        self.err = C.create_string_buffer(512)
        self.h = L.ref_fwd_open(path.encode(), n_ctx, self.err, 512)
        if not self.h:
            raise RuntimeError(self.err.value.decode())
        info = (C.c_int * 8)()
        L.ref_fwd_info(self.h, info)
        self.n_layer, self.n_embd, self.n_vocab, self.n_expert, self.n_used, self.n_ctx, _, self.head_dim = list(info)

    def step(self, token: int):
        """-> (logits [n_vocab] f32, sel [n_layer, n_used] int32, wt [n_layer, n_used] f32)"""
        logits = np.zeros(self.n_vocab, np.float32)
        sel = np.zeros((self.n_layer, self.n_used), np.int32)
        wt = np.zeros((self.n_layer, self.n_used), np.float32)
        if self.L.ref_fwd_step(self.h, token, logits.ctypes.data, sel.ctypes.data, wt.ctypes.data, self.err, 512):
            raise RuntimeError(self.err.value.decode())
        return logits, sel, wt

    def prefill(self, tokens, logits: bool = True):
        """cl_fwd_prefill: the tokens in batches (CLUTOR_PS_B in the environment shrinks them); the logits after the last."""
        t = np.ascontiguousarray(tokens, np.int32)
        out = np.zeros(self.n_vocab, np.float32) if logits else None
        if self.L.ref_fwd_prefill(self.h, t.ctypes.data, len(t), None if out is None else out.ctypes.data, self.err, 512):
            raise RuntimeError(self.err.value.decode())
        return out

    def greedy(self, first: int, n: int) -> list[int]:
        """The reference's generate loop (c/src/main.c:342-360) on ids: feed `first`, then each arg-max, n tokens."""
        out, cur = [], first
        for _ in range(n):
            logits, _, _ = self.step(cur)
            cur = int(np.argmax(logits))   # first maximum: the reference's strict > scan
            out.append(cur)
        return out

    def close(self) -> None:
        if self.h:
            self.L.ref_fwd_close(self.h)
            self.h = None

    def __del__(self):
        self.close()


class RouteResult(C.Structure):
    """cl_route_result (c/src/route.h:16-22) and clb200_route_result: the same layout."""
    _fields_ = [("selected", C.c_int * 32), ("k", C.c_int), ("substituted", C.c_int), ("dropped_mass", C.c_double),
                ("max_delta", C.c_double)]


class Smart(C.Structure):
    """cl_smart (c/src/route.h:14) and clb200_smart."""
    _fields_ = [("enabled", C.c_int), ("J", C.c_int), ("M", C.c_int), ("tau", C.c_double)]


_RESIDENT_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_int)


def smart_route(logits: np.ndarray, K: int, smart: tuple | None = None, resident: np.ndarray | None = None,
                which: str = "oracle") -> dict | None:
    """cl_route (c/src/route.c:13-52) of one token: ``which`` "oracle" (orc_smart_route, the restatement) or "ref" (the
    reference's own cl_route, its resident callback reading ``resident``). smart = (J, M, tau) or None (plain routing).
    Returns {"selected": [K] ints, "substituted", "dropped_mass", "max_delta"}, or None when cl_route refuses the arguments."""
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    E = lg.shape[0]
    res = None if resident is None else np.ascontiguousarray(resident, dtype=np.uint8)
    if which == "oracle":
        sel = (C.c_int * 32)()
        subs, dropped, maxd = C.c_int(0), C.c_double(0), C.c_double(0)
        J, M, tau = smart if smart else (0, 0, 0.0)
        lib = oracle_lib()
        lib.orc_smart_route.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_double, C.c_void_p,
                                        C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
        rc = lib.orc_smart_route(lg.ctypes.data, E, K, 1 if smart else 0, J, M, tau,
                                 None if res is None else res.ctypes.data, C.addressof(sel), C.addressof(subs),
                                 C.addressof(dropped), C.addressof(maxd))
        if rc:
            return None
        return {"selected": list(sel[:K]), "substituted": subs.value, "dropped_mass": dropped.value, "max_delta": maxd.value}
    L = ref_lib()
    L.cl_route.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, _RESIDENT_FN, C.c_void_p, C.POINTER(RouteResult)]
    L.cl_route.restype = C.c_int
    out = RouteResult()
    cb = _RESIDENT_FN(lambda ctx, e: int(res[e]) if res is not None and 0 <= e < E else 0)
    sm = Smart(1, *smart) if smart else None
    rc = L.cl_route(lg.ctypes.data, E, K, C.addressof(sm) if sm else None, cb if res is not None else _RESIDENT_FN(),
                    None, C.byref(out))
    if rc:
        return None
    return {"selected": list(out.selected[:K]), "substituted": out.substituted, "dropped_mass": out.dropped_mass,
            "max_delta": out.max_delta}


def router_probs(layer, x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """The router of one token (c/src/forward.c:950-958): logits = dotf(router row, rmsnorm(x)) and the float softmax
    probabilities, by the restatement. layer: a clutor_b200.synth.HostLayer. -> (logits [NE], probs [NE]) float32."""
    lib = oracle_lib()
    lib.orc_rmsnorm.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_float]
    lib.orc_dotf.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
    lib.orc_dotf.restype = C.c_float
    lib.orc_route.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
    x = np.ascontiguousarray(x, np.float32)
    xn = np.zeros(layer.E, np.float32)
    lib.orc_rmsnorm(xn.ctypes.data, x.ctypes.data, _ptr(layer.ffn_norm), layer.E, layer.rms_eps)
    router = np.ascontiguousarray(layer.router, np.float32).reshape(layer.NE, layer.E)
    logits = np.array([lib.orc_dotf(router[e].ctypes.data, xn.ctypes.data, layer.E) for e in range(layer.NE)], np.float32)
    probs = logits.copy()
    sel = np.zeros(layer.K, np.int32)
    wt = np.zeros(layer.K, np.float32)
    lib.orc_route(probs.ctypes.data, layer.NE, layer.K, layer.norm_topk, sel.ctypes.data, wt.ctypes.data)
    return logits, probs


def router_ahead(next_layer, x: np.ndarray, n: int) -> np.ndarray:
    """Router-ahead (c/src/forward.c:937-946): the NEXT layer's norm and router applied to this layer's x, and its top n
    experts by raw logit, by repeated arg-max with ties to the lower id (a pure-Python loop: NE is small). next_layer: a
    clutor_b200.synth.HostLayer. -> [n] int32 expert ids in pick order."""
    logits, _ = router_probs(next_layer, x)
    taken = np.zeros(next_layer.NE, bool)
    picks = []
    for _k in range(n):
        best = -1
        for e in range(next_layer.NE):
            if not taken[e] and (best < 0 or logits[e] > logits[best]):
                best = e
        taken[best] = True
        picks.append(best)
    return np.array(picks, np.int32)

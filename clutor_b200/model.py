"""Whole models on the device: the reference's forward-pass interface (c/src/forward.h:113-117) over clb200_model_*."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import ClutorError, Context, lib


class ModelInfo(C.Structure):
    """clb200_model_info."""
    _fields_ = [("arch", C.c_char * 16)] + [(n, C.c_int) for n in (
        "n_layer", "n_embd", "n_head", "n_head_kv", "head_dim", "n_ff_exp", "n_expert", "n_used", "n_vocab", "n_ctx")] + [
        ("device_bytes", C.c_uint64), ("smem_bytes", C.c_uint32)]


def _bind(L) -> None:
    if getattr(L, "_model_bound", False):
        return
    L.clb200_model_open.restype = C.c_void_p
    L.clb200_model_open.argtypes = [C.c_void_p, C.c_char_p, C.c_int, C.c_char_p, C.c_size_t]
    L.clb200_model_open_image.restype = C.c_void_p
    L.clb200_model_open_image.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int, C.c_char_p, C.c_size_t]
    L.clb200_model_close.argtypes = [C.c_void_p]
    L.clb200_model_reset.argtypes = [C.c_void_p]
    L.clb200_model_pos.argtypes = [C.c_void_p]
    L.clb200_model_get_info.argtypes = [C.c_void_p, C.POINTER(ModelInfo)]
    L.clb200_model_step.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.POINTER(C.c_int), C.c_void_p, C.c_void_p, C.c_char_p,
                                    C.c_size_t]
    L.clb200_model_generate.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_char_p, C.c_size_t]
    L.clb200_model_generate_async.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_char_p, C.c_size_t]
    L.clb200_model_tokens.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_char_p, C.c_size_t]
    L.clb200_model_prefill.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_char_p, C.c_size_t]
    L.clb200_model_set_batch.argtypes = [C.c_void_p, C.c_int]
    L._model_bound = True


class Model:
    """A GGUF mixture-of-experts model in HBM (clb200_model_open / _open_image) with a key/value cache of n_ctx positions."""

    def __init__(self, ctx: Context, source, n_ctx: int = 512):
        L = lib()
        _bind(L)
        self.L, self.ctx = L, ctx
        self._err = C.create_string_buffer(512)
        if isinstance(source, str):
            self.h = L.clb200_model_open(ctx.handle, source.encode(), n_ctx, self._err, 512)
        else:
            img = np.ascontiguousarray(np.frombuffer(source, dtype=np.uint8) if not isinstance(source, np.ndarray) else source)
            self.h = L.clb200_model_open_image(ctx.handle, img.ctypes.data, img.nbytes, n_ctx, self._err, 512)
        if not self.h:
            raise ClutorError(self._err.value.decode())
        info = ModelInfo()
        L.clb200_model_get_info(self.h, C.byref(info))
        self.info = info
        self.n_vocab, self.n_layer, self.n_used = info.n_vocab, info.n_layer, info.n_used

    def close(self) -> None:
        if getattr(self, "h", None):
            self.L.clb200_model_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def pos(self) -> int:
        return self.L.clb200_model_pos(self.h)

    def reset(self) -> None:
        self.L.clb200_model_reset(self.h)

    def step(self, token: int, logits: bool = True, route: bool = False):
        """cl_fwd_step: -> (logits [n_vocab] or None, next token, (sel, wt) [n_layer, n_used] or None)."""
        lg = np.zeros(self.n_vocab, np.float32) if logits else None
        sel = np.zeros((self.n_layer, self.n_used), np.int32) if route else None
        wt = np.zeros((self.n_layer, self.n_used), np.float32) if route else None
        nxt = C.c_int(-1)
        if self.L.clb200_model_step(self.h, token, lg.ctypes.data if lg is not None else None, C.byref(nxt),
                                    sel.ctypes.data if route else None, wt.ctypes.data if route else None, self._err, 512):
            raise ClutorError(self._err.value.decode())
        return lg, nxt.value, ((sel, wt) if route else None)

    def prefill(self, tokens, logits: bool = True):
        """cl_fwd_prefill (clb200_model_prefill): the tokens in batches; the logits after the last one, or None."""
        t = np.ascontiguousarray(tokens, np.int32)
        lg = np.zeros(self.n_vocab, np.float32) if logits else None
        if self.L.clb200_model_prefill(self.h, t.ctypes.data, len(t), lg.ctypes.data if lg is not None else None, self._err, 512):
            raise ClutorError(self._err.value.decode())
        return lg

    def set_batch(self, tokens: int) -> None:
        """Tokens per prefill batch (the reference's CLUTOR_PS_B), 1..512."""
        if self.L.clb200_model_set_batch(self.h, tokens):
            raise ClutorError(f"a prefill batch of {tokens} tokens is out of range")

    def generate(self, token: int, n: int) -> list[int]:
        """Greedy generation on the device: feeds `token`, then each arg-max; returns the n chosen tokens."""
        out = np.zeros(n, np.int32)
        if self.L.clb200_model_generate(self.h, token, n, out.ctypes.data, self._err, 512):
            raise ClutorError(self._err.value.decode())
        return out.tolist()

    def generate_async(self, token: int, n: int, stream: int = 0) -> None:
        if self.L.clb200_model_generate_async(self.h, token, n, C.c_void_p(stream) if stream else None, self._err, 512):
            raise ClutorError(self._err.value.decode())

    def tokens(self, start: int, n: int) -> list[int]:
        out = np.zeros(n, np.int32)
        if self.L.clb200_model_tokens(self.h, start, n, out.ctypes.data, self._err, 512):
            raise ClutorError(self._err.value.decode())
        return out.tolist()

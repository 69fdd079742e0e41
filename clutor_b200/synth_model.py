"""Seeded synthetic mixture-of-experts models as GGUF files or images.

There are no model files here, so whole-model workloads use random weights with a real model's shapes and tensor types.
The tensors and metadata are the ones the reference's forward pass binds (c/src/forward.c:110-240) for the qwen3moe
architecture (and olmoe / granitemoe by name); the "Q4_K_M" mix follows llama.cpp's: Q4_K for the embedding, attn_q,
attn_k, attn_output and the gate/up experts, Q6_K for attn_v, the down experts and the output matrix.

Weights follow the distributions of ``synth.quant_tensor`` (random 6-bit scales and mins, fp16 block scales
~ U(0.001, 0.02)); norm weights are 1 + N(0, 0.1^2), routers N(0, 0.02^2). Small models draw every byte from the
reproducible splitmix64 streams of ``synth``; large ones (``fast``) draw quant bytes from numpy's PCG64 for speed.
"""
from __future__ import annotations

from dataclasses import dataclass, replace

import numpy as np

from . import gguf
from .synth import BLOCK_BYTES, BLOCK_ELEMS, T_F32, T_Q4_K, T_Q6_K, _normal, quant_tensor, row_bytes


@dataclass(frozen=True)
class Spec:
    arch: str = "qwen3moe"
    n_layer: int = 48
    E: int = 2048
    n_head: int = 32
    n_kv: int = 4
    hd: int = 128
    FF: int = 768
    NE: int = 128
    K: int = 8
    vocab: int = 151936
    ctx: int = 40960          # context_length (the cache is sized by the caller's n_ctx)
    eps: float = 1e-6
    theta: float = 1e6
    embd_type: int = T_Q4_K
    q_type: int = T_Q4_K
    k_type: int = T_Q4_K
    v_type: int = T_Q6_K
    o_type: int = T_Q4_K
    gate_type: int = T_Q4_K
    down_type: int = T_Q6_K
    out_type: int = T_Q6_K

    @property
    def n_q(self) -> int:
        return self.n_head * self.hd

    @property
    def n_kvw(self) -> int:
        return self.n_kv * self.hd


QWEN3_30B_A3B = Spec()


def tiny(**kw) -> Spec:
    """A small qwen3moe-shaped model for parity tests: 2 layers, width 256, GQA 2:1 with head_dim 128, 8 experts, top 2."""
    base = Spec(n_layer=2, E=256, n_head=2, n_kv=1, hd=128, FF=256, NE=8, K=2, vocab=512, ctx=1024)
    return replace(base, **kw)


def _quant(type_: int, rows: int, cols: int, seed: int, stream: int, fast: bool) -> np.ndarray:
    n = rows * cols
    if not fast:
        return quant_tensor(type_, n, seed, stream)
    nblk = n // BLOCK_ELEMS[type_]
    bb = BLOCK_BYTES[type_]
    rng = np.random.Generator(np.random.PCG64([seed, stream]))
    raw = np.frombuffer(rng.bytes(nblk * bb), dtype=np.uint8).reshape(nblk, bb).copy()
    d = (0.001 + 0.019 * rng.random(nblk, dtype=np.float32)).astype(np.float16).view(np.uint8).reshape(nblk, 2)
    if type_ == T_Q4_K:
        raw[:, 0:2] = d
        raw[:, 2:4] = (0.001 + 0.019 * rng.random(nblk, dtype=np.float32)).astype(np.float16).view(np.uint8).reshape(nblk, 2)
    elif type_ == T_Q6_K:
        raw[:, 208:210] = d
    else:
        raw[:, 0:2] = d
    return raw.reshape(-1)


def _floats(n: int, seed: int, stream: int, base: float, scale: float) -> np.ndarray:
    return (base + scale * _normal(seed, stream, n)).astype(np.float32)


def writer(spec: Spec, seed: int = 1, fast: bool | None = None) -> gguf.Writer:
    """A GGUF writer holding every tensor of the model (as lazily generated arrays) and its metadata."""
    s = spec
    if fast is None:
        fast = s.n_layer * s.NE * s.FF * s.E > (1 << 30)
    w = gguf.Writer()
    A = s.arch
    w.add("general.architecture", gguf.STR, A)
    w.add("general.name", gguf.STR, f"synthetic-{A}-{s.n_layer}x{s.E}")
    w.add("general.alignment", gguf.U32, gguf.ALIGN)
    w.add(f"{A}.block_count", gguf.U32, s.n_layer)
    w.add(f"{A}.context_length", gguf.U32, s.ctx)
    w.add(f"{A}.embedding_length", gguf.U32, s.E)
    w.add(f"{A}.expert_feed_forward_length" if A in ("qwen3moe", "qwen3vlmoe") else f"{A}.feed_forward_length", gguf.U32, s.FF)
    w.add(f"{A}.attention.head_count", gguf.U32, s.n_head)
    w.add(f"{A}.attention.head_count_kv", gguf.U32, s.n_kv)
    w.add(f"{A}.rope.freq_base", gguf.F32, s.theta)
    w.add(f"{A}.attention.layer_norm_rms_epsilon", gguf.F32, s.eps)
    w.add(f"{A}.expert_used_count", gguf.U32, s.K)
    w.add(f"{A}.expert_count", gguf.U32, s.NE)
    if A in ("qwen3moe", "qwen3vlmoe"):
        w.add(f"{A}.attention.key_length", gguf.U32, s.hd)
        w.add(f"{A}.attention.value_length", gguf.U32, s.hd)
    stream = [0]

    def nxt() -> int:
        stream[0] += 16
        return stream[0]

    def q(name, type_, rows, cols, ne=None):
        st = nxt()
        dims = [cols, rows] + ([ne] if ne else [])
        n_rows = rows * (ne or 1)
        w.add_tensor(name, dims, type_, _Lazy(lambda: _quant(type_, n_rows, cols, seed, st, fast), n_rows * row_bytes(type_, cols)))

    def f(name, n, base, scale, dims=None):
        st = nxt()
        w.add_tensor(name, dims or [n], T_F32, _Lazy(lambda: _floats(n, seed, st, base, scale), 4 * n))

    q("token_embd.weight", s.embd_type, s.vocab, s.E)
    f("output_norm.weight", s.E, 1.0, 0.1)
    q("output.weight", s.out_type, s.vocab, s.E)
    qk_per_head = A in ("qwen3moe", "qwen3vlmoe")
    for l in range(s.n_layer):
        p = f"blk.{l}."
        f(p + "attn_norm.weight", s.E, 1.0, 0.1)
        q(p + "attn_q.weight", s.q_type, s.n_q, s.E)
        q(p + "attn_k.weight", s.k_type, s.n_kvw, s.E)
        q(p + "attn_v.weight", s.v_type, s.n_kvw, s.E)
        q(p + "attn_output.weight", s.o_type, s.E, s.n_q)
        if A != "granitemoe":
            f(p + "attn_q_norm.weight", s.hd if qk_per_head else s.n_q, 1.0, 0.1)
            f(p + "attn_k_norm.weight", s.hd if qk_per_head else s.n_kvw, 1.0, 0.1)
        f(p + "ffn_norm.weight", s.E, 1.0, 0.1)
        f(p + "ffn_gate_inp.weight", s.NE * s.E, 0.0, 0.02, dims=[s.E, s.NE])
        q(p + "ffn_gate_exps.weight", s.gate_type, s.FF, s.E, s.NE)
        q(p + "ffn_up_exps.weight", s.gate_type, s.FF, s.E, s.NE)
        q(p + "ffn_down_exps.weight", s.down_type, s.E, s.FF, s.NE)
    return w


class _Lazy:
    """Tensor data made when the file or image is written (so a 20 GB model never sits in memory twice)."""

    def __init__(self, make, nbytes: int):
        self.make, self._n = make, nbytes

    @property
    def nbytes(self) -> int:
        return self._n

    def __call__(self) -> np.ndarray:
        a = self.make()
        assert a.nbytes == self._n, (a.nbytes, self._n)
        return a


def write(path: str, spec: Spec, seed: int = 1, fast: bool | None = None) -> int:
    """Writes the model to a GGUF file; returns its size."""
    return writer(spec, seed, fast).write(path)


def image(spec: Spec, seed: int = 1, fast: bool | None = None) -> np.ndarray:
    """The model as one GGUF image in host memory (a uint8 array), for clb200_model_open_image."""
    return writer(spec, seed, fast).image()


def model_bytes(spec: Spec) -> dict:
    """Bytes one token reads, by part (weights only; the key/value cache adds 2 * 2 * n_kvw bytes per layer and position)."""
    s = spec
    experts = s.n_layer * s.K * (2 * s.FF * row_bytes(s.gate_type, s.E) + s.E * row_bytes(s.down_type, s.FF))
    attention = s.n_layer * (s.n_q * row_bytes(s.q_type, s.E) + s.n_kvw * (row_bytes(s.k_type, s.E) + row_bytes(s.v_type, s.E))
                             + s.E * row_bytes(s.o_type, s.n_q))
    routers = s.n_layer * s.NE * s.E * 4
    output = s.vocab * row_bytes(s.out_type, s.E)
    return {"experts": experts, "attention": attention, "routers": routers, "output": output,
            "embedding_row": row_bytes(s.embd_type, s.E), "total": experts + attention + routers + output}

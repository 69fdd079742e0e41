"""Seeded synthetic MoE layers in GGUF block layout.

There are no model files or datasets here, so every workload is synthetic, with the shapes and value distributions of the
Qwen3-30B-A3B / Qwen3-235B-A22B MoE layers:

* expert weights are fused GGUF tensors (gate/up ``[E, FF, NE]``, down ``[FF, E, NE]``), one expert's slab after another,
  stored as ggml blocks:
  - Q4_K: fp16 d and dmin ~ U(0.001, 0.02), 12 random scale bytes (random 6-bit scales and mins), 128 random nibble bytes;
  - Q6_K: random low/high bits, random int8 scales, fp16 d ~ U(0.001, 0.02);
  - Q8_0: fp16 d ~ U(0.001, 0.02), uniform int8 quants;
* the router is fp32 ``[NE, E]`` ~ N(0, 0.02^2); the RMSNorm weight is fp32 1 + N(0, 0.1^2); activations are N(0, 1)
  (host normals are a four-uniform Irwin-Hall approximation, bit-reproducible across machines).

``HostLayer`` holds numpy arrays, generated with a splitmix64 stream per tensor (deterministic on any machine).
``device_layer`` fills the same structure on a CUDA device with torch's generator (fast, for full-size benchmarks).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

T_F32, T_F16, T_Q8_0, T_Q4_K, T_Q6_K = 0, 1, 8, 12, 14
BLOCK_ELEMS = {T_F32: 1, T_F16: 1, T_Q8_0: 32, T_Q4_K: 256, T_Q6_K: 256}
BLOCK_BYTES = {T_F32: 4, T_F16: 2, T_Q8_0: 34, T_Q4_K: 144, T_Q6_K: 210}
TYPE_NAMES = {"q4_k": T_Q4_K, "q6_k": T_Q6_K, "q8_0": T_Q8_0}


def row_bytes(type_: int, n: int) -> int:
    return n // BLOCK_ELEMS[type_] * BLOCK_BYTES[type_]


_MASK = (1 << 64) - 1


def splitmix64(seed: int, stream: int, n: int) -> np.ndarray:
    """n outputs of splitmix64 (Steele, Lea, Flood 2014) started at a state derived from (seed, stream)."""
    base = np.uint64(((seed * 0x9E3779B97F4A7C15) ^ (stream * 0xD1B54A32D192ED03) ^ 0x5851F42D4C957F2D) & _MASK)
    z = base + np.arange(1, n + 1, dtype=np.uint64) * np.uint64(0x9E3779B97F4A7C15)
    z ^= z >> np.uint64(30)
    z *= np.uint64(0xBF58476D1CE4E5B9)
    z ^= z >> np.uint64(27)
    z *= np.uint64(0x94D049BB133111EB)
    z ^= z >> np.uint64(31)
    return z


def _bytes(seed: int, stream: int, n: int) -> np.ndarray:
    return splitmix64(seed, stream, (n + 7) // 8).view(np.uint8)[:n].copy()


def _uniform(seed: int, stream: int, n: int) -> np.ndarray:
    return (splitmix64(seed, stream, n) >> np.uint64(11)).astype(np.float64) * (1.0 / (1 << 53))


def _normal(seed: int, stream: int, n: int) -> np.ndarray:
    """Approximately N(0, 1): the Irwin-Hall sum of four uniforms, centred and scaled to unit variance. Only additions and
    multiplications, so the values are the same bits on every machine (no library transcendental functions)."""
    u = _uniform(seed, stream, 4 * n).reshape(4, n)
    return ((u[0] + u[1]) + (u[2] + u[3]) - 2.0) * np.sqrt(3.0)


def quant_tensor(type_: int, n_elems: int, seed: int, stream: int) -> np.ndarray:
    """n_elems weights of a GGUF block type as raw bytes, with the distributions described in the module docstring."""
    nblk = n_elems // BLOCK_ELEMS[type_]
    bb = BLOCK_BYTES[type_]
    raw = _bytes(seed, stream, nblk * bb).reshape(nblk, bb)
    d = (0.001 + 0.019 * _uniform(seed, stream + 1, nblk)).astype(np.float16).view(np.uint16)
    if type_ == T_Q4_K:
        dm = (0.001 + 0.019 * _uniform(seed, stream + 2, nblk)).astype(np.float16).view(np.uint16)
        raw[:, 0:2] = d.view(np.uint8).reshape(nblk, 2)
        raw[:, 2:4] = dm.view(np.uint8).reshape(nblk, 2)
    elif type_ == T_Q6_K:
        raw[:, 208:210] = d.view(np.uint8).reshape(nblk, 2)
    elif type_ == T_Q8_0:
        raw[:, 0:2] = d.view(np.uint8).reshape(nblk, 2)
    else:
        raise ValueError(f"unsupported type {type_}")
    return raw.reshape(-1)


@dataclass
class HostLayer:
    """One MoE layer's tensors on the host, laid out as the reference binds them (c/src/forward.h:18-29)."""
    E: int
    FF: int
    NE: int
    K: int
    gate_type: int
    up_type: int
    down_type: int
    ffn_norm: np.ndarray
    router: np.ndarray
    gate: np.ndarray
    up: np.ndarray
    down: np.ndarray
    norm_topk: int = 1
    resid_scale: float = 1.0
    rms_eps: float = 1e-6

    @property
    def gate_slab(self) -> int:
        return self.FF * row_bytes(self.gate_type, self.E)

    @property
    def up_slab(self) -> int:
        return self.FF * row_bytes(self.up_type, self.E)

    @property
    def down_slab(self) -> int:
        return self.E * row_bytes(self.down_type, self.FF)

    @property
    def expert_bytes(self) -> int:
        return self.gate_slab + self.up_slab + self.down_slab


def host_layer(E: int = 2048, FF: int = 768, NE: int = 128, K: int = 8, gate_type: int = T_Q4_K,
               down_type: int | None = None, seed: int = 1, router_scale: float = 0.02, norm_topk: int = 1,
               resid_scale: float = 1.0, rms_eps: float = 1e-6) -> HostLayer:
    """A seeded layer. gate and up share gate_type; down defaults to gate_type (the Q4_K_M mix uses Q6_K for down)."""
    down_type = gate_type if down_type is None else down_type
    s = 1000 * seed
    return HostLayer(
        E=E, FF=FF, NE=NE, K=K, gate_type=gate_type, up_type=gate_type, down_type=down_type,
        ffn_norm=(1.0 + 0.1 * _normal(seed, s + 1, E)).astype(np.float32),
        router=(router_scale * _normal(seed, s + 3, NE * E)).astype(np.float32).reshape(NE, E),
        gate=quant_tensor(gate_type, NE * FF * E, seed, s + 10),
        up=quant_tensor(gate_type, NE * FF * E, seed, s + 20),
        down=quant_tensor(down_type, NE * E * FF, seed, s + 30),
        norm_topk=norm_topk, resid_scale=resid_scale, rms_eps=rms_eps)


def activations(T: int, E: int, seed: int = 7) -> np.ndarray:
    """x ~ N(0, 1) fp32 [T, E]."""
    return _normal(seed, 99, T * E).astype(np.float32).reshape(T, E)


# ---------------------------------------------------------------------------------------------------------------------
# Device generation (torch): same layout and distributions, a different (torch) random stream.

def device_quant_tensor(type_: int, n_elems: int, gen, device):
    import torch
    nblk = n_elems // BLOCK_ELEMS[type_]
    bb = BLOCK_BYTES[type_]
    raw = torch.randint(0, 256, (nblk, bb), dtype=torch.uint8, device=device, generator=gen)

    def scales():
        return (0.001 + 0.019 * torch.rand(nblk, device=device, generator=gen)).to(torch.float16).view(torch.uint8).view(nblk, 2)
    if type_ == T_Q4_K:
        raw[:, 0:2] = scales()
        raw[:, 2:4] = scales()
    elif type_ == T_Q6_K:
        raw[:, 208:210] = scales()
    elif type_ == T_Q8_0:
        raw[:, 0:2] = scales()
    else:
        raise ValueError(f"unsupported type {type_}")
    return raw.view(-1)


@dataclass
class DeviceLayer:
    """A layer whose tensors are torch CUDA tensors (same fields as HostLayer)."""
    E: int
    FF: int
    NE: int
    K: int
    gate_type: int
    up_type: int
    down_type: int
    ffn_norm: object
    router: object
    gate: object
    up: object
    down: object
    norm_topk: int = 1
    resid_scale: float = 1.0
    rms_eps: float = 1e-6

    gate_slab = HostLayer.gate_slab
    up_slab = HostLayer.up_slab
    down_slab = HostLayer.down_slab
    expert_bytes = HostLayer.expert_bytes


def device_layer(E: int = 2048, FF: int = 768, NE: int = 128, K: int = 8, gate_type: int = T_Q4_K,
                 down_type: int | None = None, seed: int = 1, device="cuda", router_scale: float = 0.02,
                 norm_topk: int = 1, resid_scale: float = 1.0, rms_eps: float = 1e-6) -> DeviceLayer:
    import torch
    down_type = gate_type if down_type is None else down_type
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    return DeviceLayer(
        E=E, FF=FF, NE=NE, K=K, gate_type=gate_type, up_type=gate_type, down_type=down_type,
        ffn_norm=(1.0 + 0.1 * torch.randn(E, device=device, generator=gen)).float(),
        router=(router_scale * torch.randn(NE, E, device=device, generator=gen)).float(),
        gate=device_quant_tensor(gate_type, NE * FF * E, gen, device),
        up=device_quant_tensor(gate_type, NE * FF * E, gen, device),
        down=device_quant_tensor(down_type, NE * E * FF, gen, device),
        norm_topk=norm_topk, resid_scale=resid_scale, rms_eps=rms_eps)


def to_host(layer: DeviceLayer) -> HostLayer:
    """Copies a DeviceLayer's tensors to numpy (for checking a device-generated layer with the oracle)."""
    return HostLayer(E=layer.E, FF=layer.FF, NE=layer.NE, K=layer.K, gate_type=layer.gate_type, up_type=layer.up_type,
                     down_type=layer.down_type, ffn_norm=layer.ffn_norm.cpu().numpy(), router=layer.router.cpu().numpy(),
                     gate=layer.gate.cpu().numpy(), up=layer.up.cpu().numpy(), down=layer.down.cpu().numpy(),
                     norm_topk=layer.norm_topk, resid_scale=layer.resid_scale, rms_eps=layer.rms_eps)


# ---- synthetic expert-selection stream for the cache stress workload -----------------------------------------------------
# The reference's own stress harness draws router logits with this generator (c/src/stream.c:114-140): per layer a fixed
# Zipf-like popularity (a seeded permutation of experts, logit -3 * locality * ln(rank + 1) / ln(E)), 8 "topics" that each
# lift 12 experts per layer by 1.5 and change every 16 tokens, and unit Gaussian noise per (token, layer, expert); the
# predictor's logits share the noise with correlation rho. Restated here (vectorised) so the cache workload sees the
# reference's key stream; routing from these logits is the plain top-K (c/src/route.c:13-30).

_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def _mix64(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.uint64)
    with np.errstate(over="ignore"):
        x = x + np.uint64(0x9E3779B97F4A7C15)
        x = (x ^ (x >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        x = (x ^ (x >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return x ^ (x >> np.uint64(31))


def _unit(x: np.ndarray) -> np.ndarray:
    return (_mix64(x) >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)


def _gauss(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        return (_unit(x) + _unit(x + np.uint64(1)) + _unit(x + np.uint64(2)) + _unit(x + np.uint64(3)) - 2.0) * 1.7320508


class ExpertStream:
    """Router logits of the reference's stress harness: logits(t, l) for token t and layer l, float32 [E]."""

    TOPICS, TOPIC_LEN = 8, 16

    def __init__(self, L: int, E: int, locality: float = 1.0, seed: int = 1, rho: float = 0.8):
        self.L, self.E, self.seed, self.rho, self.sigma = L, E, seed, rho, 1.0
        self.base = np.zeros((L, E), np.float32)
        self.bonus = np.zeros((self.TOPICS, L, E), np.float32)
        s = np.uint64(seed)
        for l in range(L):
            perm = list(range(E))
            for i in range(E - 1, 0, -1):
                j = int(_mix64(s ^ np.uint64(l << 20) ^ np.uint64(i)) % np.uint64(i + 1))
                perm[i], perm[j] = perm[j], perm[i]
            for rank in range(E):
                self.base[l, perm[rank]] = np.float32(-3.0 * locality * np.log(rank + 1.0) / np.log(E))
            for tp in range(self.TOPICS):
                for k in range(min(12, E)):
                    e = int(_mix64(s ^ np.uint64(0xABCDEF) ^ np.uint64(tp << 32) ^ np.uint64(l << 16) ^ np.uint64(k)) % np.uint64(E))
                    self.bonus[tp, l, e] += np.float32(1.5)

    def logits(self, t: np.ndarray | int, l: int, predicted: bool = False) -> np.ndarray:
        """[len(t), E] float32 logits of layer l for tokens t (topics drift every 16 tokens)."""
        t = np.atleast_1d(np.asarray(t, dtype=np.int64))
        e = np.arange(self.E, dtype=np.uint64)
        with np.errstate(over="ignore"):
            k = (np.uint64(self.seed) ^ (t.astype(np.uint64)[:, None] << np.uint64(24)) ^ np.uint64(l << 12)
                 ^ (e[None, :] * np.uint64(0x9E3779B1)))
            n = _gauss(k * np.uint64(4) + np.uint64(1))
            if predicted:
                n = self.rho * n + np.sqrt(max(0.0, 1.0 - self.rho * self.rho)) * _gauss(k * np.uint64(4) + np.uint64(7777))
        tp = (t // self.TOPIC_LEN) % self.TOPICS
        out = (self.base[l][None, :] + self.bonus[tp, l]).astype(np.float64) + self.sigma * n   # float sum, then double
        return out.astype(np.float32)


def route_topk(logits: np.ndarray, K: int) -> tuple[np.ndarray, np.ndarray]:
    """Plain top-K of each row of logits (c/src/route.c:17-23): softmax in double, best first, ties to the lower id.
    Returns (sel int32 [n, K], p float32 [n, K] -- the chosen probabilities, not renormalised)."""
    lg = np.atleast_2d(logits).astype(np.float64)
    p = np.exp(lg - lg.max(axis=1, keepdims=True))
    p /= p.sum(axis=1, keepdims=True)
    order = np.lexsort((np.broadcast_to(np.arange(lg.shape[1]), lg.shape), -p), axis=1)[:, :K]
    return order.astype(np.int32), np.take_along_axis(p, order, axis=1).astype(np.float32)

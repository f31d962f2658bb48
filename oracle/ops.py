"""Oracle per-op math: numpy float32 restatements of the reference's torch ops.

Each function follows the torch reference backend in breezetoken/backends.py
line by line (TEST INFRASTRUCTURE: see oracle/__init__.py).
"""

from __future__ import annotations

import numpy as np

F32 = np.float32


def linear(x: np.ndarray, w_kn: np.ndarray) -> np.ndarray:
    """backends.py:109-112 / 182-184: x.reshape(-1) @ w with w (K, N), f32."""
    return (x.reshape(-1).astype(F32) @ w_kn.astype(F32, copy=False)).reshape(-1)


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """backends.py:119-123 / 187-189: x * rsqrt(mean(x^2) + eps) * w."""
    xf = x.astype(F32)
    r = F32(1.0) / np.sqrt(np.mean(xf * xf, axis=-1, keepdims=True, dtype=F32) + F32(eps))
    return (xf * r) * w.astype(F32)


def fused_add_rms_norm(a: np.ndarray, b: np.ndarray, w: np.ndarray, eps: float):
    """backends.py:229-238: h = a + b; (h, rms_norm(h))."""
    h = a.astype(F32) + b.reshape(a.shape).astype(F32)
    return h, rms_norm(h, w, eps)


def silu(x: np.ndarray) -> np.ndarray:
    """torch.nn.functional.silu: x * sigmoid(x)."""
    x = x.astype(F32)
    return x / (F32(1.0) + np.exp(-x))


def sigmoid(x: np.ndarray) -> np.ndarray:
    return F32(1.0) / (F32(1.0) + np.exp(-x.astype(F32)))


def softplus(x: np.ndarray) -> np.ndarray:
    """torch.nn.functional.softplus (beta 1, threshold 20)."""
    x = x.astype(F32)
    return np.where(x > 20, x, np.log1p(np.exp(np.minimum(x, 20)))).astype(F32)


def silu_mul(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """backends.py:160-163."""
    return silu(gate) * up.astype(F32)


def rope_tables(rope_dim: int, theta: float, cap: int) -> tuple[np.ndarray, np.ndarray]:
    """model/layers.py:26-32: inv = theta^(-arange(half)/half), freqs = [phases, phases]."""
    half = rope_dim // 2
    inv = (F32(theta) ** (-np.arange(0, half, dtype=F32) / F32(half))).astype(F32)
    phases = np.outer(np.arange(cap, dtype=F32), inv).astype(F32)
    freqs = np.concatenate([phases, phases], axis=-1)
    return np.cos(freqs).astype(F32), np.sin(freqs).astype(F32)


def rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, p: int, rope_dim: int) -> np.ndarray:
    """backends.py:218-226: partial rotate-half RoPE at position p."""
    rot = x[..., :rope_dim].astype(F32)
    tail = x[..., rope_dim:].astype(F32)
    half = rope_dim // 2
    turned = rot * cos[p] + np.concatenate([-rot[..., half:], rot[..., :half]], axis=-1) * sin[p]
    return np.concatenate([turned, tail], axis=-1).astype(F32)


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float) -> np.ndarray:
    """backends.py:196-215: q (H, D), k/v (S, Hkv, D); head h uses KV head h // (H/Hkv)."""
    heads, dim = q.shape
    groups = k.shape[1]
    group = heads // groups
    qg = q.astype(F32).reshape(groups, group, dim)
    kf = k.astype(F32)
    vf = v.astype(F32)
    scores = np.einsum("kgd,skd->kgs", qg, kf) * F32(scale)
    scores = scores - scores.max(axis=-1, keepdims=True)
    e = np.exp(scores)
    probs = e / e.sum(axis=-1, keepdims=True)
    return np.einsum("kgs,skd->kgd", probs, vf).reshape(heads, dim).astype(F32)


def gdn_decode(q, k, v, g, beta, state, scale: float, eps: float = 1e-6) -> np.ndarray:
    """backends.py:241-271: one gated-delta-rule step; ``state`` updated in place."""
    heads_k, dim = q.shape
    heads_v = v.shape[0]
    qf, kf, vf = q.astype(F32), k.astype(F32), v.astype(F32)
    qn = qf / np.sqrt((qf * qf).sum(-1, keepdims=True) + F32(eps)) * F32(scale)
    kn = kf / np.sqrt((kf * kf).sum(-1, keepdims=True) + F32(eps))
    index = np.arange(heads_v) % heads_k
    decayed = state * np.exp(g.astype(F32)).reshape(heads_v, 1, 1)
    recalled = np.einsum("hdv,hd->hv", decayed, kn[index])
    delta = (vf - recalled) * sigmoid(beta).reshape(heads_v, 1)
    state[...] = decayed + kn[index][:, :, None] * delta[:, None, :]
    return np.einsum("hdv,hd->hv", state, qn[index]).astype(F32)


def argmax_first(x: np.ndarray) -> int:
    """torch.argmax / np.argmax: index of the first maximum."""
    return int(np.argmax(x))

"""Oracle MoE routing and expert evaluation (TEST INFRASTRUCTURE ONLY).

* route: breezetoken/model/moe.py:33-39 -- softmax over the router logits,
  top-k, renormalise by the (clamped) sum.
* experts: moe.py:225-233 -- dequantise the selected experts' gate/up rows,
  gu = rows @ x, act = silu(gate) * up, dequantise down, weighted sum.
* shared expert: model/qwen36_moe.py:634-642 -- sigmoid(x . g_sh) *
  down(silu(gate x) * up x), added to the routed output.
"""

from __future__ import annotations

import numpy as np

from oracle import ops
from oracle.dequant import dequant_iq3_s

F32 = np.float32
WEIGHT_SUM_MIN = F32(6.103515625e-5)


def route(logits: np.ndarray, top_k: int) -> tuple[np.ndarray, np.ndarray]:
    """(weights f32, expert ids) in descending weight order; ties -> lower id."""
    lg = logits.astype(F32)
    e = np.exp(lg - lg.max())
    probs = (e / e.sum(dtype=F32)).astype(F32)
    ids = np.argsort(-probs, kind="stable")[:top_k]
    w = probs[ids]
    return (w / max(w.sum(dtype=F32), WEIGHT_SUM_MIN)).astype(F32), ids.astype(np.int64)


def experts(x, gate_raw, up_raw, down_raw, ids, weights, hidden: int, ffn: int) -> np.ndarray:
    """Routed output of one token; *_raw are the full IQ3_S tensors as (E*rows, row_bytes) bytes."""
    xf = x.astype(F32).reshape(-1)
    out = np.zeros(hidden, F32)
    for e, w in zip(ids, weights, strict=True):
        g = dequant_iq3_s(gate_raw[e * ffn : (e + 1) * ffn], ffn, hidden) @ xf
        u = dequant_iq3_s(up_raw[e * ffn : (e + 1) * ffn], ffn, hidden) @ xf
        act = ops.silu(g) * u
        d = dequant_iq3_s(down_raw[e * hidden : (e + 1) * hidden], hidden, ffn) @ act
        out += d * F32(w)
    return out


def shared_expert(x, sh_gate, sh_up, sh_down, sh_gate_inp) -> np.ndarray:
    xf = x.astype(F32).reshape(-1)
    act = ops.silu(sh_gate @ xf) * (sh_up @ xf)
    return ops.sigmoid(np.array(sh_gate_inp @ xf, dtype=F32)) * (sh_down @ act)

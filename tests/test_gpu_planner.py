"""The planner's byte model against the buffers the loaders actually
allocate (the tiny checkpoints with the real per-layer shapes)."""

from __future__ import annotations

import pytest
import torch

from breezetoken_b200.planner import model_bytes

pytestmark = pytest.mark.gpu


def _bytes(t) -> int:
    return t.numel() * t.element_size()


def test_weight_bytes_match_the_qwen36_loader(cuda, qwen36_tiny_gguf) -> None:
    from breezetoken_b200.qwen36_moe import Qwen36Moe

    m = Qwen36Moe(qwen36_tiny_gguf, max_context=64)
    try:
        got = _bytes(m.embd) + _bytes(m.head) + _bytes(m.norm_f)
        for layer in m.layers:
            for v in layer.values():
                if isinstance(v, torch.Tensor):
                    got += _bytes(v)
            ex, sh = layer["experts"], layer["shared"]
            got += _bytes(ex.gate) + _bytes(ex.up) + _bytes(ex.down)
            got += _bytes(sh.gate) + _bytes(sh.up) + _bytes(sh.down) + _bytes(sh.gate_inp)
        assert got == model_bytes(m.cfg).weights
        p = m.placement
        assert p.gpu_layers == m.cfg.n_layers and p.n_gpus == 1 and p.weight_bytes == got
    finally:
        m.close()


def test_weight_and_state_bytes_match_the_qwen35_loader(cuda, tiny_gguf) -> None:
    from breezetoken_b200.model import Qwen35

    m = Qwen35(tiny_gguf, max_context=64, batch=2)
    try:
        mb = model_bytes(m.cfg)
        assert m.placement.weight_bytes == mb.weights
        q8 = m.weight_bytes  # the Q8_0 matrices (embedding / head included)
        assert 0 < mb.weights - q8 < 0.05 * mb.weights  # the rest: f32 norms, conv and SSM parameters
        assert m.placement.state_bytes_per_sequence == mb.state_per_sequence + 64 * mb.kv_per_token
    finally:
        m.close()

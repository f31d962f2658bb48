"""The config-5 decoder's host composition, checked on the CPU.

``Qwen36Moe`` (and the ``B200Backend`` / MoE helpers under it) reach the
library only through ``_native.call`` and ``_native.load``.  Here every C-ABI
entry point they use is emulated on host memory with numpy, following the
contract in include/bt_b200.h and the oracle's restatement of the reference
math, and the unchanged Python mirror decodes the seeded 4-layer checkpoint
with the config-5 layer shapes.  Its greedy tokens must be the reference's
(``Qwen36Moe(device="cpu", dtype="f32")``, golden fixture) and its first
logits within 1e-4 of their scale.  What this covers is the host side: weight
loading and orientation, the stacked [beta | alpha] projection, the strided
q / k / v / beta views handed to the recurrence, the residual adds fused with
the following norm, the KV writes and attended lengths, routing and the
shared expert's inputs.  The kernels themselves are checked on the GPU.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from breezetoken_b200 import qwen36_moe
from tests.abi_emulator import install
from tests.conftest import golden


@pytest.fixture()
def emulated(monkeypatch):
    return install(monkeypatch)


def test_qwen36_host_composition_reproduces_reference(emulated, qwen36_tiny_gguf) -> None:
    g = golden("qwen36_tiny")
    m = qwen36_moe.Qwen36Moe(qwen36_tiny_gguf, device="cpu", max_context=int(g["max_context"]))
    prompt, steps = g["prompt"].tolist(), 12
    m.reset()
    for i, t in enumerate(prompt):
        logits = m.forward_token(t, i, logits=(i == len(prompt) - 1))
    got, want = logits.numpy(), g["logits"][0]
    assert np.abs(got - want).max() <= 1e-4 * np.abs(want).max()
    toks = m.generate(prompt, steps)
    assert toks == g["tokens"][:steps].tolist(), f"margins {g['margins'][:steps]}"
    # every entry point the mirror's decode path uses was exercised
    assert {"bt_linear_rows", "bt_gdn_gated_scan", "bt_add_rms_norm_planes", "bt_attention_layer",
            "bt_moe_layer_iq3s_add_norm", "bt_moe_route", "bt_conv_silu_scan", "bt_bf16_planes",
            "bt_argmax"} <= emulated.names
    m.close()


@pytest.mark.parametrize("chunk", [4, 6])
def test_qwen36_chunked_prefill_host_composition(emulated, qwen36_tiny_gguf, chunk) -> None:
    """prefill() in chunks (4 + 2 tokens, or all 6 at once) hands every
    entry point token-major rows, per-token positions and the chunk's row
    offsets such that the last prompt token's logits are the reference's."""
    g = golden("qwen36_tiny")
    m = qwen36_moe.Qwen36Moe(qwen36_tiny_gguf, device="cpu", max_context=int(g["max_context"]))
    prompt = g["prompt"].tolist()
    m.reset()
    m.prefill(torch.tensor([prompt[:-1]]), chunk=chunk)
    logits = m.forward_token(prompt[-1], len(prompt) - 1)
    got, want = logits.numpy(), g["logits"][0]
    assert np.abs(got - want).max() <= 1e-4 * np.abs(want).max()
    m.close()

"""Pin the CPU oracle against golden vectors produced by the reference.

The fixtures in tests/golden were written by tests/golden/make_golden.py,
which runs the reference's own torch f32 code; these tests check that the
numpy oracle reproduces them, so the oracle can stand in for the reference
on the GPU box (where the reference is not installed).
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

from oracle import ops
from oracle.dequant import dequant_iq3_s, dequant_q8_0
from tests.conftest import golden
from tests.golden.make_golden import STATE_SAMPLE, moe_inputs, ops_inputs


def test_q8_0_dequant_bit_exact() -> None:
    g = golden("dequant")
    got = dequant_q8_0(g["q8_raw"], 64, 32)
    assert np.array_equal(got.view(np.uint32), g["q8_out"].view(np.uint32))


def test_iq3_s_dequant_bit_exact() -> None:
    g = golden("dequant")
    got = dequant_iq3_s(g["iq3s_raw"], 64, 256)
    assert np.array_equal(got.view(np.uint32), g["iq3s_out"].view(np.uint32))
    fixed = dequant_iq3_s(g["iq3s_fixed_raw"], 1, 256)
    assert np.array_equal(fixed.reshape(-1), g["iq3s_fixed_out"].reshape(-1))
    # the reference's hand-computed vector (test_quant_dequant.py:268-279)
    assert np.array_equal(fixed.reshape(-1), np.array([1.0] * 32 + [3.0] * 32 + [1.0] * 192, dtype=np.float32))
    q = dequant_iq3_s(g["iq3s_quant_raw"].reshape(-1), 8, 512)
    assert np.array_equal(q.view(np.uint32), g["iq3s_quant_out"].view(np.uint32))


def test_gdn_decode_matches_reference() -> None:
    g, inp = golden("ops"), ops_inputs()
    for name in ("gdn16", "gdn8_16", "gdn16_32"):
        state = inp[f"{name}_state0"].copy()
        o = ops.gdn_decode(
            inp[f"{name}_q"], inp[f"{name}_k"], inp[f"{name}_v"], inp[f"{name}_g"], inp[f"{name}_beta"], state,
            128**-0.5, 1e-6,
        )
        np.testing.assert_allclose(o, g[f"{name}_out"], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(state.reshape(-1)[::STATE_SAMPLE], g[f"{name}_state1_sample"], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(state.astype(np.float64).sum(axis=(1, 2)), g[f"{name}_state1_sum"], rtol=1e-5, atol=1e-3)


def test_attention_rope_norms_match_reference() -> None:
    g, inp = golden("ops"), ops_inputs()
    for seq in (1, 17, 128):
        o = ops.attention(inp[f"attn{seq}_q"], inp[f"attn{seq}_k"], inp[f"attn{seq}_v"], 256**-0.5)
        np.testing.assert_allclose(o, g[f"attn{seq}_out"], rtol=1e-5, atol=1e-6)
    r = ops.rope(inp["rope_x"], inp["rope_cos"], inp["rope_sin"], int(inp["rope_pos"][0]), 64)
    np.testing.assert_allclose(r, g["rope_out"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(ops.rms_norm(inp["norm_x"], inp["norm_gamma"], 1e-6), g["norm_out"], rtol=1e-6, atol=1e-6)
    h, xn = ops.fused_add_rms_norm(inp["norm_x"], inp["norm_other"], inp["norm_gamma"], 1e-6)
    np.testing.assert_array_equal(h, g["fused_h"])
    np.testing.assert_allclose(xn, g["fused_xn"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(ops.silu_mul(inp["silu_gate"], inp["silu_up"]), g["silu_out"], rtol=1e-6, atol=1e-6)


def test_moe_route_and_experts_match_reference() -> None:
    from oracle.moe import experts, route

    g, m = golden("moe"), moe_inputs()
    digest = hashlib.sha256(m["gate"].tobytes() + m["up"].tobytes() + m["down"].tobytes()).hexdigest()
    assert digest == str(g["bytes_sha256"]), "IQ3_S quantiser no longer reproduces the fixture bytes"
    w, ids = route(m["logits"], 8)
    assert ids.tolist() == g["route_ids"].tolist()
    np.testing.assert_allclose(w, g["route_w"], rtol=1e-6, atol=1e-7)
    y = experts(m["x"], m["gate"], m["up"], m["down"], m["ids"], m["w"], m["hidden"], m["ffn"])
    np.testing.assert_allclose(y, g["y"], rtol=1e-4, atol=1e-5)


def test_moe_shared_expert_matches_reference() -> None:
    """routed + sigmoid(x . gate_inp) * shared(x) against the reference's
    Qwen36Moe._moe (model/qwen36_moe.py:634-642) on the same inputs."""
    from oracle.moe import shared_expert
    from tests.golden.make_golden import moe_shared_inputs

    g, m, sh = golden("moe_shared"), moe_inputs(), moe_shared_inputs()
    y = golden("moe")["y"] + shared_expert(m["x"], sh["gate"], sh["up"], sh["down"], sh["gate_inp"])
    assert np.abs(y - g["y"]).max() <= 1e-6 * np.abs(g["y"]).max()


def test_tiny_model_greedy_tokens_match_reference(tiny_gguf) -> None:
    from oracle.qwen35 import Qwen35Oracle

    g = golden("qwen35_tiny")
    o = Qwen35Oracle(tiny_gguf, max_context=int(g["max_context"]))
    toks, logits = o.generate(g["prompt"].tolist(), int(g["steps"]), return_logits=True)
    assert toks == g["tokens"].tolist()
    for i in range(g["logits"].shape[0]):
        np.testing.assert_allclose(logits[i], g["logits"][i], rtol=1e-4, atol=1e-5)


@pytest.mark.slow
def test_0_8b_model_greedy_tokens_match_reference(gguf_0_8b) -> None:
    from oracle.qwen35 import Qwen35Oracle

    g = golden("qwen35_0_8b")
    o = Qwen35Oracle(gguf_0_8b, max_context=int(g["max_context"]))
    toks, logits = o.generate(g["prompt"].tolist(), int(g["steps"]), return_logits=True)
    assert toks == g["tokens"].tolist()
    # 24 layers of differently ordered f32 sums: bound the error by the logit scale
    scale = np.abs(g["logits"][0]).max()
    assert np.abs(logits[0] - g["logits"][0]).max() <= 1e-4 * scale

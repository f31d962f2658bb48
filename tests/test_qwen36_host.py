"""Config-5 host logic on the CPU: the synthetic qwen35moe checkpoint parses
into the reference's config, and its golden prompt is reproducible."""

from __future__ import annotations

import numpy as np

from breezetoken_b200.gguf import GGML_BF16, GGML_IQ3_S, GGUFFile
from breezetoken_b200.qwen36_moe import Qwen36Config, rope_tables
from breezetoken_b200.synth import QWEN36_TINY
from tests.conftest import golden


def test_qwen36_tiny_config(qwen36_tiny_gguf) -> None:
    with GGUFFile(qwen36_tiny_gguf) as g:
        cfg = Qwen36Config.from_gguf(g, 64)
        assert (cfg.hidden, cfg.n_layers, cfg.n_heads, cfg.n_kv, cfg.head_dim) == (2048, 4, 16, 2, 256)
        assert (cfg.gdn_key_heads, cfg.gdn_value_heads, cfg.gdn_k_dim, cfg.gdn_inner) == (16, 32, 128, 4096)
        assert (cfg.n_experts, cfg.top_k, cfg.expert_ffn, cfg.shared_ffn, cfg.vocab) == (16, 8, 512, 512, 8192)
        assert cfg.attn_layers == (3,) and cfg.conv_dim == 8192
        assert g.tensor_layout("blk.0.attn_qkv.weight")[:2] == ((8192, 2048), GGML_BF16)
        assert g.tensor_layout("blk.0.ffn_gate_exps.weight")[:2] == ((16, 512, 2048), GGML_IQ3_S)


def test_qwen36_rope_tables_are_duplicated_halves() -> None:
    cfg = Qwen36Config(hidden=2048, n_layers=4, n_heads=16, n_kv=2, head_dim=256, rope_dim=64, rope_theta=1e7,
                       max_context=16, n_experts=16, top_k=8, expert_ffn=512, shared_ffn=512, gdn_key_heads=16,
                       gdn_value_heads=32, gdn_k_dim=128, gdn_inner=4096, gdn_conv=4, vocab=8192, eps=1e-6)
    cos, sin = rope_tables(cfg)
    assert cos.shape == (16, 64)
    assert (cos[:, :32] == cos[:, 32:]).all() and (sin[:, :32] == sin[:, 32:]).all()
    assert cos[0].eq(1).all() and sin[0].eq(0).all()


def test_qwen36_golden_prompt_is_seeded() -> None:
    g = golden("qwen36_tiny")
    assert g["prompt"].tolist() == np.random.default_rng(4).integers(0, QWEN36_TINY.vocab, 7).tolist()
    assert len(g["tokens"]) == int(g["steps"]) == 24

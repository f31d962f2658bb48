"""The all-GPU planner (breezetoken/planner.py's API): byte model of the
device layout, context candidates, sequence shards and the errors, on CPU
with a stand-in Hardware record."""

from __future__ import annotations

from types import SimpleNamespace as NS

import pytest

from breezetoken_b200.planner import Hardware, expected_distinct_experts, model_bytes, plan, shard, step_bytes

GIB = 1 << 30
C1 = NS(hidden=1024, n_layers=24, n_heads=8, n_kv=2, head_dim=256, ffn=3584, vocab=151936, ssm_inner=2048,
        ssm_state=128, ssm_heads=16, conv_k=4, attn_layers=tuple(i for i in range(24) if (i + 1) % 4 == 0),
        context_length=262144)
C5 = NS(hidden=2048, n_layers=40, n_heads=16, n_kv=2, head_dim=256, vocab=151936, n_experts=256, top_k=8,
        expert_ffn=512, shared_ffn=512, gdn_key_heads=16, gdn_value_heads=32, gdn_k_dim=128, gdn_inner=4096,
        gdn_conv=4, attn_layers=tuple(i for i in range(40) if (i + 1) % 4 == 0), max_context=262144)


def _b200(n: int = 8, free: int = 178 * GIB) -> Hardware:
    return Hardware(cpu_count=16, cpu_ram=196 * GIB, cuda=True, gpu_name="NVIDIA B200", gpu_total=179 * GIB,
                    gpu_free=free, sm_count=148, smem_optin=232448, compute_cap=(10, 0), n_gpus=n)


def test_step_bytes_match_the_published_byte_model() -> None:
    """The 0.8B batch-1 step: 736,419,072 + 24,576 L bytes (Q8_0 weights,
    f32 parameters, GDN and conv state read + written, f32 KV read)."""
    assert step_bytes(C1, 1, 0) == 736_419_072
    assert step_bytes(C1, 1, 100) - step_bytes(C1, 1, 0) == 100 * 24_576
    mb = model_bytes(C5)
    assert mb.expert_bytes == 1_351_680  # gate + up + down of one expert in IQ3_S
    assert abs(expected_distinct_experts(256, 8, 64) - 222.4) < 0.1
    # 64 sequences: dense weights + 40 x U experts + state + KV
    per_seq = step_bytes(C5, 2, 640) - step_bytes(C5, 1, 640)
    assert per_seq > 0


def test_plan_shards_sequences_and_keeps_every_layer_on_the_gpu() -> None:
    p = plan(C5, _b200(8), max_context=769, batch=64)
    assert p.n_gpus == 8 and p.shards == tuple((8 * r, 8) for r in range(8))
    assert p.gpu_layers == C5.n_layers and p.head_on_gpu and p.cpu_bytes == 0
    assert p.weight_bytes > 17 * 10**9 and p.gpu_bytes > p.weight_bytes
    assert list(p.sequences(3)) == list(range(24, 32))
    q = plan(C5, _b200(8), max_context=769, batch=10, n_gpus=4)
    assert [c for _, c in q.shards] == [3, 3, 2, 2] and sum(c for _, c in q.shards) == 10
    with pytest.raises(RuntimeError):
        shard(3, 8)


def test_plan_lowers_the_automatic_context_and_raises_when_nothing_fits() -> None:
    # 0.8B at 8 sequences on a GPU with ~3 GiB free: 8192 does not fit, a lower context does
    small = _b200(1, free=int(3.6 * GIB))
    p = plan(C1, small, batch=8)
    assert p.max_context < 8192
    with pytest.raises(RuntimeError, match="GPU memory"):
        plan(C1, small, max_context=262144, batch=8)
    with pytest.raises(RuntimeError):
        plan(C5, _b200(1, free=8 * GIB), max_context=1024, batch=1)
    with pytest.raises(ValueError):
        plan(C1, _b200(), max_context=0)
    with pytest.raises(RuntimeError, match="CUDA"):
        plan(C1, Hardware(cpu_count=8, cpu_ram=GIB, cuda=False))

"""Placement for the B200 backend: context, GPUs and sequences per GPU.

Mirrors breezetoken/planner.py (``Hardware`` :49-85, ``Placement`` :88-104,
``plan`` :149-191, ``_plan_at`` :194-282): the same names, the same
context candidates when none is requested (8192, 4096, 2048, 1024, lowered
under memory pressure) and the same error kinds (``ValueError`` for bad
arguments, ``RuntimeError`` when nothing fits).  What changes is the
placement itself.  The reference keeps the longest GPU prefix of layers and
runs the rest on the CPU; on a B200 box the whole model is resident on every
GPU it uses (``gpu_layers`` = all layers, the head on the GPU, no CPU
suffix), and a batch of independent sequences is sharded across the GPUs of
one box: each GPU holds a full replica of the weights and the KV / GDN state
of its own sequences, with no collective on the data path.

The byte model counts the library's device layout: Q8_0 "q8 rows" for the
Qwen3.5 checkpoints, bf16 / f32 rows and IQ3_S tile chunks (136 bytes per
256 weights) for the Qwen3.6-MoE ones, plus per sequence the GDN conv
window and recurrent state and the f32 KV cache at the planned context.
``step_bytes`` is the matching per-step traffic of one decode step on one
GPU (every weight read once, the selected experts, state read and written,
the KV read at a context), the roofline numerator of the benchmarks.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from pathlib import Path

import torch

_GIB = 1 << 30
#: Preferred context when none is requested (planner.py:30).
AUTO_CONTEXT = 8192
#: Per-GPU reserve for the CUDA context, graphs, workspaces and activations.
RESERVE_BYTES = 2 * _GIB
IQ3S_DEVICE_BYTES_PER_256 = 136  # bt_iq3s_row_bytes: 4-bit codes (128) + scales and d (8)
IQ3S_BYTES_PER_256 = 110  # the format's own bytes: what a step must read


def _available_ram() -> int:
    try:
        for line in Path("/proc/meminfo").read_text().splitlines():
            if line.startswith("MemAvailable:"):
                return int(line.split()[1]) * 1024
    except OSError:
        pass
    return 0


@dataclass(frozen=True)
class Hardware:
    """planner.py:49-85, with the number of GPUs of the box (taken as
    identical: the figures are the current device's)."""

    cpu_count: int
    cpu_ram: int
    cuda: bool
    gpu_name: str = ""
    gpu_total: int = 0
    gpu_free: int = 0
    sm_count: int = 0
    smem_optin: int = 0
    compute_cap: tuple[int, int] = (0, 0)
    n_gpus: int = 0

    @classmethod
    def detect(cls) -> Hardware:
        cuda = torch.cuda.is_available()
        name, total, free, sm, smem, cap, n = "", 0, 0, 0, 0, (0, 0), 0
        if cuda:
            n = torch.cuda.device_count()
            props = torch.cuda.get_device_properties(0)
            name, total, sm = props.name, int(props.total_memory), int(props.multi_processor_count)
            smem = int(getattr(props, "shared_memory_per_block_optin", 0))
            cap = (int(props.major), int(props.minor))
            free = int(torch.cuda.mem_get_info()[0])  # this process's device (no context on the others)
        return cls(cpu_count=os.cpu_count() or 1, cpu_ram=_available_ram(), cuda=cuda, gpu_name=name,
                   gpu_total=total, gpu_free=free, sm_count=sm, smem_optin=smem, compute_cap=cap, n_gpus=n)


@dataclass(frozen=True)
class Placement:
    """planner.py:88-104 plus the sequence shards: GPU r decodes sequences
    [shards[r][0], shards[r][0] + shards[r][1])."""

    max_context: int
    gpu_layers: int
    head_on_gpu: bool
    gpu_bytes: int
    cpu_bytes: int
    reason: str
    gpu_name: str = ""
    n_gpus: int = 1
    shards: tuple[tuple[int, int], ...] = ((0, 1),)
    weight_bytes: int = 0
    state_bytes_per_sequence: int = 0

    def summary(self, total_layers: int) -> str:
        per = "/".join(str(c) for _, c in self.shards)
        return (f"cuda x{self.n_gpus} ({per} sequences) gpu_layers={self.gpu_layers}/{total_layers} head=cuda "
                f"ctx={self.max_context}")

    def sequences(self, rank: int) -> range:
        start, count = self.shards[rank]
        return range(start, start + count)


@dataclass(frozen=True)
class ModelBytes:
    """Device bytes of a model: weights (once per GPU), and per sequence the
    fixed recurrent state and the KV bytes per cached position."""

    weights: int
    state_per_sequence: int
    kv_per_token: int
    # per decode step: the weights one step reads (the embedding is a row
    # gather, not a read of the matrix), and one expert's IQ3_S bytes
    # (gate + up + down, the format's 110 bytes per 256 weights)
    step_weights: int = 0
    expert_bytes: int = 0
    n_layers: int = 0
    n_experts: int = 0
    top_k: int = 0


def _q8_row_bytes(k: int) -> int:
    return (k // 32 * 2 + 15) // 16 * 16 + k


def model_bytes(cfg) -> ModelBytes:
    """The device layout's bytes of a Qwen3.5 (model.Qwen35Config) or
    Qwen3.6-MoE (qwen36_moe.Qwen36Config) configuration."""
    attn = set(cfg.attn_layers)
    f32, bf16 = 4, 2
    if hasattr(cfg, "n_experts"):  # qwen35moe: bf16 projections, IQ3_S experts
        h, D, E = cfg.hidden, cfg.head_dim, cfg.n_experts
        dv = cfg.gdn_inner // cfg.gdn_value_heads
        expert = 3 * cfg.expert_ffn * h // 256 * IQ3S_DEVICE_BYTES_PER_256  # gate + up + down, device layout
        shared = 3 * cfg.shared_ffn * h * bf16 + h * f32
        weights = 2 * cfg.vocab * h * bf16 + h * f32  # embedding, head, final norm
        step_weights = cfg.vocab * h * bf16 + h * f32
        state = kv = 0
        for i in range(cfg.n_layers):
            layer = 2 * h * f32 + E * h * f32 + shared  # norms, router, shared expert
            if i in attn:
                layer += (2 * cfg.n_heads + 2 * cfg.n_kv) * D * h * bf16 + h * cfg.n_heads * D * bf16 + 2 * D * f32
                kv += 2 * cfg.n_kv * D * f32
            else:
                conv_dim = 2 * cfg.gdn_key_heads * cfg.gdn_k_dim + cfg.gdn_inner
                layer += (conv_dim + cfg.gdn_inner) * h * bf16 + h * cfg.gdn_inner * bf16  # qkv, z, out
                layer += 2 * cfg.gdn_value_heads * h * f32 + conv_dim * cfg.gdn_conv * f32  # beta/alpha, conv
                layer += 2 * cfg.gdn_value_heads * f32 + cfg.gdn_k_dim * f32  # a, dt bias, norm
                state += conv_dim * (cfg.gdn_conv - 1) * f32 + cfg.gdn_value_heads * cfg.gdn_k_dim * dv * f32
            weights += layer + E * expert
            step_weights += layer
        return ModelBytes(weights, state, kv, step_weights, 3 * cfg.expert_ffn * h // 256 * IQ3S_BYTES_PER_256,
                          cfg.n_layers, E, cfg.top_k)
    # qwen35: Q8_0 rows, f32 norms / conv / SSM parameters
    h = cfg.hidden
    embed = cfg.vocab * _q8_row_bytes(h)
    weights = embed + h * f32
    state = kv = 0
    for i in range(cfg.n_layers):
        layer = 2 * h * f32 + 2 * cfg.ffn * _q8_row_bytes(h) + h * _q8_row_bytes(cfg.ffn)
        if i in attn:
            rows = cfg.n_heads * 2 * cfg.head_dim + 2 * cfg.n_kv * cfg.head_dim
            layer += rows * _q8_row_bytes(h) + h * _q8_row_bytes(cfg.n_heads * cfg.head_dim) + 2 * cfg.head_dim * f32
            kv += 2 * cfg.n_kv * cfg.head_dim * f32
        else:
            rows = 4 * cfg.ssm_inner + 2 * cfg.ssm_heads
            layer += rows * _q8_row_bytes(h) + h * _q8_row_bytes(cfg.ssm_inner)
            layer += 3 * cfg.ssm_inner * cfg.conv_k * f32 + 2 * cfg.ssm_heads * f32 + cfg.ssm_state * f32
            state += 3 * cfg.ssm_inner * (cfg.conv_k - 1) * f32 + cfg.ssm_heads * cfg.ssm_state ** 2 * f32
        weights += layer
    return ModelBytes(weights, state, kv, weights, 0, cfg.n_layers)


def expected_distinct_experts(n_experts: int, top_k: int, sequences: int) -> float:
    """E[distinct experts a step of `sequences` tokens selects] under uniform
    routing: n (1 - (1 - k/n)^S)."""
    return n_experts * (1.0 - (1.0 - top_k / n_experts) ** sequences)


def step_bytes(cfg, sequences: int, context: float, distinct_experts: float | None = None) -> float:
    """Algorithmic bytes of one decode step of `sequences` sequences on one
    GPU at mean context `context`: the weights the step reads once (the
    selected experts, `distinct_experts` per layer, measured or else the
    uniform-routing expectation), the recurrent state read and written, the
    KV cache read over the context."""
    mb = model_bytes(cfg)
    total = float(mb.step_weights)
    if mb.n_experts:
        u = distinct_experts if distinct_experts is not None else expected_distinct_experts(
            mb.n_experts, mb.top_k, sequences)
        total += mb.n_layers * u * mb.expert_bytes
    # the conv windows and recurrent states are read and written once each
    return total + sequences * (2 * mb.state_per_sequence + context * mb.kv_per_token)


def shard(batch: int, n_gpus: int) -> tuple[tuple[int, int], ...]:
    """Contiguous sequence ranges, as even as possible, the larger first."""
    if batch < 1 or n_gpus < 1:
        raise ValueError("batch and n_gpus must be positive")
    if batch < n_gpus:
        raise RuntimeError(f"{batch} sequences cannot occupy {n_gpus} GPUs")
    base, extra = divmod(batch, n_gpus)
    out, start = [], 0
    for r in range(n_gpus):
        c = base + (1 if r < extra else 0)
        out.append((start, c))
        start += c
    return tuple(out)


def plan(cfg, hw: Hardware | None = None, *, max_context: int | None = None, batch: int = 1,
         n_gpus: int | None = None) -> Placement:
    """Choose the context and the sequences per GPU (planner.py:149-191).

    ``max_context`` is a hard request (raises when it cannot fit); ``None``
    tries 8192, 4096, 2048 and 1024 in turn, capped by the model's context.
    ``n_gpus`` defaults to every GPU of the box (at most one per sequence).
    """
    hw = hw or Hardware.detect()
    if max_context is not None and max_context <= 0:
        raise ValueError("max_context must be positive")
    if batch < 1:
        raise ValueError("batch must be positive")
    if n_gpus is not None and n_gpus < 1:
        raise ValueError("n_gpus must be positive")
    if not hw.cuda or hw.n_gpus < 1:
        raise RuntimeError("the b200 backend needs a CUDA GPU; none is available")
    gpus = min(n_gpus or hw.n_gpus, batch)
    if gpus > hw.n_gpus:
        raise RuntimeError(f"{gpus} GPUs requested, {hw.n_gpus} available")
    limit = int(getattr(cfg, "context_length", 0) or getattr(cfg, "max_context", 0) or AUTO_CONTEXT)
    if max_context is not None:
        candidates = [min(max_context, limit)]
    else:
        candidates = [c for c in (AUTO_CONTEXT, 4096, 2048, 1024) if c <= limit] or [min(limit, 1024)]
    mb = model_bytes(cfg)
    shards = shard(batch, gpus)
    per_gpu = max(c for _, c in shards)
    budget = max(0, min(hw.gpu_free, int(hw.gpu_total * 0.92)) - RESERVE_BYTES)
    last = ""
    for cap in candidates:
        seq_bytes = mb.state_per_sequence + cap * mb.kv_per_token
        need = mb.weights + per_gpu * seq_bytes
        if need <= budget:
            return Placement(
                max_context=cap, gpu_layers=cfg.n_layers, head_on_gpu=True, gpu_bytes=need, cpu_bytes=0,
                reason=f"weights replicated on {gpus} GPU(s), {per_gpu} sequence(s) per GPU at context {cap}",
                gpu_name=hw.gpu_name, n_gpus=gpus, shards=shards, weight_bytes=mb.weights,
                state_bytes_per_sequence=seq_bytes)
        last = (f"GPU memory: need {need / _GIB:.1f} GiB per GPU ({per_gpu} sequences at context {cap}), "
                f"budget {budget / _GIB:.1f} GiB")
    raise RuntimeError(last or "no placement fits this model")


__all__ = ["AUTO_CONTEXT", "Hardware", "ModelBytes", "Placement", "expected_distinct_experts", "model_bytes",
           "plan", "shard", "step_bytes"]

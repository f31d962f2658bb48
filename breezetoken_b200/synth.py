"""Seeded synthetic checkpoints in GGUF form.

No real checkpoint is available to this project, so the benchmarks and parity
tests run on random-initialised models written as GGUF files that both this
backend and the reference's loader (breezetoken/gguf.py, model/qwen35.py:166-219)
read.  Generation is deterministic for a given seed and independent of the
thread count: every tensor is filled in fixed 1 Mi-element chunks, chunk c of
tensor t drawing from ``default_rng(SeedSequence(seed, spawn_key=(t, c)))``.

Distributions (Q8_0 matrices follow the benchmark definition, N(0, 0.02)
before quantisation; the f32 parameters are chosen so the recurrence and
norms stay in a realistic range):

* projection / embedding matrices: N(0, 0.02) -> Q8_0;
* RMSNorm gammas (stored pre-folded, model/qwen35.py:9): 1 + N(0, 0.02);
* ssm_a = -exp(U(0, log 16)) (GGUF stores -exp(A_log));
* ssm_dt.bias = log(expm1(dt)), dt log-uniform in [1e-3, 1e-1];
* ssm_conv1d: N(0, 0.25).
"""

from __future__ import annotations

import concurrent.futures as cf
import os
from dataclasses import asdict, dataclass
from pathlib import Path

import numpy as np

from breezetoken_b200.gguf import GGML_BF16, GGML_F32, GGML_IQ3_S, GGML_Q8_0, GGUFWriter
from breezetoken_b200.quant import quantize_iq3_s, quantize_q8_0

CHUNK = 1 << 20


@dataclass(frozen=True)
class Qwen35Spec:
    """Shape of a Qwen3.5 hybrid decoder (qwen35 GGUF metadata)."""

    hidden: int = 1024
    n_layers: int = 24
    n_heads: int = 8
    n_kv: int = 2
    head_dim: int = 256
    rope_dim: int = 64
    rope_theta: float = 1e7
    ffn: int = 3584
    vocab: int = 151936
    ssm_inner: int = 2048
    ssm_state: int = 128
    ssm_heads: int = 16
    conv_k: int = 4
    attn_interval: int = 4
    eps: float = 1e-6
    context_length: int = 262144


#: The Qwen3.5-0.8B shape (the batch-1 decode benchmark).
QWEN35_0_8B = Qwen35Spec()
#: A small model with the same per-layer kernel shapes (GQA 8/2x256, GDN 16x128)
#: and one full [GDN, GDN, GDN, GQA] period, for fast parity tests.
QWEN35_TINY = Qwen35Spec(hidden=512, n_layers=4, ffn=1024, vocab=8192)

SPECS = {"qwen35-0.8b": QWEN35_0_8B, "qwen35-tiny": QWEN35_TINY}


def _threads() -> int:
    return max(1, min(16, os.cpu_count() or 1))


def _fill(seed: int, tensor_id: int, n: int, kind: str, pool: cf.Executor) -> np.ndarray:
    """n float32 values of distribution `kind`, chunked and seeded deterministically."""
    out = np.empty(n, dtype=np.float32)

    def chunk(c: int) -> None:
        rng = np.random.default_rng(np.random.SeedSequence(seed, spawn_key=(tensor_id, c)))
        view = out[c * CHUNK : min(n, (c + 1) * CHUNK)]
        if kind == "normal":
            rng.standard_normal(view.shape[0], dtype=np.float32, out=view)
        else:  # uniform [0, 1)
            rng.random(view.shape[0], dtype=np.float32, out=view)

    list(pool.map(chunk, range((n + CHUNK - 1) // CHUNK)))
    return out


def _q8_rows(values: np.ndarray, rows: int, k: int, pool: cf.Executor) -> np.ndarray:
    m = values.reshape(rows, k)
    step = max(1, CHUNK // k)
    parts = list(pool.map(lambda r: quantize_q8_0(m[r : r + step]), range(0, rows, step)))
    return np.concatenate(parts, axis=0)


def qwen35_tensors(spec: Qwen35Spec) -> list[tuple[str, tuple[int, ...], str]]:
    """(name, logical shape, role) of every tensor, in file order."""
    s = spec
    t: list[tuple[str, tuple[int, ...], str]] = [
        ("token_embd.weight", (s.vocab, s.hidden), "q8"),
        ("output_norm.weight", (s.hidden,), "gamma"),
    ]
    for i in range(s.n_layers):
        p = f"blk.{i}."
        t += [
            (p + "attn_norm.weight", (s.hidden,), "gamma"),
            (p + "post_attention_norm.weight", (s.hidden,), "gamma"),
            (p + "ffn_gate.weight", (s.ffn, s.hidden), "q8"),
            (p + "ffn_up.weight", (s.ffn, s.hidden), "q8"),
            (p + "ffn_down.weight", (s.hidden, s.ffn), "q8"),
        ]
        if (i + 1) % s.attn_interval == 0:
            t += [
                (p + "attn_q.weight", (2 * s.n_heads * s.head_dim, s.hidden), "q8"),
                (p + "attn_k.weight", (s.n_kv * s.head_dim, s.hidden), "q8"),
                (p + "attn_v.weight", (s.n_kv * s.head_dim, s.hidden), "q8"),
                (p + "attn_output.weight", (s.hidden, s.n_heads * s.head_dim), "q8"),
                (p + "attn_q_norm.weight", (s.head_dim,), "gamma"),
                (p + "attn_k_norm.weight", (s.head_dim,), "gamma"),
            ]
        else:
            t += [
                (p + "attn_qkv.weight", (3 * s.ssm_inner, s.hidden), "q8"),
                (p + "attn_gate.weight", (s.ssm_inner, s.hidden), "q8"),
                (p + "ssm_conv1d.weight", (3 * s.ssm_inner, s.conv_k), "conv"),
                (p + "ssm_alpha.weight", (s.ssm_heads, s.hidden), "q8"),
                (p + "ssm_beta.weight", (s.ssm_heads, s.hidden), "q8"),
                (p + "ssm_a", (s.ssm_heads,), "ssm_a"),
                (p + "ssm_dt.bias", (s.ssm_heads,), "dt_bias"),
                (p + "ssm_out.weight", (s.hidden, s.ssm_inner), "q8"),
                (p + "ssm_norm.weight", (s.ssm_state,), "gamma"),
            ]
    return t


def write_qwen35_gguf(path: str | Path, spec: Qwen35Spec = QWEN35_0_8B, seed: int = 0) -> Path:
    """Write a seeded random Qwen3.5-shaped Q8_0/F32 GGUF to ``path``."""
    s = spec
    w = GGUFWriter()
    w.add("general.architecture", "qwen35")
    w.add("general.name", f"synthetic-qwen35-seed{seed}")
    w.add("general.alignment", 32)
    w.add("qwen35.block_count", s.n_layers)
    w.add("qwen35.context_length", s.context_length)
    w.add("qwen35.embedding_length", s.hidden)
    w.add("qwen35.feed_forward_length", s.ffn)
    w.add("qwen35.attention.head_count", s.n_heads)
    w.add("qwen35.attention.head_count_kv", s.n_kv)
    w.add("qwen35.attention.key_length", s.head_dim)
    w.add("qwen35.attention.value_length", s.head_dim)
    w.add("qwen35.attention.layer_norm_rms_epsilon", float(s.eps))
    w.add("qwen35.rope.dimension_count", s.rope_dim)
    w.add("qwen35.rope.freq_base", float(s.rope_theta))
    w.add("qwen35.ssm.inner_size", s.ssm_inner)
    w.add("qwen35.ssm.state_size", s.ssm_state)
    w.add("qwen35.ssm.group_count", s.ssm_heads)
    w.add("qwen35.ssm.conv_kernel", s.conv_k)
    w.add("qwen35.full_attention_interval", s.attn_interval)
    with cf.ThreadPoolExecutor(_threads()) as pool:
        for tid, (name, shape, role) in enumerate(qwen35_tensors(s)):
            n = int(np.prod(shape))
            if role == "q8":
                vals = _fill(seed, tid, n, "normal", pool) * np.float32(0.02)
                w.add_tensor(name, shape, GGML_Q8_0, _q8_rows(vals, shape[0], shape[1], pool))
                continue
            if role == "gamma":
                vals = np.float32(1.0) + _fill(seed, tid, n, "normal", pool) * np.float32(0.02)
            elif role == "conv":
                vals = _fill(seed, tid, n, "normal", pool) * np.float32(0.25)
            elif role == "ssm_a":
                vals = -np.exp(_fill(seed, tid, n, "uniform", pool) * np.float32(np.log(16.0)))
            elif role == "dt_bias":
                u = _fill(seed, tid, n, "uniform", pool)
                dt = np.exp(np.log(1e-3) + u * (np.log(1e-1) - np.log(1e-3)))
                vals = np.log(np.expm1(dt))
            else:
                raise AssertionError(role)
            w.add_tensor(name, shape, GGML_F32, np.asarray(vals, dtype=np.float32).reshape(shape))
    return w.write(path)


def spec_dict(spec: Qwen35Spec) -> dict:
    return asdict(spec)


# --------------------------------------------------------------------------
# MoE expert layer (the Qwen3.6-35B-A3B expert FFN shape)
# --------------------------------------------------------------------------
@dataclass(frozen=True)
class MoeSpec:
    hidden: int = 2048
    n_experts: int = 256
    top_k: int = 8
    ffn: int = 512


def make_moe_layer(spec: MoeSpec = MoeSpec(), seed: int = 3, n_experts: int | None = None):
    """IQ3_S expert tensors of one MoE layer as GGUF-stored bytes.

    Returns dict with ``gate``/``up`` (E, ffn, hidden) and ``down`` (E, hidden,
    ffn) as uint8 arrays of shape (E * rows, row_bytes), plus the bf16 shared
    expert (gate/up (ffn, hidden), down (hidden, ffn)) as float32 values
    already rounded to bf16, and the shared-expert gate vector.
    """
    e = spec.n_experts if n_experts is None else n_experts
    out: dict[str, np.ndarray] = {}
    with cf.ThreadPoolExecutor(_threads()) as pool:
        for tid, (name, rows, k) in enumerate(
            (("gate", e * spec.ffn, spec.hidden), ("up", e * spec.ffn, spec.hidden), ("down", e * spec.hidden, spec.ffn))
        ):
            vals = (_fill(seed, 100 + tid, rows * k, "normal", pool) * np.float32(0.02)).reshape(rows, k)
            step = max(1, CHUNK // k)
            parts = list(pool.map(lambda r, v=vals: quantize_iq3_s(v[r : r + step]), range(0, rows, step)))
            out[name] = np.concatenate(parts, axis=0)
        import torch  # noqa: PLC0415 - bf16 rounding only

        for tid, (name, shape) in enumerate(
            (("sh_gate", (spec.ffn, spec.hidden)), ("sh_up", (spec.ffn, spec.hidden)), ("sh_down", (spec.hidden, spec.ffn)))
        ):
            vals = _fill(seed, 200 + tid, int(np.prod(shape)), "normal", pool) * np.float32(0.02)
            out[name] = torch.from_numpy(vals.reshape(shape)).to(torch.bfloat16).float().numpy()
        out["sh_gate_inp"] = _fill(seed, 210, spec.hidden, "normal", pool) * np.float32(0.02)
    return out


def moe_layer_inputs(tokens: int, spec: MoeSpec = MoeSpec(), seed: int = 3) -> tuple[np.ndarray, np.ndarray]:
    """The MoE-layer benchmark's per-step inputs for T tokens: activations
    x (T, hidden) drawn N(0, 1) and rounded to bf16 (returned as f32), and
    router logits (T, n_experts) drawn N(0, 1); one seeded stream per T."""
    import torch  # noqa: PLC0415 - bf16 rounding only

    rng = np.random.default_rng(np.random.SeedSequence(seed, spawn_key=(1000, tokens)))
    x = rng.standard_normal((tokens, spec.hidden), dtype=np.float32)
    x = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    logits = rng.standard_normal((tokens, spec.n_experts), dtype=np.float32)
    return x, logits


# --------------------------------------------------------------------------
# Qwen3.6-35B-A3B-shaped hybrid MoE decoder (qwen35moe GGUF)
# --------------------------------------------------------------------------
@dataclass(frozen=True)
class Qwen36Spec:
    """Shape of a qwen35moe decoder (the 35B-A3B benchmark shape with the defaults)."""

    hidden: int = 2048
    n_layers: int = 40
    n_heads: int = 16
    n_kv: int = 2
    head_dim: int = 256
    rope_dim: int = 64
    rope_theta: float = 1e7
    vocab: int = 151936
    n_experts: int = 256
    top_k: int = 8
    expert_ffn: int = 512
    shared_ffn: int = 512
    gdn_key_heads: int = 16
    gdn_value_heads: int = 32
    gdn_dim: int = 128
    conv_k: int = 4
    attn_interval: int = 4
    eps: float = 1e-6
    context_length: int = 262144

    @property
    def gdn_inner(self) -> int:
        return self.gdn_value_heads * self.gdn_dim

    @property
    def conv_dim(self) -> int:
        return 2 * self.gdn_key_heads * self.gdn_dim + self.gdn_inner


#: The Qwen3.6-35B-A3B benchmark shape.
QWEN36_35B = Qwen36Spec()
#: The config-5 layer shapes (hidden 2048, GQA 16/2x256, GDN 16K/32V x128,
#: experts of ffn 512 + a shared expert) with one [GDN, GDN, GDN, GQA]
#: period, 16 experts and a small vocabulary, for parity against the
#: reference's CPU path.
QWEN36_TINY = Qwen36Spec(n_layers=4, vocab=8192, n_experts=16)


def qwen36_tensors(spec: Qwen36Spec) -> list[tuple[str, tuple[int, ...], str]]:
    """(name, logical shape, role) of every tensor of a qwen35moe GGUF, in
    the names and orientations model/qwen36_moe.py:259-307 loads."""
    s = spec
    t: list[tuple[str, tuple[int, ...], str]] = [
        ("token_embd.weight", (s.vocab, s.hidden), "bf16"),
        ("output.weight", (s.vocab, s.hidden), "bf16"),
        ("output_norm.weight", (s.hidden,), "gamma"),
    ]
    for i in range(s.n_layers):
        p = f"blk.{i}."
        t += [
            (p + "attn_norm.weight", (s.hidden,), "gamma"),
            (p + "post_attention_norm.weight", (s.hidden,), "gamma"),
            (p + "ffn_gate_inp.weight", (s.n_experts, s.hidden), "f32w"),
            (p + "ffn_gate_inp_shexp.weight", (s.hidden,), "f32w"),
            (p + "ffn_gate_shexp.weight", (s.shared_ffn, s.hidden), "bf16"),
            (p + "ffn_up_shexp.weight", (s.shared_ffn, s.hidden), "bf16"),
            (p + "ffn_down_shexp.weight", (s.hidden, s.shared_ffn), "bf16"),
            (p + "ffn_gate_exps.weight", (s.n_experts, s.expert_ffn, s.hidden), "iq3s"),
            (p + "ffn_up_exps.weight", (s.n_experts, s.expert_ffn, s.hidden), "iq3s"),
            (p + "ffn_down_exps.weight", (s.n_experts, s.hidden, s.expert_ffn), "iq3s"),
        ]
        if (i + 1) % s.attn_interval == 0:
            t += [
                (p + "attn_q.weight", (2 * s.n_heads * s.head_dim, s.hidden), "bf16"),
                (p + "attn_k.weight", (s.n_kv * s.head_dim, s.hidden), "bf16"),
                (p + "attn_v.weight", (s.n_kv * s.head_dim, s.hidden), "bf16"),
                (p + "attn_output.weight", (s.hidden, s.n_heads * s.head_dim), "bf16"),
                (p + "attn_q_norm.weight", (s.head_dim,), "gamma"),
                (p + "attn_k_norm.weight", (s.head_dim,), "gamma"),
            ]
        else:
            t += [
                (p + "attn_qkv.weight", (s.conv_dim, s.hidden), "bf16"),
                (p + "attn_gate.weight", (s.gdn_inner, s.hidden), "bf16"),
                (p + "ssm_conv1d.weight", (s.conv_dim, s.conv_k), "conv"),
                (p + "ssm_alpha.weight", (s.gdn_value_heads, s.hidden), "f32w"),
                (p + "ssm_beta.weight", (s.gdn_value_heads, s.hidden), "f32w"),
                (p + "ssm_a", (s.gdn_value_heads,), "ssm_a"),
                (p + "ssm_dt.bias", (s.gdn_value_heads,), "dt_bias"),
                (p + "ssm_out.weight", (s.hidden, s.gdn_inner), "bf16"),
                (p + "ssm_norm.weight", (s.gdn_dim,), "gamma"),
            ]
    return t


#: IQ3_S block scale d of the random-byte experts (fp16 2^-12, little-endian):
#: with random scale nibbles, grid entries and signs the weights have the
#: magnitude an N(0, 0.02) quantisation gives.
IQ3S_RANDOM_D = (0x00, 0x0C)


def iq3s_random_bytes(seed: int, tensor_id: int, rows: int, k: int, pool: cf.Executor) -> np.ndarray:
    """Seeded uniform random IQ3_S blocks (rows, k/256 * 110) with the block
    scale d fixed to IQ3S_RANDOM_D: every byte pattern is a valid IQ3_S block,
    so this is a checkpoint of the format's full range without quantising."""
    nb = rows * (k // 256)
    out = np.empty((nb, 110), dtype=np.uint8)
    per = max(1, CHUNK // 110)

    def chunk(c: int) -> None:
        rng = np.random.default_rng(np.random.SeedSequence(seed, spawn_key=(tensor_id, c)))
        view = out[c * per : min(nb, (c + 1) * per)]
        view[:] = rng.integers(0, 256, view.shape, dtype=np.uint8)
        view[:, 0], view[:, 1] = IQ3S_RANDOM_D

    list(pool.map(chunk, range((nb + per - 1) // per)))
    return out.reshape(rows, -1)


def write_qwen36_gguf(path: str | Path, spec: Qwen36Spec = QWEN36_TINY, seed: int = 4,
                      experts: str = "quantized") -> Path:
    """Write a seeded random qwen35moe GGUF: bf16 projections, IQ3_S experts,
    f32 router, gate vectors, norms and SSM parameters (distributions as for
    the Qwen3.5 checkpoints).  ``experts="quantized"`` quantises N(0, 0.02)
    weights to IQ3_S; ``experts="random"`` writes seeded random IQ3_S blocks
    (iq3s_random_bytes), minutes faster for the full 35B-A3B shape.  Tensors
    are generated while the file is written, one at a time."""
    import torch  # noqa: PLC0415 - bf16 rounding

    if experts not in ("quantized", "random"):
        raise ValueError(f"experts must be 'quantized' or 'random', got {experts!r}")
    s = spec
    w = GGUFWriter()
    w.add("general.architecture", "qwen35moe")
    w.add("general.name", f"synthetic-qwen35moe-seed{seed}")
    w.add("general.alignment", 32)
    a = "qwen35moe."
    for key, val in (
        ("block_count", s.n_layers), ("context_length", s.context_length), ("embedding_length", s.hidden),
        ("attention.head_count", s.n_heads), ("attention.head_count_kv", s.n_kv),
        ("attention.key_length", s.head_dim), ("attention.value_length", s.head_dim),
        ("attention.layer_norm_rms_epsilon", float(s.eps)), ("rope.dimension_count", s.rope_dim),
        ("rope.freq_base", float(s.rope_theta)), ("expert_count", s.n_experts), ("expert_used_count", s.top_k),
        ("expert_feed_forward_length", s.expert_ffn), ("expert_shared_feed_forward_length", s.shared_ffn),
        ("ssm.group_count", s.gdn_key_heads), ("ssm.inner_size", s.gdn_inner), ("ssm.state_size", s.gdn_dim),
        ("ssm.conv_kernel", s.conv_k), ("full_attention_interval", s.attn_interval), ("nextn_predict_layers", 0),
    ):
        w.add(a + key, val)
    def tensor(tid: int, shape: tuple[int, ...], role: str, pool: cf.Executor) -> np.ndarray:
        n = int(np.prod(shape))
        if role == "bf16":
            vals = _fill(seed, tid, n, "normal", pool) * np.float32(0.02)
            return torch.from_numpy(vals).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
        if role == "iq3s":
            k = shape[-1]
            rows = n // k
            if experts == "random":
                return iq3s_random_bytes(seed, tid, rows, k, pool)
            vals = (_fill(seed, tid, n, "normal", pool) * np.float32(0.02)).reshape(rows, k)
            step = max(1, CHUNK // k)
            parts = list(pool.map(lambda r, v=vals: quantize_iq3_s(v[r : r + step]), range(0, rows, step)))
            return np.concatenate(parts, axis=0)
        if role == "gamma":
            vals = np.float32(1.0) + _fill(seed, tid, n, "normal", pool) * np.float32(0.02)
        elif role == "f32w":
            vals = _fill(seed, tid, n, "normal", pool) * np.float32(0.02)
        elif role == "conv":
            vals = _fill(seed, tid, n, "normal", pool) * np.float32(0.25)
        elif role == "ssm_a":
            vals = -np.exp(_fill(seed, tid, n, "uniform", pool) * np.float32(np.log(16.0)))
        elif role == "dt_bias":
            u = _fill(seed, tid, n, "uniform", pool)
            dt = np.exp(np.log(1e-3) + u * (np.log(1e-1) - np.log(1e-3)))
            vals = np.log(np.expm1(dt))
        else:
            raise AssertionError(role)
        return np.asarray(vals, dtype=np.float32)

    kinds = {"bf16": GGML_BF16, "iq3s": GGML_IQ3_S}
    with cf.ThreadPoolExecutor(_threads()) as pool:
        for tid, (name, shape, role) in enumerate(qwen36_tensors(s)):
            w.add_tensor(name, shape, kinds.get(role, GGML_F32),
                         lambda tid=tid, shape=shape, role=role: tensor(tid, shape, role, pool))
        return w.write(path)


def cached_qwen36_full(directory: str | Path | None = None) -> Path:
    """The full Qwen3.6-35B-A3B-shaped checkpoint (seed 4, random-byte
    experts, ~18 GB), written once into `directory` (default: $BT_BENCH_DIR,
    else <tmp>/bt_bench) and reused by later calls on the same machine."""
    import os
    import tempfile

    d = Path(directory or os.environ.get("BT_BENCH_DIR", Path(tempfile.gettempdir()) / "bt_bench"))
    d.mkdir(parents=True, exist_ok=True)
    path, done = d / "qwen36-35b-seed4.gguf", d / "qwen36-35b-seed4.ok"
    if not done.exists():
        write_qwen36_gguf(path, QWEN36_35B, seed=4, experts="random")
        done.write_text("ok")
    return path


__all__ = [
    "cached_qwen36_full",
    "GGML_IQ3_S",
    "QWEN36_35B",
    "QWEN36_TINY",
    "Qwen36Spec",
    "qwen36_tensors",
    "write_qwen36_gguf",
    "MoeSpec",
    "QWEN35_0_8B",
    "QWEN35_TINY",
    "Qwen35Spec",
    "SPECS",
    "make_moe_layer",
    "moe_layer_inputs",
    "qwen35_tensors",
    "write_qwen35_gguf",
]


def main() -> None:
    """``python -m breezetoken_b200.synth {0.8b,tiny} OUT.gguf [--seed N]``:
    write a seeded random-init Qwen3.5-shaped Q8_0 GGUF."""
    import argparse

    ap = argparse.ArgumentParser(description=main.__doc__)
    ap.add_argument("shape", choices=("0.8b", "tiny"))
    ap.add_argument("out")
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args()
    spec = QWEN35_0_8B if args.shape == "0.8b" else QWEN35_TINY
    print(write_qwen35_gguf(args.out, spec, seed=args.seed))


if __name__ == "__main__":
    main()

"""Generate the golden fixtures by running the reference implementation.

Imports breezetoken from a reference checkout (argument ``--reference``) and
records, on seeded inputs, what its torch f32 path computes:

* ``dequant.npz``   -- Q8_0 and IQ3_S blocks (the block builders of the
  reference's tests/test_quant_dequant.py:177-233, rng 1234) and the
  reference's ``dequantize`` output; plus the hand-computed IQ3_S vector of
  test_quant_dequant.py:268-279;
* ``ops.npz``       -- inputs/outputs of ``_torch_gdn_decode`` (16/16, 8/16 and
  16/32 heads x 128, like tests/test_cuda.py:56-77,170-191),
  ``_torch_attention`` (seq 1, 17, 128; tests/test_cuda.py:195-211),
  ``_torch_rope``, rms_norm, fused_add_rms_norm, silu_mul;
* ``moe.npz``       -- ``route`` on N(0,1) router logits (the 35B-A3B MoE layer
  shape) and one ``ExpertPool``-style expert evaluation from IQ3_S bytes;
* ``moe_shared.npz`` -- ``Qwen36Moe._moe`` (routed output + gated bf16 shared
  expert) run on a stand-in object around moe.npz's routed output;
* ``qwen36_tiny.npz`` -- greedy token ids, top-2 margins and the first
  logits of the reference's ``Qwen36Moe`` (CPU, f32) on the seeded tiny
  qwen35moe checkpoint (35B-A3B layer shapes);
* ``qwen35_tiny.npz`` / ``qwen35_0_8b.npz`` -- greedy token ids of
  ``Qwen35(backend="torch", device="cpu").generate`` on the seeded synthetic
  checkpoints of breezetoken_b200.synth, with per-step top-2 logit margins and
  a slice of the logits.

Run from the repository root:
    python tests/golden/make_golden.py --reference <breezetoken checkout>
"""

from __future__ import annotations

import argparse
import sys
import tempfile
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from breezetoken_b200.quant import quantize_iq3_s  # noqa: E402
from breezetoken_b200.synth import QWEN35_0_8B, QWEN35_TINY, write_qwen35_gguf  # noqa: E402

PROMPT_LEN = 16


def _f16(x: float) -> bytes:
    return np.float16(x).tobytes()


def make_q8_0(rng) -> bytes:
    return _f16(rng.uniform(0.01, 2.0)) + rng.integers(-127, 128, 32, dtype=np.int16).astype(np.int8).tobytes()


def make_iq3_s(rng) -> bytes:
    return (
        _f16(rng.uniform(0.01, 2.0))
        + rng.integers(0, 256, 64, dtype=np.uint8).tobytes()
        + rng.integers(0, 256, 8, dtype=np.uint8).tobytes()
        + rng.integers(0, 256, 32, dtype=np.uint8).tobytes()
        + rng.integers(0, 256, 4, dtype=np.uint8).tobytes()
    )


def gen_dequant(out: Path) -> None:
    from breezetoken.quant.dequant import dequantize
    from breezetoken.quant.formats import FORMATS, GGMLType

    rng = np.random.default_rng(1234)
    q8 = np.frombuffer(b"".join(make_q8_0(rng) for _ in range(64)), dtype=np.uint8).copy()
    iq = np.frombuffer(b"".join(make_iq3_s(rng) for _ in range(64)), dtype=np.uint8).copy()
    q8_out = dequantize(torch.from_numpy(q8), FORMATS[GGMLType.Q8_0], (64, 32)).numpy()
    iq_out = dequantize(torch.from_numpy(iq), FORMATS[GGMLType.IQ3_S], (64, 256)).numpy()
    fixed = _f16(1.0) + bytes(64) + bytes(8) + bytes(32) + bytes([0x10, 0, 0, 0])
    fixed_raw = np.frombuffer(fixed, dtype=np.uint8).copy()
    fixed_out = dequantize(torch.from_numpy(fixed_raw), FORMATS[GGMLType.IQ3_S], (256,)).numpy()
    # quantiser output of this project, decoded by the reference
    w = np.random.default_rng(3).standard_normal((8, 512)).astype(np.float32) * 0.02
    qz = quantize_iq3_s(w)
    qz_out = dequantize(torch.from_numpy(qz.reshape(-1).copy()), FORMATS[GGMLType.IQ3_S], (8, 512)).numpy()
    np.savez_compressed(
        out,
        q8_raw=q8, q8_out=q8_out, iq3s_raw=iq, iq3s_out=iq_out, iq3s_fixed_raw=fixed_raw,
        iq3s_fixed_out=fixed_out, iq3s_quant_raw=qz, iq3s_quant_out=qz_out,
    )


def ops_inputs() -> dict[str, np.ndarray]:
    """Seeded op inputs; tests regenerate them with this same function."""
    rec: dict[str, np.ndarray] = {}
    for name, hk, hv, seed in (("gdn16", 16, 16, 3), ("gdn8_16", 8, 16, 5), ("gdn16_32", 16, 32, 7)):
        rng = np.random.default_rng(seed)
        dim = 128
        rec[f"{name}_q"] = rng.standard_normal((hk, dim), dtype=np.float32)
        rec[f"{name}_k"] = rng.standard_normal((hk, dim), dtype=np.float32)
        rec[f"{name}_v"] = rng.standard_normal((hv, dim), dtype=np.float32)
        rec[f"{name}_g"] = rng.standard_normal(hv, dtype=np.float32) * np.float32(0.1)
        rec[f"{name}_beta"] = rng.standard_normal(hv, dtype=np.float32)
        rec[f"{name}_state0"] = rng.standard_normal((hv, dim, dim), dtype=np.float32)
    rng = np.random.default_rng(6)
    for seq in (1, 17, 128):
        rec[f"attn{seq}_q"] = rng.standard_normal((8, 256), dtype=np.float32)
        rec[f"attn{seq}_k"] = rng.standard_normal((seq, 2, 256), dtype=np.float32)
        rec[f"attn{seq}_v"] = rng.standard_normal((seq, 2, 256), dtype=np.float32)
    rng = np.random.default_rng(4)
    rec["rope_x"] = rng.standard_normal((8, 256), dtype=np.float32)
    rec["rope_cos"] = rng.standard_normal((128, 64), dtype=np.float32)
    rec["rope_sin"] = rng.standard_normal((128, 64), dtype=np.float32)
    rec["rope_pos"] = np.array([17], dtype=np.int32)
    rng = np.random.default_rng(0)
    rec["norm_x"] = rng.standard_normal((2, 3, 256), dtype=np.float32)
    rec["norm_gamma"] = rng.standard_normal(256, dtype=np.float32)
    rec["norm_other"] = rng.standard_normal((2, 3, 256), dtype=np.float32)
    rec["silu_gate"] = rng.standard_normal(3584, dtype=np.float32)
    rec["silu_up"] = rng.standard_normal(3584, dtype=np.float32)
    return rec


#: stride of the recorded sample of the updated GDN state
STATE_SAMPLE = 97


def gen_ops(out: Path) -> None:
    from breezetoken.backends import (
        _torch_attention,
        _torch_fused_add_rms_norm,
        _torch_gdn_decode,
        _torch_rms_norm,
        _torch_rope,
        _torch_silu_mul,
    )

    inp = {k: torch.from_numpy(v.copy()) for k, v in ops_inputs().items()}
    rec: dict[str, np.ndarray] = {}
    for name in ("gdn16", "gdn8_16", "gdn16_32"):
        state = inp[f"{name}_state0"].clone()
        o = _torch_gdn_decode(
            inp[f"{name}_q"], inp[f"{name}_k"], inp[f"{name}_v"], inp[f"{name}_g"], inp[f"{name}_beta"], state,
            128**-0.5, 1e-6,
        )
        rec[f"{name}_out"] = o.numpy()
        rec[f"{name}_state1_sample"] = state.reshape(-1)[::STATE_SAMPLE].numpy()
        rec[f"{name}_state1_sum"] = state.double().sum(dim=(1, 2)).numpy()
    for seq in (1, 17, 128):
        rec[f"attn{seq}_out"] = _torch_attention(inp[f"attn{seq}_q"], inp[f"attn{seq}_k"], inp[f"attn{seq}_v"], 256**-0.5).numpy()
    rec["rope_out"] = _torch_rope(inp["rope_x"], inp["rope_cos"], inp["rope_sin"], inp["rope_pos"], 64).numpy()
    h, xn = _torch_fused_add_rms_norm(inp["norm_x"], inp["norm_other"], inp["norm_gamma"], 1e-6)
    rec.update(
        norm_out=_torch_rms_norm(inp["norm_x"], inp["norm_gamma"], 1e-6).numpy(), fused_h=h.numpy(),
        fused_xn=xn.numpy(), silu_out=_torch_silu_mul(inp["silu_gate"], inp["silu_up"]).numpy(),
    )
    np.savez_compressed(out, **rec)


def moe_inputs():
    """Seeded MoE-layer inputs (35B-A3B layer shapes, 16 experts)."""
    rng = np.random.default_rng(3)
    hidden, ffn, n_exp = 2048, 512, 16
    logits = rng.standard_normal(256).astype(np.float32)
    gate = quantize_iq3_s(rng.standard_normal((n_exp * ffn, hidden)).astype(np.float32) * np.float32(0.02))
    up = quantize_iq3_s(rng.standard_normal((n_exp * ffn, hidden)).astype(np.float32) * np.float32(0.02))
    down = quantize_iq3_s(rng.standard_normal((n_exp * hidden, ffn)).astype(np.float32) * np.float32(0.02))
    x = rng.standard_normal(hidden).astype(np.float32)
    return dict(hidden=hidden, ffn=ffn, logits=logits, gate=gate, up=up, down=down, x=x,
                ids=[1, 5, 7, 11], w=np.array([0.4, 0.3, 0.2, 0.1], dtype=np.float32))


def gen_moe(out: Path) -> None:
    """route() on router logits plus the torch dequant-then-matmul expert path (moe.py:225-233)."""
    import hashlib

    import torch.nn.functional as F
    from breezetoken.model.moe import route
    from breezetoken.quant.dequant import dequantize
    from breezetoken.quant.formats import FORMATS, GGMLType

    m = moe_inputs()
    hidden, ffn, ids = m["hidden"], m["ffn"], m["ids"]
    # route() computes logits = gate_inp @ x; an identity gate makes them = x
    r = route(torch.from_numpy(m["logits"]), torch.eye(256), 8)
    fmt = FORMATS[GGMLType.IQ3_S]
    g_rows = np.concatenate([m["gate"][e * ffn : (e + 1) * ffn] for e in ids] + [m["up"][e * ffn : (e + 1) * ffn] for e in ids])
    gu = dequantize(torch.from_numpy(g_rows.reshape(-1).copy()), fmt, (2 * len(ids) * ffn, hidden)) @ torch.from_numpy(m["x"])
    n = len(ids)
    act = F.silu(gu[: n * ffn].view(n, ffn)) * gu[n * ffn :].view(n, ffn)
    d_rows = np.concatenate([m["down"][e * hidden : (e + 1) * hidden] for e in ids])
    dn = dequantize(torch.from_numpy(d_rows.reshape(-1).copy()), fmt, (n * hidden, ffn)).view(n, hidden, ffn)
    y = ((dn @ act.unsqueeze(-1)).squeeze(-1) * torch.from_numpy(m["w"]).view(-1, 1)).sum(0)
    digest = hashlib.sha256(m["gate"].tobytes() + m["up"].tobytes() + m["down"].tobytes()).hexdigest()
    np.savez_compressed(
        out, route_w=r.weights.numpy(), route_ids=r.expert_ids.numpy(), y=y.numpy(), act=act.numpy(),
        bytes_sha256=np.array(digest),
    )


def moe_shared_inputs():
    """Seeded bf16 shared expert for moe_inputs() (the 35B-A3B layer: one
    bf16 shared expert of ffn 512), as f32 arrays holding bf16 values."""
    rng = np.random.default_rng(4)
    m = moe_inputs()
    hidden, ffn = m["hidden"], 512

    def bf16(a: np.ndarray) -> np.ndarray:
        return torch.from_numpy(a.astype(np.float32)).bfloat16().float().numpy()

    return dict(
        gate=bf16(rng.standard_normal((ffn, hidden)) * 0.02), up=bf16(rng.standard_normal((ffn, hidden)) * 0.02),
        down=bf16(rng.standard_normal((hidden, ffn)) * 0.02),
        gate_inp=(rng.standard_normal(hidden) * 0.02).astype(np.float32), ffn=ffn,
    )


def gen_moe_shared(out: Path) -> None:
    """The reference's Qwen36Moe._moe (model/qwen36_moe.py:634-642), run on a
    stand-in object: the routed output is moe.npz's `y` (the stand-in expert
    pool returns it), the shared expert is moe_shared_inputs() in f32."""
    import types

    from breezetoken.model.qwen36_moe import Qwen36Moe

    m, sh = moe_inputs(), moe_shared_inputs()
    routed = torch.from_numpy(np.load(HERE / "moe.npz")["y"])
    stub = types.SimpleNamespace()
    stub.cfg = types.SimpleNamespace(top_k=8, shared_ffn=sh["ffn"])
    stub.layers = [{
        "router": torch.zeros(16, m["hidden"]),
        "shexp_gu": torch.from_numpy(np.concatenate([sh["gate"], sh["up"]])),
        "shexp_down": torch.from_numpy(sh["down"]),
        "shexp_gate": torch.from_numpy(sh["gate_inp"]),
    }]
    stub.experts = types.SimpleNamespace(forward=lambda i, gguf, xn, routing: routed.clone())
    stub._gguf = None
    stub._linear = lambda w, x: Qwen36Moe._linear(stub, w, x)
    y = Qwen36Moe._moe(stub, 0, torch.from_numpy(m["x"]))
    np.savez_compressed(out, y=y.numpy())


def gen_qwen36_tiny(out: Path, steps: int = 24) -> None:
    """Greedy decode of the reference's Qwen36Moe (model/qwen36_moe.py,
    device="cpu", dtype="f32") on the seeded tiny qwen35moe checkpoint of
    breezetoken_b200.synth (35B-A3B layer shapes, 4 layers, 16
    experts).  The 7-token prompt stays below the reference's batched-prefill
    threshold (8 tokens), so every token takes its per-token f32 path."""
    from breezetoken.model.qwen36_moe import Qwen36Moe

    from breezetoken_b200.synth import QWEN36_TINY, write_qwen36_gguf

    with tempfile.TemporaryDirectory() as d:
        path = write_qwen36_gguf(Path(d) / "q36.gguf", QWEN36_TINY, seed=4)
        m = Qwen36Moe(str(path), device="cpu", dtype="f32", max_context=64)
        prompt = np.random.default_rng(4).integers(0, QWEN36_TINY.vocab, 7).tolist()
        t0 = time.time()
        with torch.inference_mode():
            m.reset()
            for i, tok in enumerate(prompt):
                logits = m.forward_token(tok, i, logits=(i == len(prompt) - 1))
            tokens, margins, first = [], [], logits.numpy().copy()
            for step in range(steps):
                top2 = torch.topk(logits, 2).values
                margins.append(float(top2[0] - top2[1]))
                tok = int(logits.argmax())
                tokens.append(tok)
                if step + 1 < steps:
                    logits = m.forward_token(tok, len(prompt) + step, logits=True)
        np.savez_compressed(
            out, prompt=np.array(prompt), tokens=np.array(tokens), margins=np.array(margins, dtype=np.float32),
            logits=first[None], steps=np.array(steps), max_context=np.array(64), seconds=np.array(time.time() - t0),
        )


#: The config-5 full-shape parity case: two 7-token prompts (below the
#: reference's 8-token batched-prefill threshold, so every token takes its
#: per-token f32 path), 8 greedy steps each.
QWEN36_FULL_PROMPTS, QWEN36_FULL_PROMPT_LEN, QWEN36_FULL_STEPS = 2, 7, 8


def qwen36_full_prompts() -> np.ndarray:
    from breezetoken_b200.synth import QWEN36_35B

    return np.random.default_rng(5).integers(0, QWEN36_35B.vocab, (QWEN36_FULL_PROMPTS, QWEN36_FULL_PROMPT_LEN))


def gen_qwen36_full(out: Path, gguf: Path | None = None) -> None:
    """Greedy decode of the reference's Qwen36Moe (device="cpu", dtype="f32")
    on the full Qwen3.6-35B-A3B-shaped checkpoint (40 layers, 256 IQ3_S
    experts, vocab 151936; seed 4, random-byte experts: synth.write_qwen36_gguf
    experts="random"), for the two prompts of qwen36_full_prompts()."""
    from breezetoken.model.qwen36_moe import Qwen36Moe

    from breezetoken_b200.synth import QWEN36_35B, write_qwen36_gguf

    with tempfile.TemporaryDirectory() as d:
        path = gguf or write_qwen36_gguf(Path(d) / "q36_full.gguf", QWEN36_35B, seed=4, experts="random")
        m = Qwen36Moe(str(path), device="cpu", dtype="f32", max_context=64)
        prompts = qwen36_full_prompts()
        t0 = time.time()
        tokens, margins, top_idx, top_val, first = [], [], [], [], None
        with torch.inference_mode():
            for b, prompt in enumerate(prompts.tolist()):
                m.reset()
                for i, tok in enumerate(prompt):
                    logits = m.forward_token(tok, i, logits=(i == len(prompt) - 1))
                if b == 0:
                    first = logits.numpy().copy()
                seq_t, seq_m, seq_i, seq_v = [], [], [], []
                for step in range(QWEN36_FULL_STEPS):
                    top = torch.topk(logits, 16)
                    seq_m.append(float(top.values[0] - top.values[1]))
                    seq_i.append(top.indices.numpy())
                    seq_v.append(top.values.numpy())
                    tok = int(logits.argmax())
                    seq_t.append(tok)
                    if step + 1 < QWEN36_FULL_STEPS:
                        logits = m.forward_token(tok, len(prompt) + step, logits=True)
                tokens.append(seq_t)
                margins.append(seq_m)
                top_idx.append(np.stack(seq_i))
                top_val.append(np.stack(seq_v))
        np.savez_compressed(
            out, prompts=prompts, tokens=np.array(tokens), margins=np.array(margins, dtype=np.float32),
            top_idx=np.stack(top_idx), top_val=np.stack(top_val), logits=first[None], max_context=np.array(64),
            seconds=np.array(time.time() - t0), threads=np.array(torch.get_num_threads()),
        )


def gen_model(out: Path, spec, steps: int, max_context: int, keep_logits: int) -> None:
    from breezetoken.gguf import GGUFFile
    from breezetoken.model.qwen35 import Qwen35

    with tempfile.TemporaryDirectory() as td:
        path = write_qwen35_gguf(Path(td) / "m.gguf", spec, seed=0)
        prompt = np.random.default_rng(0).integers(0, spec.vocab, PROMPT_LEN).tolist()
        with GGUFFile(path) as g:
            model = Qwen35(g, backend="torch", device="cpu", max_context=max_context)
        t0 = time.time()
        toks, margins, top_idx, top_val, first = [], [], [], [], []
        logits = model._prefill_batch(prompt)
        for step in range(steps):
            lv = logits.float()
            nxt = int(lv.argmax())
            top = torch.topk(lv, 64)
            toks.append(nxt)
            margins.append(float(top.values[0] - top.values[1]))
            top_idx.append(top.indices.numpy())
            top_val.append(top.values.numpy())
            if step < keep_logits:
                first.append(lv.numpy())
            if step + 1 < steps:
                logits = model.forward_token(nxt, PROMPT_LEN + step, logits=True)
        # must match the reference's public generate()
        assert model.generate(prompt, steps, 0.0) == toks
        elapsed = time.time() - t0
    np.savez_compressed(
        out, prompt=np.array(prompt), tokens=np.array(toks), margins=np.array(margins, dtype=np.float32),
        top_idx=np.stack(top_idx), top_val=np.stack(top_val), logits=np.stack(first), steps=steps,
        max_context=max_context, seconds=elapsed, threads=torch.get_num_threads(),
    )


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--skip-0_8b", action="store_true")
    ap.add_argument("--only", help="regenerate one fixture (e.g. moe_shared)")
    ap.add_argument("--gguf", help="qwen36_full: an already written full-shape checkpoint (seed 4, random experts)")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    if args.only == "moe_shared":
        gen_moe_shared(HERE / "moe_shared.npz")
        return
    if args.only == "qwen36_tiny":
        gen_qwen36_tiny(HERE / "qwen36_tiny.npz")
        return
    if args.only == "qwen36_full":
        gen_qwen36_full(HERE / "qwen36_full.npz", Path(args.gguf) if args.gguf else None)
        return
    gen_dequant(HERE / "dequant.npz")
    gen_ops(HERE / "ops.npz")
    gen_moe(HERE / "moe.npz")
    gen_moe_shared(HERE / "moe_shared.npz")
    gen_qwen36_tiny(HERE / "qwen36_tiny.npz")
    gen_qwen36_full(HERE / "qwen36_full.npz")
    gen_model(HERE / "qwen35_tiny.npz", QWEN35_TINY, steps=32, max_context=512, keep_logits=4)
    if not args.skip_0_8b:
        gen_model(HERE / "qwen35_0_8b.npz", QWEN35_0_8B, steps=128, max_context=1024, keep_logits=1)
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()

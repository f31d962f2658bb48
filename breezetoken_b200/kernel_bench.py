"""Kernel microbenchmarks through the C ABI (CUDA-event timing).

    python -m breezetoken_b200.kernel_bench gemv --n 151936 --k 1024
    python -m breezetoken_b200.kernel_bench gdn --batch 64 --steps 256
    python -m breezetoken_b200.kernel_bench attn --batch 64 --ctx 32768
    python -m breezetoken_b200.kernel_bench moe --tokens 8
    python -m breezetoken_b200.kernel_bench qwen36 --batch 64 --prompt 512 --steps 256
    python -m breezetoken_b200.kernel_bench linear --tokens 64
    python -m breezetoken_b200.kernel_bench trace --gguf model.gguf
    python -m breezetoken_b200.kernel_bench attn-layer --batch 64 --pos 648 --splits 2
    python -m breezetoken_b200.kernel_bench load
    python -m breezetoken_b200.kernel_bench precision
    torchrun --nproc-per-node 2 -m breezetoken_b200.kernel_bench moe-ep --tokens 8

Each prints one JSON line: average launch time and achieved HBM GB/s from
the algorithmic bytes of one launch (weights / state / KV read once).
``moe`` is the 35B-A3B MoE-layer benchmark: one MoE layer (hidden 2048, 256
IQ3_S experts of ffn 512 quantised from N(0, 0.02), top-8 over N(0,1) router
logits, the bf16 shared expert, seed 3), its output checked once against a
dequantise-then-matmul, then timed per call after reading a 256 MB buffer
(the experts are not in L2); its bytes are the U * 1,351,680 of the U
distinct experts the routing selects, the shared expert and x in and out.
``qwen36`` is the 35B-A3B decode benchmark on one GPU (Qwen3.6-35B-A3B shape, seeded
random weights built on the device, 64 sequences in lockstep).
``linear`` times ``bt_linear_rows`` (bf16 weight rows x three bf16 planes of
x) at the 35B-A3B decoder's projection shapes (GDN qkv 8192 x 2048, z 4096 x 2048, out
2048 x 4096, the 151936 x 2048 head) for T tokens, cycling over weight
copies larger than L2 together.
``trace`` prints the device-side timeline of one Qwen3.5 decode step (per
kernel kind: release gap, prologue, body) after a 16-token prefill.
``load`` times loading the full-shape checkpoint (parse, upload, repack).
``moe-ep`` times the ``moe`` layer expert-parallel over the torchrun ranks
against the replicated layer.
``precision`` prints, per projection path at the decoders' shapes, the worst
error against an f64 product (of the output scale, and per element).
``gdn`` and ``attn`` are the stand-alone GDN-step and split-KV attention decode
benchmarks with their synthetic inputs (seeds 1 and 2).
"""

from __future__ import annotations

import argparse
import json
import time
from pathlib import Path

import numpy as np
import torch

from breezetoken_b200 import _native as N
from breezetoken_b200.backends import Q8Weight
from breezetoken_b200.quant import quantize_q8_0


def _time_graph(fn, iters: int, stream: torch.cuda.Stream) -> float:
    """Device time per call with `iters` calls captured in one CUDA graph (no
    host launch cost between them), averaged over 3 replays."""
    with torch.cuda.stream(stream):
        for _ in range(3):
            fn()
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for _ in range(iters):
            fn()
    with torch.cuda.stream(stream):
        g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(3):
            g.replay()
        e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) / 1e3 / (3 * iters)


def _time(fn, iters: int, stream: torch.cuda.Stream) -> float:
    with torch.cuda.stream(stream):
        for _ in range(3):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(iters):
            fn()
        e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) / 1e3 / iters


def bench_gemv(n: int, k: int, iters: int) -> dict:
    rng = np.random.default_rng(0)
    # random bytes are a valid Q8_0 stream for timing; quantise a small tile and tile it
    tile = quantize_q8_0(rng.standard_normal((256, k)).astype(np.float32) * 0.02)
    raw = np.tile(tile, ((n + 255) // 256, 1))[:n]
    w = Q8Weight.from_gguf(raw, n, k, "cuda")
    x = torch.randn(k, device="cuda")
    y = torch.empty(n, device="cuda")
    s = torch.cuda.Stream()
    lib = N.load()

    def run():
        N.check(lib.bt_linear_q8(w.data.data_ptr(), x.data_ptr(), y.data_ptr(), n, k, 1, s.cuda_stream), "gemv")

    sec = _time(run, iters, s)
    nbytes = w.data.numel() + 4 * (k + n)
    return {"kernel": "gemv_q8", "n": n, "k": k, "us": sec * 1e6, "bytes": nbytes, "gbs": nbytes / sec / 1e9}


def bench_linear(n: int, k: int, t: int, iters: int) -> dict:
    g = torch.Generator(device="cuda").manual_seed(5)
    nbytes_w = n * k * 2
    copies = max(1, -(-(256 << 20) // nbytes_w))  # together larger than L2
    ws = [(torch.randn(n, k, device="cuda", generator=g) * 0.02).to(torch.bfloat16) for _ in range(copies)]
    x = torch.randn(t, k, device="cuda", generator=g)
    planes = torch.empty(t, 3, k, dtype=torch.bfloat16, device="cuda")
    y = torch.empty(t, n, device="cuda")
    s = torch.cuda.Stream()
    lib = N.load()
    N.check(lib.bt_bf16_planes(x.data_ptr(), planes.data_ptr(), t, k, s.cuda_stream), "planes")
    it = [0]

    def run():
        w = ws[it[0] % copies]
        it[0] += 1
        N.check(lib.bt_linear_rows(w.data_ptr(), N.BT_BF16, planes.data_ptr(), y.data_ptr(), n, k, t, s.cuda_stream),
                "linear_rows")

    sec = _time_graph(run, max(iters, copies), s)
    nbytes = nbytes_w + t * 3 * k * 2 + t * n * 4
    return {"kernel": "linear_rows", "n": n, "k": k, "tokens": t, "us": sec * 1e6, "bytes": nbytes,
            "gbs": nbytes / sec / 1e9, "tflops": 2 * n * k * t / sec / 1e12,
            "tflops_planes": 3 * 2 * n * k * t / sec / 1e12, "l2": f"{copies} weight copies cycled"}


def _errors(y: np.ndarray, want: np.ndarray, host_f32: np.ndarray) -> dict:
    """Errors of f32 outputs `y` against an f64 product `want`: relative to the
    output scale (max |want|), and per element over the elements of at least
    1e-3 of the scale (smaller ones are cancellations, whose relative error
    says nothing about the kernel); `host_f32` (the same product in f32 by
    the host's BLAS, as a torch f32 CPU path computes it) measured the same
    way for comparison."""
    scale = float(np.abs(want).max())
    big = np.abs(want) >= 1e-3 * scale

    def measure(v: np.ndarray) -> tuple[float, float, float]:
        err = np.abs(v.astype(np.float64) - want)
        rel = err[big] / np.abs(want[big])
        return float(err.max() / scale), float(rel.max()), float(np.quantile(rel, 0.999))

    a, b, c = measure(y)
    ha, hb, _ = measure(host_f32)
    return {"rel_of_scale": a, "rel_elem_max": b, "rel_elem_p999": c, "host_f32_rel_of_scale": ha,
            "host_f32_rel_elem_max": hb, "elements": int(y.size)}


def bench_precision() -> list[dict]:
    """Worst errors of each projection path on seeded N(0, 0.02) weights and
    N(0, 1) activations, against f64 products of the same (device-dequantised)
    weights: the Q8_0 GEMV of a batch-1 step (its activations carried to 2^-22
    of each 32-element block's maximum), bf16 rows for 8 tokens (CUDA cores)
    and 64 tokens (tcgen05), f32 rows (the router) for 64 tokens."""
    rng = np.random.default_rng(21)
    out = []
    lib = N.load()
    for n, k in ((3584, 1024), (1024, 3584), (8224, 1024)):  # 0.8B gate/up, down, GDN in-projection
        w = Q8Weight.from_gguf(quantize_q8_0(rng.standard_normal((n, k)).astype(np.float32) * 0.02), n, k, "cuda")
        deq32 = w.dequantize().cpu().numpy()
        deq = deq32.astype(np.float64)
        x = rng.standard_normal(k).astype(np.float32)
        y = torch.empty(n, device="cuda")
        xd = torch.from_numpy(x).cuda()
        N.check(lib.bt_linear_q8(w.data.data_ptr(), xd.data_ptr(), y.data_ptr(), n, k, 1, 0), "gemv")
        out.append({"path": "q8_0 gemv", "n": n, "k": k, "tokens": 1,
                    **_errors(y.cpu().numpy(), deq @ x.astype(np.float64), deq32 @ x)})
    for n, k, t, dt in ((2048, 4096, 8, N.BT_BF16), (8192, 2048, 8, N.BT_BF16), (8192, 2048, 64, N.BT_BF16),
                        (2048, 4096, 64, N.BT_BF16), (256, 2048, 64, N.BT_F32)):
        wf = rng.standard_normal((n, k)).astype(np.float32) * 0.02
        w = torch.from_numpy(wf).to(torch.bfloat16 if dt == N.BT_BF16 else torch.float32).cuda().contiguous()
        x = rng.standard_normal((t, k)).astype(np.float32)
        xd = torch.from_numpy(x).cuda()
        planes = torch.empty(t, 3, k, dtype=torch.bfloat16, device="cuda")
        y = torch.empty(t, n, device="cuda")
        N.check(lib.bt_bf16_planes(xd.data_ptr(), planes.data_ptr(), t, k, 0), "planes")
        N.check(lib.bt_linear_rows(w.data_ptr(), dt, planes.data_ptr(), y.data_ptr(), n, k, t, 0), "linear_rows")
        w32 = w.float().cpu().numpy()
        want = x.astype(np.float64) @ w32.astype(np.float64).T
        out.append({"path": ("bf16" if dt == N.BT_BF16 else "f32") + " rows", "n": n, "k": k, "tokens": t,
                    **_errors(y.cpu().numpy(), want, x @ w32.T)})
    torch.cuda.synchronize()
    return out


def bench_gdn(batch: int, steps: int, heads: int = 16, dim: int = 128) -> dict:
    rng = np.random.default_rng(1)
    q = torch.from_numpy(rng.standard_normal((batch, heads, dim), dtype=np.float32)).to("cuda", torch.bfloat16)
    k = torch.from_numpy(rng.standard_normal((batch, heads, dim), dtype=np.float32)).to("cuda", torch.bfloat16)
    v = torch.from_numpy(rng.standard_normal((batch, heads, dim), dtype=np.float32)).to("cuda", torch.bfloat16)
    g = -torch.nn.functional.softplus(torch.from_numpy(rng.standard_normal((batch, heads), dtype=np.float32))).cuda()
    beta = torch.from_numpy(rng.standard_normal((batch, heads), dtype=np.float32)).cuda()
    state = torch.zeros(batch, heads, dim, dim, device="cuda")
    out = torch.empty(batch, heads, dim, device="cuda")
    s = torch.cuda.Stream()
    lib = N.load()

    def run():
        N.check(
            lib.bt_gdn_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), N.BT_BF16, g.data_ptr(), beta.data_ptr(),
                              state.data_ptr(), out.data_ptr(), batch, heads, heads, dim, 1.0, 1e-6, s.cuda_stream),
            "gdn",
        )

    sec = _time(run, steps, s)
    gsec = _time_graph(run, steps, s)
    # the same steps with a 256 MB read before each (L2 holds none of the
    # state when a step starts): device time of (flush + step) minus flush
    flush = torch.ones(256 << 20, dtype=torch.uint8, device="cuda")

    def flush_l2() -> None:
        flush.sum(dtype=torch.int32)

    fsec = _time_graph(lambda: (flush_l2(), run()), steps, s) - _time_graph(flush_l2, steps, s)
    nbytes = batch * (2 * heads * dim * dim * 4 + 3 * heads * dim * 2 + 2 * heads * 4 + heads * dim * 4)
    return {"kernel": "gdn_decode", "batch": batch, "steps": steps, "us_per_step": sec * 1e6,
            "us_per_step_graph": gsec * 1e6, "us_per_step_l2_flushed": fsec * 1e6, "bytes": nbytes,
            "gbs": nbytes / sec / 1e9, "gbs_graph": nbytes / gsec / 1e9, "gbs_l2_flushed": nbytes / fsec / 1e9,
            "note": "graph: the steps captured in one CUDA graph, back to back (a state of up to ~126 MB partly "
                    "stays in L2 between steps); l2_flushed: a 256 MB read before every step"}


def bench_gdn_scan(batch: int, steps: int, iters: int = 5, heads: int = 16, dim: int = 128) -> dict:
    """The config-2 op's `steps` tokens as one prefill scan (bt_gdn_prefill):
    q/k/v (steps, B, 16, 128) bf16, g/beta (steps, B, 16) f32, state read and
    written once; L2 flushed before each launch.  Compared with `steps`
    launches of the decode step on the same inputs."""
    gen = torch.Generator(device="cuda").manual_seed(1)
    q = torch.nn.functional.normalize(torch.randn(steps, batch, heads, dim, device="cuda", generator=gen), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(steps, batch, heads, dim, device="cuda", generator=gen), dim=-1)
    q, k = q.to(torch.bfloat16), k.to(torch.bfloat16)
    v = torch.randn(steps, batch, heads, dim, device="cuda", generator=gen).to(torch.bfloat16)
    g = -torch.nn.functional.softplus(torch.randn(steps, batch, heads, device="cuda", generator=gen))
    beta = torch.randn(steps, batch, heads, device="cuda", generator=gen)
    state = torch.zeros(batch, heads, dim, dim, device="cuda")
    out = torch.empty(steps, batch, heads, dim, device="cuda")
    flush = torch.ones(256 << 20, dtype=torch.uint8, device="cuda")
    s = torch.cuda.Stream()
    lib = N.load()
    nk = heads * dim

    def scan():
        N.check(lib.bt_gdn_prefill(q.data_ptr(), k.data_ptr(), v.data_ptr(), N.BT_BF16, nk, nk, nk, batch * nk,
                                   batch * nk, batch * nk, g.data_ptr(), heads, batch * heads, beta.data_ptr(), heads,
                                   batch * heads, state.data_ptr(), out.data_ptr(), nk, batch * nk, steps, batch,
                                   heads, heads, dim, 1.0, 1e-6, s.cuda_stream), "gdn_prefill")

    def steps_loop():
        for t in range(steps):
            N.check(lib.bt_gdn_decode(q[t].data_ptr(), k[t].data_ptr(), v[t].data_ptr(), N.BT_BF16, g[t].data_ptr(),
                                      beta[t].data_ptr(), state.data_ptr(), out[t].data_ptr(), batch, heads, heads,
                                      dim, 1.0, 1e-6, s.cuda_stream), "gdn_decode")

    def timed(fn) -> float:
        tot = 0.0
        with torch.cuda.stream(s):
            for i in range(iters + 1):
                flush.sum(dtype=torch.int32)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(s)
                fn()
                e1.record(s)
                e1.synchronize()
                if i:
                    tot += e0.elapsed_time(e1) / 1e3
        return tot / iters

    scan_s, loop_s = timed(scan), timed(steps_loop)
    nbytes = batch * heads * dim * dim * 4 * 2 + steps * batch * heads * (3 * dim * 2 + 2 * 4 + dim * 4)
    return {"kernel": "gdn_prefill", "batch": batch, "steps": steps, "us": scan_s * 1e6,
            "us_per_token": scan_s * 1e6 / steps, "decode_steps_us": loop_s * 1e6, "speedup": loop_s / scan_s,
            "bytes": nbytes, "gbs": nbytes / scan_s / 1e9,
            "note": "one launch over all steps (state on chip) vs one decode launch per step; L2 flushed before each"}


def attn_inputs(batch: int, ctx: int, seed: int = 2):
    """The flash-decode benchmark's inputs (8 q heads, 2 KV heads of 256, one
    query per sequence, bf16 K/V N(0, 1), uniform length ctx), drawn on the
    device from a seeded generator: q (B, 8, 256) f32, k and v (B, ctx, 2,
    256) bf16, lens (B,) int32."""
    heads, kv_heads, dim = 8, 2, 256
    gen = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(batch, heads, dim, device="cuda", generator=gen)
    kc = torch.randn(batch, ctx, kv_heads, dim, device="cuda", generator=gen).to(torch.bfloat16)
    vc = torch.randn(batch, ctx, kv_heads, dim, device="cuda", generator=gen).to(torch.bfloat16)
    lens = torch.full((batch,), ctx, dtype=torch.int32, device="cuda")
    return q, kc, vc, lens


def attn_splits(batch: int, kv_heads: int, ctx: int) -> int:
    """KV splits per (sequence, KV head): about two CTAs per SM in total, at
    least 256 keys per split, at most 256 splits."""
    return max(1, min(256, (2 * N.load().bt_sm_count() + batch * kv_heads - 1) // (batch * kv_heads), ctx // 256))


def bench_attn(batch: int, ctx: int, splits: int, iters: int) -> dict:
    heads, kv_heads, dim = 8, 2, 256
    q, kc, vc, lens = attn_inputs(batch, ctx)
    out = torch.empty(batch, heads, dim, device="cuda")
    lib = N.load()
    if splits <= 0:
        splits = attn_splits(batch, kv_heads, ctx)
    ws = torch.zeros(int(lib.bt_attention_workspace_bytes(batch, kv_heads, heads, dim, splits)), dtype=torch.uint8,
                     device="cuda")
    s = torch.cuda.Stream()

    def run():
        N.check(
            lib.bt_attention_decode(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), N.BT_BF16, lens.data_ptr(),
                                    out.data_ptr(), batch, heads, kv_heads, dim, ctx, 1.0 / 16, splits,
                                    ws.data_ptr(), s.cuda_stream),
            "attn",
        )

    sec = _time(run, iters, s)
    gsec = _time_graph(run, iters, s)
    nbytes = batch * ctx * kv_heads * dim * 2 * 2 + 2 * batch * heads * dim * 4
    return {"kernel": "attn_decode", "batch": batch, "ctx": ctx, "splits": splits, "us": sec * 1e6,
            "us_graph": gsec * 1e6, "bytes": nbytes, "gbs": nbytes / sec / 1e9, "gbs_graph": nbytes / gsec / 1e9}


def bench_attn_layer(batch: int, pos: int, splits: int, iters: int) -> dict:
    """bt_attention_layer (the fused Qwen3.6 attention layer: q/k norms, RoPE,
    KV write, attention, gate) at the 35B-A3B shape (16 q / 2 KV heads x 256,
    f32 cache of 769 positions), every sequence at position `pos` - 7 b, seed
    3; timed per call in a CUDA graph of `iters` calls (no host launch time),
    L2 flushed by a 256 MB read between calls outside the events.  Bytes: the
    K and V rows attended (f32)."""
    from breezetoken_b200.qwen36_moe import Qwen36Config, rope_tables
    from breezetoken_b200.synth import QWEN36_35B

    heads, kv, dim, cap = 16, 2, 256, 769
    cfg = Qwen36Config.from_spec(QWEN36_35B, cap)
    cos, sin = (t.cuda() for t in rope_tables(cfg))
    g = torch.Generator(device="cuda").manual_seed(3)
    proj = torch.randn(batch, (2 * heads + 2 * kv) * dim, device="cuda", generator=g)
    qn = 1 + 0.02 * torch.randn(dim, device="cuda", generator=g)
    kn = 1 + 0.02 * torch.randn(dim, device="cuda", generator=g)
    kc = torch.randn(batch, cap, kv, dim, device="cuda", generator=g)
    vc = torch.randn(batch, cap, kv, dim, device="cuda", generator=g)
    pos_t = torch.tensor([max(0, pos - 7 * b) for b in range(batch)], dtype=torch.int32, device="cuda")
    lib = N.load()
    ws = torch.zeros(max(256, int(lib.bt_attention_workspace_bytes(batch, kv, heads, dim, splits))),
                     dtype=torch.uint8, device="cuda")
    out = torch.empty(batch, heads, dim, device="cuda")
    flush = torch.ones(256 << 20, dtype=torch.uint8, device="cuda")
    s = torch.cuda.Stream()

    def call() -> None:
        N.call("bt_attention_layer", proj.data_ptr(), proj.shape[1], qn.data_ptr(), kn.data_ptr(), cos.data_ptr(),
               sin.data_ptr(), cfg.rope_dim, pos_t.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), batch,
               heads, kv, dim, cap, float(dim ** -0.5), float(cfg.eps), splits, ws.data_ptr(), None,
               torch.cuda.current_stream().cuda_stream)

    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            call()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        call()
    total = 0.0
    with torch.cuda.stream(s):
        for i in range(iters + 3):
            flush.sum(dtype=torch.int32)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(s)
            graph.replay()
            b.record(s)
            b.synchronize()
            if i >= 3:
                total += a.elapsed_time(b) * 1e3
    us = total / iters
    nbytes = int(sum(int(p) + 1 for p in pos_t.tolist())) * kv * dim * 4 * 2
    return {"kernel": "attention_layer", "batch": batch, "pos": pos, "splits": splits, "us": us,
            "bytes": nbytes, "gbs": nbytes / us / 1e3, "l2": "flushed before each call (256 MB read)",
            "timing": "one graph replay of one call between CUDA events"}


def bench_moe(tokens: int, iters: int, shared: bool = True) -> dict:
    from breezetoken_b200.moe import IQ3SExperts, SharedExpert, moe_forward, route_logits
    from breezetoken_b200.synth import MoeSpec, make_moe_layer, moe_layer_inputs

    hidden, ffn, n_exp, top_k = 2048, 512, 256, 8
    # the MoE-layer benchmark's layer: 256 distinct IQ3_S experts quantised
    # from N(0, 0.02) and the bf16 shared expert, seed 3
    m = make_moe_layer(MoeSpec(), seed=3)
    ex = IQ3SExperts.from_gguf_bytes(m["gate"], m["up"], m["down"], n_exp, hidden, ffn, "cuda")
    xh, lh = moe_layer_inputs(tokens)
    x, logits = torch.from_numpy(xh).cuda(), torch.from_numpy(lh).cuda()
    r = route_logits(logits, top_k)
    u = int(torch.unique(r.expert_ids).numel())
    se = None
    if shared:
        se = SharedExpert.from_tensors(torch.from_numpy(m["sh_gate"]), torch.from_numpy(m["sh_up"]),
                                       torch.from_numpy(m["sh_down"]), torch.from_numpy(m["sh_gate_inp"]), "cuda")
        ws = torch.zeros(int(N.load().bt_moe_layer_workspace_bytes(tokens, hidden, ffn, ffn, n_exp, top_k)),
                         dtype=torch.uint8, device="cuda")
    else:
        ws = torch.zeros(int(N.load().bt_moe_workspace_bytes(tokens, hidden, ffn, n_exp, top_k)), dtype=torch.uint8,
                         device="cuda")
    flush = torch.ones(256 << 20, dtype=torch.uint8, device="cuda")
    s = torch.cuda.Stream()

    def flush_l2() -> None:
        flush.sum(dtype=torch.int32)  # read 256 MB: afterwards L2 holds only clean lines

    def call() -> torch.Tensor:
        return moe_forward(ex, se, x, r.expert_ids, r.weights, ws)

    # self-check of up to 4 tokens against a dequantise-then-matmul in f64 on
    # the bit-exact device dequantisation (bt_dequant_iq3_s)
    got = call()
    worst = 0.0
    for t in range(min(tokens, 4)):
        ref = torch.zeros(hidden, dtype=torch.float64, device="cuda")
        xt = x[t].double()
        for e, w in zip(r.expert_ids[t].tolist(), r.weights[t].tolist(), strict=True):
            deq = []
            for name, rows, k in (("gate", ffn, hidden), ("up", ffn, hidden), ("down", hidden, ffn)):
                raw = torch.from_numpy(m[name][e * rows:(e + 1) * rows].reshape(-1).copy()).cuda()
                out = torch.empty(rows, k, device="cuda")
                N.call("bt_dequant_iq3_s", raw.data_ptr(), out.data_ptr(), rows, k, 0)
                torch.cuda.synchronize()
                deq.append(out.double())
            act = torch.nn.functional.silu(deq[0] @ xt) * (deq[1] @ xt)
            ref += w * (deq[2] @ act)
        if se is not None:
            g = torch.sigmoid(se.gate_inp.double() @ xt)
            act = torch.nn.functional.silu(se.gate.double() @ xt) * (se.up.double() @ xt)
            ref += g * (se.down.double() @ act)
        worst = max(worst, float((got[t].double() - ref).abs().max() / ref.abs().max()))
    if worst > 1e-5:
        raise AssertionError(f"MoE layer output off by {worst:.2e} of scale")

    # launch-timed: events around each call, L2 flushed before it
    total = 0.0
    with torch.cuda.stream(s):
        for i in range(iters + 3):
            flush_l2()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            call()
            e1.record(s)
            e1.synchronize()
            if i >= 3:
                total += e0.elapsed_time(e1) / 1e3
    sec = total / iters
    # device time: (flush + call) and flush alone, each captured `iters` times
    # in one CUDA graph (no host launch gaps)
    both = _time_graph(lambda: (flush_l2(), call()), iters, s)
    alone = _time_graph(flush_l2, iters, s)
    gsec = both - alone
    # algorithmic bytes: the selected experts, the bf16 shared expert, x in and out
    nbytes = u * 1_351_680 + (6_291_456 if shared else 0) + tokens * hidden * 8
    return {"kernel": "moe_layer_iq3s", "tokens": tokens, "unique_experts": u, "shared_expert": shared,
            "us": sec * 1e6, "us_graph": gsec * 1e6, "bytes": nbytes, "gbs": nbytes / sec / 1e9,
            "gbs_graph": nbytes / gsec / 1e9, "check_rel_err": worst,
            "l2": "flushed before each call (256 MB read)"}


def _kernel_timeline(run, n_steps: int) -> dict:
    """Device timeline of `run()` (n_steps decode steps) under the CUDA
    profiling interface (torch.profiler): per kernel name the launches and the
    summed device time per step, and the span from the first kernel's start
    to the last one's end per step.  Kernels launched early with programmatic
    dependent launch count their wait for the predecessor, so the per-kernel
    sums exceed the span; `excl_us_per_step` charges each launch only the time
    from the previous kernel's end (or its own start, if later) to its own end,
    which sums to the span less the idle gaps."""
    import collections

    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        run()
        torch.cuda.synchronize()
    evs = [e for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA and e.time_range.elapsed_us() > 0
           and "Memcpy" not in e.name and "Memset" not in e.name]
    span = max(e.time_range.end for e in evs) - min(e.time_range.start for e in evs)
    agg = collections.defaultdict(lambda: [0, 0.0, 0.0])
    prev_end = None
    for e in sorted(evs, key=lambda e: e.time_range.start):
        name = e.name.replace("(anonymous namespace)::", "").split("(")[0].replace("void ", "").replace("bt::", "")
        agg[name][0] += 1
        agg[name][1] += e.time_range.elapsed_us()
        start = e.time_range.start if prev_end is None else max(prev_end, e.time_range.start)
        agg[name][2] += max(0.0, e.time_range.end - start)
        prev_end = e.time_range.end if prev_end is None else max(prev_end, e.time_range.end)
    rows = sorted(agg.items(), key=lambda kv: -kv[1][2])
    return {"span_us_per_step": span / n_steps, "kernels_per_step": len(evs) / n_steps,
            "kernels": [{"kernel": k, "launches_per_step": c / n_steps, "us_per_step": t / n_steps,
                         "excl_us_per_step": x / n_steps} for k, (c, t, x) in rows]}


def bench_qwen36(batch: int, prompt: int, steps: int, layers: int, timeline: bool = False) -> dict | None:
    """The 35B-A3B decode benchmark: `batch` sequences of a `prompt`-token random prompt,
    fed in lockstep, then `steps` greedy steps timed with CUDA events; seeded
    random weights of the Qwen3.6-35B-A3B shape (with `layers` layers) built
    on the device.  Under torchrun the sequences are sharded: each of the N
    ranks holds a full replica and decodes batch / N sequences, the timed
    region is bracketed by barriers and the slowest rank's time counts; rank
    0 returns the result, the others None."""
    import os
    from dataclasses import replace

    from breezetoken_b200.qwen36_moe import Qwen36Moe
    from breezetoken_b200.shard import aggregate_rate, max_over_ranks
    from breezetoken_b200.synth import QWEN36_35B

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
        if batch % world:
            raise ValueError(f"batch {batch} does not split over {world} GPUs")
    local = batch // world
    spec = replace(QWEN36_35B, n_layers=layers)
    m = Qwen36Moe.random(spec, batch=local, max_context=prompt + steps + 1)
    rng = np.random.default_rng(4 + rank)
    toks = torch.from_numpy(rng.integers(0, spec.vocab, (prompt, local))).cuda()
    t0 = time.time()
    m.prefill(toks[: prompt - 1].t().contiguous())  # the chunked batched prefill
    nxt = m.decode_batch(toks[prompt - 1], prompt - 1)
    torch.cuda.synchronize()
    prefill_s = time.time() - t0
    m.graph_decode(nxt, prompt, 1)  # capture (and one step)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    h0 = time.perf_counter()
    m.graph_decode(nxt, prompt, steps)  # one CUDA graph replay per step, no host sync
    host = time.perf_counter() - h0  # enqueue time: close to `sec` when launches, not kernels, bound the step
    e1.record()
    e1.synchronize()
    sec, prefill_s = max_over_ranks([e0.elapsed_time(e1) / 1e3, prefill_s], "cuda")
    if world > 1:
        dist.barrier()
    tl = None
    if timeline and rank == 0:
        n_tl = min(steps, 4)
        m.set_decode(nxt, prompt)
        tl = _kernel_timeline(lambda: m.replay(n_tl), n_tl)
    cfg = m.cfg
    # per-step algorithmic bytes (bf16 non-expert weights without the
    # embedding gather, selected experts at the expected number of distinct
    # experts per layer, GDN state r+w, f32 KV read at the mean context)
    u = cfg.n_experts * (1 - (1 - cfg.top_k / cfg.n_experts) ** local)
    dense = sum(t.numel() * t.element_size() for layer in m.layers for k, t in layer.items()
                if isinstance(t, torch.Tensor)) + m.head.numel() * 2
    dense += sum(sum(x.numel() * x.element_size() for x in (la["shared"].gate, la["shared"].up, la["shared"].down))
                 for la in m.layers)
    n_gdn = cfg.n_layers - len(cfg.attn_layers)
    state = local * n_gdn * cfg.gdn_value_heads * cfg.gdn_k_dim * cfg.gdn_value_dim * 4 * 2
    kv = local * (prompt + steps / 2) * len(cfg.attn_layers) * 2 * cfg.n_kv * cfg.head_dim * 4
    step_bytes = dense + cfg.n_layers * u * 1_351_680 + state + kv  # per GPU
    m.close()
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return None
    return {"kernel": "qwen36_35b_decode", "layers": layers, "n_gpus": world, "batch": batch, "batch_per_gpu": local,
            "prompt": prompt, "steps": steps, "tok_s": aggregate_rate(local * steps, world, sec),
            "scaling": "strong (64 sequences split over the GPUs)", "ms_per_step": sec / steps * 1e3,
            "host_enqueue_ms_per_step": host / steps * 1e3, "prefill_s": prefill_s,
            "expected_unique_experts": u, "step_bytes_per_gpu": step_bytes,
            "gbs_per_gpu": step_bytes * steps / sec / 1e9, **({"timeline": tl} if tl else {})}


def bench_moe_ep(tokens: int, iters: int) -> dict | None:
    """The MoE-layer benchmark's layer placed expert-parallel over the N
    ranks of torchrun (breezetoken_b200.expert_parallel): each rank holds 256 / N
    experts and T tokens of its own (seed 3 + rank), and one layer call is
    dispatch all-to-all -> local experts over N T tokens -> combine all-to-all
    + shared expert.  Timed per call with CUDA events after a 256 MB read and a
    barrier, slowest rank; beside it the same rank's tokens through the
    replicated layer (all 256 experts on the GPU, no collective) and the parts
    of the EP call.  Rank 0 returns the result."""
    import datetime
    import os

    import torch.distributed as dist

    from breezetoken_b200.expert_parallel import ExpertParallelMoE
    from breezetoken_b200.moe import IQ3SExperts, SharedExpert, moe_forward, route_logits
    from breezetoken_b200.synth import MoeSpec, make_moe_layer, moe_layer_inputs

    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    spec = MoeSpec()
    m = make_moe_layer(spec, seed=3)
    ex = IQ3SExperts.from_gguf_bytes(m["gate"], m["up"], m["down"], spec.n_experts, spec.hidden, spec.ffn, "cuda")
    se = SharedExpert.from_tensors(torch.from_numpy(m["sh_gate"]), torch.from_numpy(m["sh_up"]),
                                   torch.from_numpy(m["sh_down"]), torch.from_numpy(m["sh_gate_inp"]), "cuda")
    xh, lh = moe_layer_inputs(tokens, spec, seed=3 + rank)
    x = torch.from_numpy(xh).cuda()
    r = route_logits(torch.from_numpy(lh).cuda(), spec.top_k)
    ep = ExpertParallelMoE(ex, se)
    ws = torch.zeros(int(N.load().bt_moe_layer_workspace_bytes(tokens, spec.hidden, spec.ffn, spec.ffn,
                                                               spec.n_experts, spec.top_k)),
                     dtype=torch.uint8, device="cuda")
    want = moe_forward(ex, se, x, r.expert_ids, r.weights, ws)
    got = ep(x, r.expert_ids, r.weights)
    err = float((got - want).abs().max() / want.abs().max())
    rows_in, r_ids, r_w = ep.dispatch(x, r.expert_ids, r.weights)
    part = ep.local_experts(rows_in, r_ids, r_w)
    local_u = int(torch.unique(r_ids[r_ids >= 0]).numel())
    flush = torch.ones(256 << 20, dtype=torch.uint8, device="cuda")

    def timed(fn) -> float:
        total = 0.0
        for i in range(iters + 3):
            flush.sum(dtype=torch.int32)  # the experts are not in L2
            dist.barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            b.synchronize()
            if i >= 3:
                total += a.elapsed_time(b) * 1e3
        t = torch.tensor([total / iters], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def captured(fn):
        """fn captured in a CUDA graph (its collectives included), after a
        warm-up call on a side stream; every rank captures the same calls."""
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            fn()
        torch.cuda.current_stream().wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        graphs.append(g)
        return g.replay

    graphs: list = []
    res = {
        "ep_graph_us": timed(captured(lambda: ep(x, r.expert_ids, r.weights))),
        "replicated_graph_us": timed(captured(lambda: moe_forward(ex, se, x, r.expert_ids, r.weights, ws))),
        "ep_us": timed(lambda: ep(x, r.expert_ids, r.weights)),
        "ep_dispatch_us": timed(lambda: ep.dispatch(x, r.expert_ids, r.weights)),
        "ep_local_experts_us": timed(lambda: ep.local_experts(rows_in, r_ids, r_w)),
        "ep_combine_us": timed(lambda: ep.combine(part, x)),
        "replicated_us": timed(lambda: moe_forward(ex, se, x, r.expert_ids, r.weights, ws)),
    }
    errs = torch.tensor([err, float(local_u)], device="cuda")
    dist.all_reduce(errs, op=dist.ReduceOp.MAX)
    dist.barrier()
    torch.cuda.synchronize()
    graphs.clear()  # graphs holding NCCL calls go before the process group
    dist.destroy_process_group()
    if rank != 0:
        return None
    return {"kernel": "moe_expert_parallel", "ranks": world, "tokens_per_rank": tokens,
            "experts_per_rank": ep.per_rank, "max_local_unique_experts": int(errs[1].item()),
            "exchange_bytes_per_rank": (world * tokens * spec.hidden * 4 * 2 + world * tokens * spec.top_k * 8),
            **res, "check_rel_err_vs_replicated": float(errs[0].item()),
            "l2": "256 MB read before each call",
            "timing": "CUDA events per call (eager: host launches included; graph: one replay) after a barrier, "
                      "max over ranks"}


def bench_load(path: str | None) -> dict:
    """Load time of the full 35B-A3B-shaped checkpoint (written once per
    machine by synth.cached_qwen36_full when no path is given): the GGUF
    bytes read and uploaded, against the time the repack kernels take on the
    device (CUDA events around the whole load)."""
    from breezetoken_b200.gguf import GGUFFile
    from breezetoken_b200.qwen36_moe import Qwen36Moe
    from breezetoken_b200.synth import cached_qwen36_full

    path = path or str(cached_qwen36_full())
    nbytes = Path(path).stat().st_size
    t0 = time.perf_counter()
    with open(path, "rb") as f:  # the file into the page cache, timed on its own
        while f.read(1 << 28):
            pass
    read_s = time.perf_counter() - t0
    lib = N.load()
    before = int(lib.bt_launch_count())
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    g = GGUFFile(path)
    m = Qwen36Moe(g, max_context=64, batch=1)
    torch.cuda.synchronize()
    load_s = time.perf_counter() - t0
    launches = int(lib.bt_launch_count()) - before
    g.close()
    m.close()
    return {"kernel": "qwen36_load", "gguf_bytes": nbytes, "file_read_s": read_s,
            "file_read_gbs": nbytes / read_s / 1e9, "load_s": load_s, "load_gbs": nbytes / load_s / 1e9,
            "library_launches": launches,
            "note": "load = open + parse + host->device upload + repack kernels, the file already in the page cache"}


def trace_step(gguf: str, max_context: int, steps: int) -> str:
    """Per-kernel-kind device timeline of a decode step (model.Qwen35.trace_step):
    entered = previous kernel's last CTA exit -> this kernel's last CTA entry
    (negative: resident before the previous kernel ended);
    gap = previous kernel's last CTA exit -> this kernel's last CTA past the
    dependency wait; prologue = -> last CTA ready for its main loop; body =
    -> last CTA exit; loads = -> last CTA with its activation loads back (GEMV)."""
    from breezetoken_b200.model import Qwen35

    m = Qwen35(gguf, max_context=max_context)
    try:
        prompt = np.random.default_rng(0).integers(0, m.cfg.vocab, 16).tolist()
        m.prefill([prompt])
        for _ in range(4):
            m.replay(1)
        m.stream.synchronize()
        tl = m.trace_step(steps=steps)
    finally:
        m.close()
    agg: dict[str, list[float]] = {}
    prev_end = 0.0
    for t in tl:
        kind = t["name"].split(".")[-1]
        a = agg.setdefault(kind, [0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0])
        a[0] += 1
        a[1] += t["released"] - prev_end
        a[2] += t["ready"] - t["released"]
        a[3] += t["end"] - t["ready"]
        a[4] += t["end"] - prev_end
        a[5] += (t["loaded"] - t["released"]) if t.get("loaded") else 0.0
        a[6] += t["entered"] - prev_end
        prev_end = t["end"]
    lines = [f"step: {len(tl)} kernels, {tl[-1]['end']:.1f} us from first entry to last exit",
             f"{'kind':11s} {'n':>3s} {'total us':>9s} {'entered':>8s} {'gap':>6s} {'prologue':>9s} {'(loads)':>8s}"
             f" {'body':>7s}"]
    for k, (n, gap, pro, body, tot, ld, ent) in sorted(agg.items(), key=lambda x: -x[1][4]):
        lines.append(f"{k:11s} {n:3d} {tot:9.1f} {ent / n:8.2f} {gap / n:6.2f} {pro / n:9.2f} {ld / n:8.2f} "
                     f"{body / n:7.2f}")
    return "\n".join(lines)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    sub = ap.add_subparsers(dest="cmd", required=True)
    a = sub.add_parser("gemv")
    a.add_argument("--n", type=int, default=151936)
    a.add_argument("--k", type=int, default=1024)
    a.add_argument("--iters", type=int, default=20)
    b = sub.add_parser("gdn")
    b.add_argument("--batch", type=int, default=1)
    b.add_argument("--steps", type=int, default=256)
    b.add_argument("--scan", action="store_true", help="all steps as one prefill scan (bt_gdn_prefill)")
    c = sub.add_parser("attn")
    c.add_argument("--batch", type=int, default=1)
    c.add_argument("--ctx", type=int, default=8192)
    c.add_argument("--splits", type=int, default=0)
    c.add_argument("--iters", type=int, default=20)
    al = sub.add_parser("attn-layer", help="the fused Qwen3.6 attention layer at the 35B shape")
    al.add_argument("--batch", type=int, default=64)
    al.add_argument("--pos", type=int, default=648)
    al.add_argument("--splits", type=int, default=2)
    al.add_argument("--iters", type=int, default=20)
    sub.add_parser("precision")
    mo = sub.add_parser("moe")
    mo.add_argument("--tokens", type=int, default=1)
    mo.add_argument("--iters", type=int, default=50)
    mo.add_argument("--no-shared", action="store_true", help="routed experts only")
    li = sub.add_parser("linear")
    li.add_argument("--tokens", type=int, default=64)
    li.add_argument("--n", type=int, default=0, help="0: the 35B-A3B decoder's projection shapes")
    li.add_argument("--k", type=int, default=2048)
    li.add_argument("--iters", type=int, default=20)
    q6 = sub.add_parser("qwen36")
    q6.add_argument("--batch", type=int, default=64)
    q6.add_argument("--prompt", type=int, default=512)
    q6.add_argument("--steps", type=int, default=256)
    q6.add_argument("--layers", type=int, default=40)
    q6.add_argument("--timeline", action="store_true", help="per-kernel device times of a few graph replays")
    ep = sub.add_parser("moe-ep", help="under torchrun: the MoE layer expert-parallel over the ranks")
    ep.add_argument("--tokens", type=int, default=8, help="tokens per rank")
    ep.add_argument("--iters", type=int, default=30)
    ld = sub.add_parser("load")
    ld.add_argument("--gguf", default=None, help="default: the cached full-shape checkpoint")
    t = sub.add_parser("trace")
    t.add_argument("--gguf", required=True)
    t.add_argument("--max-context", type=int, default=1024)
    t.add_argument("--steps", type=int, default=3)
    args = ap.parse_args()
    if args.cmd == "trace":
        print(trace_step(args.gguf, args.max_context, args.steps), flush=True)
        return
    if args.cmd == "linear":
        shapes = [(args.n, args.k)] if args.n else [(8192, 2048), (4096, 2048), (2048, 4096), (151936, 2048)]
        for n, k in shapes:
            print(json.dumps(bench_linear(n, k, args.tokens, args.iters)), flush=True)
        return
    if args.cmd == "gemv":
        r = bench_gemv(args.n, args.k, args.iters)
    elif args.cmd == "attn-layer":
        r = bench_attn_layer(args.batch, args.pos, args.splits, args.iters)
    elif args.cmd == "moe-ep":
        r = bench_moe_ep(args.tokens, args.iters)
    elif args.cmd == "load":
        r = bench_load(args.gguf)
    elif args.cmd == "qwen36":
        r = bench_qwen36(args.batch, args.prompt, args.steps, args.layers, args.timeline)
    elif args.cmd == "moe":
        r = bench_moe(args.tokens, args.iters, shared=not args.no_shared)
    elif args.cmd == "precision":
        for line in bench_precision():
            print(json.dumps(line), flush=True)
        r = None
    elif args.cmd == "gdn":
        r = bench_gdn_scan(args.batch, args.steps) if args.scan else bench_gdn(args.batch, args.steps)
    else:
        r = bench_attn(args.batch, args.ctx, args.splits, args.iters)
    if r is not None:
        print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()

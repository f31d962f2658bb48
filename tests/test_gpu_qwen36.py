"""GPU parity of the config-5 (Qwen3.6-35B-A3B-shaped, qwen35moe) decoder.

The tiny checkpoint has the config-5 layer shapes (hidden 2048, GQA 16q/2kv
x 256, GDN 16 key / 32 value heads x 128, IQ3_S experts of ffn 512 + a bf16
shared expert) with 4 layers and 16 experts.  Greedy tokens must be
identical to the reference's Qwen36Moe (CPU, f32) over 24 steps; the first
logits within 1e-4 of the logit scale.  The golden fixture records the top-2
margin of every step.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from breezetoken_b200 import _native as N
from breezetoken_b200.qwen36_moe import Qwen36Moe
from tests.conftest import golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model(cuda, qwen36_tiny_gguf):
    m = Qwen36Moe(qwen36_tiny_gguf, max_context=int(golden("qwen36_tiny")["max_context"]))
    yield m
    m.close()


def test_qwen36_first_logits_match_reference(model) -> None:
    g = golden("qwen36_tiny")
    prompt = g["prompt"].tolist()
    model.reset()
    for i, t in enumerate(prompt):
        logits = model.forward_token(t, i, logits=(i == len(prompt) - 1))
    got, want = logits.cpu().numpy(), g["logits"][0]
    assert np.abs(got - want).max() <= 1e-4 * np.abs(want).max()


def test_qwen36_greedy_tokens_match_reference(model) -> None:
    g = golden("qwen36_tiny")
    got = model.generate(g["prompt"].tolist(), int(g["steps"]))
    want = g["tokens"].tolist()
    first = next((i for i, (a, b) in enumerate(zip(got, want, strict=True)) if a != b), None)
    assert got == want, f"first mismatch at {first} (margins {g['margins'][:8]})"


def test_qwen36_batch_lockstep(cuda, qwen36_tiny_gguf, model) -> None:
    """Four sequences decoded together match each decoded alone."""
    g = golden("qwen36_tiny")
    p0 = g["prompt"].tolist()
    rng = np.random.default_rng(11)
    prompts = [p0] + [rng.integers(0, 8192, len(p0)).tolist() for _ in range(3)]
    solo = [model.generate(p, 6) for p in prompts]
    mb = Qwen36Moe(qwen36_tiny_gguf, max_context=64, batch=4)
    try:
        toks = torch.tensor([p[0] for p in prompts], device="cuda")
        for i in range(1, len(p0)):
            mb._step(toks, i - 1, logits=False)
            toks = torch.tensor([p[i] for p in prompts], device="cuda")
        together = [[] for _ in prompts]
        for step in range(6):
            toks = mb.decode_batch(toks, len(p0) - 1 + step)
            for b, t in enumerate(toks.tolist()):
                together[b].append(t)
    finally:
        mb.close()
    assert together == solo


def test_qwen36_graph_decode_matches_reference(model) -> None:
    """The CUDA-graph decode (device-side token, position and history)
    reproduces the reference's greedy tokens."""
    g = golden("qwen36_tiny")
    prompt = g["prompt"].tolist()
    model.reset()
    for i, t in enumerate(prompt[:-1]):
        model._step(torch.tensor([t], device="cuda"), i, logits=False)
    got = model.graph_decode(torch.tensor([prompt[-1]], device="cuda"), len(prompt) - 1, int(g["steps"]))
    assert got[0].tolist() == g["tokens"].tolist()


@pytest.fixture(scope="module")
def full_gguf(cuda):
    """The full Qwen3.6-35B-A3B-shaped checkpoint of the golden (40 layers,
    256 IQ3_S experts, vocab 151936, seed 4, random-byte experts), ~18 GB,
    written once per machine (the benchmark's CPU arm loads the same file)."""
    from breezetoken_b200.synth import cached_qwen36_full

    return cached_qwen36_full()


def test_qwen36_full_shape_64_sequences_match_reference(full_gguf) -> None:
    """The 35B-A3B decode benchmark's shape and batch: 64 sequences in
    lockstep through the CUDA-graph decode (tcgen05 projections at 64 tokens,
    the 256-expert MoE layers, 40 layers).  Sequences 0 and 1 carry the
    golden prompts: their first logits are within 1e-4 of the logit scale of
    the reference's Qwen36Moe (CPU, f32) and all 8 greedy tokens are
    identical; the other 62 sequences are random prompts."""
    from tests.golden.make_golden import qwen36_full_prompts

    g = golden("qwen36_full")
    prompts = g["prompts"]
    assert (prompts == qwen36_full_prompts()).all()
    B, L = 64, prompts.shape[1]
    steps = g["tokens"].shape[1]
    rng = np.random.default_rng(12)
    allp = np.concatenate([prompts, rng.integers(0, 151936, (B - len(prompts), L))])
    m = Qwen36Moe(full_gguf, max_context=int(g["max_context"]), batch=B)
    try:
        toks = torch.from_numpy(allp).cuda()
        # the prompts' first L - 1 tokens token by token, then as one chunk
        # (the default prefill): the same bits, since no projection's sums
        # depend on how many tokens share the call
        m.reset()
        m.prefill(toks[:, : L - 1], chunk=1)
        by_token = m._step(toks[:, L - 1], L - 1, logits=True)
        m.reset()
        m.prefill(toks[:, : L - 1])
        logits = m._step(toks[:, L - 1], L - 1, logits=True)
        assert torch.equal(logits, by_token)
        for b in range(len(prompts)):
            got = logits[b].cpu().numpy()
            want = g["top_val"][b, 0]
            assert (np.argsort(-got, kind="stable")[:4] == g["top_idx"][b, 0, :4]).all()
            assert np.abs(got[g["top_idx"][b, 0]] - want).max() <= 1e-4 * np.abs(want).max()
        want0 = g["logits"][0]
        assert np.abs(logits[0].cpu().numpy() - want0).max() <= 1e-4 * np.abs(want0).max()
        first = m.backend.argmax(logits).long()
        rest = m.graph_decode(first, L, steps - 1)
        out = torch.cat([first[:, None], rest], 1).cpu().numpy()
    finally:
        m.close()
    for b in range(len(prompts)):
        assert out[b].tolist() == g["tokens"][b].tolist(), f"sequence {b} (margins {g['margins'][b]})"


@pytest.mark.parametrize("n,k,dtype", [(8192, 2048, torch.bfloat16), (2048, 4096, torch.bfloat16),
                                       (256, 2048, torch.float32), (64, 2048, torch.float32)])
def test_linear_rows_sums_do_not_depend_on_token_count(cuda, n, k, dtype) -> None:
    """A token's outputs are the same bits whether it is projected with 8+
    others (bf16, the tensor-core path) or with any number of others (f32):
    the chunked prefill relies on it to reproduce the decode step."""
    rng = np.random.default_rng(19)
    w = torch.from_numpy(rng.standard_normal((n, k), dtype=np.float32) * 0.02).to(dtype).cuda()
    x = torch.from_numpy(rng.standard_normal((448, k), dtype=np.float32)).cuda()
    dt = N.BT_BF16 if dtype == torch.bfloat16 else N.BT_F32

    def lin(xs):
        t = xs.shape[0]
        p = torch.empty(t, 3, k, dtype=torch.bfloat16, device="cuda")
        N.call("bt_bf16_planes", xs.data_ptr(), p.data_ptr(), t, k, 0)
        y = torch.empty(t, n, device="cuda")
        N.call("bt_linear_rows", w.data_ptr(), dt, p.data_ptr(), y.data_ptr(), n, k, t, 0)
        return y

    full = lin(x)
    spans = [(64, 128), (0, 32), (0, 17), (3, 12), (100, 292)] + ([(5, 6), (0, 8)] if dtype == torch.float32 else [])
    for a, b in spans:
        assert torch.equal(lin(x[a:b].contiguous()), full[a:b]), (a, b)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("t", [1, 5, 20, 70])
def test_linear_rows_matches_f64(cuda, dtype, t) -> None:
    """y = x W^T against an f64 product: within 2e-6 of sum |x||w| per output."""
    rng = np.random.default_rng(12)
    n, k = 96, 512
    w = torch.from_numpy(rng.standard_normal((n, k)).astype(np.float32) * 0.02).to(dtype)
    x = torch.from_numpy(rng.standard_normal((t, k)).astype(np.float32))
    y = torch.empty(t, n, device="cuda")
    wd, xd = w.cuda().contiguous(), x.cuda().contiguous()
    planes = torch.empty(t, 3, k, dtype=torch.bfloat16, device="cuda")
    N.call("bt_bf16_planes", xd.data_ptr(), planes.data_ptr(), t, k, 0)
    assert torch.equal(planes.float().sum(1), xd)  # the planes hold x exactly
    N.call("bt_linear_rows", wd.data_ptr(), N.BT_BF16 if dtype == torch.bfloat16 else N.BT_F32, planes.data_ptr(),
           y.data_ptr(), n, k, t, 0)
    wf = w.double().numpy()
    want = x.double().numpy() @ wf.T
    bound = np.abs(x.double().numpy()) @ np.abs(wf).T
    assert (np.abs(y.cpu().double().numpy() - want) <= 2e-6 * bound).all()


@pytest.mark.parametrize("n,k", [(2048, 4096), (4096, 2048)])
def test_linear_rows_small_batch_bf16_split_matches_f64(cuda, n, k) -> None:
    """The 35B out- and z-projections' bf16 rows for <= 8 tokens (the first
    with its K split over a 4-CTA cluster, the second not): within 2e-6 of
    sum |x||w| of an f64 product, and a token's sums the same bits for any
    T <= 8 (the split is chosen from N and K)."""
    rng = np.random.default_rng(21)
    w = torch.from_numpy(rng.standard_normal((n, k)).astype(np.float32) * 0.02).to(torch.bfloat16)
    x = torch.from_numpy(rng.standard_normal((8, k)).astype(np.float32))
    wd, xd = w.cuda().contiguous(), x.cuda().contiguous()

    def lin(xs):
        t = xs.shape[0]
        planes = torch.empty(t, 3, k, dtype=torch.bfloat16, device="cuda")
        N.call("bt_bf16_planes", xs.data_ptr(), planes.data_ptr(), t, k, 0)
        y = torch.empty(t, n, device="cuda")
        N.call("bt_linear_rows", wd.data_ptr(), N.BT_BF16, planes.data_ptr(), y.data_ptr(), n, k, t, 0)
        return y

    full = lin(xd)
    wf = w.double().numpy()
    want = x.double().numpy() @ wf.T
    bound = np.abs(x.double().numpy()) @ np.abs(wf).T
    assert (np.abs(full.cpu().double().numpy() - want) <= 2e-6 * bound).all()
    for a, b in [(0, 1), (0, 5), (3, 8), (7, 8)]:
        assert torch.equal(lin(xd[a:b].contiguous()), full[a:b]), (a, b)


@pytest.mark.parametrize("n,t", [(256, 64), (64, 64), (64, 9), (256, 130)])
def test_linear_rows_f32_cluster_split_matches_f64(cuda, n, t) -> None:
    """f32 weight rows of the router / GDN beta-alpha shapes (K = 2048) for a
    batch: the K range split over a cluster of CTAs whose sums are added in
    rank order: within 2e-6 of sum |x||w| of an f64 product and the same bits
    on a second call."""
    rng = np.random.default_rng(14)
    k = 2048
    w = torch.from_numpy(rng.standard_normal((n, k)).astype(np.float32) * 0.02)
    x = torch.from_numpy(rng.standard_normal((t, k)).astype(np.float32))
    wd, xd = w.cuda().contiguous(), x.cuda().contiguous()
    planes = torch.empty(t, 3, k, dtype=torch.bfloat16, device="cuda")
    N.call("bt_bf16_planes", xd.data_ptr(), planes.data_ptr(), t, k, 0)
    ys = []
    for _ in range(2):
        y = torch.full((t, n), float("nan"), device="cuda")
        N.call("bt_linear_rows", wd.data_ptr(), N.BT_F32, planes.data_ptr(), y.data_ptr(), n, k, t, 0)
        ys.append(y)
    want = x.double().numpy() @ w.double().numpy().T
    bound = np.abs(x.double().numpy()) @ np.abs(w.double().numpy()).T
    got = ys[0].cpu().double().numpy()
    assert np.isfinite(got).all()
    assert (np.abs(got - want) <= 2e-6 * bound).all()
    assert torch.equal(ys[0], ys[1])


@pytest.mark.parametrize("t", [9, 16, 17, 32, 33, 64, 130])
@pytest.mark.parametrize("n,k", [(64, 256), (192, 2048), (128, 256), (256, 2048), (512, 4096)])
def test_linear_rows_tiled_matches_f64(cuda, t, n, k) -> None:
    """The tiled paths for bf16 weights and > 8 tokens (N % 128 == 0: tcgen05
    MMAs with TMEM accumulators; else N % 64 == 0: ldmatrix-fed MMAs), K split
    over 1 to 8 CTAs of a cluster: y = x W^T within 2e-6 of sum |x||w| per
    output, ragged token counts included, the same bits on a second call (the
    splits are added in a fixed order), and no bounded wait gave up."""
    rng = np.random.default_rng(13)
    w = torch.from_numpy(rng.standard_normal((n, k)).astype(np.float32) * 0.02).to(torch.bfloat16)
    x = torch.from_numpy(rng.standard_normal((t, k)).astype(np.float32))
    wd, xd = w.cuda().contiguous(), x.cuda().contiguous()
    planes = torch.empty(t, 3, k, dtype=torch.bfloat16, device="cuda")
    N.call("bt_bf16_planes", xd.data_ptr(), planes.data_ptr(), t, k, 0)
    y = torch.full((t, n), float("nan"), device="cuda")
    N.call("bt_linear_rows", wd.data_ptr(), N.BT_BF16, planes.data_ptr(), y.data_ptr(), n, k, t, 0)
    y2 = torch.empty_like(y)
    N.call("bt_linear_rows", wd.data_ptr(), N.BT_BF16, planes.data_ptr(), y2.data_ptr(), n, k, t, 0)
    wf = w.double().numpy()
    want = x.double().numpy() @ wf.T
    bound = np.abs(x.double().numpy()) @ np.abs(wf).T
    got = y.cpu().double().numpy()
    assert N.load().bt_linear_rows_timeouts() == 0
    assert np.isfinite(got).all()
    assert (np.abs(got - want) <= 2e-6 * bound).all()
    assert torch.equal(y, y2)


def test_linear_rows_rejects_bad_shapes(cuda) -> None:
    buf = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    p = buf.data_ptr()
    assert N.load().bt_linear_rows(p, N.BT_BF16, p, p, 24, 512, 1, 0) == N.BT_ERR_UNSUPPORTED
    assert N.load().bt_linear_rows(p, N.BT_BF16, p, p, 32, 500, 1, 0) == N.BT_ERR_UNSUPPORTED


def test_sequence_shards_decode_the_same_bits(cuda) -> None:
    """Sharding the benchmark's 64 sequences over two GPUs (32 per GPU, the
    planner's split) changes nothing in any sequence's arithmetic: a model
    of the 35B-A3B layer shapes (4 layers, 256 experts, seeded random
    weights) decoding sequences 0..31 alone and 32..63 alone reproduces the
    bits of decoding all 64 together -- logits after a chunked prefill and 4
    greedy steps (64 and 32 tokens take the same projection and MoE paths,
    whose per-token sums do not depend on the other tokens)."""
    from dataclasses import replace

    from breezetoken_b200.synth import QWEN36_35B

    spec = replace(QWEN36_35B, n_layers=4)
    rng = np.random.default_rng(61)
    prompts = torch.from_numpy(rng.integers(0, spec.vocab, (64, 9))).cuda()

    def run(rows: slice):
        m = Qwen36Moe.random(spec, batch=rows.stop - rows.start, max_context=16, seed=4)
        try:
            p = prompts[rows]
            m.prefill(p[:, :8])
            logits = m._step(p[:, 8], 8, logits=True)
            toks = [m.backend.argmax(logits).long()]
            for s in range(3):
                toks.append(m.decode_batch(toks[-1], 9 + s).long())
            m.check_pipeline()
            return logits.clone(), torch.stack(toks, 1)
        finally:
            m.close()

    l_all, t_all = run(slice(0, 64))
    for rows in (slice(0, 32), slice(32, 64)):
        l_s, t_s = run(rows)
        assert torch.equal(l_s, l_all[rows])
        assert torch.equal(t_s, t_all[rows])


def test_uploader_moves_the_bytes_unchanged(cuda, tmp_path) -> None:
    """The checkpoint uploader (pinned double buffering, host copies split over
    threads) delivers every byte: empty, small and multi-chunk arrays, a
    read-only memory map and a non-byte dtype, with chunks smaller than the
    arrays so both buffers are reused several times."""
    from breezetoken_b200.upload import Uploader

    rng = np.random.default_rng(61)
    up = Uploader("cuda", chunk_bytes=8 << 20, threads=4)
    try:
        for n in (0, 1000, (8 << 20) + 3, (20 << 20) + 7):
            src = rng.integers(0, 256, n, dtype=np.uint8)
            got = up.to_device(src)
            assert got.dtype == torch.uint8 and got.numel() == n
            assert torch.equal(got.cpu(), torch.from_numpy(src))
        path = tmp_path / "blob.bin"
        blob = rng.integers(0, 256, (17 << 20) + 11, dtype=np.uint8)
        blob.tofile(path)
        mm = np.memmap(path, dtype=np.uint8, mode="r")
        assert torch.equal(up.to_device(mm[5:]).cpu(), torch.from_numpy(blob[5:]))
        f = rng.standard_normal(3 << 20).astype(np.float32)
        assert torch.equal(up.to_device(f).view(torch.float32).cpu(), torch.from_numpy(f))
    finally:
        up.close()

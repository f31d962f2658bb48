"""GPU parity of the prefill scans: the GDN recurrence, the config-5 gated
GDN mixer and the short conv over many tokens per launch, and the chunked
batched prefill of the config-5 decoder.

The reference runs the recurrence of a prompt token by token
(model/prefill.py:106-110, model/qwen36_moe.py:520-530).  The scans run the
same per-token arithmetic with the state on chip between tokens, so:

* bt_gdn_prefill over the config-2 benchmark's 256 steps matches the oracle
  (relative 1e-4, as the stepwise config-2 test) and, where the stepwise op
  takes the one-CTA-per-head kernel (64 sequences x 16 heads), gives the
  same bits as 256 bt_gdn_decode calls;
* bt_gdn_gated_scan and bt_conv_silu_scan give the same bits as one
  bt_gdn_gated_step / bt_conv_silu call per token;
* a chunked prefill of the 4-layer config-5-shaped model reaches the same
  greedy tokens as a token-by-token one, with logits within 1e-4 of scale
  (4 sequences: the token-by-token steps project 4 tokens on the CUDA cores,
  the chunks 80 on the tensor cores; with more than 8 sequences both take
  the tensor cores and the full-shape test in test_gpu_qwen36.py finds the
  same bits).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from breezetoken_b200 import _native as N
from breezetoken_b200.backends import make_backend
from breezetoken_b200.qwen36_moe import Qwen36Moe
from oracle import ops
from tests.conftest import golden

pytestmark = pytest.mark.gpu


def _config2_inputs(batch: int, steps: int):
    """The config-2 op benchmark's inputs (16 heads x 128, seed 1), drawn in
    the stepwise test's order: (steps, batch, ...) arrays."""
    rng = np.random.default_rng(1)
    H, D = 16, 128
    qs, ks, vs, gs, bs = [], [], [], [], []
    for _ in range(steps):
        q = rng.standard_normal((batch, H, D), dtype=np.float32)
        k = rng.standard_normal((batch, H, D), dtype=np.float32)
        q /= np.linalg.norm(q, axis=-1, keepdims=True)
        k /= np.linalg.norm(k, axis=-1, keepdims=True)
        v = rng.standard_normal((batch, H, D), dtype=np.float32)
        beta = rng.standard_normal((batch, H), dtype=np.float32)
        g = -ops.softplus(rng.standard_normal((batch, H), dtype=np.float32))
        qs.append(q), ks.append(k), vs.append(v), gs.append(g), bs.append(beta)
    return tuple(np.stack(a) for a in (qs, ks, vs, gs, bs))


def _prefill(q, k, v, g, beta, state, out, steps, batch, heads_k, heads_v, dim, dtype, scale=1.0, eps=1e-6):
    """bt_gdn_prefill on token-major contiguous (steps, batch, heads, dim) operands."""
    nk, nv = heads_k * dim, heads_v * dim
    N.call("bt_gdn_prefill", q.data_ptr(), k.data_ptr(), v.data_ptr(), dtype, nk, nk, nv, batch * nk, batch * nk,
           batch * nv, g.data_ptr(), heads_v, batch * heads_v, beta.data_ptr(), heads_v, batch * heads_v,
           state.data_ptr(), out.data_ptr(), nv, batch * nv, steps, batch, heads_k, heads_v, dim, scale, eps, 0)


@pytest.mark.parametrize("batch", [1, 8, 64])
def test_gdn_prefill_config2_256_steps_in_one_launch(cuda, batch) -> None:
    steps, H, D = 256, 16, 128
    q, k, v, g, beta = _config2_inputs(batch, steps)
    qb, kb, vb = (torch.from_numpy(a).to(torch.bfloat16).cuda() for a in (q, k, v))
    gd, bd = torch.from_numpy(g).cuda(), torch.from_numpy(beta).cuda()
    state = torch.zeros(batch, H, D, D, device="cuda")
    out = torch.empty(steps, batch, H, D, device="cuda")
    _prefill(qb, kb, vb, gd, bd, state, out, steps, batch, H, H, D, N.BT_BF16)
    o = out.cpu().numpy()
    # the oracle, step by step on the same bf16-rounded inputs
    qf, kf, vf = (t.float().cpu().numpy() for t in (qb, kb, vb))
    ref_state = np.zeros((batch, H, D, D), np.float32)
    worst = 0.0
    for s in range(steps):
        for b in range(batch):
            ro = ops.gdn_decode(qf[s, b], kf[s, b], vf[s, b], g[s, b], beta[s, b], ref_state[b], 1.0, 1e-6)
            worst = max(worst, float(np.abs(o[s, b] - ro).max() / (np.abs(ro).max() + 1e-6)))
    assert worst < 1e-4, worst
    np.testing.assert_allclose(state.cpu().numpy(), ref_state, rtol=1e-4, atol=1e-4)
    if batch == 64:
        # 64 x 16 heads take the stepwise op's one-CTA-per-head kernel: same bits
        s2 = torch.zeros_like(state)
        o2 = torch.empty_like(out)
        for s in range(steps):
            N.call("bt_gdn_decode", qb[s].data_ptr(), kb[s].data_ptr(), vb[s].data_ptr(), N.BT_BF16,
                   gd[s].data_ptr(), bd[s].data_ptr(), s2.data_ptr(), o2[s].data_ptr(), batch, H, H, D, 1.0, 1e-6, 0)
        assert torch.equal(o2, out)
        assert torch.equal(s2, state)


def test_gdn_prefill_chunks_strides_and_gqa(cuda) -> None:
    """A scan split into chunks (17 + 23 tokens, and an empty one) gives the
    bits of one 40-token scan; the operands are strided views of packed
    token-major rows (q | k | v of the conv output, beta | alpha), with 32
    value heads over 16 key heads; the output's row padding is not written."""
    rng = np.random.default_rng(41)
    S, B, HK, HV, D = 40, 24, 16, 32, 128
    c = 2 * HK * D + HV * D
    mixed = torch.from_numpy(rng.standard_normal((S, B, c), dtype=np.float32) * 0.3).cuda()
    ba = torch.from_numpy(rng.standard_normal((S, B, 2 * HV), dtype=np.float32)).cuda()
    g = -torch.nn.functional.softplus(torch.from_numpy(rng.standard_normal((S, B, HV), dtype=np.float32))).cuda()
    s0 = torch.from_numpy(rng.standard_normal((B, HV, D, D), dtype=np.float32) * 0.1).cuda()
    pad = HV * D + 32

    def run(state, out, t0, t1):
        m, b_, g_, o_ = mixed[t0:], ba[t0:], g[t0:], out[t0:]
        N.call("bt_gdn_prefill", m.data_ptr(), m[..., HK * D:].data_ptr(), m[..., 2 * HK * D:].data_ptr(), N.BT_F32,
               c, c, c, B * c, B * c, B * c, g_.data_ptr(), HV, B * HV, b_.data_ptr(), 2 * HV, B * 2 * HV,
               state.data_ptr(), o_.data_ptr(), pad, B * pad, t1 - t0, B, HK, HV, D, float(D ** -0.5), 1e-6, 0)

    s1, s2 = s0.clone(), s0.clone()
    o1 = torch.full((S, B, pad), float("nan"), device="cuda")
    o2 = torch.full((S, B, pad), float("nan"), device="cuda")
    run(s1, o1, 0, S)
    run(s2, o2, 0, 17)
    run(s2, o2, 17, 17)  # steps == 0: no-op
    run(s2, o2, 17, S)
    assert torch.equal(torch.nan_to_num(o1, 7.0), torch.nan_to_num(o2, 7.0))
    assert torch.equal(s1, s2)
    assert torch.isnan(o1[..., HV * D:]).all()
    # against the oracle for two sequences
    mm, bb, gg = mixed.cpu().numpy(), ba.cpu().numpy(), g.cpu().numpy()
    for b in (0, B - 1):
        st = s0[b].cpu().numpy().copy()
        for s in range(S):
            q = mm[s, b, : HK * D].reshape(HK, D)
            k = mm[s, b, HK * D : 2 * HK * D].reshape(HK, D)
            v = mm[s, b, 2 * HK * D :].reshape(HV, D)
            ro = ops.gdn_decode(q, k, v, gg[s, b], bb[s, b, :HV], st, float(D ** -0.5), 1e-6)
            np.testing.assert_allclose(o1[s, b, : HV * D].cpu().numpy(), ro.reshape(-1), rtol=1e-4, atol=1e-5)
        np.testing.assert_allclose(s1[b].cpu().numpy(), st, rtol=1e-4, atol=1e-5)


def test_gdn_prefill_rejects_other_head_dims(cuda) -> None:
    x = torch.zeros(4, 64, device="cuda")
    with pytest.raises(N.B200Error):
        N.call("bt_gdn_prefill", x.data_ptr(), x.data_ptr(), x.data_ptr(), N.BT_F32, 64, 64, 64, 64, 64, 64,
               x.data_ptr(), 1, 1, x.data_ptr(), 1, 1, x.data_ptr(), x.data_ptr(), 64, 64, 2, 1, 1, 1, 64, 1.0,
               1e-6, 0)


def test_backend_gdn_prefill_equals_decode_loop(cuda) -> None:
    """B200Backend.gdn_prefill is the reference's prefill loop over
    Backend.gdn_decode (model/prefill.py:106-110) in one call."""
    be = make_backend("b200", "cuda")
    rng = np.random.default_rng(43)
    S, H, D = 33, 16, 128
    q = torch.from_numpy(rng.standard_normal((S, H, D), dtype=np.float32)).cuda()
    k = torch.from_numpy(rng.standard_normal((S, H, D), dtype=np.float32)).cuda()
    v = torch.from_numpy(rng.standard_normal((S, H, D), dtype=np.float32)).cuda()
    g = -torch.nn.functional.softplus(torch.from_numpy(rng.standard_normal((S, H), dtype=np.float32))).cuda()
    beta = torch.from_numpy(rng.standard_normal((S, H), dtype=np.float32)).cuda()
    s1 = torch.zeros(H, D, D, device="cuda")
    s2 = torch.zeros(H, D, D, device="cuda")
    got = be.gdn_prefill(q, k, v, g, beta, s1, D ** -0.5, 1e-6)
    want = torch.stack([be.gdn_decode(q[t], k[t], v[t], g[t], beta[t], s2, D ** -0.5, 1e-6) for t in range(S)])
    torch.testing.assert_close(got, want, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(s1, s2, rtol=1e-4, atol=1e-5)
    with pytest.raises(ValueError):
        be.gdn_prefill(q, k, v[:, :5], g, beta, s1, 1.0)


def test_gdn_gated_scan_and_conv_scan_equal_steps(cuda) -> None:
    """The config-5 GDN mixer (16 key / 32 value heads x 128) over a 5-token
    chunk of 8 sequences: the same bits as five single-token launches."""
    rng = np.random.default_rng(47)
    S, B, HK, HV, D, taps = 5, 8, 16, 32, 128, 4
    c, inner = 2 * HK * D + HV * D, HV * D
    entry = torch.from_numpy(rng.standard_normal((S * B, c), dtype=np.float32) * 0.5).cuda()
    conv_w = torch.from_numpy(rng.standard_normal((c, taps), dtype=np.float32) * 0.25).cuda()
    cs0 = torch.from_numpy(rng.standard_normal((B, c, taps - 1), dtype=np.float32)).cuda()
    ba = torch.from_numpy(rng.standard_normal((S * B, 2 * HV), dtype=np.float32)).cuda()
    z = torch.from_numpy(rng.standard_normal((S * B, inner), dtype=np.float32)).cuda()
    a_log = -torch.exp(torch.from_numpy(rng.uniform(0, np.log(16.0), HV).astype(np.float32))).cuda()
    dt_bias = torch.from_numpy(rng.standard_normal(HV, dtype=np.float32) * 0.5).cuda()
    norm_w = torch.from_numpy(1 + rng.standard_normal(D, dtype=np.float32) * 0.02).cuda()
    st0 = torch.from_numpy(rng.standard_normal((B, HV, D, D), dtype=np.float32) * 0.1).cuda()

    def mixer(steps, rows, conv_state, state):
        mixed = torch.empty(steps * B, c, device="cuda")
        planes = torch.empty(steps * B, 3, inner, dtype=torch.bfloat16, device="cuda")
        e, b_, z_ = entry[rows:], ba[rows:], z[rows:]
        if steps == 1:
            N.call("bt_conv_silu", e.data_ptr(), conv_state.data_ptr(), conv_w.data_ptr(), mixed.data_ptr(), B, c,
                   taps, 0)
            N.call("bt_gdn_gated_step", mixed.data_ptr(), c, b_.data_ptr(), 2 * HV, a_log.data_ptr(),
                   dt_bias.data_ptr(), state.data_ptr(), z_.data_ptr(), inner, norm_w.data_ptr(), planes.data_ptr(),
                   B, HK, HV, D, float(D ** -0.5), 1e-6, 1e-6, 0)
        else:
            N.call("bt_conv_silu_scan", e.data_ptr(), conv_state.data_ptr(), conv_w.data_ptr(), mixed.data_ptr(),
                   steps, B, c, taps, 0)
            N.call("bt_gdn_gated_scan", mixed.data_ptr(), c, b_.data_ptr(), 2 * HV, a_log.data_ptr(),
                   dt_bias.data_ptr(), state.data_ptr(), z_.data_ptr(), inner, norm_w.data_ptr(), planes.data_ptr(),
                   steps, B, HK, HV, D, float(D ** -0.5), 1e-6, 1e-6, 0)
        return mixed, planes

    cs1, st1 = cs0.clone(), st0.clone()
    m1, p1 = mixer(S, 0, cs1, st1)
    cs2, st2 = cs0.clone(), st0.clone()
    parts = [mixer(1, s * B, cs2, st2) for s in range(S)]
    assert torch.equal(m1, torch.cat([m for m, _ in parts]))
    assert torch.equal(p1, torch.cat([p for _, p in parts]))
    assert torch.equal(cs1, cs2)
    assert torch.equal(st1, st2)


def test_qwen36_chunked_prefill_matches_token_by_token(cuda, qwen36_tiny_gguf) -> None:
    """Four sequences of a 21-token prompt: a chunked prefill (the default
    single chunk, and chunks of 6 with a ragged last one) leaves the model
    where a token-by-token prefill does: the next logits within 1e-4 of
    their scale and the same 8 greedy tokens.  Sequence 0 carries the
    golden prompt's first tokens."""
    g = golden("qwen36_tiny")
    rng = np.random.default_rng(53)
    B, L = 4, 21
    prompts = rng.integers(0, 8192, (B, L))
    prompts[0, : len(g["prompt"])] = g["prompt"]
    toks = torch.from_numpy(prompts).cuda()
    m = Qwen36Moe(qwen36_tiny_gguf, max_context=64, batch=B)
    try:
        results = []
        for chunk in (1, None, 6):
            m.reset()
            m.prefill(toks[:, : L - 1], chunk=chunk)
            logits = m._step(toks[:, L - 1], L - 1, logits=True)
            first = m.backend.argmax(logits).long()
            rest = [first]
            for s in range(7):
                rest.append(m.decode_batch(rest[-1], L + s).long())
            results.append((logits.cpu().numpy(), torch.stack(rest, 1).cpu().numpy()))
        m.check_pipeline()
    finally:
        m.close()
    base_logits, base_toks = results[0]
    for logits, tokens in results[1:]:
        assert np.abs(logits - base_logits).max() <= 1e-4 * np.abs(base_logits).max()
        assert (tokens == base_toks).all()

"""GPU parity of every stand-alone op, through the C ABI, against the oracle
and the reference's golden vectors.

Tolerances: integer/byte work (dequantisation, repacking, argmax) is
bit-exact; f32 arithmetic is compared at rel <= 1e-5 (the reference's own
kernel tests use atol 1e-5 for GDN/RoPE/norms, tests/test_cuda.py), with
GEMV sums bounded by 1e-5 * sum|x||w| (order-dependent f32 accumulation).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from breezetoken_b200 import _native as N
from breezetoken_b200.backends import Q8Weight, make_backend
from breezetoken_b200.quant import quantize_iq3_s, quantize_q8_0
from oracle import ops
from oracle.dequant import dequant_iq3_s, dequant_q8_0
from tests.conftest import golden
from tests.golden.make_golden import STATE_SAMPLE, ops_inputs

pytestmark = pytest.mark.gpu


def _t(a, dev="cuda"):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _gemv_bound(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    return 1e-5 * (np.abs(x)[None, :] @ np.abs(w).T).reshape(-1) + 1e-6


@pytest.fixture(scope="module")
def be(cuda):
    return make_backend("b200", "cuda")


def test_dequant_bit_exact(be) -> None:
    g = golden("dequant")
    out = torch.empty(64, 256, device="cuda")
    raw_d = _t(g["iq3s_raw"])  # keep device inputs alive until the kernel ran
    N.call("bt_dequant_iq3_s", raw_d.data_ptr(), out.data_ptr(), 64, 256, 0)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), g["iq3s_out"].view(np.uint32))
    w = Q8Weight.from_gguf(g["q8_raw"], 64, 32, "cuda")
    assert np.array_equal(w.dequantize().cpu().numpy().view(np.uint32), g["q8_out"].view(np.uint32))
    # larger random IQ3_S tensor vs the oracle decoder
    rng = np.random.default_rng(11)
    raw = quantize_iq3_s(rng.standard_normal((96, 1024)).astype(np.float32))
    out = torch.empty(96, 1024, device="cuda")
    raw_d = _t(raw)
    N.call("bt_dequant_iq3_s", raw_d.data_ptr(), out.data_ptr(), 96, 1024, 0)
    assert np.array_equal(out.cpu().numpy(), dequant_iq3_s(raw.reshape(-1), 96, 1024))


@pytest.mark.parametrize("n,k", [(4, 32), (37, 1024), (6144, 1024), (1024, 3584), (1024, 2048), (16, 1024), (8224, 1024)])
def test_linear_q8_matches_oracle(be, n, k) -> None:
    rng = np.random.default_rng(n * 7 + k)
    wf = rng.standard_normal((n, k)).astype(np.float32) * 0.02
    raw = quantize_q8_0(wf)
    deq = dequant_q8_0(raw, n, k)
    w = Q8Weight.from_gguf(raw, n, k, "cuda")
    assert np.array_equal(w.dequantize().cpu().numpy(), deq)  # repack is lossless
    x = rng.standard_normal(k).astype(np.float32)
    y = be.linear(_t(x), w).cpu().numpy()
    ref = ops.linear(x, deq.T)
    assert np.all(np.abs(y - ref) <= _gemv_bound(x, deq))


@pytest.mark.parametrize("n,k", [(151936, 1024), (40000, 2048), (9000, 3584)])
def test_linear_q8_ring_refill(be, n, k) -> None:
    """Row counts far above what one CTA's shared-memory ring holds, so every
    consumer warp cycles its stages many times (the lm-head shape first)."""
    rng = np.random.default_rng(k)
    raw = quantize_q8_0(rng.standard_normal((n, k)).astype(np.float32) * 0.02)
    deq = dequant_q8_0(raw, n, k)
    w = Q8Weight.from_gguf(raw, n, k, "cuda")
    x = rng.standard_normal(k).astype(np.float32)
    xd = _t(x)
    for _ in range(3):
        y = be.linear(xd, w).cpu().numpy()
        assert np.all(np.abs(y - deq @ x) <= _gemv_bound(x, deq))


@pytest.mark.parametrize("nv", [2, 4, 8])
def test_linear_q8_multi_vector(be, nv) -> None:
    rng = np.random.default_rng(nv)
    n, k = 3000, 1024
    raw = quantize_q8_0(rng.standard_normal((n, k)).astype(np.float32) * 0.02)
    deq = dequant_q8_0(raw, n, k)
    w = Q8Weight.from_gguf(raw, n, k, "cuda")
    x = rng.standard_normal((nv, k)).astype(np.float32)
    y = be.linear_batch(_t(x), w).cpu().numpy()
    for i in range(nv):
        assert np.all(np.abs(y[i] - x[i] @ deq.T) <= _gemv_bound(x[i], deq))


def test_linear_dense_kn(be) -> None:
    """Backend.linear with the reference's dense (K, N) weights (tests/test_cuda.py:22-33)."""
    torch.manual_seed(0)
    x = torch.randn(1024, device="cuda")
    for dt in (torch.bfloat16, torch.float32):
        w = torch.randn(1024, 1000, device="cuda", dtype=dt)
        got = be.linear(x, w)
        ref = x.double() @ w.double()
        assert (got.double() - ref).abs().max().item() < 1e-5 * ref.abs().max().item() + 1e-4


def test_norms_silu_rope_match_reference(be) -> None:
    g, inp = golden("ops"), ops_inputs()
    y = be.rms_norm(_t(inp["norm_x"]), _t(inp["norm_gamma"]), 1e-6).cpu().numpy()
    np.testing.assert_allclose(y, g["norm_out"], rtol=1e-5, atol=1e-5)
    h, xn = be.fused_add_rms_norm(_t(inp["norm_x"]), _t(inp["norm_other"]), _t(inp["norm_gamma"]), 1e-6)
    np.testing.assert_array_equal(h.cpu().numpy(), g["fused_h"])
    np.testing.assert_allclose(xn.cpu().numpy(), g["fused_xn"], rtol=1e-5, atol=1e-5)
    s = be.silu_mul(_t(inp["silu_gate"]), _t(inp["silu_up"])).cpu().numpy()
    np.testing.assert_allclose(s, g["silu_out"], rtol=1e-5, atol=1e-6)
    r = be.rope(_t(inp["rope_x"]), _t(inp["rope_cos"]), _t(inp["rope_sin"]), _t(inp["rope_pos"]), 64).cpu().numpy()
    np.testing.assert_allclose(r, g["rope_out"], rtol=1e-5, atol=1e-5)


def test_gdn_decode_matches_reference(be) -> None:
    g, inp = golden("ops"), ops_inputs()
    for name in ("gdn16", "gdn8_16", "gdn16_32"):
        state = _t(inp[f"{name}_state0"])
        o = be.gdn_decode(
            _t(inp[f"{name}_q"]), _t(inp[f"{name}_k"]), _t(inp[f"{name}_v"]), _t(inp[f"{name}_g"]),
            _t(inp[f"{name}_beta"]), state, 128**-0.5,
        )
        np.testing.assert_allclose(o.cpu().numpy(), g[f"{name}_out"], rtol=1e-5, atol=1e-5)
        st = state.cpu().numpy()
        np.testing.assert_allclose(st.reshape(-1)[::STATE_SAMPLE], g[f"{name}_state1_sample"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("batch", [1, 8, 64])
def test_gdn_decode_config2_256_steps(be, batch) -> None:
    """The GDN op benchmark: 16 heads x 128, bf16 q/k/v, 256 steps, seed 1, vs the oracle."""
    steps = 256
    rng = np.random.default_rng(1)
    H, D = 16, 128
    state = torch.zeros(batch, H, D, D, device="cuda")
    ref_state = np.zeros((batch, H, D, D), np.float32)
    worst = 0.0
    for _ in range(steps):
        q = rng.standard_normal((batch, H, D), dtype=np.float32)
        k = rng.standard_normal((batch, H, D), dtype=np.float32)
        q /= np.linalg.norm(q, axis=-1, keepdims=True)
        k /= np.linalg.norm(k, axis=-1, keepdims=True)
        v = rng.standard_normal((batch, H, D), dtype=np.float32)
        beta = rng.standard_normal((batch, H), dtype=np.float32)
        g = -ops.softplus(rng.standard_normal((batch, H), dtype=np.float32))
        qb, kb, vb = (torch.from_numpy(a).to(torch.bfloat16) for a in (q, k, v))
        out = torch.empty(batch, H, D, device="cuda")
        # device copies held in locals: they must outlive the asynchronous kernel
        qd, kd, vd, gd, bd = qb.cuda(), kb.cuda(), vb.cuda(), _t(g), _t(beta)
        N.call(
            "bt_gdn_decode", qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), N.BT_BF16,
            gd.data_ptr(), bd.data_ptr(), state.data_ptr(), out.data_ptr(), batch, H, H, D,
            1.0, 1e-6, 0,
        )
        o = out.cpu().numpy()
        for b in range(batch):
            ro = ops.gdn_decode(qb[b].float().numpy(), kb[b].float().numpy(), vb[b].float().numpy(), g[b], beta[b],
                                ref_state[b], 1.0, 1e-6)
            worst = max(worst, float(np.abs(o[b] - ro).max() / (np.abs(ro).max() + 1e-6)))
    assert worst < 1e-4, worst
    np.testing.assert_allclose(state.cpu().numpy(), ref_state, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("B", [5, 40])
def test_gdn_decode_strided_views_equal_contiguous(cuda, B) -> None:
    """bt_gdn_decode_strided on views of one packed row per sequence (q | k |
    v as the conv output holds them, beta | alpha as one projection, out with
    padding) gives the same bits as bt_gdn_decode on contiguous copies, with
    the GQA head mapping (32 value heads over 16 key heads); 40 sequences
    take the one-CTA-per-head kernel, checked against the oracle as well."""
    rng = np.random.default_rng(31)
    HK, HV, D = 16, 32, 128
    c = 2 * HK * D + HV * D
    mixed = torch.from_numpy(rng.standard_normal((B, c), dtype=np.float32) * 0.3).cuda()
    ba = torch.from_numpy(rng.standard_normal((B, 2 * HV), dtype=np.float32)).cuda()
    g = -torch.nn.functional.softplus(torch.from_numpy(rng.standard_normal((B, HV), dtype=np.float32))).cuda()
    q, k, v = mixed[:, : HK * D], mixed[:, HK * D : 2 * HK * D], mixed[:, 2 * HK * D :]
    beta = ba[:, :HV]
    s0 = torch.from_numpy(rng.standard_normal((B, HV, D, D), dtype=np.float32) * 0.1).cuda()
    s1, s2 = s0.clone(), s0.clone()
    o1 = torch.empty(B, HV, D, device="cuda")
    o2 = torch.full((B, HV * D + 64), float("nan"), device="cuda")
    qc, kc, vc, bc = q.contiguous(), k.contiguous(), v.contiguous(), beta.contiguous()
    N.call("bt_gdn_decode", qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), N.BT_F32, g.data_ptr(), bc.data_ptr(),
           s1.data_ptr(), o1.data_ptr(), B, HK, HV, D, float(D ** -0.5), 1e-6, 0)
    N.call("bt_gdn_decode_strided", q.data_ptr(), k.data_ptr(), v.data_ptr(), N.BT_F32, c, c, c, g.data_ptr(), HV,
           beta.data_ptr(), 2 * HV, s2.data_ptr(), o2.data_ptr(), HV * D + 64, B, HK, HV, D, float(D ** -0.5), 1e-6,
           0)
    assert torch.equal(o2[:, : HV * D].reshape(B, HV, D), o1)
    assert torch.isnan(o2[:, HV * D :]).all()  # the padding is not written
    assert torch.equal(s2, s1)
    ref_state = s0.cpu().numpy().copy()
    for b in range(B):
        ro = ops.gdn_decode(q[b].reshape(HK, D).cpu().numpy(), k[b].reshape(HK, D).cpu().numpy(),
                            v[b].reshape(HV, D).cpu().numpy(), g[b].cpu().numpy(), beta[b].cpu().numpy(),
                            ref_state[b], float(D ** -0.5), 1e-6)
        np.testing.assert_allclose(o1[b].cpu().numpy(), ro, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(s1.cpu().numpy(), ref_state, rtol=1e-4, atol=1e-5)
    assert N.load().bt_gdn_decode_strided(q.data_ptr(), k.data_ptr(), v.data_ptr(), N.BT_F32, HK * D - 1, c, c,
                                          g.data_ptr(), HV, beta.data_ptr(), 2 * HV, s2.data_ptr(), o2.data_ptr(),
                                          HV * D, B, HK, HV, D, 1.0, 1e-6, None) == N.BT_ERR_INVALID


def test_attention_matches_reference(be) -> None:
    g, inp = golden("ops"), ops_inputs()
    for seq in (1, 17, 128):
        o = be.attention(_t(inp[f"attn{seq}_q"]), _t(inp[f"attn{seq}_k"]), _t(inp[f"attn{seq}_v"]), 256**-0.5)
        np.testing.assert_allclose(o.cpu().numpy(), g[f"attn{seq}_out"], rtol=1e-5, atol=2e-6)


@pytest.mark.parametrize(
    "batch,ctx,splits",
    # (splits > 16 merge in two levels: groups of 16 splits, the last group ragged for 40)
    [(1, 1024, 8), (16, 1024, 4), (4, 8192, 16), (2, 32768, 64), (1, 8192, 40), (3, 777, 5)],
)
def test_attention_config3_bf16(be, batch, ctx, splits) -> None:
    """The flash-decode benchmark shapes: 8q/2kv x 256, bf16 KV N(0,1), scale 1/16, vs the f32 oracle."""
    rng = np.random.default_rng(2)
    q = rng.standard_normal((batch, 8, 256), dtype=np.float32)
    k = torch.from_numpy(rng.standard_normal((batch, ctx, 2, 256), dtype=np.float32)).to(torch.bfloat16)
    v = torch.from_numpy(rng.standard_normal((batch, ctx, 2, 256), dtype=np.float32)).to(torch.bfloat16)
    lens = np.full(batch, ctx, dtype=np.int32)
    lens[-1] = max(1, ctx - 3)  # ragged last sequence
    out = torch.empty(batch, 8, 256, device="cuda")
    ws = torch.zeros(int(N.load().bt_attention_workspace_bytes(batch, 2, 8, 256, splits)), dtype=torch.uint8,
                     device="cuda")
    kc, vc, qd, ld = k.cuda(), v.cuda(), _t(q), _t(lens)  # alive until the kernels ran
    for _ in range(2):  # second call checks the workspace is re-armed
        N.call(
            "bt_attention_decode", qd.data_ptr(), kc.data_ptr(), vc.data_ptr(), N.BT_BF16, ld.data_ptr(),
            out.data_ptr(), batch, 8, 2, 256, ctx, 1.0 / 16, splits, ws.data_ptr(), 0,
        )
        o = out.cpu().numpy()
        for b in range(batch):
            L = int(lens[b])
            ref = ops.attention(q[b], k[b, :L].float().numpy(), v[b, :L].float().numpy(), 1.0 / 16)
            np.testing.assert_allclose(o[b], ref, rtol=1e-4, atol=1e-5)
    groups = -(-splits // 16) if splits > 16 else 0
    part_bytes = (4 * batch * 2 * (splits + groups) * 4 * (256 + 2) + 255) // 256 * 256
    assert int(ws[part_bytes:].sum().item()) == 0  # split and group counters re-armed


@pytest.mark.parametrize("batch", [1, 16, 64])
@pytest.mark.parametrize("ctx", [1024, 8192, 32768])
def test_attention_config3_benchmark_inputs(be, batch, ctx) -> None:
    """The flash-decode benchmark exactly as measured (kernel_bench attn: its
    device-drawn inputs, seed 2, and its split count), every (batch, context)
    of the benchmark, up to four sequences per case (first, last, two drawn)
    against the f32 oracle, on two calls in a row."""
    from breezetoken_b200.kernel_bench import attn_inputs, attn_splits

    q, kc, vc, lens = attn_inputs(batch, ctx)
    splits = attn_splits(batch, 2, ctx)
    out = torch.empty(batch, 8, 256, device="cuda")
    ws = torch.zeros(int(N.load().bt_attention_workspace_bytes(batch, 2, 8, 256, splits)), dtype=torch.uint8,
                     device="cuda")
    picks = sorted({0, batch - 1, *np.random.default_rng(batch * 7 + ctx).integers(0, batch, 2).tolist()})
    for _ in range(2):
        N.call("bt_attention_decode", q.data_ptr(), kc.data_ptr(), vc.data_ptr(), N.BT_BF16, lens.data_ptr(),
               out.data_ptr(), batch, 8, 2, 256, ctx, 1.0 / 16, splits, ws.data_ptr(), 0)
        for b in picks:
            ref = ops.attention(q[b].cpu().numpy(), kc[b].float().cpu().numpy(), vc[b].float().cpu().numpy(),
                                1.0 / 16)
            np.testing.assert_allclose(out[b].cpu().numpy(), ref, rtol=1e-4, atol=1e-5)


def test_argmax_first_index(be) -> None:
    x = torch.zeros(3, 151936, device="cuda")
    x[0, 5] = 2.0
    x[0, 151935] = 2.0  # tie -> first index
    x[1, 77777] = -1e-3
    x[1] -= 1.0
    x[2, 123456] = float("inf")
    got = be.argmax(x).cpu().tolist()
    assert got == [5, int(torch.argmax(x[1]).item()), 123456]
    y = torch.randn(2, 100000, device="cuda")
    assert be.argmax(y).cpu().tolist() == torch.argmax(y, dim=-1).cpu().tolist()


def test_errors_raise(be) -> None:
    with pytest.raises(ValueError):
        be.linear(torch.zeros(5, device="cuda"), torch.zeros(4, 4, device="cuda"))
    with pytest.raises(N.B200Error):
        N.call("bt_linear_q8", 0, 0, 0, 4, 33, 1, 0)
    with pytest.raises(N.B200Error):
        N.call("bt_gdn_decode", 1, 1, 1, 0, 1, 1, 1, 1, 1, 3, 16, 120, 1.0, 1e-6, 0)

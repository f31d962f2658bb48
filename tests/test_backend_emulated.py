"""The ``Backend`` mirror's host side, checked on the CPU.

``B200Backend`` is the drop-in for the reference's ``Backend`` (backends.py:
28-98).  With its library calls emulated on host memory (tests/abi_emulator.py)
the unchanged methods must give the reference's golden op outputs and the
oracle's: argument conversions, (K, N) versus (N, K) orientation, the Q8_0
repack and multi-vector batching, attention lengths (full and fixed
capacity), the in-place GDN state update, and ``ValueError`` on mismatched
shapes as the reference raises it.  The kernels themselves are checked on the
GPU.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from breezetoken_b200.backends import B200Backend, Q8Weight
from breezetoken_b200.quant import quantize_q8_0
from oracle import ops
from oracle.dequant import dequant_q8_0
from tests.abi_emulator import install
from tests.conftest import golden
from tests.golden.make_golden import STATE_SAMPLE, ops_inputs


@pytest.fixture()
def be(monkeypatch):
    em = install(monkeypatch)
    b = B200Backend("cpu")
    b.emulator = em
    return b


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a))


def test_norms_silu_rope_match_reference(be) -> None:
    g, inp = golden("ops"), ops_inputs()
    np.testing.assert_allclose(be.rms_norm(_t(inp["norm_x"]), _t(inp["norm_gamma"]), 1e-6).numpy(), g["norm_out"],
                               rtol=1e-5, atol=1e-5)
    h, xn = be.fused_add_rms_norm(_t(inp["norm_x"]), _t(inp["norm_other"]), _t(inp["norm_gamma"]), 1e-6)
    np.testing.assert_array_equal(h.numpy(), g["fused_h"])
    np.testing.assert_allclose(xn.numpy(), g["fused_xn"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(be.silu_mul(_t(inp["silu_gate"]), _t(inp["silu_up"])).numpy(), g["silu_out"],
                               rtol=1e-5, atol=1e-6)
    r = be.rope(_t(inp["rope_x"]), _t(inp["rope_cos"]), _t(inp["rope_sin"]), _t(inp["rope_pos"]), 64)
    np.testing.assert_allclose(r.numpy(), g["rope_out"], rtol=1e-5, atol=1e-5)


def test_gdn_decode_updates_state_in_place(be) -> None:
    g, inp = golden("ops"), ops_inputs()
    for name in ("gdn16", "gdn8_16", "gdn16_32"):
        state = _t(inp[f"{name}_state0"]).clone()
        o = be.gdn_decode(_t(inp[f"{name}_q"]), _t(inp[f"{name}_k"]), _t(inp[f"{name}_v"]), _t(inp[f"{name}_g"]),
                          _t(inp[f"{name}_beta"]), state, 128**-0.5)
        np.testing.assert_allclose(o.numpy(), g[f"{name}_out"], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(state.numpy().reshape(-1)[::STATE_SAMPLE], g[f"{name}_state1_sample"], rtol=1e-5,
                                   atol=1e-5)
    with pytest.raises(ValueError):
        be.gdn_decode(_t(inp["gdn16_q"]), _t(inp["gdn16_k"]), _t(inp["gdn16_v"]), _t(inp["gdn16_g"]),
                      _t(inp["gdn16_beta"]), torch.zeros(3, 128, 128), 1.0)


def test_attention_full_and_fixed_capacity(be) -> None:
    g, inp = golden("ops"), ops_inputs()
    for seq in (1, 17, 128):
        q, k, v = _t(inp[f"attn{seq}_q"]), _t(inp[f"attn{seq}_k"]), _t(inp[f"attn{seq}_v"])
        np.testing.assert_allclose(be.attention(q, k, v, 256**-0.5).numpy(), g[f"attn{seq}_out"], rtol=1e-5,
                                   atol=2e-6)
    # fixed capacity: a 64-row cache of which rows [0, pos] are live (graph.py:55-61)
    q, k, v = _t(inp["attn17_q"]), _t(inp["attn17_k"]), _t(inp["attn17_v"])
    cap_k, cap_v = torch.full((64, *k.shape[1:]), 1e3), torch.full((64, *v.shape[1:]), 1e3)
    cap_k[:17], cap_v[:17] = k, v
    o = be.attention_fixed(q, cap_k, cap_v, torch.tensor([16], dtype=torch.int32), 256**-0.5)
    np.testing.assert_allclose(o.numpy(), g["attn17_out"], rtol=1e-5, atol=2e-6)
    with pytest.raises(ValueError):
        be.attention(q, k[:, :1, :8], v, 1.0)


def test_q8_linear_and_batches(be) -> None:
    rng = np.random.default_rng(3)
    n, k = 40, 1024
    raw = quantize_q8_0(rng.standard_normal((n, k)).astype(np.float32) * 0.02)
    deq = dequant_q8_0(raw, n, k)
    w = Q8Weight.from_gguf(raw, n, k, "cpu")
    assert w.shape == (k, n)  # the reference's (K, N) GEMV orientation
    assert np.array_equal(w.dequantize().numpy(), deq)  # the repack keeps every byte
    x = rng.standard_normal((5, k)).astype(np.float32)  # 5 vectors: batches of 4 and 1
    np.testing.assert_allclose(be.linear(_t(x[0]), w).numpy(), ops.linear(x[0], deq.T), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(be.linear_batch(_t(x), w).numpy(), (x.astype(np.float64) @ deq.T).astype(np.float32),
                               rtol=1e-5, atol=1e-6)
    assert {"bt_repack_q8_0", "bt_linear_q8"} <= be.emulator.names
    with pytest.raises(ValueError):
        be.linear(_t(x[0, :512]), w)


def test_dense_linear_kn_orientation(be) -> None:
    """Backend.linear with the reference's dense (K, N) weights in bf16 and f32."""
    torch.manual_seed(0)
    x = torch.randn(256)
    for dt in (torch.bfloat16, torch.float32):
        w = torch.randn(256, 100).to(dt)
        ref = x.double() @ w.double()
        assert (be.linear(x, w).double() - ref).abs().max().item() < 1e-5 * ref.abs().max().item() + 1e-5
    with pytest.raises(ValueError):
        be.silu_mul(torch.zeros(4), torch.zeros(5))
    with pytest.raises(ValueError):
        be.rms_norm(torch.zeros(2, 8), torch.ones(7), 1e-6)

"""GPU parity of the routed-expert (MoE) path against the oracle and the
reference's golden output (the 35B-A3B layer shapes: hidden 2048, ffn 512,
IQ3_S experts, top-8 routing).

f32 tolerance: outputs within 1e-5 of the output scale (max |ref|): the
expert GEMVs sum exact integer sub-block dots in a different order than the
reference's dequantise-then-matmul, and the activations are encoded to 22
bits of their 32-element block maximum.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from breezetoken_b200 import _native as N
from breezetoken_b200.moe import IQ3SExperts, SharedExpert, experts_forward, moe_forward, route_logits
from breezetoken_b200.quant import quantize_iq3_s
from oracle.moe import experts as oracle_experts
from oracle.moe import route as oracle_route
from oracle.moe import shared_expert as oracle_shared
from tests.conftest import golden
from tests.golden.make_golden import moe_inputs, moe_shared_inputs

pytestmark = pytest.mark.gpu

TOL = 1e-5


def _close(got: np.ndarray, want: np.ndarray) -> None:
    err = np.abs(got - want).max()
    assert err <= TOL * np.abs(want).max(), f"max |diff| {err:.3e} vs scale {np.abs(want).max():.3e}"


@pytest.fixture(scope="module")
def layer(cuda):
    m = moe_inputs()
    ex = IQ3SExperts.from_gguf_bytes(m["gate"], m["up"], m["down"], 16, m["hidden"], m["ffn"], "cuda")
    return m, ex


#: Bit of a code word where code i (weight 8t + i of a lane's sub-block
#: slice) starts; its 4 bits are at (CODE_BIT[i] + b) % 32 (moe.cu code_bit).
CODE_BIT = (1, 17, 5, 21, 9, 25, 13, 29)


def iq3s_signed_values(raw: np.ndarray, rows: int, k: int) -> np.ndarray:
    """The signed codebook value v (odd, -15..15) of every weight, (rows, k)
    int8: weight = d * (1 + 2 * scale nibble) * v (quant/dequant.py:164-185)."""
    from oracle.dequant import iq3s_grid

    b = np.ascontiguousarray(raw).reshape(rows, k // 256, 110)
    qs = b[..., 2:66].astype(np.int64)  # (rows, blocks, 64 groups)
    qh = b[..., 66:74].astype(np.int64)
    hb = (qh[..., np.arange(64) // 8] >> (np.arange(64) % 8)) & 1
    grid = iq3s_grid().astype(np.int64) & 255  # (512, 4)
    mag = grid[qs | (hb << 8)]  # (rows, blocks, 64, 4)
    signs = b[..., 74:106].astype(np.int64)  # (rows, blocks, 32): byte j = weights 8j .. 8j+7
    neg = (signs[..., np.arange(256) // 8] >> (np.arange(256) % 8)) & 1
    v = mag.reshape(rows, k // 256, 256) * (1 - 2 * neg)
    return v.reshape(rows, k).astype(np.int8)


def pack_iq3s_tiles(raw: np.ndarray, rows: int, k: int) -> np.ndarray:
    """The device layout of bt_repack_iq3_s, restated in numpy: per 16-row
    tile and 256-weight block, a 2176-byte chunk of [4-bit codes (2048 B),
    per-row scales + d (128 B)].  Code c = (v + 15) / 2 of each weight's
    signed codebook value v; part j (sub-blocks 2j, 2j+1) at 512 j, lane
    L = 4g + t's 16 bytes at 512 j + 16 L = the words of (row g, sub-block
    2j), (row g+8, 2j), (row g, 2j+1), (row g+8, 2j+1); a word holds the
    codes of weights 8t .. 8t+7 of its sub-block at CODE_BIT."""
    kb = k // 256
    codes = ((iq3s_signed_values(raw, rows, k).astype(np.int64) + 15) >> 1).astype(np.uint64)
    c = codes.reshape(rows // 16, 2, 8, kb, 8, 4, 8)  # (tile, r, g, block, sub-block, t, i)
    word = np.zeros(c.shape[:-1], np.uint64)
    for i in range(8):
        for bit in range(4):
            word |= ((c[..., i] >> np.uint64(bit)) & np.uint64(1)) << np.uint64((CODE_BIT[i] + bit) % 32)
    word = word.astype(np.uint32)  # (tile, r, g, block, sb, t)
    w = word.reshape(rows // 16, 2, 8, kb, 4, 2, 4)  # (.., part j, S, t)
    w = w.transpose(0, 3, 4, 2, 6, 5, 1)  # (tile, block, j, g, t, S, r): 16 bytes per lane = (S, r) words
    codes_b = w.reshape(rows // 16, kb, 2048 // 4).view(np.uint8).reshape(rows // 16, kb, 2048)
    b = np.ascontiguousarray(raw).reshape(rows // 16, 16, kb, 110)
    rec = np.concatenate([b[..., 106:110], b[..., 0:2], np.zeros(b.shape[:-1] + (2,), np.uint8)], -1)
    rec = rec.transpose(0, 2, 1, 3).reshape(rows // 16, kb, 128)  # (tile, block, row 0..15, 8 B)
    return np.concatenate([codes_b, rec], -1).reshape(-1)


def test_iq3s_repack_matches_layout(layer) -> None:
    """The device layout holds the GGUF bytes exactly where the restated
    packer puts them (every field of every block of the 16 experts)."""
    m, ex = layer
    for dev, raw, rows, k in ((ex.gate, m["gate"], 16 * m["ffn"], m["hidden"]),
                              (ex.down, m["down"], 16 * m["hidden"], m["ffn"])):
        want = pack_iq3s_tiles(raw, rows, k)
        got = dev.cpu().numpy()
        assert got.shape == want.shape
        assert (got == want).all()


def test_moe_experts_match_reference_golden(layer) -> None:
    """One token, the golden fixture's 4 experts and weights (the reference's
    ExpertPool torch path produced `y`)."""
    m, ex = layer
    g = golden("moe")
    x = torch.from_numpy(m["x"]).cuda()
    ids = torch.tensor([m["ids"]], dtype=torch.int32, device="cuda")
    w = torch.from_numpy(m["w"]).reshape(1, -1).cuda()
    ws = torch.zeros(int(N.load().bt_moe_workspace_bytes(1, m["hidden"], m["ffn"], 16, 4)), dtype=torch.uint8,
                     device="cuda")
    for _ in range(2):  # the workspace's arrival counters are re-armed by each call
        got = experts_forward(ex, x.reshape(1, -1), ids, w, ws).cpu().numpy()[0]
        _close(got, g["y"])


def test_moe_experts_batch_shares_experts(layer) -> None:
    """8 tokens routed top-8 over 16 experts: most experts serve several
    tokens in one pass; every token matches the oracle."""
    m, ex = layer
    rng = np.random.default_rng(5)
    t, k = 8, 8
    x = rng.standard_normal((t, m["hidden"])).astype(np.float32)
    logits = rng.standard_normal((t, 16)).astype(np.float32)
    ids, ws = zip(*[(oracle_route(lg, k)[1], oracle_route(lg, k)[0]) for lg in logits], strict=True)
    ids, ws = np.stack(ids).astype(np.int32), np.stack(ws)
    got = experts_forward(ex, torch.from_numpy(x).cuda(), torch.from_numpy(ids).cuda(),
                          torch.from_numpy(ws).cuda()).cpu().numpy()
    gr = np.ascontiguousarray(m["gate"]).reshape(16 * m["ffn"], -1)
    ur = np.ascontiguousarray(m["up"]).reshape(16 * m["ffn"], -1)
    dr = np.ascontiguousarray(m["down"]).reshape(16 * m["hidden"], -1)
    for i in range(t):
        want = oracle_experts(x[i], gr, ur, dr, ids[i], ws[i], m["hidden"], m["ffn"])
        _close(got[i], want)


def test_moe_experts_passes_of_eight_tokens(layer) -> None:
    """20 tokens that all select expert 3 (and 7 others): the expert's 20
    pairs take three 8-token MMA passes; every token matches the oracle."""
    m, ex = layer
    rng = np.random.default_rng(6)
    t = 20
    x = rng.standard_normal((t, m["hidden"])).astype(np.float32)
    others = [e for e in range(16) if e != 3]
    ids = np.array([[3] + [others[(i + j) % 15] for j in range(7)] for i in range(t)], np.int32)
    ws = rng.random((t, 8)).astype(np.float32)
    ws /= ws.sum(1, keepdims=True)
    got = experts_forward(ex, torch.from_numpy(x).cuda(), torch.from_numpy(ids).cuda(),
                          torch.from_numpy(ws).cuda()).cpu().numpy()
    gr = np.ascontiguousarray(m["gate"]).reshape(16 * m["ffn"], -1)
    ur = np.ascontiguousarray(m["up"]).reshape(16 * m["ffn"], -1)
    dr = np.ascontiguousarray(m["down"]).reshape(16 * m["hidden"], -1)
    for i in range(t):
        _close(got[i], oracle_experts(x[i], gr, ur, dr, ids[i], ws[i], m["hidden"], m["ffn"]))


@pytest.fixture(scope="module")
def shared(cuda):
    sh = moe_shared_inputs()
    return sh, SharedExpert.from_tensors(torch.from_numpy(sh["gate"]), torch.from_numpy(sh["up"]),
                                         torch.from_numpy(sh["down"]), torch.from_numpy(sh["gate_inp"]), "cuda")


def test_moe_layer_with_shared_expert_matches_reference_golden(layer, shared) -> None:
    """One token: routed experts + the gated bf16 shared expert against the
    reference's Qwen36Moe._moe output (moe_shared golden)."""
    m, ex = layer
    _, se = shared
    x = torch.from_numpy(m["x"]).cuda().reshape(1, -1)
    ids = torch.tensor([m["ids"]], dtype=torch.int32, device="cuda")
    w = torch.from_numpy(m["w"]).reshape(1, -1).cuda()
    for _ in range(2):
        got = moe_forward(ex, se, x, ids, w).cpu().numpy()[0]
        _close(got, golden("moe_shared")["y"])


def test_moe_layer_with_shared_expert_batch(layer, shared) -> None:
    """12 tokens (two 8-token passes of the shared expert) against the oracle."""
    m, ex = layer
    sh, se = shared
    rng = np.random.default_rng(8)
    t = 12
    x = rng.standard_normal((t, m["hidden"])).astype(np.float32)
    logits = rng.standard_normal((t, 16)).astype(np.float32)
    ids, ws = zip(*[(oracle_route(lg, 8)[1], oracle_route(lg, 8)[0]) for lg in logits], strict=True)
    ids, ws = np.stack(ids).astype(np.int32), np.stack(ws)
    got = moe_forward(ex, se, torch.from_numpy(x).cuda(), torch.from_numpy(ids).cuda(),
                      torch.from_numpy(ws).cuda()).cpu().numpy()
    gr = np.ascontiguousarray(m["gate"]).reshape(16 * m["ffn"], -1)
    ur = np.ascontiguousarray(m["up"]).reshape(16 * m["ffn"], -1)
    dr = np.ascontiguousarray(m["down"]).reshape(16 * m["hidden"], -1)
    for i in range(t):
        want = oracle_experts(x[i], gr, ur, dr, ids[i], ws[i], m["hidden"], m["ffn"])
        want = want + oracle_shared(x[i], sh["gate"], sh["up"], sh["down"], sh["gate_inp"])
        _close(got[i], want)


def test_moe_route_matches_oracle(cuda) -> None:
    """softmax -> top-8 -> renormalise over 256 experts for 16 tokens."""
    rng = np.random.default_rng(3)
    logits = rng.standard_normal((16, 256)).astype(np.float32)
    r = route_logits(torch.from_numpy(logits).cuda(), 8)
    ids, w = r.expert_ids.cpu().numpy(), r.weights.cpu().numpy()
    for i in range(16):
        w_ref, ids_ref = oracle_route(logits[i], 8)
        assert (ids[i] == ids_ref).all()
        np.testing.assert_allclose(w[i], w_ref, rtol=2e-6, atol=1e-7)


def test_moe_golden_routing(cuda) -> None:
    """The reference's route() on the fixture's 256 router logits."""
    g, m = golden("moe"), moe_inputs()
    r = route_logits(torch.from_numpy(m["logits"]).cuda(), 8)
    assert (r.expert_ids.cpu().numpy() == g["route_ids"]).all()
    np.testing.assert_allclose(r.weights.cpu().numpy(), g["route_w"], rtol=2e-6, atol=1e-7)


def test_moe_invalid_ids_contribute_nothing(layer) -> None:
    m, ex = layer
    x = torch.from_numpy(m["x"]).cuda().reshape(1, -1)
    w = torch.tensor([[0.5, 0.5]], device="cuda")
    good = experts_forward(ex, x, torch.tensor([[3, 3]], dtype=torch.int32, device="cuda"),
                           torch.tensor([[0.5, 0.0]], device="cuda"))
    bad = experts_forward(ex, x, torch.tensor([[3, 99]], dtype=torch.int32, device="cuda"), w)
    np.testing.assert_array_equal(bad.cpu().numpy(), good.cpu().numpy())


def test_moe_rejects_unsupported_shapes(cuda) -> None:
    lib = N.load()
    buf = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    p = buf.data_ptr()
    rc = lib.bt_moe_experts_iq3s(p, p, p, p, 1, 3072, 512, 4, p, p, 2, p, p, 0)
    assert rc == N.BT_ERR_UNSUPPORTED
    # a quantiser round trip keeps the op honest for the supported shapes
    assert quantize_iq3_s(np.zeros((1, 256), np.float32)).shape == (1, 110)


# ----------------------------------------------------------- config-4 shape
@pytest.fixture(scope="module")
def layer256(cuda):
    """The MoE-layer benchmark's layer exactly: 256 IQ3_S experts (hidden
    2048, ffn 512) quantised from N(0, 0.02), seed 3, and the bf16 shared expert."""
    from breezetoken_b200.synth import MoeSpec, make_moe_layer

    m = make_moe_layer(MoeSpec(), seed=3)
    ex = IQ3SExperts.from_gguf_bytes(m["gate"], m["up"], m["down"], 256, 2048, 512, "cuda")
    se = SharedExpert.from_tensors(torch.from_numpy(m["sh_gate"]), torch.from_numpy(m["sh_up"]),
                                   torch.from_numpy(m["sh_down"]), torch.from_numpy(m["sh_gate_inp"]), "cuda")
    return m, ex, se


class _DequantCache:
    """The oracle's dequantised expert matrices, each decoded once."""

    def __init__(self, m) -> None:
        from oracle.dequant import dequant_iq3_s

        self.m, self.deq, self.cache = m, dequant_iq3_s, {}

    def get(self, name: str, e: int) -> np.ndarray:
        key = (name, e)
        if key not in self.cache:
            rows, k = (512, 2048) if name != "down" else (2048, 512)
            raw = self.m[name][e * rows : (e + 1) * rows]
            self.cache[key] = self.deq(np.ascontiguousarray(raw).reshape(-1), rows, k)
        return self.cache[key]

    def routed(self, x: np.ndarray, ids, weights) -> np.ndarray:
        """oracle.moe.experts on the cached matrices (model/moe.py:225-233)."""
        from oracle import ops

        out = np.zeros(2048, np.float32)
        for e, w in zip(ids, weights, strict=True):
            act = ops.silu(self.get("gate", int(e)) @ x) * (self.get("up", int(e)) @ x)
            out += (self.get("down", int(e)) @ act) * np.float32(w)
        return out


@pytest.mark.parametrize("t", [1, 8, 16, 64])
def test_moe_layer_config4_full_shape(layer256, t) -> None:
    """The MoE-layer benchmark exactly as measured: 256 experts, top-8 over
    N(0, 1) router logits, T tokens of bf16 N(0, 1) activations, seed 3:
    device routing equals the oracle's, and every token's routed + shared
    output is within 1e-5 of the output scale of the oracle's
    dequantise-then-matmul, on two calls in a row (workspace re-armed)."""
    from breezetoken_b200.synth import moe_layer_inputs

    m, ex, se = layer256
    x, logits = moe_layer_inputs(t)
    r = route_logits(torch.from_numpy(logits).cuda(), 8)
    ids, w = r.expert_ids.cpu().numpy(), r.weights.cpu().numpy()
    cache = _DequantCache(m)
    xd = torch.from_numpy(x).cuda()
    ws = torch.zeros(int(N.load().bt_moe_layer_workspace_bytes(t, 2048, 512, 512, 256, 8)), dtype=torch.uint8,
                     device="cuda")
    outs = [moe_forward(ex, se, xd, r.expert_ids, r.weights, ws).cpu().numpy() for _ in range(2)]
    for i in range(t):
        w_ref, ids_ref = oracle_route(logits[i], 8)
        assert (ids[i] == ids_ref).all()
        np.testing.assert_allclose(w[i], w_ref, rtol=2e-6, atol=1e-7)
        want = cache.routed(x[i], ids[i], w[i]) + oracle_shared(x[i], m["sh_gate"], m["sh_up"], m["sh_down"],
                                                                 m["sh_gate_inp"])
        for got in outs:
            _close(got[i], want)


@pytest.mark.parametrize("t", [1, 8, 16, 17, 64])
def test_moe_layer_add_norm_equals_layer_then_norm(layer256, t) -> None:
    """bt_moe_layer_iq3s_add_norm (the combine fused with the residual add,
    RMSNorm and bf16 planes for T > 1) gives the bits of bt_moe_layer_iq3s
    followed by bt_add_rms_norm_planes, on the static (T <= 16), pulled (T > 16)
    and one-token paths."""
    from breezetoken_b200.moe import moe_forward, route_logits
    from breezetoken_b200.synth import moe_layer_inputs

    m, ex, se = layer256
    xh, lh = moe_layer_inputs(t)
    x, logits = torch.from_numpy(xh).cuda(), torch.from_numpy(lh).cuda()
    r = route_logits(logits, 8)
    rng = np.random.default_rng(57)
    h = torch.from_numpy(rng.standard_normal((t, 2048), dtype=np.float32)).cuda()
    gamma = torch.from_numpy(1 + 0.02 * rng.standard_normal(2048, dtype=np.float32)).cuda()
    out = moe_forward(ex, se, x, r.expert_ids, r.weights)
    h1, y1 = torch.empty_like(h), torch.empty_like(h)
    p1 = torch.empty(t, 3, 2048, dtype=torch.bfloat16, device="cuda")
    N.call("bt_add_rms_norm_planes", h.data_ptr(), out.data_ptr(), gamma.data_ptr(), h1.data_ptr(), y1.data_ptr(),
           p1.data_ptr(), t, 2048, 1e-6, 0)
    h2, y2, p2 = moe_forward(ex, se, x, r.expert_ids, r.weights, norm=(h, gamma, 1e-6))
    assert torch.equal(h2, h1)
    assert torch.equal(y2, y1)
    assert torch.equal(p2, p1)


@pytest.mark.parametrize("t", [1, 8, 16, 17, 64])
def test_moe_prepared_layer_equals_layer(layer256, t) -> None:
    """bt_moe_route_sort_iq3s then bt_moe_layer_iq3s_add_norm_prepared: the
    routing and the bits of bt_moe_route + the one-call layer, on the static,
    pulled and one-token paths, from a workspace left dirty by another layer
    call, twice (the routing ticket re-armed)."""
    from breezetoken_b200.moe import moe_forward, route_logits, route_sort
    from breezetoken_b200.synth import moe_layer_inputs

    m, ex, se = layer256
    xh, lh = moe_layer_inputs(t)
    x, logits = torch.from_numpy(xh).cuda(), torch.from_numpy(lh).cuda()
    rng = np.random.default_rng(58)
    h = torch.from_numpy(rng.standard_normal((t, 2048), dtype=np.float32)).cuda()
    gamma = torch.from_numpy(1 + 0.02 * rng.standard_normal(2048, dtype=np.float32)).cuda()
    r = route_logits(logits, 8)
    want = moe_forward(ex, se, x, r.expert_ids, r.weights, norm=(h, gamma, 1e-6))
    ws = torch.zeros(int(N.load().bt_moe_layer_workspace_bytes(t, 2048, 512, 512, 256, 8)), dtype=torch.uint8,
                     device="cuda")
    other = torch.from_numpy(moe_layer_inputs(t, seed=9)[0]).cuda()
    moe_forward(ex, se, other, r.expert_ids, r.weights, ws, norm=(h, gamma, 1e-6))  # dirty workspace
    for _ in range(2):
        r2 = route_sort(logits, x, 8, ex, se, ws)
        assert torch.equal(r2.expert_ids, r.expert_ids) and torch.equal(r2.weights, r.weights)
        got = moe_forward(ex, se, x, r2.expert_ids, r2.weights, ws, norm=(h, gamma, 1e-6), prepared=True)
        for a, b in zip(got, want, strict=True):
            assert torch.equal(a, b)


def test_moe_wide_passes_equal_narrow_batches(layer256) -> None:
    """512 tokens over 256 experts (a prefill chunk: 16 pairs per expert on
    average) run on wide passes, where each decoded weight tile serves up to
    16 tokens; every token's output has the bits of the same token in 64-token
    calls (4-token passes), through the one-call layer, the fused add + norm
    and the prepared (route + sort) call, and a sample of tokens is within
    1e-5 of the output scale of the oracle's dequantise-then-matmul."""
    from breezetoken_b200.moe import route_sort
    from breezetoken_b200.synth import moe_layer_inputs

    m, ex, se = layer256
    t, step = 512, 64
    xh, lh = moe_layer_inputs(t)
    x, logits = torch.from_numpy(xh).cuda(), torch.from_numpy(lh).cuda()
    r = route_logits(logits, 8)
    counts = np.bincount(r.expert_ids.cpu().numpy().reshape(-1), minlength=256)
    assert counts.max() > 16 and (counts % 4).any()  # several and ragged wide passes
    got = moe_forward(ex, se, x, r.expert_ids, r.weights)
    want = torch.cat([moe_forward(ex, se, x[i:i + step], r.expert_ids[i:i + step], r.weights[i:i + step])
                      for i in range(0, t, step)])
    assert torch.equal(got, want)
    rng = np.random.default_rng(59)
    h = torch.from_numpy(rng.standard_normal((t, 2048), dtype=np.float32)).cuda()
    gamma = torch.from_numpy(1 + 0.02 * rng.standard_normal(2048, dtype=np.float32)).cuda()
    fused = moe_forward(ex, se, x, r.expert_ids, r.weights, norm=(h, gamma, 1e-6))
    parts = [moe_forward(ex, se, x[i:i + step], r.expert_ids[i:i + step], r.weights[i:i + step],
                         norm=(h[i:i + step], gamma, 1e-6)) for i in range(0, t, step)]
    for j, a in enumerate(fused):
        assert torch.equal(a, torch.cat([p[j] for p in parts]))
    ws = torch.zeros(int(N.load().bt_moe_layer_workspace_bytes(t, 2048, 512, 512, 256, 8)), dtype=torch.uint8,
                     device="cuda")
    for _ in range(2):
        r2 = route_sort(logits, x, 8, ex, se, ws)
        assert torch.equal(r2.expert_ids, r.expert_ids) and torch.equal(r2.weights, r.weights)
        prep = moe_forward(ex, se, x, r2.expert_ids, r2.weights, ws, norm=(h, gamma, 1e-6), prepared=True)
        for a, b in zip(prep, fused, strict=True):
            assert torch.equal(a, b)
    cache = _DequantCache(m)
    ids, w, out = r.expert_ids.cpu().numpy(), r.weights.cpu().numpy(), got.cpu().numpy()
    for i in (0, 1, 255, 511):
        ref = cache.routed(xh[i], ids[i], w[i]) + oracle_shared(xh[i], m["sh_gate"], m["sh_up"], m["sh_down"],
                                                                m["sh_gate_inp"])
        _close(out[i], ref)

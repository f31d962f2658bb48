"""bt_attention_layer (the fused Qwen3.6 full-attention layer: q/k RMSNorm,
partial RoPE at the position, KV-cache write, attention over the cached
prefix, sigmoid gate; model/qwen36_moe.py:432-457) at the 35B-A3B shape,
16 query / 2 KV heads x 256, against the oracle's ops
(oracle/ops.py rms_norm, rope, attention, sigmoid), at ragged positions and
across split counts: single-position slices, slices that end on and off a
warp batch of 4 positions, up to 16 splits and the full 64-sequence batch."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from breezetoken_b200 import _native as N
from breezetoken_b200.qwen36_moe import Qwen36Config, rope_tables
from breezetoken_b200.synth import QWEN36_35B
from oracle import ops

pytestmark = pytest.mark.gpu

H, KV, D, CAP = 16, 2, 256, 769


def _reference(proj, qn, kn, cos, sin, rope_dim, pos, kc, vc, eps):
    """Per sequence, the oracle's restatement of the layer on host copies
    (updates kc / vc at the position like the kernel)."""
    batch = proj.shape[0]
    out = np.empty((batch, H, D), np.float32)
    for b in range(batch):
        row = proj[b]
        qg = row[: 2 * H * D].reshape(H, 2 * D)
        q, gate = qg[:, :D], qg[:, D:]
        k = row[2 * H * D : (2 * H + KV) * D].reshape(KV, D)
        v = row[(2 * H + KV) * D :].reshape(KV, D)
        p = int(pos[b])
        q = ops.rope(ops.rms_norm(q, qn, eps), cos, sin, p, rope_dim)
        k = ops.rope(ops.rms_norm(k, kn, eps), cos, sin, p, rope_dim)
        kc[b, p], vc[b, p] = k, v
        out[b] = ops.attention(q, kc[b, : p + 1], vc[b, : p + 1], D**-0.5) * ops.sigmoid(gate)
    return out


@pytest.mark.parametrize(
    "batch,top,step,splits",
    [
        (4, 0, 0, 1),  # one position
        (4, 17, 5, 1),  # 17, 12, 7, 2 positions: one stage and its ragged tail
        (3, 64, 1, 2),  # slices of 32 positions (two stages each)
        (4, 200, 17, 3),  # uneven splits, slice ends off the stage boundary
        (2, 767, 300, 8),  # the last cache row, eight slices
        (2, 700, 350, 16),  # 16 splits: short contexts run fewer
        (64, 660, 3, 2),  # the benchmark's batch and split count
    ],
)
def test_attention_layer_matches_oracle(cuda, batch, top, step, splits) -> None:
    cfg = Qwen36Config.from_spec(QWEN36_35B, CAP)
    cos, sin = rope_tables(cfg)
    rng = np.random.default_rng(7)
    proj = rng.standard_normal((batch, (2 * H + 2 * KV) * D), dtype=np.float32)
    qn = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    kc = rng.standard_normal((batch, CAP, KV, D), dtype=np.float32)
    vc = rng.standard_normal((batch, CAP, KV, D), dtype=np.float32)
    pos = np.array([max(0, top - step * b) for b in range(batch)], dtype=np.int32)
    kc_ref, vc_ref = kc.copy(), vc.copy()
    want = _reference(proj, qn, kn, cos.numpy(), sin.numpy(), cfg.rope_dim, pos, kc_ref, vc_ref, cfg.eps)

    lib = N.load()
    ws = torch.zeros(max(256, int(lib.bt_attention_workspace_bytes(batch, KV, H, D, splits))), dtype=torch.uint8,
                     device="cuda")
    dev = {name: torch.from_numpy(a).cuda() for name, a in
           (("proj", proj), ("qn", qn), ("kn", kn), ("kc", kc), ("vc", vc), ("pos", pos))}
    cd, sd = cos.cuda(), sin.cuda()
    out = torch.empty(batch, H, D, device="cuda")
    for _ in range(2):  # the second call finds the merge counters re-armed
        N.call("bt_attention_layer", dev["proj"].data_ptr(), proj.shape[1], dev["qn"].data_ptr(),
               dev["kn"].data_ptr(), cd.data_ptr(), sd.data_ptr(), cfg.rope_dim, dev["pos"].data_ptr(),
               dev["kc"].data_ptr(), dev["vc"].data_ptr(), out.data_ptr(), batch, H, KV, D, CAP, float(D**-0.5),
               float(cfg.eps), splits, ws.data_ptr(), None, 0)
        got = out.cpu().numpy()
        for b in range(batch):
            np.testing.assert_allclose(got[b], want[b], rtol=1e-4, atol=1e-5, err_msg=f"sequence {b}")
    # the cache holds the new rows at each position and nothing else changed
    np.testing.assert_allclose(dev["kc"].cpu().numpy(), kc_ref, rtol=1e-5, atol=1e-5)
    np.testing.assert_array_equal(dev["vc"].cpu().numpy(), vc_ref)


def test_attention_layer_repeats_bit_for_bit(cuda) -> None:
    """Same inputs, same bits, whichever CTA of a split finishes last."""
    cfg = Qwen36Config.from_spec(QWEN36_35B, CAP)
    cos, sin = (t.cuda() for t in rope_tables(cfg))
    g = torch.Generator(device="cuda").manual_seed(5)
    batch, splits = 16, 4
    proj = torch.randn(batch, (2 * H + 2 * KV) * D, device="cuda", generator=g)
    qn = 1 + 0.02 * torch.randn(D, device="cuda", generator=g)
    kn = 1 + 0.02 * torch.randn(D, device="cuda", generator=g)
    kc = torch.randn(batch, CAP, KV, D, device="cuda", generator=g)
    vc = torch.randn(batch, CAP, KV, D, device="cuda", generator=g)
    pos = torch.full((batch,), 600, dtype=torch.int32, device="cuda")
    lib = N.load()
    ws = torch.zeros(int(lib.bt_attention_workspace_bytes(batch, KV, H, D, splits)), dtype=torch.uint8, device="cuda")
    outs = []
    for _ in range(3):
        out = torch.empty(batch, H, D, device="cuda")
        N.call("bt_attention_layer", proj.data_ptr(), proj.shape[1], qn.data_ptr(), kn.data_ptr(), cos.data_ptr(),
               sin.data_ptr(), cfg.rope_dim, pos.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), batch, H,
               KV, D, CAP, float(D**-0.5), float(cfg.eps), splits, ws.data_ptr(), None, 0)
        outs.append(out.cpu())
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])

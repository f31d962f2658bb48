"""The allocation-free attention entry point against the workspace one.

bt_attention_decode_noalloc exists for callers that cannot allocate GPU
memory at the moment they call us -- an inference server whose memory pool
was sized at start-up and owns every allocation, or a foreign-language
binding that only holds the buffers it was handed -- so it keeps its scratch
(split partials and merge counters) in a fixed static device array instead
of asking for a workspace.  This file is collected last on purpose: if it
fails, a run that stops at the first failure has already run everything else.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from breezetoken_b200 import _native as N

pytestmark = pytest.mark.gpu


def _inputs(seed: int, batch: int, ctx: int, kv_dtype=torch.bfloat16):
    rng = np.random.default_rng(seed)
    q = torch.from_numpy(rng.standard_normal((batch, 8, 256), dtype=np.float32)).cuda()
    k = torch.from_numpy(rng.standard_normal((batch, ctx, 2, 256), dtype=np.float32)).to("cuda", kv_dtype)
    v = torch.from_numpy(rng.standard_normal((batch, ctx, 2, 256), dtype=np.float32)).to("cuda", kv_dtype)
    lens = torch.tensor([max(1, ctx - 7 * b) for b in range(batch)], dtype=torch.int32, device="cuda")
    return q, k, v, lens


def _dt(k) -> int:
    return N.BT_BF16 if k.dtype == torch.bfloat16 else N.BT_F32


def _with_workspace(lib, q, k, v, lens, batch, ctx, splits):
    out = torch.empty(batch, 8, 256, device="cuda")
    ws = torch.zeros(int(lib.bt_attention_workspace_bytes(batch, 2, 8, 256, splits)), dtype=torch.uint8, device="cuda")
    N.check(
        lib.bt_attention_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), _dt(k), lens.data_ptr(), out.data_ptr(),
                                batch, 8, 2, 256, ctx, 1.0 / 16, splits, ws.data_ptr(), 0),
        "bt_attention_decode",
    )
    torch.cuda.synchronize()
    return out


def _noalloc(lib, q, k, v, lens, batch, ctx, splits):
    out = torch.empty(batch, 8, 256, device="cuda")
    N.check(
        lib.bt_attention_decode_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), _dt(k), lens.data_ptr(),
                                        out.data_ptr(), batch, 8, 2, 256, ctx, 1.0 / 16, splits, 0),
        "bt_attention_decode_noalloc",
    )
    torch.cuda.synchronize()
    return out


def test_noalloc_attention_matches_workspace_entry_point(cuda) -> None:
    lib = N.load()
    batch, ctx, splits = 4, 1500, 8
    # two calls in a row, with different inputs: the second must not see the
    # first call's partials or counters
    for seed in (21, 22):
        q, k, v, lens = _inputs(seed, batch, ctx)
        want = _with_workspace(lib, q, k, v, lens, batch, ctx, splits).cpu().numpy()
        got = _noalloc(lib, q, k, v, lens, batch, ctx, splits).cpu().numpy()
        np.testing.assert_allclose(got, want, rtol=1e-5, atol=2e-6)
    # a shape whose scratch exceeds the fixed maximum is rejected, not
    # truncated (buffers are sized for the shape all the same)
    bq, bk, bv, bl = _inputs(23, 64, 16)
    bout = torch.empty(64, 8, 256, device="cuda")
    big = lib.bt_attention_decode_noalloc(bq.data_ptr(), bk.data_ptr(), bv.data_ptr(), N.BT_BF16, bl.data_ptr(),
                                          bout.data_ptr(), 64, 8, 2, 256, 16, 1.0 / 16, 256, 0)
    assert big == N.BT_ERR_INVALID
    assert b"maximum" in lib.bt_last_error()


@pytest.mark.parametrize(
    "calls",
    [
        # more than 16 splits merge in two levels (group records and group
        # counters sit after the split counters in the fixed array); the
        # smaller call after it checks the counters are cleared for another layout
        [(31, 3, 8192, 40, torch.bfloat16), (32, 2, 2000, 4, torch.bfloat16)],
        # f32 KV, then bf16 with more splits than the first call
        [(33, 2, 3000, 12, torch.float32), (34, 5, 4096, 24, torch.bfloat16)],
    ],
)
def test_noalloc_attention_two_level_merge_and_f32(cuda, calls) -> None:
    lib = N.load()
    for seed, batch, ctx, splits, kv_dtype in calls:
        q, k, v, lens = _inputs(seed, batch, ctx, kv_dtype)
        want = _with_workspace(lib, q, k, v, lens, batch, ctx, splits).cpu().numpy()
        got = _noalloc(lib, q, k, v, lens, batch, ctx, splits).cpu().numpy()
        np.testing.assert_allclose(got, want, rtol=1e-5, atol=2e-6)


def test_noalloc_attention_rejects_bad_heads(cuda) -> None:
    """heads not a multiple of kv_heads, and sizes above the bounds, are
    rejected before any scratch arithmetic or launch."""
    lib = N.load()
    q, k, v, lens = _inputs(35, 1, 16)
    out = torch.empty(1, 8, 256, device="cuda")
    args = (q.data_ptr(), k.data_ptr(), v.data_ptr(), N.BT_BF16, lens.data_ptr(), out.data_ptr())
    assert lib.bt_attention_decode_noalloc(*args, 1, 7, 2, 256, 16, 1.0 / 16, 1, 0) == N.BT_ERR_INVALID
    assert lib.bt_attention_decode_noalloc(*args, 1, 1 << 20, 2, 256, 16, 1.0 / 16, 1, 0) == N.BT_ERR_INVALID
    assert lib.bt_attention_decode_noalloc(*args, 1, 8, 2, 1 << 20, 16, 1.0 / 16, 1, 0) == N.BT_ERR_INVALID

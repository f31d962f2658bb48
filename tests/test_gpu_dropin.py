"""The drop-in on the reference's own code: breezetoken's unchanged Qwen3.5
model layer (model/qwen35.py, layers.py, prefill.py) running every Backend
call on this library's B200Backend.

The only change is the one INTEGRATION.md describes for backends.py:860-903:
``make_backend("b200", ...)`` returns ``breezetoken_b200.backends.B200Backend``.
The test patches that factory in the installed reference (baseline/_ref, see
baseline/install_reference.py) and decodes the seeded tiny checkpoint: the
16-token prompt takes the reference's batched prefill (linear_batch,
rms_norm, gdn_decode with the state updated in place, silu_mul,
fused_add_rms_norm), then the per-token path (linear, rope, attention,
gdn_decode, ...).  Greedy tokens must equal the golden ones the reference's
torch f32 backend produced, and the prefill's logits must be within 1e-4 of
their scale.  Skipped when the reference is not installed.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from tests.conftest import ROOT, golden

REF = ROOT / "baseline" / "_ref"

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not (REF / "breezetoken" / "model" / "qwen35.py").is_file(),
                       reason="reference not installed (python baseline/install_reference.py <checkout>)"),
]


@pytest.fixture()
def reference(monkeypatch, cuda):
    """The installed reference with make_backend serving kind "b200"."""
    monkeypatch.syspath_prepend(str(REF))
    for name in [m for m in sys.modules if m == "breezetoken" or m.startswith("breezetoken.")]:
        monkeypatch.delitem(sys.modules, name)
    import breezetoken.backends as rb
    import breezetoken.model.qwen35 as rq

    from breezetoken_b200.backends import B200Backend
    from breezetoken_b200.backends import make_backend as make_b200

    stock = rb.make_backend

    def make_backend(kind="auto", device="auto", dtype=None):
        if str(kind).lower() == "b200":
            return make_b200("b200", device, dtype)
        return stock(kind, device, dtype)

    monkeypatch.setattr(rb, "make_backend", make_backend)
    monkeypatch.setattr(rq, "make_backend", make_backend)
    assert Path(rq.__file__).resolve().is_relative_to(REF.resolve())
    return rq, B200Backend


def test_reference_qwen35_decodes_on_b200_backend(reference, tiny_gguf) -> None:
    rq, B200Backend = reference
    from breezetoken.gguf import GGUFFile

    g = golden("qwen35_tiny")
    with GGUFFile(str(tiny_gguf)) as f:
        model = rq.Qwen35(f, backend="b200", device="cuda", dtype="float32", max_context=int(g["max_context"]))
    assert all(isinstance(b, B200Backend) for b in model.layer_backends)
    assert isinstance(model.head_backend, B200Backend)
    prompt = g["prompt"].tolist()
    with torch.inference_mode():
        first = model._prefill_batch(prompt).float().cpu().numpy()
    want = g["logits"][0]
    assert np.abs(first - want).max() <= 1e-4 * np.abs(want).max()
    got = model.generate(prompt, int(g["steps"]), 0.0)
    assert got == g["tokens"].tolist()


def test_reference_qwen35_per_token_prompt_on_b200_backend(reference, tiny_gguf) -> None:
    """A 7-token prompt stays on the reference's per-token path (attention over
    the f32 KV cache view, RoPE from the device position, the GDN step) and
    must reproduce the reference torch backend's greedy continuation."""
    rq, _ = reference
    from breezetoken.gguf import GGUFFile

    prompt = golden("qwen35_tiny")["prompt"].tolist()[:7]
    with GGUFFile(str(tiny_gguf)) as f:
        ours = rq.Qwen35(f, backend="b200", device="cuda", dtype="float32", max_context=64)
        theirs = rq.Qwen35(f, backend="torch", device="cpu", dtype="float32", max_context=64)
    assert ours.generate(prompt, 12, 0.0) == theirs.generate(prompt, 12, 0.0)

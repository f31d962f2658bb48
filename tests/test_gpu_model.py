"""GPU parity of the fused Qwen3.5 decode step against the reference.

Greedy token ids must be identical to the reference's (golden fixtures from
``Qwen35(backend="torch", device="cpu")``) over the whole run; logits must
agree within 1e-4 of the logit scale (f32 sums in a different order through
24 layers).  A mismatching token is only tolerated nowhere: the fixtures
record the top-2 margin of every step so a failure can be told apart from a
genuine near-tie.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from breezetoken_b200.model import Qwen35
from tests.conftest import golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny(cuda, tiny_gguf):
    g = golden("qwen35_tiny")
    m = Qwen35(tiny_gguf, max_context=int(g["max_context"]))
    yield m
    m.close()


def _first_mismatch(a, b) -> int | None:
    for i, (x, y) in enumerate(zip(a, b, strict=False)):
        if x != y:
            return i
    return None


def test_tiny_forward_token_logits(tiny) -> None:
    """Token-wise prefill through the eager step; last-prompt logits vs the reference."""
    g = golden("qwen35_tiny")
    prompt = g["prompt"].tolist()
    tiny.reset()
    for i, t in enumerate(prompt):
        logits = tiny.forward_token(t, i, logits=(i == len(prompt) - 1))
    ref = g["logits"][0]
    got = logits.cpu().numpy()
    assert np.abs(got - ref).max() <= 1e-4 * np.abs(ref).max()
    assert int(got.argmax()) == int(g["tokens"][0])


def test_tiny_generate_matches_reference(tiny) -> None:
    g = golden("qwen35_tiny")
    got = tiny.generate(g["prompt"].tolist(), int(g["steps"]))
    want = g["tokens"].tolist()
    assert got == want, f"first mismatch at {_first_mismatch(got, want)}; margins {g['margins'][:8]}"


def test_tiny_graph_burst_equals_stepwise(tiny) -> None:
    """decode_greedy (n-step graphs, no host sync) == generate (1-step graph + sync)."""
    g = golden("qwen35_tiny")
    prompt = g["prompt"].tolist()
    burst = tiny.decode_greedy([prompt], int(g["steps"]), chunk=8)[0]
    assert burst == g["tokens"].tolist()


@pytest.mark.parametrize("batch", [2, 4, 8])
def test_tiny_batch_lockstep(cuda, tiny_gguf, batch) -> None:
    """Sequences decoded together in one step match each decoded alone
    (every batch width the step serves: the GEMV specialises per width)."""
    g = golden("qwen35_tiny")
    p0 = g["prompt"].tolist()
    rng = np.random.default_rng(9)
    prompts = [p0] + [rng.integers(0, 8192, len(p0)).tolist() for _ in range(batch - 1)]
    m1 = Qwen35(tiny_gguf, max_context=256)
    solo = [m1.decode_greedy([p], 12)[0] for p in prompts]
    m1.close()
    mb = Qwen35(tiny_gguf, max_context=256, batch=batch)
    together = mb.decode_greedy(prompts, 12)
    mb.close()
    assert together == solo
    assert together[0] == g["tokens"][:12].tolist()


def test_invalid_inputs_raise(tiny) -> None:
    with pytest.raises(ValueError):
        tiny.forward_token(10**9, 0)
    with pytest.raises(ValueError):
        tiny.forward_token(1, tiny.cfg.max_context)
    with pytest.raises(ValueError):
        tiny.generate([], 4)


def test_0_8b_greedy_128_steps_match_reference(cuda, gguf_0_8b) -> None:
    """The 0.8B decode benchmark: 16-token prompt, 128 greedy steps, identical ids."""
    g = golden("qwen35_0_8b")
    m = Qwen35(gguf_0_8b, max_context=int(g["max_context"]))
    try:
        got = m.decode_greedy([g["prompt"].tolist()], int(g["steps"]), chunk=16)[0]
        want = g["tokens"].tolist()
        assert got == want, f"first mismatch at {_first_mismatch(got, want)} (margin {g['margins']})"
        stepwise = m.generate(g["prompt"].tolist(), 16)
        assert stepwise == want[:16]
        logits = m.logits[0].cpu().numpy()
        assert np.isfinite(logits).all()
    finally:
        m.close()
    torch.cuda.synchronize()


_PATH_SCRIPT = """
import sys
import numpy as np
sys.path.insert(0, sys.argv[1])
from breezetoken_b200.model import Qwen35
m = Qwen35(sys.argv[2], max_context=64)
tok, rows = 3, []
for pos in range(12):
    lg = m.forward_token(tok, pos).cpu().numpy()
    rows.append(lg)
    tok = int(lg.argmax())
np.save(sys.argv[3], np.stack(rows))
m.close()
"""


def test_gdn_fused_layer_matches_three_kernel_path(cuda, tiny_gguf, tmp_path) -> None:
    """The fused GDN layer kernel (in-projection, conv, recurrence and gated
    norm in one cluster launch) against the in-projection GEMV, recurrence
    kernel and gated-norm out-projection it replaces: same greedy tokens,
    logits within 1e-5 of their scale (the gated norm's sum of squares is
    added in a different order)."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    root = str(Path(__file__).resolve().parents[1])
    out = {}
    for fused in ("1", "0"):
        dst = tmp_path / f"logits_{fused}.npy"
        env = dict(os.environ, BT_GDN_FUSED=fused)
        subprocess.run([sys.executable, "-c", _PATH_SCRIPT, root, str(tiny_gguf), str(dst)], env=env, check=True,
                       timeout=600)
        out[fused] = np.load(dst)
    a, b = out["1"], out["0"]
    assert (a.argmax(-1) == b.argmax(-1)).all()
    assert np.abs(a - b).max() <= 1e-5 * np.abs(b).max()

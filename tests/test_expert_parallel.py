"""Expert-parallel MoE placement (breezetoken_b200.expert_parallel): the
routing rebased per rank, expert slices as views, and the dispatch / local
experts / combine exchange on two ranks against the replicated layer
(model/moe.py:205-233 with the shared expert of model/qwen36_moe.py:634-642).

The two-rank CPU test runs gloo ranks with the library calls emulated on
host memory (tests/abi_emulator.py); the GPU test runs the kernels over NCCL
on two GPUs when the box has them."""

from __future__ import annotations

import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from breezetoken_b200.expert_parallel import expert_slice, rebase_routing
from breezetoken_b200.moe import IQ3SExperts
from breezetoken_b200.synth import MoeSpec

SPEC = MoeSpec(hidden=1024, n_experts=4, top_k=2, ffn=512)
TOL = 1e-5


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_rebase_routing_keeps_each_ranks_experts() -> None:
    ids = torch.tensor([[0, 5], [7, 2], [4, 3]], dtype=torch.int32)
    w = torch.tensor([[0.6, 0.4], [0.7, 0.3], [0.5, 0.5]])
    r = rebase_routing(ids, w, world=2, per_rank=4)
    assert r.shape == (2, 3, 4)
    assert r[0, :, :2].tolist() == [[0, -1], [-1, 2], [-1, 3]]
    assert r[1, :, :2].tolist() == [[-1, 1], [3, -1], [0, -1]]
    assert torch.equal(r[0, :, 2:], w) and torch.equal(r[1, :, 2:], w)


def test_expert_slice_is_a_view_of_whole_experts() -> None:
    rb_h, rb_f = 1024 // 256 * 136, 512 // 256 * 136
    gate = torch.arange(4 * 512 * rb_h, dtype=torch.int64).to(torch.uint8)
    down = torch.zeros(4 * 1024 * rb_f, dtype=torch.uint8)
    ex = IQ3SExperts(gate, gate.clone(), down, 4, 1024, 512)
    s = expert_slice(ex, 2, 4)
    assert s.n_experts == 2 and s.gate.data_ptr() == gate.data_ptr() + 2 * 512 * rb_h
    assert s.down.numel() == 2 * 1024 * rb_f and s.down.data_ptr() == down.data_ptr() + 2 * 1024 * rb_f
    with pytest.raises(ValueError):
        expert_slice(ex, 3, 5)


def _layer(device: str, spec: MoeSpec, rank: int, tokens: int):
    from breezetoken_b200.moe import SharedExpert, route_logits
    from breezetoken_b200.synth import make_moe_layer, moe_layer_inputs

    m = make_moe_layer(spec, seed=5)
    ex = IQ3SExperts.from_gguf_bytes(m["gate"], m["up"], m["down"], spec.n_experts, spec.hidden, spec.ffn, device)
    se = SharedExpert.from_tensors(torch.from_numpy(m["sh_gate"]), torch.from_numpy(m["sh_up"]),
                                   torch.from_numpy(m["sh_down"]), torch.from_numpy(m["sh_gate_inp"]), device)
    x, logits = moe_layer_inputs(tokens, spec, seed=11 + rank)  # every rank its own tokens
    r = route_logits(torch.from_numpy(logits).to(device), spec.top_k)
    return ex, se, torch.from_numpy(x).to(device), r.expert_ids, r.weights


def _ep_worker(rank: int, world: int, port: int, backend: str, q) -> None:
    import torch.distributed as dist

    from breezetoken_b200.expert_parallel import ExpertParallelMoE
    from breezetoken_b200.moe import moe_forward

    patch = pytest.MonkeyPatch()
    try:
        if backend == "gloo":
            from tests.abi_emulator import install

            install(patch)
            device, spec, tokens = "cpu", SPEC, 3
        else:
            torch.cuda.set_device(rank)
            device, spec, tokens = "cuda", MoeSpec(n_experts=16), 8
        dist.init_process_group(backend, init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        try:
            ex, se, x, ids, w = _layer(device, spec, rank, tokens)
            ep = ExpertParallelMoE(ex, se)
            got = ep(x, ids, w)
            again = ep(x, ids, w)
            want = moe_forward(ex, se, x, ids, w)
            q.put((rank, got.cpu().numpy(), again.cpu().numpy(), want.cpu().numpy(), ep.per_rank))
        finally:
            dist.destroy_process_group()
    finally:
        patch.undo()


def _run_two_ranks(backend: str):
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_ep_worker, args=(r, world, port, backend, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            rank, *rest = q.get(timeout=300)
            res[rank] = rest
    finally:
        for p in procs:
            p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    return res


def _check(res, per_rank: int) -> None:
    for rank, (got, again, want, pr) in res.items():
        assert pr == per_rank
        # a fixed summation order: the same bits every call
        np.testing.assert_array_equal(got, again)
        # other order than the replicated combine: within f32 rounding of the layer
        err = np.abs(got - want).max()
        assert err <= TOL * np.abs(want).max(), f"rank {rank}: |diff| {err:.3e} vs scale {np.abs(want).max():.3e}"


def test_two_ranks_match_the_replicated_layer_on_cpu() -> None:
    _check(_run_two_ranks("gloo"), per_rank=SPEC.n_experts // 2)


@pytest.mark.gpu
def test_two_gpus_match_the_replicated_layer() -> None:
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    _check(_run_two_ranks("nccl"), per_rank=8)

"""Expert-parallel placement of the Qwen3.6-MoE experts over the GPUs of a box.

The decode path shards independent sequences over the GPUs and replicates
every weight (no collective; `planner.plan`).  This module is the other
placement the survey of the reference lists for the 35B-A3B shape: rank r of
N holds experts [r E/N, (r+1) E/N) of a layer, the routed part of the MoE
layer (model/moe.py:205-233) runs where the experts are, and the tokens
travel over NVLink with NCCL all-to-all:

1. dispatch: every rank sends all its T tokens' rows (T, hidden) f32, and
   their routing with the ids rebased to the destination's experts (ids of
   other ranks' experts become -1, which the expert kernels skip), to every
   rank: one all-to-all of rows and one of routing (fixed sizes, so the
   collectives are the same every step);
2. each rank runs its experts over the N T tokens it received
   (bt_moe_experts_iq3s on its expert slice);
3. combine: the partial outputs go back with one more all-to-all and the
   source rank adds them in rank order, plus its own shared expert (the
   layer call with no routed ids).

Every sum is in a fixed order, so the result is deterministic; it is not the
same bits as the replicated layer (whose combine adds the eight experts in
routing order before the shared expert).  The NCCL collectives are this
placement's baseline exchange; the replicated placement stays the default
(see the module's measurement in kernel_bench `moe-ep`).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from breezetoken_b200.moe import IQ3SExperts, SharedExpert, experts_forward, moe_forward


def expert_slice(ex: IQ3SExperts, lo: int, hi: int) -> IQ3SExperts:
    """Experts [lo, hi) of a layer's device tensors as views (each expert's
    rows are contiguous tiles in the bt_repack_iq3_s layout)."""
    if not 0 <= lo < hi <= ex.n_experts:
        raise ValueError(f"expert range [{lo}, {hi}) outside [0, {ex.n_experts})")
    gate_b = ex.gate.numel() // ex.n_experts
    down_b = ex.down.numel() // ex.n_experts
    return IQ3SExperts(ex.gate[lo * gate_b:hi * gate_b], ex.up[lo * gate_b:hi * gate_b],
                       ex.down[lo * down_b:hi * down_b], hi - lo, ex.hidden, ex.ffn)


def rebase_routing(ids: torch.Tensor, weights: torch.Tensor, world: int, per_rank: int) -> torch.Tensor:
    """(world, T, 2 k) f32: for destination d the ids rebased to d's experts
    (-1 where the expert lives elsewhere) and the routing weights; ids are
    exact in f32 (< 2^24)."""
    lo = torch.arange(world, device=ids.device, dtype=torch.int64).view(world, 1, 1) * per_rank
    local = ids.to(torch.int64).unsqueeze(0) - lo
    local = torch.where((local >= 0) & (local < per_rank), local, torch.full_like(local, -1))
    w = weights.float().unsqueeze(0).expand(world, -1, -1)
    return torch.cat([local.float(), w], dim=-1).contiguous()


class ExpertParallelMoE:
    """The routed experts of one layer split over the ranks of `group`, and
    the layer's shared expert replicated (model/qwen36_moe.py:634-642)."""

    def __init__(self, experts: IQ3SExperts, shared: SharedExpert | None, group=None) -> None:
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if experts.n_experts % self.world:
            raise ValueError(f"{experts.n_experts} experts do not split over {self.world} ranks")
        self.per_rank = experts.n_experts // self.world
        lo = self.rank * self.per_rank
        self.local = expert_slice(experts, lo, lo + self.per_rank)
        self.shared = shared
        self.n_experts, self.hidden = experts.n_experts, experts.hidden
        self._ws: dict = {}

    def __call__(self, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
        """out (T, hidden) f32 for this rank's tokens x (T, hidden), routing
        ids / weights (T, k); every rank calls it with the same T and k."""
        x2 = x.float().reshape(-1, self.hidden).contiguous()
        rows_in, r_ids, r_w = self.dispatch(x2, ids, weights)
        return self.combine(self.local_experts(rows_in, r_ids, r_w), x2)

    def dispatch(self, x2: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor):
        """Every rank's rows (N T, hidden) and their routing rebased to this
        rank's experts (N T, k): two all-to-alls of fixed size."""
        n, h = self.world, self.hidden
        t, k = x2.shape[0], ids.shape[-1]
        rows_in = torch.empty(n * t, h, dtype=torch.float32, device=x2.device)
        dist.all_to_all_single(rows_in, x2.repeat(n, 1), group=self.group)
        route = rebase_routing(ids.reshape(t, k), weights.reshape(t, k), n, self.per_rank)
        route_in = torch.empty_like(route)
        dist.all_to_all_single(route_in, route, group=self.group)
        r_ids = route_in[..., :k].reshape(n * t, k).to(torch.int32)
        r_w = route_in[..., k:].reshape(n * t, k).contiguous()
        return rows_in, r_ids, r_w

    def local_experts(self, rows_in: torch.Tensor, r_ids: torch.Tensor, r_w: torch.Tensor) -> torch.Tensor:
        """This rank's experts over the received tokens (bt_moe_experts_iq3s;
        pairs of other ranks' experts carry id -1 and add nothing)."""
        return experts_forward(self.local, rows_in, r_ids, r_w,
                               self._workspace("experts", rows_in.shape[0], r_ids.shape[-1]))

    def combine(self, part: torch.Tensor, x2: torch.Tensor) -> torch.Tensor:
        """The partial outputs back to their tokens' rank (one all-to-all),
        added in rank order, plus the shared expert of this rank's tokens."""
        n, h, t = self.world, self.hidden, x2.shape[0]
        back = torch.empty_like(part)
        dist.all_to_all_single(back, part, group=self.group)
        back = back.view(n, t, h)
        out = back[0].clone()
        for d in range(1, n):
            out = out + back[d]
        if self.shared is not None:
            k = 1
            none = torch.full((t, k), -1, dtype=torch.int32, device=x2.device)
            out = out + moe_forward(self.local, self.shared, x2, none, torch.zeros(t, k, device=x2.device),
                                    self._workspace("shared", t, k))
        return out

    def _workspace(self, key: str, t: int, k: int) -> torch.Tensor:
        from breezetoken_b200 import _native as N

        lib = N.load()
        sffn = self.shared.ffn if self.shared is not None else 0
        need = int(lib.bt_moe_layer_workspace_bytes(t, self.hidden, self.local.ffn, sffn, self.local.n_experts, k))
        ws = self._ws.get(key)
        if ws is None or ws.numel() < need:
            ws = self._ws[key] = torch.zeros(need, dtype=torch.uint8, device=self.local.gate.device)
        return ws


__all__ = ["ExpertParallelMoE", "expert_slice", "rebase_routing"]

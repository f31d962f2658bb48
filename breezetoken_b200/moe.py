"""Routed MoE experts on the GPU, mirroring breezetoken/model/moe.py.

``route`` and ``ExpertPool.forward`` keep the reference's names, argument
meaning and results (model/moe.py:33-39, :205-233); the difference is where
the experts live.  The reference keeps them as quantized bytes in the GGUF
mmap and stages the selected experts' rows to the device every step; here
every layer's IQ3_S experts are repacked once into HBM (a 35B-A3B model's
~13.8 GB of experts fits a B200 several times over) and decoded inside the
expert GEMVs.  ``forward_batch`` runs T tokens in one call, reading each
selected expert once for all the tokens that chose it.  Everything raises
on an unsupported shape or a missing library; there is no CPU path.
"""

from __future__ import annotations

import ctypes
import warnings
from dataclasses import dataclass

import numpy as np
import torch

from breezetoken_b200 import _native as N
from breezetoken_b200.backends import _stream


@dataclass(frozen=True)
class RouterOutput:
    weights: torch.Tensor  # (top_k,) or (T, top_k) f32, renormalised
    expert_ids: torch.Tensor  # same shape, int32 on the device


def route_logits(logits: torch.Tensor, top_k: int) -> RouterOutput:
    """Softmax top-k routing of router logits (T, n_experts) or (n_experts,)."""
    lg = logits.float().contiguous()
    squeeze = lg.dim() == 1
    lg2 = lg.reshape(1, -1) if squeeze else lg
    t, e = lg2.shape
    ids = torch.empty(t, top_k, dtype=torch.int32, device=lg.device)
    w = torch.empty(t, top_k, dtype=torch.float32, device=lg.device)
    N.call("bt_moe_route", lg2.data_ptr(), t, e, top_k, ids.data_ptr(), w.data_ptr(), _stream())
    return RouterOutput(w[0] if squeeze else w, ids[0] if squeeze else ids)


def route(x: torch.Tensor, gate_inp: torch.Tensor, top_k: int) -> RouterOutput:
    """model/moe.py:33-39: ``gate_inp`` is (n_experts, hidden) f32."""
    logits = gate_inp.float() @ x.reshape(-1).float()
    return route_logits(logits, top_k)


@dataclass
class IQ3SExperts:
    """One layer's gate/up (E*ffn rows of K=hidden) and down (E*hidden rows of
    K=ffn) IQ3_S experts in the library's device layout."""

    gate: torch.Tensor
    up: torch.Tensor
    down: torch.Tensor
    n_experts: int
    hidden: int
    ffn: int

    @staticmethod
    def _repack(raw, rows: int, k: int, device: str, uploader=None) -> torch.Tensor:
        if isinstance(raw, np.ndarray) and uploader is not None:
            src = uploader.to_device(raw)
        elif isinstance(raw, np.ndarray):
            with warnings.catch_warnings():
                # GGUF bytes are a read-only memory map; the tensor is only read (the upload's source)
                warnings.filterwarnings("ignore", message="The given NumPy array is not writable")
                src = torch.as_tensor(np.ascontiguousarray(raw))
        else:
            src = torch.as_tensor(raw)
        src = src.reshape(-1).to(device)  # (a no-op for the uploader's device bytes)
        if src.numel() != rows * k // 256 * 110:
            raise ValueError(f"expected {rows * k // 256 * 110} IQ3_S bytes, got {src.numel()}")
        out = torch.empty(rows * int(N.load().bt_iq3s_row_bytes(k)), dtype=torch.uint8, device=device)
        N.call("bt_repack_iq3_s", src.data_ptr(), out.data_ptr(), rows, k, _stream())
        return out

    @classmethod
    def from_gguf_bytes(cls, gate, up, down, n_experts: int, hidden: int, ffn: int, device: str,
                        uploader=None) -> IQ3SExperts:
        """GGUF-stored expert tensors (ffn_{gate,up,down}_exps) as raw bytes;
        `uploader` (breezetoken_b200.upload.Uploader): stage host bytes
        through its pinned buffers."""
        return cls(
            cls._repack(gate, n_experts * ffn, hidden, device, uploader),
            cls._repack(up, n_experts * ffn, hidden, device, uploader),
            cls._repack(down, n_experts * hidden, ffn, device, uploader),
            n_experts, hidden, ffn,
        )


def experts_forward(ex: IQ3SExperts, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor,
                    workspace: torch.Tensor | None = None) -> torch.Tensor:
    """sum_k weights[t,k] * expert_{ids[t,k]}(x[t]) for x (T, hidden) f32."""
    x2 = x.float().reshape(-1, ex.hidden).contiguous()
    t = x2.shape[0]
    ids2 = ids.to(torch.int32).reshape(t, -1).contiguous()
    w2 = weights.float().reshape(t, -1).contiguous()
    top_k = ids2.shape[1]
    lib = N.load()
    need = int(lib.bt_moe_workspace_bytes(t, ex.hidden, ex.ffn, ex.n_experts, top_k))
    if workspace is None or workspace.numel() < need:
        workspace = torch.zeros(need, dtype=torch.uint8, device=x2.device)
    out = torch.empty(t, ex.hidden, dtype=torch.float32, device=x2.device)
    N.call("bt_moe_experts_iq3s", ex.gate.data_ptr(), ex.up.data_ptr(), ex.down.data_ptr(), x2.data_ptr(), t,
           ex.hidden, ex.ffn, ex.n_experts, ids2.data_ptr(), w2.data_ptr(), top_k, out.data_ptr(),
           workspace.data_ptr(), _stream())
    return out


@dataclass
class SharedExpert:
    """A layer's shared expert (model/qwen36_moe.py:276-283): gate, up (ffn,
    hidden) and down (hidden, ffn) bf16 rows in the GGUF orientation, and
    the f32 gate vector (hidden,)."""

    gate: torch.Tensor
    up: torch.Tensor
    down: torch.Tensor
    gate_inp: torch.Tensor

    @property
    def ffn(self) -> int:
        return int(self.gate.shape[0])

    @classmethod
    def from_tensors(cls, gate, up, down, gate_inp, device: str = "cuda") -> SharedExpert:
        def rows(w) -> torch.Tensor:
            return torch.as_tensor(w).to(device=device, dtype=torch.bfloat16).contiguous()

        g, u, d = rows(gate), rows(up), rows(down)
        gi = torch.as_tensor(gate_inp).to(device=device, dtype=torch.float32).reshape(-1).contiguous()
        ffn, hidden = g.shape
        if u.shape != g.shape or d.shape != (hidden, ffn) or gi.numel() != hidden:
            raise ValueError(f"shared expert shapes: gate {tuple(g.shape)}, up {tuple(u.shape)}, "
                             f"down {tuple(d.shape)}, gate_inp {gi.numel()}")
        return cls(g, u, d, gi)


def _shared_arg(shared: SharedExpert | None, hidden: int):
    if shared is None:
        return None
    if shared.gate.shape[1] != hidden:
        raise ValueError(f"shared expert hidden {shared.gate.shape[1]} != {hidden}")
    return N.BtMoeShared(shared.gate.data_ptr(), shared.up.data_ptr(), shared.down.data_ptr(),
                         shared.gate_inp.data_ptr(), shared.ffn)


def route_sort(logits: torch.Tensor, x: torch.Tensor, top_k: int, ex: IQ3SExperts, shared: SharedExpert | None,
               workspace: torch.Tensor) -> RouterOutput:
    """route_logits (the same ids and weights) plus the layer's pair sort and
    the encoding of x (T, hidden) f32 into `workspace`, in one launch
    (bt_moe_route_sort_iq3s), for moe_forward(x, ..., prepared=True) next."""
    lg = logits.float().reshape(-1, ex.n_experts).contiguous()
    t = lg.shape[0]
    x2 = x.float().reshape(-1, ex.hidden)
    if x2.shape[0] != t or not x2.is_contiguous():
        raise ValueError(f"route_sort needs contiguous f32 x of {t} rows (the layer call reads the same buffer)")
    sffn = shared.ffn if shared is not None else 0
    need = int(N.load().bt_moe_layer_workspace_bytes(t, ex.hidden, ex.ffn, sffn, ex.n_experts, top_k))
    if workspace.numel() < need:
        raise ValueError(f"MoE workspace of {workspace.numel()} bytes < {need}")
    ids = torch.empty(t, top_k, dtype=torch.int32, device=lg.device)
    w = torch.empty(t, top_k, dtype=torch.float32, device=lg.device)
    N.call("bt_moe_route_sort_iq3s", lg.data_ptr(), x2.data_ptr(), t, ex.hidden, ex.ffn, ex.n_experts, top_k, sffn,
           ids.data_ptr(), w.data_ptr(), workspace.data_ptr(), _stream())
    return RouterOutput(w, ids)


def moe_forward(ex: IQ3SExperts, shared: SharedExpert | None, x: torch.Tensor, ids: torch.Tensor,
                weights: torch.Tensor, workspace: torch.Tensor | None = None, norm: tuple | None = None,
                prepared: bool = False):
    """Qwen36Moe._moe after routing (model/qwen36_moe.py:634-642) for x (T,
    hidden) f32: the routed experts plus, when given, the shared expert gated
    by sigmoid(x . gate_inp).

    With norm = (h, gamma, eps) the layer's output goes straight into the
    decoder's residual add and the next RMSNorm (bt_moe_layer_iq3s_add_norm,
    the same bits as the separate ops) and (h + out, rms_norm(h + out) *
    gamma, its bf16 planes (T, 3, hidden)) is returned instead of out.
    prepared (with norm): route_sort (whose ids and weights these are)
    already ran on this x and workspace."""
    x2 = x.float().reshape(-1, ex.hidden).contiguous()
    t = x2.shape[0]
    ids2 = ids.to(torch.int32).reshape(t, -1).contiguous()
    w2 = weights.float().reshape(t, -1).contiguous()
    top_k = ids2.shape[1]
    sffn = shared.ffn if shared is not None else 0
    lib = N.load()
    need = int(lib.bt_moe_layer_workspace_bytes(t, ex.hidden, ex.ffn, sffn, ex.n_experts, top_k))
    if prepared and (norm is None or workspace is None or workspace.numel() < need):
        raise ValueError("a prepared MoE layer call takes the norm and the workspace route_sort filled")
    if workspace is None or workspace.numel() < need:
        workspace = torch.zeros(need, dtype=torch.uint8, device=x2.device)
    out = torch.empty(t, ex.hidden, dtype=torch.float32, device=x2.device)
    sh = _shared_arg(shared, ex.hidden)
    if norm is None:
        N.call("bt_moe_layer_iq3s", ex.gate.data_ptr(), ex.up.data_ptr(), ex.down.data_ptr(),
               None if sh is None else ctypes.byref(sh), x2.data_ptr(), t, ex.hidden, ex.ffn, ex.n_experts,
               ids2.data_ptr(), w2.data_ptr(), top_k, out.data_ptr(), workspace.data_ptr(), _stream())
        return out
    h, gamma, eps = norm
    if h.shape != (t, ex.hidden) or h.dtype != torch.float32 or not h.is_contiguous():
        raise ValueError(f"residual must be contiguous f32 {(t, ex.hidden)}")
    h_out, y = torch.empty_like(h), torch.empty_like(h)
    planes = torch.empty(t, 3, ex.hidden, dtype=torch.bfloat16, device=x2.device)
    N.call("bt_moe_layer_iq3s_add_norm_prepared" if prepared else "bt_moe_layer_iq3s_add_norm",
           ex.gate.data_ptr(), ex.up.data_ptr(), ex.down.data_ptr(),
           None if sh is None else ctypes.byref(sh), x2.data_ptr(), t, ex.hidden, ex.ffn, ex.n_experts,
           ids2.data_ptr(), w2.data_ptr(), top_k, h.data_ptr(), gamma.data_ptr(), float(eps), h_out.data_ptr(),
           y.data_ptr(), planes.data_ptr(), out.data_ptr(), workspace.data_ptr(), _stream())
    return h_out, y, planes


class ExpertPool:
    """Per-layer IQ3_S expert tensors resident on the device (model/moe.py:42-233)."""

    def __init__(self, gguf, n_layers: int, device: str = "cuda") -> None:
        self.device = device
        self.layers: list[IQ3SExperts] = []
        self._ws: torch.Tensor | None = None
        for i in range(n_layers):
            names = [f"blk.{i}.ffn_{n}_exps.weight" for n in ("gate", "up", "down")]
            shape, _ = gguf.tensor_info(names[0])  # (n_experts, ffn, hidden), outermost first
            n_exp, ffn, hidden = shape
            raws = [gguf.raw(n) for n in names]
            self.layers.append(IQ3SExperts.from_gguf_bytes(*raws, n_exp, hidden, ffn, device))

    @classmethod
    def from_layers(cls, layers: list[IQ3SExperts], device: str = "cuda") -> ExpertPool:
        pool = cls.__new__(cls)
        pool.device, pool.layers, pool._ws = device, list(layers), None
        return pool

    def forward(self, i: int, gguf, x: torch.Tensor, routing: RouterOutput) -> torch.Tensor:
        """Routed expert output for one token (``gguf`` is accepted for the
        reference's signature and unused: the experts are on the device)."""
        return self.forward_batch(i, x.reshape(1, -1), routing.expert_ids.reshape(1, -1),
                                  routing.weights.reshape(1, -1))[0]

    def forward_batch(self, i: int, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
        ex = self.layers[i]
        t, k = x.reshape(-1, ex.hidden).shape[0], ids.reshape(x.reshape(-1, ex.hidden).shape[0], -1).shape[1]
        need = int(N.load().bt_moe_workspace_bytes(t, ex.hidden, ex.ffn, ex.n_experts, k))
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.zeros(need, dtype=torch.uint8, device=x.device)
        return experts_forward(ex, x, ids, weights, self._ws)


__all__ = ["ExpertPool", "IQ3SExperts", "RouterOutput", "SharedExpert", "experts_forward", "moe_forward", "route",
           "route_logits"]

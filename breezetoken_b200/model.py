"""Qwen3.5 on the B200 backend: load, decode step, CUDA-graph greedy loop.

API mirrors the reference's ``Qwen35`` (breezetoken/model/qwen35.py:36-433):
``forward_token``, ``reset``, ``generate_stream``, ``generate``, ``warmup``,
``close``, ``cfg`` and ``placement``, with the same validation errors.  The
per-token work is one call of the library's fused decode step
(``bt_qwen35_step``); greedy decoding replays a natively captured CUDA graph
whose token id and position live in device memory, exactly like the
reference's ``GraphMixin`` (model/graph.py), so the host only reads the
token back.  ``decode_greedy`` goes further and replays ``n`` steps without
any host synchronisation in between.

Weights stay Q8_0 on the device (repacked to the library's q8-row layout):
``[qkv | z | alpha | beta]`` and ``[q | k | v]`` are concatenated, gate/up
rows interleaved, the tied embedding is the head.  Activations, the KV cache
and the GDN state are f32, as in the reference's torch path.  ``batch``
sequences (1, 2, 4 or 8) decode in lock-step on one GPU.
"""

from __future__ import annotations

import ctypes as C
import threading
from collections.abc import Iterator, Sequence
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

from breezetoken_b200 import _native as N
from breezetoken_b200.backends import Q8Weight, resolve_device
from breezetoken_b200.gguf import GGML_F32, GGML_Q8_0, GGUFFile
from breezetoken_b200.planner import Placement, plan

_DEFAULT_CONTEXT = 8192


@dataclass(frozen=True)
class Qwen35Config:
    """model/config.py:15-97, read from the same GGUF keys."""

    hidden: int
    n_layers: int
    n_heads: int
    n_kv: int
    head_dim: int
    rope_dim: int
    rope_theta: float
    ffn: int
    vocab: int
    eps: float
    l2_eps: float
    ssm_inner: int
    ssm_state: int
    ssm_heads: int
    conv_k: int
    full_attention_interval: int
    context_length: int
    max_context: int

    @property
    def attn_layers(self) -> tuple[int, ...]:
        return tuple(i for i in range(self.n_layers) if (i + 1) % self.full_attention_interval == 0)

    @classmethod
    def from_gguf(cls, gguf: GGUFFile, max_context: int | None = None) -> Qwen35Config:
        md = gguf.metadata
        n_heads = int(md["qwen35.attention.head_count"])
        head_dim = int(md.get("qwen35.attention.key_length", int(md["qwen35.embedding_length"]) // n_heads))
        n_layers = int(md["qwen35.block_count"]) - int(md.get("qwen35.nextn_predict_layers", 0))
        context_length = int(md.get("qwen35.context_length", _DEFAULT_CONTEXT))
        requested = _DEFAULT_CONTEXT if max_context is None else int(max_context)
        if requested <= 0:
            raise ValueError("max_context must be positive")
        context = min(context_length, requested) if context_length > 0 else requested
        cfg = cls(
            hidden=int(md["qwen35.embedding_length"]),
            n_layers=n_layers,
            n_heads=n_heads,
            n_kv=int(md["qwen35.attention.head_count_kv"]),
            head_dim=head_dim,
            rope_dim=int(md.get("qwen35.rope.dimension_count", head_dim)),
            rope_theta=float(md["qwen35.rope.freq_base"]),
            ffn=int(md["qwen35.feed_forward_length"]),
            vocab=int(gguf.tensor_layout("token_embd.weight")[0][0]),
            eps=float(md.get("qwen35.attention.layer_norm_rms_epsilon", 1e-6)),
            l2_eps=1e-6,
            ssm_inner=int(md["qwen35.ssm.inner_size"]),
            ssm_state=int(md["qwen35.ssm.state_size"]),
            ssm_heads=int(md["qwen35.ssm.group_count"]),
            conv_k=int(md["qwen35.ssm.conv_kernel"]),
            full_attention_interval=int(md.get("qwen35.full_attention_interval", 4)),
            context_length=context_length,
            max_context=context,
        )
        cfg.validate()
        return cfg

    def validate(self) -> None:
        if self.n_layers <= 0:
            raise ValueError("n_layers must be positive")
        if self.full_attention_interval <= 0 or not self.attn_layers:
            raise ValueError("model has no full-attention layers")
        if self.rope_dim <= 0 or self.rope_dim > self.head_dim or self.rope_dim % 2:
            raise ValueError(f"invalid rope_dim {self.rope_dim}")
        if not 0 < self.max_context <= self.context_length:
            raise ValueError(f"max_context {self.max_context} outside (0, {self.context_length}]")
        if self.n_heads % self.n_kv:
            raise ValueError("n_heads must be divisible by n_kv")
        if self.ssm_heads * self.ssm_state != self.ssm_inner:
            raise ValueError("ssm group_count * state_size must equal ssm.inner_size")


def rope_tables(cfg: Qwen35Config, cap: int) -> tuple[torch.Tensor, torch.Tensor]:
    """model/layers.py:26-32, computed with the same torch f32 CPU ops."""
    half = cfg.rope_dim // 2
    inv = cfg.rope_theta ** (-torch.arange(0, half, dtype=torch.float32) / half)
    phases = torch.outer(torch.arange(cap, dtype=torch.float32), inv)
    freqs = torch.cat((phases, phases), dim=-1)
    return freqs.cos(), freqs.sin()


class Qwen35:
    """A Qwen3.5 decoder resident on one B200."""

    def __init__(
        self,
        gguf: GGUFFile | str | Path,
        *,
        backend: str = "b200",
        device: str = "cuda",
        dtype: str | torch.dtype | None = None,
        max_context: int | None = None,
        batch: int = 1,
    ) -> None:
        if backend not in ("auto", "b200"):
            raise ValueError(f"unknown backend {backend!r}")
        own = not isinstance(gguf, GGUFFile)
        g = GGUFFile(gguf) if own else gguf
        try:
            if g.arch != "qwen35":
                raise NotImplementedError(f"{g.arch} is not a qwen35 GGUF")
            for name in g.tensor_names():
                if g.tensor_layout(name)[1] not in (GGML_F32, GGML_Q8_0):
                    raise NotImplementedError(f"{name}: only f32/q8_0 tensors are supported")
            self.cfg = Qwen35Config.from_gguf(g, max_context)
            if batch not in (1, 2, 4, 8):
                raise ValueError(f"batch must be 1, 2, 4 or 8, got {batch}")
            self.batch = batch
            self.device = resolve_device(device if device != "auto" else "cuda")
            self.dtype = torch.float32
            self.lib = N.load()
            with torch.cuda.device(torch.device(self.device)):
                self.stream = torch.cuda.Stream()
                with torch.cuda.stream(self.stream):
                    self._load(g)
                    self._alloc()
                self.stream.synchronize()
        finally:
            if own:
                g.close()
        cfg = self.cfg
        self.placement = plan(cfg, max_context=cfg.max_context, batch=batch, n_gpus=1)
        self._graphs: dict[int, int] = {}
        self._lock = threading.Lock()

    # ------------------------------------------------------------------ load
    def _q8(self, g: GGUFFile, names: list[str], step: int = 1) -> Q8Weight:
        """Repack one or more GGUF Q8_0 matrices with the same K into one Q8Weight.

        step=1 concatenates rows; step=2 with two names interleaves them."""
        shapes = [g.tensor_layout(n)[0] for n in names]
        k = shapes[0][1]
        if any(s[1] != k for s in shapes):
            raise ValueError(f"cannot fuse {names}: inner dims differ")
        n_total = sum(s[0] for s in shapes)
        w = Q8Weight.empty(n_total, k, self.device)
        row0 = 0
        for j, (name, s) in enumerate(zip(names, shapes, strict=True)):
            if step == 1:
                w.load_gguf_rows(g.raw(name), s[0], row0, 1)
                row0 += s[0]
            else:
                w.load_gguf_rows(g.raw(name), s[0], j, step)
        return w

    def _f32(self, g: GGUFFile, name: str) -> torch.Tensor:
        return torch.from_numpy(np.array(g.f32(name))).to(self.device)

    def _load(self, g: GGUFFile) -> None:
        cfg = self.cfg
        self.embed = self._q8(g, ["token_embd.weight"])
        if self.embed.shape != (cfg.hidden, cfg.vocab):
            raise ValueError(f"token_embd shape {self.embed.shape} != {(cfg.hidden, cfg.vocab)}")
        attn = set(cfg.attn_layers)
        self.layers: list[dict] = []
        for i in range(cfg.n_layers):
            p = f"blk.{i}."
            L = {
                "norm_in": self._f32(g, p + "attn_norm.weight"),
                "norm_post": self._f32(g, p + "post_attention_norm.weight"),
                "w_gu": self._q8(g, [p + "ffn_gate.weight", p + "ffn_up.weight"], step=2),
                "w_down": self._q8(g, [p + "ffn_down.weight"]),
            }
            if i in attn:
                L["w_in"] = self._q8(g, [p + "attn_q.weight", p + "attn_k.weight", p + "attn_v.weight"])
                L["w_out"] = self._q8(g, [p + "attn_output.weight"])
                L["q_norm"] = self._f32(g, p + "attn_q_norm.weight")
                L["k_norm"] = self._f32(g, p + "attn_k_norm.weight")
                expect_in = 2 * cfg.n_heads * cfg.head_dim + 2 * cfg.n_kv * cfg.head_dim
                expect_out = (cfg.n_heads * cfg.head_dim, cfg.hidden)
            else:
                L["w_in"] = self._q8(
                    g, [p + "attn_qkv.weight", p + "attn_gate.weight", p + "ssm_alpha.weight", p + "ssm_beta.weight"]
                )
                L["w_out"] = self._q8(g, [p + "ssm_out.weight"])
                L["conv_w"] = self._f32(g, p + "ssm_conv1d.weight").contiguous()
                L["a_log"] = self._f32(g, p + "ssm_a")
                L["dt_bias"] = self._f32(g, p + "ssm_dt.bias")
                L["ssm_norm"] = self._f32(g, p + "ssm_norm.weight")
                expect_in = 4 * cfg.ssm_inner + 2 * cfg.ssm_heads
                expect_out = (cfg.ssm_inner, cfg.hidden)
                if tuple(L["conv_w"].shape) != (3 * cfg.ssm_inner, cfg.conv_k):
                    raise ValueError(f"blk.{i}.ssm_conv1d shape {tuple(L['conv_w'].shape)}")
            checks = {
                "w_in": (cfg.hidden, expect_in),
                "w_out": expect_out,
                "w_gu": (cfg.hidden, 2 * cfg.ffn),
                "w_down": (cfg.ffn, cfg.hidden),
            }
            for key, shape in checks.items():
                if L[key].shape != shape:
                    raise ValueError(f"blk.{i}.{key}: expected {shape}, got {L[key].shape}")
            self.layers.append(L)
        norm_f = self._f32(g, "output_norm.weight")
        for i, L in enumerate(self.layers):
            L["norm_next"] = self.layers[i + 1]["norm_in"] if i + 1 < cfg.n_layers else norm_f
        self.norm_f = norm_f
        cos, sin = rope_tables(cfg, cfg.max_context)
        self.rope_cos, self.rope_sin = cos.to(self.device), sin.to(self.device)
        self.weight_bytes = self.embed.data.numel() + sum(
            L[k].data.numel() for L in self.layers for k in ("w_in", "w_out", "w_gu", "w_down")
        )

    def _alloc(self) -> None:
        cfg, B, dev = self.cfg, self.batch, self.device
        f32 = dict(dtype=torch.float32, device=dev)
        d = N.BtQwen35Dims(
            hidden=cfg.hidden, n_layers=cfg.n_layers, n_heads=cfg.n_heads, n_kv=cfg.n_kv, head_dim=cfg.head_dim,
            rope_dim=cfg.rope_dim, ffn=cfg.ffn, vocab=cfg.vocab, ssm_inner=cfg.ssm_inner, ssm_state=cfg.ssm_state,
            ssm_heads=cfg.ssm_heads, conv_k=cfg.conv_k, max_ctx=cfg.max_context, batch=B, eps=cfg.eps,
            l2_eps=cfg.l2_eps,
        )
        self._dims = d
        proj = int(self.lib.bt_qwen35_proj_elems(C.byref(d)))
        mix = max(cfg.ssm_inner, cfg.n_heads * cfg.head_dim)
        self.pos = torch.zeros(B, dtype=torch.int32, device=dev)
        self.token = torch.zeros(B, dtype=torch.int32, device=dev)
        self.history = torch.zeros(B, cfg.max_context, dtype=torch.int32, device=dev)
        self.logits = torch.zeros(B, cfg.vocab, **f32)
        self.h = (torch.zeros(B, cfg.hidden, **f32), torch.zeros(B, cfg.hidden, **f32))
        self.delta = torch.zeros(B, cfg.hidden, **f32)
        self.proj = torch.zeros(B, proj, **f32)
        self.mix = torch.zeros(B, mix, **f32)
        self.act = torch.zeros(B, 2 * cfg.ffn, **f32)
        self.workspace = torch.zeros(int(self.lib.bt_qwen35_workspace_bytes(C.byref(d))), dtype=torch.uint8, device=dev)
        self.status = torch.zeros(N.BT_STATUS_WORDS, dtype=torch.int32, device=dev)
        attn = set(cfg.attn_layers)
        kv = cfg.n_kv * cfg.head_dim
        layer_structs = (N.BtQwen35Layer * cfg.n_layers)()
        for i, L in enumerate(self.layers):
            if i in attn:
                L["k_cache"] = torch.zeros(B, cfg.max_context, kv, **f32)
                L["v_cache"] = torch.zeros(B, cfg.max_context, kv, **f32)
            else:
                L["conv_state"] = torch.zeros(B, 3 * cfg.ssm_inner, cfg.conv_k - 1, **f32)
                L["rec_state"] = torch.zeros(B, cfg.ssm_heads, cfg.ssm_state, cfg.ssm_state, **f32)
            s = layer_structs[i]
            s.is_attn = 1 if i in attn else 0
            for key in ("norm_in", "norm_post", "norm_next", "conv_w", "a_log", "dt_bias", "ssm_norm", "q_norm",
                        "k_norm", "conv_state", "rec_state", "k_cache", "v_cache"):
                if key in L:
                    setattr(s, key, L[key].data_ptr())
            for key in ("w_in", "w_out", "w_gu", "w_down"):
                setattr(s, key, L[key].data.data_ptr())
        self._layer_structs = layer_structs
        self._model = N.BtQwen35Model(
            dims=d, embed=self.embed.data.data_ptr(), rope_cos=self.rope_cos.data_ptr(),
            rope_sin=self.rope_sin.data_ptr(), layers=C.cast(layer_structs, C.POINTER(N.BtQwen35Layer)),
        )
        self._rt = N.BtQwen35Runtime(
            pos=self.pos.data_ptr(), token=self.token.data_ptr(), history=self.history.data_ptr(),
            logits=self.logits.data_ptr(), h0=self.h[0].data_ptr(), h1=self.h[1].data_ptr(),
            delta=self.delta.data_ptr(), proj=self.proj.data_ptr(), mix=self.mix.data_ptr(), act=self.act.data_ptr(),
            workspace=self.workspace.data_ptr(), status=self.status.data_ptr(),
        )

    # ------------------------------------------------------------------ step
    def _sid(self) -> int:
        return self.stream.cuda_stream

    def _check_status(self) -> None:
        rec = self.status.cpu().tolist()
        if rec[0]:
            self.status.zero_()
            raise N.B200Error(rec[0], f"device-side check failed: {N.describe_status(rec)}")

    def step(self, with_logits: bool = True) -> None:
        """Enqueue one decode step on the model's stream (no host sync)."""
        N.check(
            self.lib.bt_qwen35_step(C.byref(self._model), C.byref(self._rt), 1 if with_logits else 0, self._sid()),
            "bt_qwen35_step",
        )

    def set_inputs(self, tokens: Sequence[int], positions: Sequence[int]) -> None:
        """Set the device token ids and positions of every sequence."""
        with torch.cuda.stream(self.stream):
            self.token.copy_(torch.tensor(list(tokens), dtype=torch.int32), non_blocking=False)
            self.pos.copy_(torch.tensor(list(positions), dtype=torch.int32), non_blocking=False)

    @torch.inference_mode()
    def forward_token(self, token: int, pos: int, *, logits: bool = True):
        """qwen35.py:252-286: consume one token at ``pos``; f32 logits or None."""
        cfg = self.cfg
        if not 0 <= pos < cfg.max_context:
            raise ValueError(f"position {pos} outside [0, {cfg.max_context})")
        if token < 0 or token >= cfg.vocab:
            raise ValueError(f"token {token} out of range [0, {cfg.vocab})")
        self.set_inputs([token] * self.batch, [pos] * self.batch)
        with torch.cuda.stream(self.stream):
            self.step(with_logits=logits)
            out = self.logits[0].clone() if logits else None
        self.stream.synchronize()
        self._check_status()
        return out

    def reset(self) -> None:
        """qwen35.py:288-292: zero the GDN states (KV rows are overwritten before use)."""
        with torch.cuda.stream(self.stream):
            for L in self.layers:
                if "rec_state" in L:
                    L["conv_state"].zero_()
                    L["rec_state"].zero_()
            self.history.zero_()

    # ------------------------------------------------------------- snapshots
    def snapshot(self) -> dict[str, torch.Tensor]:
        """Copy of every piece of per-sequence state (positions, tokens, caches,
        GDN states) so a decode can be re-run from this point."""
        upto = int(self.pos.max().item())
        snap: dict[str, torch.Tensor] = {"_upto": torch.tensor(upto)}
        with torch.cuda.stream(self.stream):
            for name in ("pos", "token", "history"):
                snap[name] = getattr(self, name).clone()
            for i, L in enumerate(self.layers):
                for key in ("conv_state", "rec_state"):
                    if key in L:
                        snap[f"{i}.{key}"] = L[key].clone()
                for key in ("k_cache", "v_cache"):
                    if key in L:
                        snap[f"{i}.{key}"] = L[key][:, :upto].clone()
        self.stream.synchronize()
        return snap

    def restore(self, snap: dict[str, torch.Tensor]) -> None:
        """Enqueue device copies that put the state back to ``snap`` (no host sync)."""
        upto = int(snap["_upto"])
        with torch.cuda.stream(self.stream):
            for name in ("pos", "token", "history"):
                getattr(self, name).copy_(snap[name], non_blocking=True)
            for i, L in enumerate(self.layers):
                for key in ("conv_state", "rec_state"):
                    if key in L:
                        L[key].copy_(snap[f"{i}.{key}"], non_blocking=True)
                for key in ("k_cache", "v_cache"):
                    if key in L:
                        L[key][:, :upto].copy_(snap[f"{i}.{key}"], non_blocking=True)

    def kernels_per_step(self) -> int:
        """Kernels one decode step launches: 5 per attention layer, 4 per GDN
        layer (in-projection and recurrence fused) or 5 where that fusion
        does not serve the shapes, plus the head."""
        return int(self.lib.bt_qwen35_kernels_per_step(C.byref(self._model)))

    def step_bytes(self, context: float) -> float:
        """Algorithmic HBM bytes of one decode step per sequence at attended length
        ``context``: every weight byte once (q8 rows incl. scales), the f32 norm /
        conv / SSM parameters, GDN recurrent and conv state read+write, and the
        f32 KV rows read (plus the new row written)."""
        cfg = self.cfg
        n_attn = len(cfg.attn_layers)
        n_gdn = cfg.n_layers - n_attn
        params = 4 * (cfg.hidden * (2 * cfg.n_layers + 1) + n_attn * 2 * cfg.head_dim
                      + n_gdn * (3 * cfg.ssm_inner * cfg.conv_k + 2 * cfg.ssm_heads + cfg.ssm_state))
        gdn_state = n_gdn * 2 * 4 * cfg.ssm_heads * cfg.ssm_state * cfg.ssm_state
        conv_state = n_gdn * 2 * 4 * 3 * cfg.ssm_inner * (cfg.conv_k - 1)
        kv = n_attn * 2 * 4 * cfg.n_kv * cfg.head_dim * context
        return float(self.weight_bytes + params + gdn_state + conv_state + kv)

    # ---------------------------------------------------------------- graph
    def _graph(self, n_steps: int) -> int:
        g = self._graphs.get(n_steps)
        if g is None:
            handle = C.c_void_p()
            self.stream.synchronize()
            N.check(
                self.lib.bt_qwen35_graph_create(
                    C.byref(self._model), C.byref(self._rt), n_steps, self._sid(), C.byref(handle)
                ),
                "bt_qwen35_graph_create",
            )
            g = handle.value
            self._graphs[n_steps] = g
        return g

    def trace_step(self, steps: int = 1) -> list[dict]:
        """Device-side timeline of the last of ``steps`` decode steps, replayed
        as one captured graph from the current state (which it advances).

        Returns one dict per launch: name, start (first CTA entry), entered
        (last CTA entry), released (last CTA past the dependency wait), ready (last CTA past its
        prologue) and end (last CTA exit), in microseconds from the step's
        first entry."""
        n = self.kernels_per_step()
        rec = torch.zeros(n, 8, dtype=torch.int64, device=self.device)
        n_attn = len(self.cfg.attn_layers)
        fused = n == 5 * n_attn + 4 * (self.cfg.n_layers - n_attn) + 1
        names = []
        for i in range(self.cfg.n_layers):
            if i in self.cfg.attn_layers:
                names += [f"{i}.attn_in", f"{i}.attention", f"{i}.attn_out"]
            elif fused:
                names += [f"{i}.gdn_fused", f"{i}.gdn_out"]
            else:
                names += [f"{i}.gdn_in", f"{i}.gdn_step", f"{i}.gdn_out"]
            names += [f"{i}.gate_up", f"{i}.down"]
        names.append("head")
        traced = N.BtQwen35Runtime.from_buffer_copy(self._rt)
        traced.trace = rec.data_ptr()
        handle = C.c_void_p()
        self.stream.synchronize()
        N.check(
            self.lib.bt_qwen35_graph_create(C.byref(self._model), C.byref(traced), 1, self._sid(), C.byref(handle)),
            "trace graph",
        )
        try:
            for _ in range(steps):
                with torch.cuda.stream(self.stream):
                    rec[:, [0, 2, 5]] = -1  # all ones: unsigned max for the *_min fields
                    rec[:, [1, 3, 4, 6, 7]] = 0
                    N.check(self.lib.bt_graph_launch(handle.value, self._sid()), "trace replay")
            self.stream.synchronize()
        finally:
            self.lib.bt_graph_destroy(handle.value)
        r = rec.cpu().numpy().view(np.uint64)
        t0 = int(r[:, 0].min())
        out = []
        for i, nm in enumerate(names):
            out.append({
                "name": nm,
                "start": (int(r[i, 0]) - t0) / 1e3,
                "entered": (int(r[i, 1]) - t0) / 1e3,
                "released": (int(r[i, 3]) - t0) / 1e3,
                "ready": (int(r[i, 4]) - t0) / 1e3,
                "loaded": (int(r[i, 7]) - t0) / 1e3 if r[i, 7] else None,
                "end": (int(r[i, 6]) - t0) / 1e3,
            })
        return out

    def replay(self, n_steps: int = 1) -> None:
        """Launch the captured n-step greedy graph (no host sync)."""
        N.check(self.lib.bt_graph_launch(self._graph(n_steps), self._sid()), "bt_graph_launch")

    def prefill(self, prompts: Sequence[Sequence[int]]) -> None:
        """Consume equal-length prompts token by token; leaves token = argmax of the last logits."""
        if len(prompts) != self.batch:
            raise ValueError(f"expected {self.batch} prompts, got {len(prompts)}")
        n = len(prompts[0])
        if n < 1 or any(len(p) != n for p in prompts):
            raise ValueError("prompts must be non-empty and of equal length")
        if n > self.cfg.max_context:
            raise ValueError("prompt longer than max_context")
        self.reset()
        for i in range(n):
            self.set_inputs([p[i] for p in prompts], [i] * self.batch)
            with torch.cuda.stream(self.stream):
                self.step(with_logits=(i == n - 1))

    @torch.inference_mode()
    def decode_greedy(self, prompts: Sequence[Sequence[int]], max_new: int, chunk: int = 16) -> list[list[int]]:
        """Greedy tokens for each prompt with no host sync between steps.

        Prefill, then replay a ``chunk``-step graph until ``max_new`` tokens
        exist; tokens accumulate in device memory and are read once."""
        n = len(prompts[0])
        if n + max_new > self.cfg.max_context:
            raise ValueError(f"prompt {n} + max_new {max_new} exceeds max_context {self.cfg.max_context}")
        self.prefill(prompts)
        # token produced by prefill is at history[n]; each replayed step adds one
        done = 1
        with torch.cuda.stream(self.stream):
            while done < max_new:
                take = min(chunk, max_new - done)
                if take == chunk:
                    self.replay(chunk)
                else:
                    for _ in range(take):
                        self.replay(1)
                done += take
        self.stream.synchronize()
        self._check_status()
        hist = self.history[:, n : n + max_new].cpu().tolist()
        return hist

    # ------------------------------------------------------------ generation
    def generate_stream(
        self,
        ids: Sequence[int],
        max_new: int,
        temperature: float = 0.0,
        *,
        top_p: float = 1.0,
        eos_ids: Sequence[int] = (),
        cancel: threading.Event | None = None,
        seed: int | None = None,
    ) -> Iterator[int]:
        """qwen35.py:320-402: yield generated ids until EOS, cancel or max_new."""
        if not ids:
            raise ValueError("prompt must contain at least one token")
        if max_new < 0:
            raise ValueError("max_new must be >= 0")
        if temperature < 0:
            raise ValueError("temperature must be >= 0")
        if not 0.0 < top_p <= 1.0:
            raise ValueError("top_p must be in (0, 1]")
        if len(ids) + max_new > self.cfg.max_context:
            raise ValueError(
                f"prompt {len(ids)} + max_new {max_new} exceeds max_context {self.cfg.max_context}"
            )
        if max_new == 0 or (cancel is not None and cancel.is_set()):
            return
        eos = frozenset(eos_ids)
        greedy = temperature == 0.0 and top_p == 1.0
        gen = None
        if not greedy and seed is not None:
            gen = torch.Generator(device=self.device)
            gen.manual_seed(int(seed))
        self.prefill([list(ids)] * self.batch)
        self.stream.synchronize()
        self._check_status()
        for step in range(max_new):
            if cancel is not None and cancel.is_set():
                return
            if greedy:
                nxt = int(self.token[0].item())
            else:
                nxt = self._sample(self.logits[0], temperature, top_p, gen)
            if nxt in eos:
                return
            yield nxt
            if step + 1 >= max_new or (cancel is not None and cancel.is_set()):
                return
            if greedy:
                with torch.cuda.stream(self.stream):
                    self.replay(1)
                self.stream.synchronize()
                self._check_status()
            else:
                self.forward_token(nxt, len(ids) + step, logits=True)

    @staticmethod
    def _sample(logits: torch.Tensor, temperature: float, top_p: float, generator) -> int:
        """qwen35.py:294-311."""
        if temperature <= 0.0:
            return int(logits.argmax())
        probs = torch.softmax(logits.float() / temperature, dim=-1)
        if top_p < 1.0:
            sp, si = torch.sort(probs, descending=True)
            cum = torch.cumsum(sp, dim=-1)
            sp = torch.where(cum - sp > top_p, 0.0, sp)
            probs = torch.zeros_like(probs).scatter_(0, si, sp)
            probs = probs / probs.sum()
        return int(torch.multinomial(probs, 1, generator=generator).item())

    def generate(self, ids: Sequence[int], max_new: int, temperature: float = 0.0, **kwargs) -> list[int]:
        return list(self.generate_stream(ids, max_new, temperature, **kwargs))

    def warmup(self) -> None:
        """qwen35.py:413-421: run one step and capture the one-step graph."""
        self.generate([0], 2, 0.0)
        self._graph(1)
        self.reset()

    def close(self) -> None:
        for g in self._graphs.values():
            self.lib.bt_graph_destroy(g)
        self._graphs.clear()

    def __del__(self) -> None:  # pragma: no cover - best effort
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass

    def __repr__(self) -> str:
        cfg = self.cfg
        return (
            f"Qwen35(hidden={cfg.hidden}, layers={cfg.n_layers}, attn={len(cfg.attn_layers)}, "
            f"max_context={cfg.max_context}, batch={self.batch}, backend=b200, weights=q8_0)"
        )


__all__ = ["Placement", "Qwen35", "Qwen35Config", "rope_tables"]

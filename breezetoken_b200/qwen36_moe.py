"""Qwen3.6-35B-A3B-shaped (qwen35moe) decoder on the B200 library.

Mirrors breezetoken/model/qwen36_moe.py: the same config keys, weight names
and orientation, and per-token math -- forward_token (:646-664), _attn
(:432-457), _gdn (:459-483), _moe (:634-642).  Every operation of the step
runs on this library's kernels, fused where one follows another: the
residual add, RMSNorm and bf16 plane split of each activation
(bt_add_rms_norm_planes); the projections (bf16 / f32 weight rows,
bt_linear_rows); the attention layer after its one stacked [q | gate, k, v]
projection (q/k norms, RoPE, KV writes, split-KV attention, sigmoid gate:
bt_attention_layer); the GDN mixer after its projections and short conv
(decay, gated delta rule, output norm and SiLU gate: bt_gdn_gated_scan);
routing, IQ3_S experts + shared expert and argmax.  Only the embedding row
gather and the graph's token/position bookkeeping are torch device ops.

B sequences decode in lockstep at one position (how the 35B-A3B benchmark's 64
sequences per GPU run).  prefill() consumes the B prompts in chunks of
several tokens per sequence (the batched prefill of _prefill_batch,
:588-612): projections, norms and MoE layers run once per chunk, the conv,
the GDN recurrence (bt_gdn_gated_scan, state on chip across the chunk) and
attention go through the chunk's tokens in order.  Its arithmetic is the
per-token path's f32 (the reference's batched prefill rounds the expert
inputs and weights to bf16, _moe_batch :536-586; this one does not), so a
chunked prefill and a token-by-token one agree to f32 rounding.  generate()
feeds its prompt token by token like forward_token.  Everything raises on an
unsupported shape or a missing library.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass

import numpy as np
import torch

from breezetoken_b200 import _native as N
from breezetoken_b200.backends import B200Backend, _stream, resolve_device
from breezetoken_b200.gguf import GGML_BF16, GGML_F32, GGUFFile
from breezetoken_b200.moe import IQ3SExperts, SharedExpert, moe_forward, route_logits, route_sort
from breezetoken_b200.upload import Uploader


@dataclass(frozen=True)
class Qwen36Config:
    """model/qwen36_moe.py Qwen36Config (from the qwen35moe GGUF metadata)."""

    hidden: int
    n_layers: int
    n_heads: int
    n_kv: int
    head_dim: int
    rope_dim: int
    rope_theta: float
    max_context: int
    n_experts: int
    top_k: int
    expert_ffn: int
    shared_ffn: int
    gdn_key_heads: int
    gdn_value_heads: int
    gdn_k_dim: int
    gdn_inner: int
    gdn_conv: int
    vocab: int
    eps: float
    l2_eps: float = 1e-6

    @property
    def attn_layers(self) -> tuple[int, ...]:
        return tuple(i for i in range(self.n_layers) if (i + 1) % 4 == 0)

    @property
    def conv_dim(self) -> int:
        return 2 * self.gdn_key_heads * self.gdn_k_dim + self.gdn_inner

    @property
    def gdn_value_dim(self) -> int:
        return self.gdn_inner // self.gdn_value_heads

    @classmethod
    def from_spec(cls, spec, max_context: int) -> Qwen36Config:
        """The configuration of a breezetoken_b200.synth.Qwen36Spec shape."""
        return cls(
            hidden=spec.hidden, n_layers=spec.n_layers, n_heads=spec.n_heads, n_kv=spec.n_kv,
            head_dim=spec.head_dim, rope_dim=spec.rope_dim, rope_theta=spec.rope_theta, max_context=max_context,
            n_experts=spec.n_experts, top_k=spec.top_k, expert_ffn=spec.expert_ffn, shared_ffn=spec.shared_ffn,
            gdn_key_heads=spec.gdn_key_heads, gdn_value_heads=spec.gdn_value_heads, gdn_k_dim=spec.gdn_dim,
            gdn_inner=spec.gdn_inner, gdn_conv=spec.conv_k, vocab=spec.vocab, eps=spec.eps,
        )

    @classmethod
    def from_gguf(cls, gguf: GGUFFile, max_context: int | None = None) -> Qwen36Config:
        md = gguf.metadata
        a = "qwen35moe."
        ctx = int(md.get(a + "context_length", 262144))
        want = 8192 if max_context is None else int(max_context)
        if want <= 0:
            raise ValueError("max_context must be positive")
        return cls(
            hidden=int(md[a + "embedding_length"]),
            n_layers=int(md[a + "block_count"]) - int(md.get(a + "nextn_predict_layers", 0)),
            n_heads=int(md[a + "attention.head_count"]),
            n_kv=int(md[a + "attention.head_count_kv"]),
            head_dim=int(md[a + "attention.key_length"]),
            rope_dim=int(md.get(a + "rope.dimension_count", 64)),
            rope_theta=float(md.get(a + "rope.freq_base", 1.0e7)),
            max_context=min(ctx, want),
            n_experts=int(md[a + "expert_count"]),
            top_k=int(md[a + "expert_used_count"]),
            expert_ffn=int(md[a + "expert_feed_forward_length"]),
            shared_ffn=int(md[a + "expert_shared_feed_forward_length"]),
            gdn_key_heads=int(md[a + "ssm.group_count"]),
            gdn_value_heads=int(md[a + "ssm.inner_size"]) // int(md[a + "ssm.state_size"]),
            gdn_k_dim=int(md[a + "ssm.state_size"]),
            gdn_inner=int(md[a + "ssm.inner_size"]),
            gdn_conv=int(md[a + "ssm.conv_kernel"]),
            vocab=int(gguf.tensor_info("token_embd.weight")[0][0]),
            eps=float(md.get(a + "attention.layer_norm_rms_epsilon", 1e-6)),
        )


def rope_tables(cfg: Qwen36Config) -> tuple[torch.Tensor, torch.Tensor]:
    """model/qwen36_moe.py:226-229 on the CPU in f32, widened to the full
    rotary width (cos | cos, sin | sin) the RoPE kernel reads."""
    half = cfg.rope_dim // 2
    inv = cfg.rope_theta ** (-torch.arange(0, half, dtype=torch.float32) / half)
    phases = torch.outer(torch.arange(cfg.max_context, dtype=torch.float32), inv)
    cos, sin = phases.cos(), phases.sin()
    return torch.cat([cos, cos], 1).contiguous(), torch.cat([sin, sin], 1).contiguous()


class Qwen36Moe:
    """A loaded qwen35moe decoder: ``forward_token`` / ``generate`` keep the
    reference's names and argument meaning; ``decode_batch`` steps B
    sequences together."""

    def __init__(self, gguf: GGUFFile | str, *, device: str = "cuda", max_context: int | None = None,
                 batch: int = 1) -> None:
        own = not isinstance(gguf, GGUFFile)
        g = GGUFFile(gguf) if own else gguf
        try:
            self.cfg = Qwen36Config.from_gguf(g, max_context)
            self.device = resolve_device(device)
            self.batch = int(batch)
            self._load(g)
        finally:
            if own:
                g.close()
        self._alloc()

    # ------------------------------------------------------------------ load
    def _rows(self, g: GGUFFile, name: str) -> torch.Tensor:
        """A 2-D bf16 or f32 weight in its (out, in) orientation."""
        shape, ttype, _ = g.tensor_layout(name)
        if ttype not in (GGML_BF16, GGML_F32):
            raise ValueError(f"{name}: dense weights must be bf16 or f32")
        raw = self._up.to_device(g.raw(name))  # the mapped bytes, staged through pinned buffers
        return raw.view(torch.bfloat16 if ttype == GGML_BF16 else torch.float32).reshape(shape)

    def _vec(self, g: GGUFFile, name: str) -> torch.Tensor:
        return torch.from_numpy(np.array(g.f32(name))).to(self.device).contiguous()

    def _load(self, g: GGUFFile) -> None:
        self._up = Uploader(self.device)
        try:
            self._load_tensors(g)
        finally:
            self._up.close()
            del self._up

    def _load_tensors(self, g: GGUFFile) -> None:
        cfg = self.cfg
        self.embd = self._rows(g, "token_embd.weight")
        self.head = self._rows(g, "output.weight")
        self.norm_f = self._vec(g, "output_norm.weight")
        self.layers: list[dict] = []
        attn = set(cfg.attn_layers)
        for i in range(cfg.n_layers):
            p = f"blk.{i}."
            layer = {
                "norm_in": self._vec(g, p + "attn_norm.weight"),
                "norm_post": self._vec(g, p + "post_attention_norm.weight"),
                "router": self._rows(g, p + "ffn_gate_inp.weight").float().contiguous(),
                "experts": IQ3SExperts.from_gguf_bytes(
                    g.raw(p + "ffn_gate_exps.weight"), g.raw(p + "ffn_up_exps.weight"),
                    g.raw(p + "ffn_down_exps.weight"), cfg.n_experts, cfg.hidden, cfg.expert_ffn, self.device,
                    uploader=self._up),
                "shared": SharedExpert.from_tensors(
                    self._rows(g, p + "ffn_gate_shexp.weight"), self._rows(g, p + "ffn_up_shexp.weight"),
                    self._rows(g, p + "ffn_down_shexp.weight"), self._vec(g, p + "ffn_gate_inp_shexp.weight"),
                    self.device),
            }
            if i in attn:
                layer.update(
                    q=self._rows(g, p + "attn_q.weight"), k=self._rows(g, p + "attn_k.weight"),
                    v=self._rows(g, p + "attn_v.weight"), o=self._rows(g, p + "attn_output.weight"),
                    q_norm=self._vec(g, p + "attn_q_norm.weight"), k_norm=self._vec(g, p + "attn_k_norm.weight"),
                )
            else:
                layer.update(
                    qkv=self._rows(g, p + "attn_qkv.weight"), z=self._rows(g, p + "attn_gate.weight"),
                    out=self._rows(g, p + "ssm_out.weight"),
                    conv=self._vec(g, p + "ssm_conv1d.weight").reshape(cfg.conv_dim, cfg.gdn_conv),
                    w_alpha=self._rows(g, p + "ssm_alpha.weight").float().contiguous(),
                    w_beta=self._rows(g, p + "ssm_beta.weight").float().contiguous(),
                    a_log=self._vec(g, p + "ssm_a"), dt_bias=self._vec(g, p + "ssm_dt.bias"),
                    ssm_norm=self._vec(g, p + "ssm_norm.weight"),
                )
            self.layers.append(layer)

    @classmethod
    def random(cls, spec, *, batch: int, max_context: int, device: str = "cuda", seed: int = 4) -> Qwen36Moe:
        """A model of `spec`'s shape (breezetoken_b200.synth.Qwen36Spec) with
        seeded random weights built on the device, for throughput runs at
        sizes whose checkpoint would take minutes to write: bf16 projections
        and the f32 router N(0, 0.02); IQ3_S experts from random quant bytes
        with d = 2^-12 (weights of the magnitude an N(0, 0.02) quantisation
        gives); gammas 1 + N(0, 0.02); SSM parameters as in the synthetic
        checkpoints.  No reference output exists for it."""
        import math

        self = cls.__new__(cls)
        self.cfg = Qwen36Config.from_spec(spec, max_context)
        self.device, self.batch = resolve_device(device), int(batch)
        cfg, dev = self.cfg, self.device
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed)

        def normal(*shape, std=0.02, dtype=torch.bfloat16):
            return (torch.randn(*shape, generator=gen, device=dev) * std).to(dtype).contiguous()

        def uniform(*shape):
            return torch.rand(*shape, generator=gen, device=dev)

        def iq3s(rows: int, k: int) -> torch.Tensor:
            raw = torch.randint(0, 256, (rows * (k // 256), 110), generator=gen, device=dev, dtype=torch.uint8)
            raw[:, 0], raw[:, 1] = 0x00, 0x0C  # d = 2^-12 (fp16 0x0C00, little-endian)
            return IQ3SExperts._repack(raw.reshape(-1), rows, k, dev)

        self.embd = normal(cfg.vocab, cfg.hidden)
        self.head = normal(cfg.vocab, cfg.hidden)
        self.norm_f = 1 + normal(cfg.hidden, dtype=torch.float32)
        self.layers = []
        e, h, f, sf = cfg.n_experts, cfg.hidden, cfg.expert_ffn, cfg.shared_ffn
        for i in range(cfg.n_layers):
            layer = {
                "norm_in": 1 + normal(h, dtype=torch.float32), "norm_post": 1 + normal(h, dtype=torch.float32),
                "router": normal(e, h, dtype=torch.float32),
                "experts": IQ3SExperts(iq3s(e * f, h), iq3s(e * f, h), iq3s(e * h, f), e, h, f),
                "shared": SharedExpert(normal(sf, h), normal(sf, h), normal(h, sf), normal(h, dtype=torch.float32)),
            }
            if i in cfg.attn_layers:
                D = cfg.head_dim
                layer.update(q=normal(2 * cfg.n_heads * D, h), k=normal(cfg.n_kv * D, h), v=normal(cfg.n_kv * D, h),
                             o=normal(h, cfg.n_heads * D), q_norm=1 + normal(D, dtype=torch.float32),
                             k_norm=1 + normal(D, dtype=torch.float32))
            else:
                hv = cfg.gdn_value_heads
                dt = torch.exp(math.log(1e-3) + uniform(hv) * (math.log(1e-1) - math.log(1e-3)))
                layer.update(qkv=normal(cfg.conv_dim, h), z=normal(cfg.gdn_inner, h), out=normal(h, cfg.gdn_inner),
                             conv=normal(cfg.conv_dim, cfg.gdn_conv, std=0.25, dtype=torch.float32),
                             w_alpha=normal(hv, h, dtype=torch.float32), w_beta=normal(hv, h, dtype=torch.float32),
                             a_log=-torch.exp(uniform(hv) * math.log(16.0)), dt_bias=torch.log(torch.expm1(dt)),
                             ssm_norm=1 + normal(cfg.gdn_k_dim, dtype=torch.float32))
            self.layers.append(layer)
        self._alloc()
        return self

    def _alloc(self) -> None:
        cfg, b, dev = self.cfg, self.batch, self.device
        self.backend = B200Backend(dev)
        self.rope_cos, self.rope_sin = (t.to(dev) for t in rope_tables(cfg))
        self.kv = {i: (torch.zeros(b, cfg.max_context, cfg.n_kv, cfg.head_dim, device=dev),
                       torch.zeros(b, cfg.max_context, cfg.n_kv, cfg.head_dim, device=dev))
                   for i in cfg.attn_layers}
        dv = cfg.gdn_value_dim
        self.conv_state = {i: torch.zeros(b, cfg.conv_dim, cfg.gdn_conv - 1, device=dev)
                           for i in range(cfg.n_layers) if i not in self.kv}
        self.rec_state = {i: torch.zeros(b, cfg.gdn_value_heads, cfg.gdn_k_dim, dv, device=dev)
                          for i in self.conv_state}
        splits = self._splits()
        nbytes = int(N.load().bt_attention_workspace_bytes(b, cfg.n_kv, cfg.n_heads, cfg.head_dim, splits))
        self._attn_ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=dev)
        self._moe_ws = torch.zeros(int(N.load().bt_moe_layer_workspace_bytes(
            b, cfg.hidden, cfg.expert_ffn, cfg.shared_ffn, cfg.n_experts, cfg.top_k)), dtype=torch.uint8, device=dev)
        # the GDN layers' small projections run beside the qkv projection on
        # this stream (a parallel branch of the step's graph)
        self._side = torch.cuda.Stream(device=dev) if torch.device(dev).type == "cuda" else None
        for i in self.conv_state:  # beta and alpha rows stacked: one projection launch for both
            layer = self.layers[i]
            layer["w_ba"] = torch.cat([layer.pop("w_beta"), layer.pop("w_alpha")]).contiguous()
        for i in self.kv:  # [q | gate per head, k, v] rows stacked: one projection, the attention layer's input
            layer = self.layers[i]
            layer["qkv_all"] = torch.cat([layer.pop("q"), layer.pop("k"), layer.pop("v")]).contiguous()

    @property
    def placement(self):
        """planner.plan for this model on one GPU: context and device bytes
        (raises RuntimeError if the weights and B sequences' state do not fit)."""
        from breezetoken_b200.planner import plan

        return plan(self.cfg, max_context=self.cfg.max_context, batch=self.batch, n_gpus=1)

    def check_pipeline(self) -> None:
        """Raise if a bounded wait of the tensor-core projections gave up since
        the last check (their outputs after such a timeout are invalid).
        Synchronises the device."""
        n = int(N.load().bt_linear_rows_timeouts())
        if n != 0:
            raise N.B200Error(N.BT_ERR_TIMEOUT, f"{n} bounded waits of bt_linear_rows gave up: outputs are invalid")

    def _splits(self) -> int:
        """K/V splits of the attention layer: about 256 CTAs over the batch's
        (sequence, KV head) groups, a power of two, at most 16 and at most one
        per 64 positions of the context.  Measured on B200 at contexts 520-760
        (16 q / 2 KV heads x 256): 64 sequences 2 splits (81 us vs 103 with 3),
        32 sequences 4, 16 and 8 sequences 8 (the best of 1-8 splits)."""
        want = min(max(1, 256 // (self.batch * self.cfg.n_kv)), 16, self.cfg.max_context // 64)
        s = 1
        while s * 2 <= want:
            s *= 2
        return s

    def reset(self) -> None:
        for st in (*self.conv_state.values(), *self.rec_state.values()):
            st.zero_()

    def close(self) -> None:
        self._graph = None
        self.layers.clear()
        self.kv.clear()
        self.backend.close()

    # ------------------------------------------------------------------ ops
    def _planes(self, x: torch.Tensor) -> torch.Tensor:
        """x (T, K) f32 as the three bf16 planes the projections read (split
        once per activation, shared by every projection of it)."""
        x2 = x.float().reshape(x.shape[0], -1).contiguous()
        p = torch.empty(x2.shape[0], 3, x2.shape[1], dtype=torch.bfloat16, device=self.device)
        N.call("bt_bf16_planes", x2.data_ptr(), p.data_ptr(), x2.shape[0], x2.shape[1], _stream())
        return p

    def _lin(self, w: torch.Tensor, xp: torch.Tensor, y: torch.Tensor | None = None) -> torch.Tensor:
        """Planes xp (T, 3, K) -> (T, N) f32 through weight rows w (N, K)
        (into y when given)."""
        n, k = w.shape
        if xp.shape[-1] != k:
            raise ValueError(f"projection of {xp.shape[-1]} columns through a ({n}, {k}) weight")
        if y is None:
            y = torch.empty(xp.shape[0], n, dtype=torch.float32, device=self.device)
        dt = N.BT_BF16 if w.dtype == torch.bfloat16 else N.BT_F32
        N.call("bt_linear_rows", w.data_ptr(), dt, xp.data_ptr(), y.data_ptr(), n, k, xp.shape[0], _stream())
        return y

    def _norm_planes(self, a: torch.Tensor, b: torch.Tensor | None, gamma: torch.Tensor):
        """h = a + b (a alone when b is None), y = rms_norm(h) * gamma and y's
        bf16 planes, in one pass: (h, y, planes)."""
        rows, n = a.shape
        y = torch.empty(rows, n, dtype=torch.float32, device=self.device)
        planes = torch.empty(rows, 3, n, dtype=torch.bfloat16, device=self.device)
        h = torch.empty_like(y) if b is not None else a
        N.call("bt_add_rms_norm_planes", a.data_ptr(), None if b is None else b.data_ptr(), gamma.data_ptr(),
               None if b is None else h.data_ptr(), y.data_ptr(), planes.data_ptr(), rows, n,
               float(self.cfg.eps), _stream())
        return h, y, planes

    def _attn(self, i: int, xp: torch.Tensor, pos_t: torch.Tensor, steps: int = 1) -> torch.Tensor:
        """model/qwen36_moe.py:432-457: one projection of [q | gate, k, v], then
        q/k norms, RoPE at the device positions, the KV writes, attention and
        the sigmoid gate in one launch (bt_attention_layer) per token.

        With steps > 1 (a prefill chunk, model/qwen36_moe.py:394-430) xp holds
        steps * B token-major rows and pos_t (steps, B) their positions: the
        projections run once over the chunk, then one launch per token in
        order, each writing its K/V before the next token attends, which is
        the causal attention over the chunk and the cached prefix."""
        cfg, layer = self.cfg, self.layers[i]
        t, H, D = xp.shape[0], cfg.n_heads, cfg.head_dim
        b = t // steps
        proj = self._lin(layer["qkv_all"], xp)
        k_cache, v_cache = self.kv[i]
        out = torch.empty(t, H, D, dtype=torch.float32, device=self.device)
        pos_t = pos_t.reshape(steps, b)
        for j in range(steps):
            N.call("bt_attention_layer", proj[j * b:].data_ptr(), proj.shape[1], layer["q_norm"].data_ptr(),
                   layer["k_norm"].data_ptr(), self.rope_cos.data_ptr(), self.rope_sin.data_ptr(), cfg.rope_dim,
                   pos_t[j].data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), out[j * b:].data_ptr(), b, H,
                   cfg.n_kv, D, cfg.max_context, float(D ** -0.5), float(cfg.eps), self._splits(),
                   self._attn_ws.data_ptr(), None, _stream())
        return self._lin(layer["o"], self._planes(out.reshape(t, -1)))

    def _gdn(self, i: int, xp: torch.Tensor, steps: int = 1) -> torch.Tensor:
        """model/qwen36_moe.py:459-483: the qkv projection and the short conv,
        the [beta | alpha] and z projections, then the decay, gated delta
        rule, output norm and SiLU gate in one launch (bt_gdn_gated_scan).

        With steps > 1 (a prefill chunk, model/qwen36_moe.py:485-534) xp holds
        steps * B token-major rows: the projections run once over the chunk,
        the conv and the recurrence scan each sequence's tokens in order
        (bt_conv_silu_scan, bt_gdn_gated_scan) with their state on chip."""
        cfg, layer = self.cfg, self.layers[i]
        t, hk, hv, dk = xp.shape[0], cfg.gdn_key_heads, cfg.gdn_value_heads, cfg.gdn_k_dim
        b, inner = t // steps, cfg.gdn_inner
        # [beta | alpha] and z on the side stream while the qkv projection and
        # the conv run (their outputs allocated here, on the main stream)
        ba = torch.empty(t, layer["w_ba"].shape[0], dtype=torch.float32, device=self.device)
        z = torch.empty(t, layer["z"].shape[0], dtype=torch.float32, device=self.device)
        side = self._side
        if side is not None:
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                self._lin(layer["w_ba"], xp, ba)
                self._lin(layer["z"], xp, z)
        entry = self._lin(layer["qkv"], xp)  # (T, C)
        mixed = torch.empty_like(entry)
        N.call("bt_conv_silu_scan", entry.data_ptr(), self.conv_state[i].data_ptr(), layer["conv"].data_ptr(),
               mixed.data_ptr(), steps, b, cfg.conv_dim, cfg.gdn_conv, _stream())
        if side is None:
            self._lin(layer["w_ba"], xp, ba)
            self._lin(layer["z"], xp, z)
        else:
            torch.cuda.current_stream().wait_stream(side)
        gated = torch.empty(t, 3, inner, dtype=torch.bfloat16, device=self.device)
        N.call("bt_gdn_gated_scan", mixed.data_ptr(), mixed.shape[1], ba.data_ptr(), 2 * hv,
               layer["a_log"].data_ptr(), layer["dt_bias"].data_ptr(), self.rec_state[i].data_ptr(), z.data_ptr(),
               inner, layer["ssm_norm"].data_ptr(), gated.data_ptr(), steps, b, hk, hv, dk, float(dk ** -0.5),
               float(cfg.l2_eps), float(cfg.eps), _stream())
        return self._lin(layer["out"], gated)

    def _moe(self, i: int, xn: torch.Tensor, xp: torch.Tensor, ws: torch.Tensor | None = None,
             norm: tuple | None = None):
        """model/qwen36_moe.py:634-642: routing, the IQ3_S experts and the
        shared expert; with norm = (h, gamma) fused with the residual add and
        the next RMSNorm + planes: (h, y, planes)."""
        layer = self.layers[i]
        ws = self._moe_ws if ws is None else ws
        chained = norm is not None and self._side is not None
        if chained:
            # routing, the pairs' sort and the token encoding in one launch;
            # the layer's kernels follow it (and each other) with early launch
            r = route_sort(self._lin(layer["router"], xp), xn, self.cfg.top_k, layer["experts"], layer["shared"], ws)
        else:
            r = route_logits(self._lin(layer["router"], xp), self.cfg.top_k)
        rec = getattr(self, "_route_record", None)
        if rec is not None:  # measurement: each layer's input and routing of this (eager) step
            rec.append((xn.clone(), r.expert_ids.clone(), r.weights.clone()))
        return moe_forward(layer["experts"], layer["shared"], xn, r.expert_ids, r.weights, ws,
                           None if norm is None else (norm[0], norm[1], float(self.cfg.eps)),
                           prepared=chained)

    # ------------------------------------------------------------------ step
    def _step_t(self, tokens: torch.Tensor, pos_t: torch.Tensor, logits: bool, steps: int = 1,
                moe_ws: torch.Tensor | None = None) -> torch.Tensor | None:
        """One step with the positions as a device tensor (int32 (B,)): no
        host synchronisation, so it can be captured in a CUDA graph.  With
        steps > 1, `steps` tokens of each sequence at once (token-major
        tokens and positions, steps * B rows): a prefill chunk."""
        cfg = self.cfg
        h = self.embd[tokens.long()].float()
        attn = set(cfg.attn_layers)
        _, xn, xp = self._norm_planes(h, None, self.layers[0]["norm_in"])
        for i in range(cfg.n_layers):
            # each residual add runs fused with the norm that follows it
            # (h = h + delta, then rms_norm(h): the same f32 operations)
            layer = self.layers[i]
            delta = self._attn(i, xp, pos_t, steps) if i in attn else self._gdn(i, xp, steps)
            h, xn, xp = self._norm_planes(h, delta, layer["norm_post"])
            nxt = self.layers[i + 1]["norm_in"] if i + 1 < cfg.n_layers else self.norm_f
            h, xn, xp = self._moe(i, xn, xp, moe_ws, norm=(h, nxt))
        if not logits:
            return None
        return self._lin(self.head, xp)

    @torch.inference_mode()
    def _step(self, tokens: torch.Tensor, pos: int, logits: bool) -> torch.Tensor | None:
        cfg = self.cfg
        if not 0 <= pos < cfg.max_context:
            raise ValueError(f"position {pos} outside [0, {cfg.max_context})")
        if int(tokens.min()) < 0 or int(tokens.max()) >= cfg.vocab:
            raise ValueError("token id outside the vocabulary")
        return self._step_t(tokens, torch.full((self.batch,), pos, dtype=torch.int32, device=self.device), logits)

    # ------------------------------------------------------------ graphs
    @torch.inference_mode()
    def capture(self, history: int = 256) -> int:
        """Capture one decode step of the B sequences as a CUDA graph (once):
        it consumes the device token at the device position, writes the
        argmax token back, records it in a history ring of `history` steps and
        advances the position, with no host synchronisation.  Call an eager
        step first so that every lazily configured kernel is set up.  Returns
        the number of this library's kernels one replay launches."""
        if getattr(self, "_graph", None) is not None and self._hist.shape[1] >= history:
            return self.kernels_per_step
        b = self.batch
        self._tok = torch.zeros(b, dtype=torch.int64, device=self.device)
        self._pos = torch.zeros(b, dtype=torch.int32, device=self.device)
        self._n = torch.zeros(1, dtype=torch.int64, device=self.device)
        self._hist = torch.zeros(b, max(history, 1), dtype=torch.int64, device=self.device)
        self.backend._workspace(("argmax", b), int(N.load().bt_argmax_workspace_bytes(b)))
        lib = N.load()
        stream = torch.cuda.Stream(device=self.device)
        stream.wait_stream(torch.cuda.current_stream())
        self._graph = torch.cuda.CUDAGraph()
        before = int(lib.bt_launch_count())
        with torch.cuda.graph(self._graph, stream=stream):
            nxt = self.backend.argmax(self._step_t(self._tok, self._pos, True)).long()
            self._hist.index_copy_(1, self._n, nxt.unsqueeze(1))
            self._tok.copy_(nxt)
            self._pos.add_(1)
            self._n.add_(1).remainder_(self._hist.shape[1])
        self.kernels_per_step = int(lib.bt_launch_count()) - before
        return self.kernels_per_step

    @torch.inference_mode()
    def set_decode(self, tokens: torch.Tensor, pos: int) -> None:
        """The next replay consumes `tokens` (B,) at position `pos` (copies on
        the current stream; `tokens` may be pinned host memory)."""
        if tokens.numel() != self.batch:
            raise ValueError(f"expected {self.batch} tokens, got {tokens.numel()}")
        self._tok.copy_(tokens.reshape(-1), non_blocking=True)
        self._pos.fill_(pos)
        self._n.zero_()

    def replay(self, steps: int = 1) -> None:
        """`steps` graph replays on the current stream (no host sync)."""
        for _ in range(steps):
            self._graph.replay()

    @torch.inference_mode()
    def graph_decode(self, tokens: torch.Tensor, pos: int, steps: int) -> torch.Tensor:
        """`steps` greedy steps of the B sequences, the first feeding `tokens`
        at position `pos`, replayed from a CUDA graph of one step (token,
        position and the generated ids stay on the device; no host sync
        between steps).  Returns the generated ids (B, steps).  Call an eager
        step first so that every lazily configured kernel is set up."""
        cfg = self.cfg
        if tokens.numel() != self.batch:
            raise ValueError(f"expected {self.batch} tokens, got {tokens.numel()}")
        if not 0 <= pos or pos + steps > cfg.max_context:
            raise ValueError(f"positions {pos}..{pos + steps - 1} outside [0, {cfg.max_context})")
        self.capture(history=max(steps, 256))
        self.set_decode(tokens, pos)
        self.replay(steps)
        out = self._hist[:, :steps].clone()
        self.check_pipeline()
        return out

    # ----------------------------------------------------------- prefill
    @torch.inference_mode()
    def prefill_chunk(self) -> int:
        """Tokens per sequence that one prefill chunk carries: as many as keep
        the chunk's expert pairs within one MoE launch (T * top_k <= 4096)."""
        return max(1, 4096 // (self.cfg.top_k * self.batch))

    @torch.inference_mode()
    def prefill(self, prompts: torch.Tensor, chunk: int | None = None) -> None:
        """Consume prompts (B, L) at positions 0 .. L-1 in lockstep (no logits):
        the next step feeds each sequence's next token at position L.

        The batched prefill of model/qwen36_moe.py:588-612, in chunks of
        `chunk` tokens per sequence (default prefill_chunk()): each chunk runs
        every projection, norm and MoE layer once over its chunk * B tokens,
        and the conv, the GDN recurrence and attention scan the chunk's
        tokens in order (bt_conv_silu_scan, bt_gdn_gated_scan, one
        bt_attention_layer per token)."""
        if prompts.dim() != 2 or prompts.shape[0] != self.batch:
            raise ValueError(f"prompts must be ({self.batch}, L), got {tuple(prompts.shape)}")
        n = prompts.shape[1]
        if n > self.cfg.max_context:
            raise ValueError("prompt longer than max_context")
        if n and (int(prompts.min()) < 0 or int(prompts.max()) >= self.cfg.vocab):
            raise ValueError("token id outside the vocabulary")
        c = self.prefill_chunk() if chunk is None else int(chunk)
        if c < 1 or c * self.batch * self.cfg.top_k > 4096:
            raise ValueError(f"chunk must be in [1, {self.prefill_chunk()}] tokens per sequence")
        toks = prompts.to(self.device)
        ws = None
        if c > 1:
            need = int(N.load().bt_moe_layer_workspace_bytes(c * self.batch, self.cfg.hidden, self.cfg.expert_ffn,
                                                             self.cfg.shared_ffn, self.cfg.n_experts, self.cfg.top_k))
            ws = getattr(self, "_moe_ws_prefill", None)
            if ws is None or ws.numel() < need:
                ws = self._moe_ws_prefill = torch.zeros(need, dtype=torch.uint8, device=self.device)
        for j0 in range(0, n, c):
            s = min(c, n - j0)
            pos = torch.arange(j0, j0 + s, dtype=torch.int32, device=self.device)
            pos_t = pos[:, None].expand(s, self.batch).contiguous()
            self._step_t(toks[:, j0:j0 + s].t().reshape(-1), pos_t, False, s, ws)

    @torch.inference_mode()
    def snapshot(self) -> dict:
        """Device copies of every per-sequence state (KV caches, conv windows,
        recurrent states), for restore()."""
        return {"kv": {i: (k.clone(), v.clone()) for i, (k, v) in self.kv.items()},
                "conv": {i: t.clone() for i, t in self.conv_state.items()},
                "rec": {i: t.clone() for i, t in self.rec_state.items()}}

    @torch.inference_mode()
    def restore(self, snap: dict) -> None:
        """Put back a snapshot (device copies on the current stream)."""
        for i, (k, v) in snap["kv"].items():
            self.kv[i][0].copy_(k)
            self.kv[i][1].copy_(v)
        for i, t in snap["conv"].items():
            self.conv_state[i].copy_(t)
        for i, t in snap["rec"].items():
            self.rec_state[i].copy_(t)

    @torch.inference_mode()
    def record_routing(self, tokens: torch.Tensor, pos: int) -> list:
        """One eager step (the state advances as usual) that records each
        layer's MoE input and routing: [(xn (B, H), ids (B, k), weights (B, k))]."""
        self._route_record = []
        try:
            self._step(tokens.reshape(-1).to(self.device), pos, True)
            return self._route_record
        finally:
            self._route_record = None

    def forward_token(self, token: int, pos: int, *, logits: bool = True) -> torch.Tensor | None:
        """model/qwen36_moe.py:646-664 for sequence 0: (V,) f32 logits."""
        if self.batch != 1:
            raise ValueError("forward_token serves batch 1; use decode_batch")
        out = self._step(torch.tensor([token], device=self.device), pos, logits)
        return None if out is None else out[0]

    def decode_batch(self, tokens: torch.Tensor, pos: int) -> torch.Tensor:
        """One greedy step of the B sequences at position `pos`: next ids (B,) int32."""
        if tokens.numel() != self.batch:
            raise ValueError(f"expected {self.batch} tokens, got {tokens.numel()}")
        return self.backend.argmax(self._step(tokens.reshape(-1).to(self.device), pos, True))

    def generate(self, ids: Sequence[int], max_new: int) -> list[int]:
        """Greedy decode of one sequence (model/qwen36_moe.py:893-900 with
        temperature 0), the prompt fed token by token."""
        if not ids:
            raise ValueError("prompt must contain at least one token")
        self.reset()
        logits = None
        for i, t in enumerate(ids):
            logits = self.forward_token(int(t), i, logits=(i == len(ids) - 1))
        out: list[int] = []
        for step in range(max_new):
            nxt = int(self.backend.argmax(logits)[0])
            out.append(nxt)
            if step + 1 < max_new:
                logits = self.forward_token(nxt, len(ids) + step)
        self.check_pipeline()
        return out


__all__ = ["Qwen36Config", "Qwen36Moe", "rope_tables"]

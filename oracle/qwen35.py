"""Oracle Qwen3.5 decoder: numpy restatement of the reference's torch path.

Follows breezetoken/model/qwen35.py (load :166-219, forward_token :252-286,
generate_stream :320-402), model/layers.py (_embed :19-24, _attn :55-82,
_gdn :84-112, _mlp :114-119) and model/prefill.py (_prefill_batch
:128-151) with backend="torch", device="cpu": f32 weights dequantised from
Q8_0, f32 KV cache and recurrent state.  TEST INFRASTRUCTURE ONLY.
"""

from __future__ import annotations

import numpy as np

from oracle import ops
from oracle.gguf_io import OracleGGUF

F32 = np.float32


class Qwen35Oracle:
    def __init__(self, path, max_context: int = 8192) -> None:
        g = OracleGGUF(path)
        md = g.metadata
        self.n_heads = int(md["qwen35.attention.head_count"])
        self.head_dim = int(md.get("qwen35.attention.key_length", int(md["qwen35.embedding_length"]) // self.n_heads))
        self.n_layers = int(md["qwen35.block_count"]) - int(md.get("qwen35.nextn_predict_layers", 0))
        self.hidden = int(md["qwen35.embedding_length"])
        self.n_kv = int(md["qwen35.attention.head_count_kv"])
        self.rope_dim = int(md.get("qwen35.rope.dimension_count", self.head_dim))
        self.theta = float(md["qwen35.rope.freq_base"])
        self.ffn = int(md["qwen35.feed_forward_length"])
        self.eps = float(md.get("qwen35.attention.layer_norm_rms_epsilon", 1e-6))
        self.l2_eps = 1e-6
        self.inner = int(md["qwen35.ssm.inner_size"])
        self.state = int(md["qwen35.ssm.state_size"])
        self.hv = int(md["qwen35.ssm.group_count"])
        self.conv_k = int(md["qwen35.ssm.conv_kernel"])
        interval = int(md.get("qwen35.full_attention_interval", 4))
        ctx = int(md.get("qwen35.context_length", 8192))
        self.max_ctx = min(ctx, max_context) if ctx > 0 else max_context
        self.attn = frozenset(i for i in range(self.n_layers) if (i + 1) % interval == 0)

        # weights in the reference's (K, N) layout (qwen35.py:148-153)
        self.head = g.get("token_embd.weight").T.copy()  # (H, V)
        self.vocab = self.head.shape[1]
        self.layers = []
        for i in range(self.n_layers):
            p = f"blk.{i}."
            L = {
                "norm_in": g.get(p + "attn_norm.weight"),
                "norm_post": g.get(p + "post_attention_norm.weight"),
                "w_gu": np.concatenate([g.get(p + "ffn_gate.weight").T, g.get(p + "ffn_up.weight").T], axis=1),
                "w_down": g.get(p + "ffn_down.weight").T.copy(),
            }
            if i in self.attn:
                L["w_qkv_attn"] = np.concatenate(
                    [g.get(p + "attn_q.weight").T, g.get(p + "attn_k.weight").T, g.get(p + "attn_v.weight").T], axis=1
                )
                L["w_o"] = g.get(p + "attn_output.weight").T.copy()
                L["q_norm"] = g.get(p + "attn_q_norm.weight")
                L["k_norm"] = g.get(p + "attn_k_norm.weight")
            else:
                L["w_qkv"] = g.get(p + "attn_qkv.weight").T.copy()
                L["w_z"] = g.get(p + "attn_gate.weight").T.copy()
                L["conv"] = g.get(p + "ssm_conv1d.weight")
                L["w_alpha"] = g.get(p + "ssm_alpha.weight").T.copy()
                L["w_beta"] = g.get(p + "ssm_beta.weight").T.copy()
                L["a_log"] = g.get(p + "ssm_a")
                L["dt_bias"] = g.get(p + "ssm_dt.bias")
                L["w_out"] = g.get(p + "ssm_out.weight").T.copy()
                L["ssm_norm"] = g.get(p + "ssm_norm.weight")
            self.layers.append(L)
        norm_f = g.get("output_norm.weight")
        for i, L in enumerate(self.layers):
            L["norm_next"] = self.layers[i + 1]["norm_in"] if i + 1 < self.n_layers else norm_f
        self.cos, self.sin = ops.rope_tables(self.rope_dim, self.theta, self.max_ctx)
        self.reset()

    # ---------------------------------------------------------------- state
    def reset(self) -> None:
        """qwen35.py:288-292 (config.py:100-127 shapes)."""
        kv = self.n_kv * self.head_dim
        self.k_cache = {i: np.zeros((self.max_ctx, kv), F32) for i in self.attn}
        self.v_cache = {i: np.zeros((self.max_ctx, kv), F32) for i in self.attn}
        self.conv = {i: np.zeros((3 * self.inner, self.conv_k - 1), F32) for i in range(self.n_layers) if i not in self.attn}
        self.rec = {i: np.zeros((self.hv, self.state, self.state), F32) for i in range(self.n_layers) if i not in self.attn}

    # ---------------------------------------------------------------- layers
    def _attn(self, i: int, xn: np.ndarray, pos: int) -> np.ndarray:
        """layers.py:55-82."""
        L = self.layers[i]
        H, D, Hk = self.n_heads, self.head_dim, self.n_kv
        qkv = ops.linear(xn, L["w_qkv_attn"])
        qg = qkv[: H * 2 * D].reshape(H, 2 * D)
        q, gate = qg[:, :D], qg[:, D:]
        k = qkv[H * 2 * D : H * 2 * D + Hk * D].reshape(Hk, D)
        v = qkv[H * 2 * D + Hk * D :].reshape(Hk, D)
        q = ops.rope(ops.rms_norm(q, L["q_norm"], self.eps), self.cos, self.sin, pos, self.rope_dim)
        k = ops.rope(ops.rms_norm(k, L["k_norm"], self.eps), self.cos, self.sin, pos, self.rope_dim)
        self.k_cache[i][pos] = k.reshape(-1)
        self.v_cache[i][pos] = v.reshape(-1)
        seq = pos + 1
        out = ops.attention(
            q, self.k_cache[i][:seq].reshape(seq, Hk, D), self.v_cache[i][:seq].reshape(seq, Hk, D), D**-0.5
        )
        out = out * ops.sigmoid(gate)
        return ops.linear(out.reshape(-1), L["w_o"])

    def _gdn(self, i: int, xn: np.ndarray) -> np.ndarray:
        """layers.py:84-112."""
        L = self.layers[i]
        hv, dk = self.hv, self.state
        entry = ops.linear(xn, L["w_qkv"])
        window = np.concatenate([self.conv[i], entry.reshape(-1, 1)], axis=1)
        mixed = ops.silu((window * L["conv"]).sum(axis=-1, dtype=F32))
        self.conv[i][...] = window[:, 1:]
        q = mixed[: self.inner].reshape(hv, dk)
        k = mixed[self.inner : 2 * self.inner].reshape(hv, dk)
        v = mixed[2 * self.inner :].reshape(hv, dk)
        beta = ops.linear(xn, L["w_beta"]).reshape(hv)
        g = L["a_log"] * ops.softplus(ops.linear(xn, L["w_alpha"]) + L["dt_bias"]).reshape(hv)
        read = ops.gdn_decode(q, k, v, g, beta, self.rec[i], dk**-0.5, self.l2_eps)
        z = ops.linear(xn, L["w_z"]).reshape(hv, dk)
        gated = (ops.rms_norm(read, L["ssm_norm"], self.eps) * ops.silu(z)).reshape(-1)
        return ops.linear(gated, L["w_out"])

    def _mlp(self, i: int, xn: np.ndarray) -> np.ndarray:
        """layers.py:114-119."""
        L = self.layers[i]
        gu = ops.linear(xn, L["w_gu"])
        return ops.linear(ops.silu_mul(gu[: self.ffn], gu[self.ffn :]), L["w_down"])

    # ------------------------------------------------------------------ step
    def forward_token(self, token: int, pos: int, logits: bool = True):
        """qwen35.py:252-286."""
        if not 0 <= token < self.vocab:
            raise ValueError(f"token {token} out of range")
        if not 0 <= pos < self.max_ctx:
            raise ValueError(f"position {pos} outside [0, {self.max_ctx})")
        h = self.head[:, token].astype(F32).copy()
        xn = ops.rms_norm(h, self.layers[0]["norm_in"], self.eps)
        for i in range(self.n_layers):
            L = self.layers[i]
            mixer = self._attn(i, xn, pos) if i in self.attn else self._gdn(i, xn)
            h, xn1 = ops.fused_add_rms_norm(h, mixer, L["norm_post"], self.eps)
            h, xn = ops.fused_add_rms_norm(h, self._mlp(i, xn1), L["norm_next"], self.eps)
        if not logits:
            return None
        return ops.linear(xn, self.head)

    # --------------------------------------------------------------- prefill
    def prefill_batch(self, ids) -> np.ndarray:
        """prefill.py:128-151 (attention :41-79, GDN :81-116, MLP :118-125)."""
        S = len(ids)
        H, D, Hk = self.n_heads, self.head_dim, self.n_kv
        h = self.head[:, list(ids)].T.astype(F32).copy()
        xn = ops.rms_norm(h, self.layers[0]["norm_in"], self.eps)
        for i in range(self.n_layers):
            L = self.layers[i]
            if i in self.attn:
                qkv = xn @ L["w_qkv_attn"]
                qg = qkv[:, : H * 2 * D].reshape(S, H, 2 * D)
                q, gate = qg[..., :D], qg[..., D:]
                k = qkv[:, H * 2 * D : H * 2 * D + Hk * D].reshape(S, Hk, D)
                v = qkv[:, H * 2 * D + Hk * D :].reshape(S, Hk, D)
                q = ops.rms_norm(q, L["q_norm"], self.eps)
                k = ops.rms_norm(k, L["k_norm"], self.eps)
                half = self.rope_dim // 2
                c = self.cos[:S].reshape(S, 1, -1)
                s = self.sin[:S].reshape(S, 1, -1)

                def rb(x):
                    rot, tail = x[..., : self.rope_dim], x[..., self.rope_dim :]
                    turned = rot * c + np.concatenate([-rot[..., half:], rot[..., :half]], axis=-1) * s
                    return np.concatenate([turned, tail], axis=-1).astype(F32)

                q, k = rb(q), rb(k)
                self.k_cache[i][:S] = k.reshape(S, -1)
                self.v_cache[i][:S] = v.reshape(S, -1)
                grp = H // Hk
                out = np.empty((S, H, D), F32)
                for t in range(S):
                    out[t] = ops.attention(q[t], k[: t + 1], v[: t + 1], D**-0.5)
                out = out * ops.sigmoid(gate)
                mixer = out.reshape(S, H * D) @ L["w_o"]
                del grp
            else:
                hv, dk = self.hv, self.state
                entry = xn @ L["w_qkv"]  # (S, C)
                seq = np.concatenate([self.conv[i], entry.T], axis=1)  # (C, S+3)
                C = seq.shape[0]
                mixed = np.zeros((C, S), F32)
                for t in range(self.conv_k):
                    mixed += seq[:, t : t + S] * L["conv"][:, t : t + 1]
                mixed = ops.silu(mixed).T  # (S, C)
                self.conv[i][...] = seq[:, -(self.conv_k - 1) :]
                q = mixed[:, : self.inner].reshape(S, hv, dk)
                k = mixed[:, self.inner : 2 * self.inner].reshape(S, hv, dk)
                v = mixed[:, 2 * self.inner :].reshape(S, hv, dk)
                beta = xn @ L["w_beta"]
                g = L["a_log"] * ops.softplus(xn @ L["w_alpha"] + L["dt_bias"])
                read = np.empty((S, hv, dk), F32)
                for t in range(S):
                    read[t] = ops.gdn_decode(q[t], k[t], v[t], g[t], beta[t], self.rec[i], dk**-0.5, self.l2_eps)
                z = (xn @ L["w_z"]).reshape(S, hv, dk)
                gated = (ops.rms_norm(read, L["ssm_norm"], self.eps) * ops.silu(z)).reshape(S, -1)
                mixer = gated @ L["w_out"]
            h, xn1 = ops.fused_add_rms_norm(h, mixer, L["norm_post"], self.eps)
            gu = xn1 @ L["w_gu"]
            mlp = ops.silu_mul(gu[:, : self.ffn], gu[:, self.ffn :]) @ L["w_down"]
            h, xn = ops.fused_add_rms_norm(h, mlp, L["norm_next"], self.eps)
        return ops.linear(xn[-1], self.head)

    # ------------------------------------------------------------- generate
    def generate(self, ids, max_new: int, prefill: str = "auto", return_logits: bool = False):
        """Greedy generate_stream (qwen35.py:320-402) without EOS/cancellation.

        prefill="auto" takes the batched path for prompts of >= 8 tokens like
        the reference (qwen35.py:358); "tokenwise" always steps token by token.
        Returns the token ids (and, with return_logits, the per-step logits).
        """
        self.reset()
        ids = list(ids)
        if prefill == "auto" and len(ids) >= 8:
            logits = self.prefill_batch(ids)
        else:
            for i, t in enumerate(ids):
                logits = self.forward_token(t, i, logits=(i == len(ids) - 1))
        out, all_logits = [], []
        for step in range(max_new):
            nxt = ops.argmax_first(logits)
            out.append(nxt)
            all_logits.append(logits)
            if step + 1 >= max_new:
                break
            logits = self.forward_token(nxt, len(ids) + step, logits=True)
        return (out, all_logits) if return_logits else out

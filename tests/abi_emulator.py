"""Host-memory emulation of the library's C-ABI entry points, for CPU tests
of the Python mirrors that sit above them.

Every emulated entry point follows its contract in include/bt_b200.h (the
argument meanings, layouts and in-place updates) with the oracle's
restatement of the reference math, reading and writing the caller's buffers
through their raw addresses, so the unchanged host code runs on CPU tensors.
It is test infrastructure: the kernels themselves are checked on the GPU.
"""

from __future__ import annotations

import ctypes

import numpy as np

from breezetoken_b200 import _native as N
from breezetoken_b200 import backends, moe, qwen36_moe
from oracle import moe as omoe
from oracle import ops
from oracle.dequant import dequant_iq3_s
from tests.test_gpu_moe import pack_iq3s_tiles

F32 = np.float32


def _view(ptr: int, dtype, count: int) -> np.ndarray:
    """`count` elements of host memory at address `ptr` (writable)."""
    nbytes = count * np.dtype(dtype).itemsize
    return np.frombuffer((ctypes.c_char * nbytes).from_address(ptr), dtype=dtype, count=count)


def _bf16_to_f32(u: np.ndarray) -> np.ndarray:
    return (u.astype(np.uint32) << 16).view(F32)


def _bf16_rn(v: np.ndarray) -> np.ndarray:
    """f32 -> bf16 bits, round to nearest even (finite inputs)."""
    b = v.astype(F32).view(np.uint32)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


class Emulator:
    """Host-memory stand-ins for the entry points the Python mirrors call."""

    def __init__(self) -> None:
        self.real = N.load()  # its row-size queries are host arithmetic
        self.packed: dict[int, tuple[np.ndarray, int, int]] = {}  # repacked buffer -> (GGUF rows, rows, k)
        self.dense: dict[tuple[int, int, int], np.ndarray] = {}  # (buffer, expert, rows) -> f32 matrix
        self.names: set[str] = set()

    # --- sizes (the library's _workspace_bytes queries and the IQ3_S row size)
    def load(self):
        real = self.real

        class Lib:
            bt_attention_workspace_bytes = staticmethod(lambda *a: 256)
            bt_moe_layer_workspace_bytes = staticmethod(lambda *a: 256)
            bt_moe_workspace_bytes = staticmethod(lambda *a: 256)
            bt_argmax_workspace_bytes = staticmethod(lambda *a: 256)
            bt_iq3s_row_bytes = staticmethod(lambda k: int(real.bt_iq3s_row_bytes(k)))
            bt_q8_row_bytes = staticmethod(lambda k: int(real.bt_q8_row_bytes(k)))
            # host emulation has no bounded device waits to give up
            bt_linear_rows_timeouts = staticmethod(lambda: 0)

        return Lib()

    def call(self, name: str, *args) -> None:
        self.names.add(name)
        getattr(self, name)(*args)

    # --- entry points
    def bt_bf16_planes(self, x, planes, t, k, stream) -> None:
        v = _view(x, F32, t * k).reshape(t, k)
        hi = _bf16_rn(v)
        r1 = v - _bf16_to_f32(hi)
        mid = _bf16_rn(r1)
        lo = _bf16_rn(r1 - _bf16_to_f32(mid))
        out = _view(planes, np.uint16, t * 3 * k).reshape(t, 3, k)
        out[:, 0], out[:, 1], out[:, 2] = hi, mid, lo

    def _planes_of(self, v: np.ndarray, planes: int) -> None:
        t, k = v.shape
        hi = _bf16_rn(v)
        r1 = v - _bf16_to_f32(hi)
        mid = _bf16_rn(r1)
        lo = _bf16_rn(r1 - _bf16_to_f32(mid))
        out = _view(planes, np.uint16, t * 3 * k).reshape(t, 3, k)
        out[:, 0], out[:, 1], out[:, 2] = hi, mid, lo

    def bt_add_rms_norm_planes(self, a, b, w, h, y, planes, rows, n, eps, stream) -> None:
        av, wv = _view(a, F32, rows * n).reshape(rows, n), _view(w, F32, n)
        if b:
            hv, yv = ops.fused_add_rms_norm(av, _view(b, F32, rows * n).reshape(rows, n), wv, eps)
            _view(h, F32, rows * n)[:] = hv.reshape(-1)
        else:
            yv = ops.rms_norm(av, wv, eps)
        _view(y, F32, rows * n)[:] = yv.reshape(-1)
        self._planes_of(yv.astype(F32), planes)

    def bt_attention_layer(self, proj, proj_bs, q_norm, k_norm, cos, sin, rope_dim, pos, k_cache, v_cache, out,
                           batch, heads, kv_heads, dim, cap, scale, eps, splits, ws, status, stream) -> None:
        qn, kn = _view(q_norm, F32, dim), _view(k_norm, F32, dim)
        cv = _view(cos, F32, cap * rope_dim).reshape(cap, rope_dim)
        sv = _view(sin, F32, cap * rope_dim).reshape(cap, rope_dim)
        kc = _view(k_cache, F32, batch * cap * kv_heads * dim).reshape(batch, cap, kv_heads, dim)
        vc = _view(v_cache, F32, batch * cap * kv_heads * dim).reshape(batch, cap, kv_heads, dim)
        o = _view(out, F32, batch * heads * dim).reshape(batch, heads, dim)
        pv = _view(pos, np.int32, batch)
        for b in range(batch):
            row = _view(proj + 4 * b * proj_bs, F32, (2 * heads + 2 * kv_heads) * dim)
            qg = row[: 2 * heads * dim].reshape(heads, 2 * dim)
            q, gate = qg[:, :dim], qg[:, dim:]
            k = row[2 * heads * dim : (2 * heads + kv_heads) * dim].reshape(kv_heads, dim)
            v = row[(2 * heads + kv_heads) * dim :].reshape(kv_heads, dim)
            p = int(pv[b])
            assert 0 <= p < cap
            q = ops.rope(ops.rms_norm(q, qn, eps), cv, sv, p, rope_dim)
            k = ops.rope(ops.rms_norm(k, kn, eps), cv, sv, p, rope_dim)
            kc[b, p], vc[b, p] = k, v
            o[b] = ops.attention(q, kc[b, : p + 1], vc[b, : p + 1], scale) * ops.sigmoid(gate)

    def bt_gdn_gated_step(self, mixed, mixed_bs, ba, ba_bs, a_log, dt_bias, state, z, z_bs, norm_w, planes, batch,
                          heads_k, heads_v, dim, scale, l2_eps, norm_eps, stream) -> None:
        sv = _view(state, F32, batch * heads_v * dim * dim).reshape(batch, heads_v, dim, dim)
        al, dt, nw = _view(a_log, F32, heads_v), _view(dt_bias, F32, heads_v), _view(norm_w, F32, dim)
        y = np.empty((batch, heads_v * dim), F32)
        for b in range(batch):
            row = _view(mixed + 4 * b * mixed_bs, F32, (2 * heads_k + heads_v) * dim)
            q = row[: heads_k * dim].reshape(heads_k, dim)
            k = row[heads_k * dim : 2 * heads_k * dim].reshape(heads_k, dim)
            v = row[2 * heads_k * dim :].reshape(heads_v, dim)
            bav = _view(ba + 4 * b * ba_bs, F32, 2 * heads_v)
            g = al * ops.softplus(bav[heads_v:] + dt)
            o = ops.gdn_decode(q, k, v, g, bav[:heads_v], sv[b], scale, l2_eps)
            zv = _view(z + 4 * b * z_bs, F32, heads_v * dim).reshape(heads_v, dim)
            y[b] = (ops.rms_norm(o, nw, norm_eps) * ops.silu(zv)).reshape(-1)
        self._planes_of(y, planes)

    def bt_gdn_gated_scan(self, mixed, mixed_bs, ba, ba_bs, a_log, dt_bias, state, z, z_bs, norm_w, planes, steps,
                          batch, heads_k, heads_v, dim, scale, l2_eps, norm_eps, stream) -> None:
        for s in range(steps):  # token s of every sequence: rows s * batch .. s * batch + batch - 1
            r = s * batch
            self.bt_gdn_gated_step(mixed + 4 * r * mixed_bs, mixed_bs, ba + 4 * r * ba_bs, ba_bs, a_log, dt_bias,
                                   state, z + 4 * r * z_bs, z_bs, norm_w, planes + 2 * r * 3 * heads_v * dim,
                                   batch, heads_k, heads_v, dim, scale, l2_eps, norm_eps, stream)

    def bt_linear_rows(self, w, w_dtype, xp, y, n, k, t, stream) -> None:
        p = _bf16_to_f32(_view(xp, np.uint16, t * 3 * k).reshape(t, 3, k)).astype(np.float64).sum(1)
        wm = _bf16_to_f32(_view(w, np.uint16, n * k)) if w_dtype == N.BT_BF16 else _view(w, F32, n * k)
        _view(y, F32, t * n)[:] = (p @ wm.reshape(n, k).astype(np.float64).T).astype(F32).reshape(-1)

    # --- the Backend op API's entry points
    def _q8_split(self, k: int) -> tuple[int, int]:
        rb = int(self.real.bt_q8_row_bytes(k))
        return rb, rb - k  # row bytes, bytes before the int8 quants

    def bt_repack_q8_0(self, src, dst, rows, k, dst_row0, step, stream) -> None:
        blocks = _view(src, np.uint8, rows * k // 32 * 34).reshape(rows, k // 32, 34)
        rb, sb = self._q8_split(k)
        n_dst = dst_row0 + (rows - 1) * step + 1
        out = _view(dst, np.uint8, n_dst * rb).reshape(n_dst, rb)
        for i in range(rows):
            r = dst_row0 + i * step
            out[r, : k // 16] = blocks[i, :, :2].reshape(-1)  # fp16 scales, in block order
            out[r, k // 16 : sb] = 0
            out[r, sb:] = blocks[i, :, 2:].reshape(-1)

    def _q8_rows(self, w, n, k) -> np.ndarray:
        rb, sb = self._q8_split(k)
        rows = _view(w, np.uint8, n * rb).reshape(n, rb)
        d = rows[:, : k // 16].copy().view(np.float16).astype(F32)  # (n, k/32)
        q = rows[:, sb:].copy().view(np.int8).astype(F32).reshape(n, k // 32, 32)
        return (q * d[:, :, None]).reshape(n, k)  # exactly d * q

    def bt_dequant_q8_rows(self, w, out, n, k, stream) -> None:
        _view(out, F32, n * k)[:] = self._q8_rows(w, n, k).reshape(-1)

    def bt_linear_q8(self, w, x, y, n, k, n_vec, stream) -> None:
        wm = self._q8_rows(w, n, k).astype(np.float64)
        xv = _view(x, F32, n_vec * k).reshape(n_vec, k).astype(np.float64)
        _view(y, F32, n_vec * n)[:] = (xv @ wm.T).astype(F32).reshape(-1)

    def bt_linear_kn(self, w, w_dtype, x, y, k, n, stream) -> None:
        wm = _bf16_to_f32(_view(w, np.uint16, k * n)) if w_dtype == N.BT_BF16 else _view(w, F32, k * n)
        _view(y, F32, n)[:] = (_view(x, F32, k).astype(np.float64) @ wm.reshape(k, n).astype(np.float64)).astype(F32)

    def bt_silu_mul(self, g, u, y, n, stream) -> None:
        _view(y, F32, n)[:] = ops.silu_mul(_view(g, F32, n), _view(u, F32, n))

    def bt_gdn_decode(self, q, k, v, in_dtype, g, beta, state, out, batch, heads_k, heads_v, dim, scale, eps,
                      stream) -> None:
        def rows(ptr, heads):
            if in_dtype == N.BT_BF16:
                return _bf16_to_f32(_view(ptr, np.uint16, batch * heads * dim)).reshape(batch, heads, dim)
            return _view(ptr, F32, batch * heads * dim).reshape(batch, heads, dim)

        qv, kv, vv = rows(q, heads_k), rows(k, heads_k), rows(v, heads_v)
        gv, bv = _view(g, F32, batch * heads_v).reshape(batch, heads_v), _view(beta, F32, batch * heads_v).reshape(
            batch, heads_v)
        sv = _view(state, F32, batch * heads_v * dim * dim).reshape(batch, heads_v, dim, dim)
        o = _view(out, F32, batch * heads_v * dim).reshape(batch, heads_v, dim)
        for b in range(batch):
            o[b] = ops.gdn_decode(qv[b], kv[b], vv[b], gv[b], bv[b], sv[b], scale, eps)

    def bt_rms_norm(self, x, w, y, rows, n, eps, stream) -> None:
        xv = _view(x, F32, rows * n).reshape(rows, n)
        _view(y, F32, rows * n)[:] = ops.rms_norm(xv, _view(w, F32, n), eps).reshape(-1)

    def bt_fused_add_rms_norm(self, a, b, w, h, xn, rows, n, eps, stream) -> None:
        hv, xv = ops.fused_add_rms_norm(_view(a, F32, rows * n).reshape(rows, n),
                                        _view(b, F32, rows * n).reshape(rows, n), _view(w, F32, n), eps)
        _view(h, F32, rows * n)[:] = hv.reshape(-1)
        _view(xn, F32, rows * n)[:] = xv.reshape(-1)

    def bt_rope(self, x, cos, sin, pos, y, rows, dim, rope_dim, cap, stream) -> None:
        p = int(_view(pos, np.int32, 1)[0])
        assert 0 <= p < cap
        cv, sv = _view(cos, F32, cap * rope_dim).reshape(cap, rope_dim), _view(sin, F32, cap * rope_dim).reshape(
            cap, rope_dim)
        _view(y, F32, rows * dim)[:] = ops.rope(_view(x, F32, rows * dim).reshape(rows, dim), cv, sv, p,
                                                rope_dim).reshape(-1)

    def bt_argmax(self, x, rows, n, out, ws, stream) -> None:
        _view(out, np.int32, rows)[:] = _view(x, F32, rows * n).reshape(rows, n).argmax(-1)

    def bt_attention_decode(self, q, k, v, kv_dtype, lens, out, batch, heads, kv_heads, dim, cap, scale, splits,
                            ws, stream) -> None:
        qv = _view(q, F32, batch * heads * dim).reshape(batch, heads, dim)
        cnt = batch * cap * kv_heads * dim
        if kv_dtype == N.BT_BF16:
            kc, vc = _bf16_to_f32(_view(k, np.uint16, cnt)), _bf16_to_f32(_view(v, np.uint16, cnt))
        else:
            kc, vc = _view(k, F32, cnt), _view(v, F32, cnt)
        kc, vc = kc.reshape(batch, cap, kv_heads, dim), vc.reshape(batch, cap, kv_heads, dim)
        ln = _view(lens, np.int32, batch)
        o = _view(out, F32, batch * heads * dim).reshape(batch, heads, dim)
        for b in range(batch):
            o[b] = ops.attention(qv[b], kc[b, : ln[b]], vc[b, : ln[b]], scale)

    def bt_conv_silu(self, entry, state, w, out, batch, channels, taps, stream) -> None:
        e = _view(entry, F32, batch * channels).reshape(batch, channels)
        st = _view(state, F32, batch * channels * (taps - 1)).reshape(batch, channels, taps - 1)
        wv = _view(w, F32, channels * taps).reshape(channels, taps)
        win = np.concatenate([st, e[:, :, None]], axis=-1)
        acc = win[..., 0] * wv[:, 0]
        for j in range(1, taps):  # taps in order, each product rounded (the kernel's order)
            acc = (acc + win[..., j] * wv[:, j]).astype(F32)
        _view(out, F32, batch * channels)[:] = ops.silu(acc.astype(F32)).reshape(-1)
        st[...] = win[..., 1:]

    def bt_conv_silu_scan(self, entry, state, w, out, steps, batch, channels, taps, stream) -> None:
        for s in range(steps):
            off = 4 * s * batch * channels
            self.bt_conv_silu(entry + off, state, w, out + off, batch, channels, taps, stream)

    def bt_gdn_decode_strided(self, q, k, v, in_dtype, q_bs, k_bs, v_bs, g, g_bs, beta, beta_bs, state, out, out_bs,
                              batch, heads_k, heads_v, dim, scale, eps, stream) -> None:
        assert in_dtype == N.BT_F32
        sv = _view(state, F32, batch * heads_v * dim * dim).reshape(batch, heads_v, dim, dim)
        for b in range(batch):  # row b of every operand starts b * its batch stride elements in
            qb = _view(q + 4 * b * q_bs, F32, heads_k * dim).reshape(heads_k, dim)
            kb = _view(k + 4 * b * k_bs, F32, heads_k * dim).reshape(heads_k, dim)
            vb = _view(v + 4 * b * v_bs, F32, heads_v * dim).reshape(heads_v, dim)
            gb, bb = _view(g + 4 * b * g_bs, F32, heads_v), _view(beta + 4 * b * beta_bs, F32, heads_v)
            _view(out + 4 * b * out_bs, F32, heads_v * dim)[:] = ops.gdn_decode(
                qb, kb, vb, gb, bb, sv[b], scale, eps).reshape(-1)

    def bt_moe_route(self, logits, t, e, top_k, ids, w, stream) -> None:
        lg = _view(logits, F32, t * e).reshape(t, e)
        iv, wv = _view(ids, np.int32, t * top_k).reshape(t, top_k), _view(w, F32, t * top_k).reshape(t, top_k)
        for r in range(t):
            wv[r], ids_r = omoe.route(lg[r], top_k)
            iv[r] = ids_r

    def bt_repack_iq3_s(self, src, dst, rows, k, stream) -> None:
        raw = _view(src, np.uint8, rows * (k // 256) * 110).copy()
        _view(dst, np.uint8, rows * (k // 256) * 136)[:] = pack_iq3s_tiles(raw, rows, k)
        self.packed[dst] = (raw.reshape(rows, -1), rows, k)

    def _expert(self, buf: int, e: int, rows: int) -> np.ndarray:
        """Expert e of the expert tensor at `buf`: a repacked buffer or a
        view that starts at one of its experts (moe.expert_slice)."""
        key = (buf, e, rows)
        if key not in self.dense:
            for base, (raw, n_rows, k) in self.packed.items():
                expert_bytes = rows * (k // 256) * 136
                if base <= buf < base + n_rows * (k // 256) * 136 and (buf - base) % expert_bytes == 0:
                    first = (buf - base) // expert_bytes + e
                    self.dense[key] = dequant_iq3_s(raw[first * rows : (first + 1) * rows], rows, k)
                    break
            else:
                raise KeyError(f"no repacked expert tensor holds address {buf:#x}")
        return self.dense[key]

    def bt_moe_layer_iq3s_add_norm(self, gate, up, down, shared, x, t, hidden, ffn, n_experts, ids, weights, top_k,
                                   h, w, eps, h_out, y, planes, out, ws, stream) -> None:
        self.bt_moe_layer_iq3s(gate, up, down, shared, x, t, hidden, ffn, n_experts, ids, weights, top_k, out, ws,
                               stream)
        self.bt_add_rms_norm_planes(h, out, w, h_out, y, planes, t, hidden, eps, stream)

    def bt_moe_experts_iq3s(self, gate, up, down, x, t, hidden, ffn, n_experts, ids, weights, top_k, out, ws,
                            stream) -> None:
        self.bt_moe_layer_iq3s(gate, up, down, None, x, t, hidden, ffn, n_experts, ids, weights, top_k, out, ws,
                               stream)

    def bt_moe_layer_iq3s(self, gate, up, down, shared, x, t, hidden, ffn, n_experts, ids, weights, top_k, out, ws,
                          stream) -> None:
        xv = _view(x, F32, t * hidden).reshape(t, hidden)
        iv, wv = _view(ids, np.int32, t * top_k).reshape(t, top_k), _view(weights, F32, t * top_k).reshape(t, top_k)
        o = _view(out, F32, t * hidden).reshape(t, hidden)
        sh = shared._obj if shared is not None else None
        for r in range(t):
            y = np.zeros(hidden, F32)  # oracle.moe.experts, with each dequantised expert kept
            for e, w in zip(iv[r], wv[r], strict=True):
                if not 0 <= e < n_experts:  # invalid ids contribute nothing
                    continue
                act = ops.silu(self._expert(gate, e, ffn) @ xv[r]) * (self._expert(up, e, ffn) @ xv[r])
                y += (self._expert(down, e, hidden) @ act) * F32(w)
            if sh is not None:
                sf = sh.ffn
                gm = _bf16_to_f32(_view(sh.gate, np.uint16, sf * hidden)).reshape(sf, hidden)
                um = _bf16_to_f32(_view(sh.up, np.uint16, sf * hidden)).reshape(sf, hidden)
                dm = _bf16_to_f32(_view(sh.down, np.uint16, hidden * sf)).reshape(hidden, sf)
                y = y + omoe.shared_expert(xv[r], gm, um, dm, _view(sh.gate_inp, F32, hidden))
            o[r] = y




def install(monkeypatch) -> Emulator:
    """Route the mirrors' library calls to a fresh Emulator on CPU tensors."""
    em = Emulator()
    monkeypatch.setattr(N, "call", em.call)
    monkeypatch.setattr(N, "load", em.load)
    for mod in (backends, qwen36_moe):
        monkeypatch.setattr(mod, "resolve_device", lambda d: "cpu")
    for mod in (backends, moe, qwen36_moe):
        monkeypatch.setattr(mod, "_stream", lambda: 0)
    return em

"""The B200 backend: breezetoken's ``Backend`` interface on sm_100a kernels.

Mirrors ``breezetoken.backends`` (breezetoken/backends.py:28-98 for the
interface, :860-903 for ``make_backend``): the same method names, argument
meaning, return shapes/dtypes (f32 outputs, ``gdn_decode`` updating ``state``
in place) and error kinds (``ValueError`` for shape mismatches,
``RuntimeError`` for an unavailable device).  Differences by design:

* there is no silent torch fallback -- an unsupported shape raises
  (``B200Error``, a ``RuntimeError``), and a missing CUDA library raises;
* ``linear`` accepts the reference's dense (K, N) weights (f32 or bf16) and
  also ``Q8Weight``: Q8_0 rows kept quantised on the device, which is what
  the decode step streams.
"""

from __future__ import annotations

import ctypes as C
import warnings
from dataclasses import dataclass

import numpy as np
import torch

from breezetoken_b200 import _native as N


def resolve_device(device: str) -> str:
    """backends.py:818-829, restricted to CUDA devices."""
    if device == "auto":
        device = "cuda"
    try:
        parsed = torch.device(device)
    except RuntimeError as exc:
        raise ValueError(f"invalid device {device!r}") from exc
    if parsed.type != "cuda":
        raise ValueError(f"the b200 backend runs on CUDA devices only, got {device!r}")
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA was requested but is not available")
    return str(parsed)


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


@dataclass
class Q8Weight:
    """A (N, K) Q8_0 matrix on the device in the library's q8-row layout.

    ``shape`` reports the reference's (K, N) GEMV layout so it can stand in
    for the dense weights the reference's model layer passes to ``linear``.
    """

    data: torch.Tensor  # uint8 (N * row_bytes,)
    n: int
    k: int

    @property
    def shape(self) -> tuple[int, int]:
        return (self.k, self.n)

    @property
    def device(self) -> torch.device:
        return self.data.device

    @staticmethod
    def row_bytes(k: int) -> int:
        return int(N.load().bt_q8_row_bytes(k))

    @classmethod
    def empty(cls, n: int, k: int, device: str) -> Q8Weight:
        return cls(torch.empty(n * cls.row_bytes(k), dtype=torch.uint8, device=device), n, k)

    def load_gguf_rows(self, raw: np.ndarray | torch.Tensor, rows: int, dst_row0: int = 0, step: int = 1) -> None:
        """Upload GGUF Q8_0 rows and repack them into rows dst_row0 + i*step."""
        if rows == 0:
            return
        if isinstance(raw, np.ndarray):
            with warnings.catch_warnings():
                # GGUF bytes are a read-only memory map; the tensor is only read (the upload's source)
                warnings.filterwarnings("ignore", message="The given NumPy array is not writable")
                src = torch.as_tensor(np.ascontiguousarray(raw))
        else:
            src = torch.as_tensor(raw)
        src = src.reshape(-1).to(self.device, non_blocking=False)
        if src.numel() != rows * self.k // 32 * 34:
            raise ValueError(f"expected {rows * self.k // 32 * 34} Q8_0 bytes, got {src.numel()}")
        if dst_row0 + (rows - 1) * step >= self.n:
            raise ValueError("repack destination rows out of range")
        N.call("bt_repack_q8_0", src.data_ptr(), self.data.data_ptr(), rows, self.k, dst_row0, step, _stream())

    @classmethod
    def from_gguf(cls, raw: np.ndarray, n: int, k: int, device: str) -> Q8Weight:
        w = cls.empty(n, k, device)
        w.load_gguf_rows(raw, n)
        return w

    def dequantize(self) -> torch.Tensor:
        """(N, K) f32, exactly d * q."""
        out = torch.empty(self.n, self.k, dtype=torch.float32, device=self.device)
        N.call("bt_dequant_q8_rows", self.data.data_ptr(), out.data_ptr(), self.n, self.k, _stream())
        return out


class B200Backend:
    """breezetoken ``Backend`` implemented with the sm_100a library."""

    def __init__(self, device: str = "cuda", weight_dtype: torch.dtype = torch.bfloat16) -> None:
        self.name = "b200"
        self.device = resolve_device(device)
        self.weight_dtype = weight_dtype
        self._lib = N.load()
        self._ws: dict[tuple, torch.Tensor] = {}

    # ------------------------------------------------------------ helpers
    def _check(self, *tensors) -> None:
        """Every tensor argument must live on this backend's device before its
        pointer reaches a kernel (a host pointer there would fault the GPU);
        a mismatch raises like the reference's torch ops do."""
        want = torch.device(self.device)
        for t in tensors:
            if t is None:
                continue
            d = t.device
            if d.type != want.type or (want.index is not None and d.index is not None and d.index != want.index):
                raise RuntimeError(f"tensor on {d}, backend on {self.device}")

    def _f32(self, t: torch.Tensor) -> torch.Tensor:
        self._check(t)
        return t.float().contiguous() if t.dtype != torch.float32 or not t.is_contiguous() else t

    def _workspace(self, key: tuple, nbytes: int) -> torch.Tensor:
        ws = self._ws.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=self.device)
            self._ws[key] = ws
        return ws

    # --------------------------------------------------------- Backend API
    def linear(self, x: torch.Tensor, w) -> torch.Tensor:
        """One decode matvec: x (..., K) times w (K, N) -> (N,) f32."""
        K, Nn = w.shape
        if x.shape[-1] != K:
            raise ValueError(f"linear shape mismatch: x {tuple(x.shape)}, w {tuple(w.shape)}")
        xf = self._f32(x).reshape(-1)
        if xf.numel() != K:
            raise ValueError(f"linear expects one vector of {K}, got {tuple(x.shape)}")
        y = torch.empty(Nn, dtype=torch.float32, device=self.device)
        if isinstance(w, Q8Weight):
            self._check(w.data)
            N.call("bt_linear_q8", w.data.data_ptr(), xf.data_ptr(), y.data_ptr(), Nn, K, 1, _stream())
            return y
        self._check(w)
        if w.dtype not in (torch.bfloat16, torch.float32):
            raise N.B200Error(N.BT_ERR_UNSUPPORTED, f"linear: weight dtype {w.dtype} not served")
        wc = w.contiguous()
        dt = N.BT_BF16 if w.dtype == torch.bfloat16 else N.BT_F32
        N.call("bt_linear_kn", wc.data_ptr(), dt, xf.data_ptr(), y.data_ptr(), K, Nn, _stream())
        return y

    def linear_batch(self, x: torch.Tensor, w) -> torch.Tensor:
        """Prefill projection: x (S, K) times w (K, N) -> (S, N) f32."""
        K, Nn = w.shape
        if x.shape[-1] != K:
            raise ValueError(f"linear_batch shape mismatch: {tuple(x.shape)} x {tuple(w.shape)}")
        xf = self._f32(x).reshape(-1, K)
        S = xf.shape[0]
        y = torch.empty(S, Nn, dtype=torch.float32, device=self.device)
        if isinstance(w, Q8Weight):
            self._check(w.data)
            r = 0
            while r < S:
                nv = 8 if S - r >= 8 else 4 if S - r >= 4 else 2 if S - r >= 2 else 1
                N.call("bt_linear_q8", w.data.data_ptr(), xf[r].data_ptr(), y[r].data_ptr(), Nn, K, nv, _stream())
                r += nv
            return y
        for r in range(S):
            y[r] = self.linear(xf[r], w)
        return y

    def rms_norm(self, x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
        if x.shape[-1] != w.numel():
            raise ValueError(f"rms_norm shape mismatch: x {tuple(x.shape)}, w {tuple(w.shape)}")
        xf, wf = self._f32(x), self._f32(w)
        n = x.shape[-1]
        y = torch.empty(x.shape, dtype=torch.float32, device=self.device)
        N.call("bt_rms_norm", xf.data_ptr(), wf.data_ptr(), y.data_ptr(), xf.numel() // n, n, float(eps), _stream())
        return y

    def fused_add_rms_norm(self, a, b, w, eps):
        if a.shape != b.shape:
            if b.numel() == a.numel():
                b = b.reshape(a.shape)
            else:
                raise ValueError(f"fused_add_rms_norm shape mismatch: {a.shape} vs {b.shape}")
        n = a.shape[-1]
        if w.numel() != n:
            raise ValueError(f"fused_add_rms_norm weight shape {tuple(w.shape)} != {n}")
        af, bf, wf = self._f32(a), self._f32(b), self._f32(w)
        h = torch.empty(a.shape, dtype=torch.float32, device=self.device)
        xn = torch.empty_like(h)
        N.call(
            "bt_fused_add_rms_norm",
            af.data_ptr(), bf.data_ptr(), wf.data_ptr(), h.data_ptr(), xn.data_ptr(),
            af.numel() // n, n, float(eps), _stream(),
        )
        # h in the inputs' promoted dtype as the reference returns it (a + b);
        # xn is normalised from the f32 sum
        hd = torch.promote_types(a.dtype, b.dtype)
        return (h if hd == torch.float32 else h.to(hd)), xn

    def silu_mul(self, gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
        if gate.shape != up.shape:
            raise ValueError(f"silu_mul shape mismatch: {tuple(gate.shape)} vs {tuple(up.shape)}")
        g, u = self._f32(gate), self._f32(up)
        y = torch.empty(gate.shape, dtype=torch.float32, device=self.device)
        N.call("bt_silu_mul", g.data_ptr(), u.data_ptr(), y.data_ptr(), g.numel(), _stream())
        return y

    def rope(self, x, cos, sin, pos, rope_dim):
        dim = x.shape[-1]
        if rope_dim > dim or rope_dim % 2 or cos.shape[-1] != rope_dim or sin.shape != cos.shape:
            raise ValueError(f"rope: rope_dim {rope_dim} incompatible with x {tuple(x.shape)} / tables {tuple(cos.shape)}")
        xf, cf_, sf = self._f32(x), self._f32(cos), self._f32(sin)
        p = pos.reshape(-1)[:1].to(device=self.device, dtype=torch.int32)
        y = torch.empty(x.shape, dtype=torch.float32, device=self.device)
        N.call(
            "bt_rope", xf.data_ptr(), cf_.data_ptr(), sf.data_ptr(), p.data_ptr(), y.data_ptr(),
            xf.numel() // dim, dim, rope_dim, cos.shape[0], _stream(),
        )
        return y.to(x.dtype)

    def _attend(self, q, k, v, lens, scale, splits):
        if q.ndim != 2 or k.ndim != 3 or v.ndim != 3:
            raise ValueError("attention expects q (H, D), k/v (S, Hkv, D)")
        heads, dim = q.shape
        cap, groups, kd = k.shape
        if kd != dim or v.shape != k.shape or heads % groups:
            raise ValueError(f"attention shape mismatch: q {tuple(q.shape)}, k {tuple(k.shape)}, v {tuple(v.shape)}")
        qf = self._f32(q)
        self._check(k, v, lens)
        if k.dtype == torch.bfloat16 and v.dtype == torch.bfloat16:
            kk, vv, dt = k.contiguous(), v.contiguous(), N.BT_BF16
        else:
            kk, vv, dt = self._f32(k), self._f32(v), N.BT_F32
        out = torch.empty(heads, dim, dtype=torch.float32, device=self.device)
        nbytes = int(self._lib.bt_attention_workspace_bytes(1, groups, heads, dim, splits))
        ws = self._workspace(("attn", groups, heads, dim, splits), nbytes)
        N.call(
            "bt_attention_decode", qf.data_ptr(), kk.data_ptr(), vv.data_ptr(), dt, lens.data_ptr(), out.data_ptr(),
            1, heads, groups, dim, cap, float(scale), splits, ws.data_ptr(), _stream(),
        )
        return out

    @staticmethod
    def _splits(seq: int) -> int:
        return max(1, min(16, seq // 256))

    def attention(self, q, k, v, scale):
        """GQA decode attention; q (H, D), k/v (S, Hkv, D) -> (H, D)."""
        seq = k.shape[0]
        lens = torch.full((1,), seq, dtype=torch.int32, device=self.device)
        return self._attend(q, k, v, lens, scale, self._splits(seq))

    def attention_fixed(self, q, k, v, pos, scale):
        """Fixed-capacity attention over keys [0, pos] (graph.py:55-61)."""
        lens = (pos.reshape(-1)[:1].to(device=self.device, dtype=torch.int32) + 1).contiguous()
        return self._attend(q, k, v, lens, scale, self._splits(k.shape[0]))

    def gdn_decode(self, q, k, v, g, beta, state, scale, eps=1e-6):
        """One gated-delta-rule step; updates ``state`` in place and returns ``o``."""
        if q.shape != k.shape or q.ndim != 2 or v.ndim != 2:
            raise ValueError("q/k must be (key_heads, dim); v must be (value_heads, dim)")
        heads_k, dim = q.shape
        heads_v = v.shape[0]
        if heads_v % heads_k:
            raise ValueError("value_heads must be a multiple of key_heads")
        if state.shape != (heads_v, dim, dim):
            raise ValueError(f"state shape {tuple(state.shape)} != {(heads_v, dim, dim)}")
        if state.dtype != torch.float32 or not state.is_contiguous():
            raise ValueError("gdn_decode state must be contiguous float32 (it is updated in place)")
        self._check(q, k, v, g, beta, state)
        if q.dtype == k.dtype == v.dtype == torch.bfloat16:
            qq, kk, vv, dt = q.contiguous(), k.contiguous(), v.contiguous(), N.BT_BF16
        else:
            qq, kk, vv, dt = self._f32(q), self._f32(k), self._f32(v), N.BT_F32
        gg, bb = self._f32(g).reshape(-1), self._f32(beta).reshape(-1)
        out = torch.empty(heads_v, dim, dtype=torch.float32, device=self.device)
        N.call(
            "bt_gdn_decode", qq.data_ptr(), kk.data_ptr(), vv.data_ptr(), dt, gg.data_ptr(), bb.data_ptr(),
            state.data_ptr(), out.data_ptr(), 1, heads_k, heads_v, dim, float(scale), float(eps), _stream(),
        )
        return out

    def gdn_prefill(self, q, k, v, g, beta, state, scale, eps=1e-6):
        """The prompt loop of model/prefill.py:106-110 in one launch:
        ``gdn_decode(q[t], k[t], v[t], g[t], beta[t], state, ...)`` for t = 0 ..
        S-1 in order, with the state kept on chip between tokens.  q/k:
        (S, key_heads, dim), v: (S, value_heads, dim), g/beta: (S,
        value_heads); ``state`` (value_heads, dim, dim) f32 is updated in
        place; returns o (S, value_heads, dim) f32.  dim must be 128."""
        if q.shape != k.shape or q.ndim != 3 or v.ndim != 3 or v.shape[0] != q.shape[0]:
            raise ValueError("q/k must be (steps, key_heads, dim); v must be (steps, value_heads, dim)")
        steps, heads_k, dim = q.shape
        heads_v = v.shape[1]
        if heads_v % heads_k or v.shape[2] != dim:
            raise ValueError("value_heads must be a multiple of key_heads, with the same dim")
        if g.shape != (steps, heads_v) or beta.shape != (steps, heads_v):
            raise ValueError(f"g and beta must be {(steps, heads_v)}")
        if state.shape != (heads_v, dim, dim):
            raise ValueError(f"state shape {tuple(state.shape)} != {(heads_v, dim, dim)}")
        if state.dtype != torch.float32 or not state.is_contiguous():
            raise ValueError("gdn_prefill state must be contiguous float32 (it is updated in place)")
        self._check(q, k, v, g, beta, state)
        if q.dtype == k.dtype == v.dtype == torch.bfloat16:
            qq, kk, vv, dt = q.contiguous(), k.contiguous(), v.contiguous(), N.BT_BF16
        else:
            qq, kk, vv, dt = self._f32(q), self._f32(k), self._f32(v), N.BT_F32
        gg, bb = self._f32(g).contiguous(), self._f32(beta).contiguous()
        out = torch.empty(steps, heads_v, dim, dtype=torch.float32, device=self.device)
        nk, nv = heads_k * dim, heads_v * dim
        N.call(
            "bt_gdn_prefill", qq.data_ptr(), kk.data_ptr(), vv.data_ptr(), dt, 0, 0, 0, nk, nk, nv,
            gg.data_ptr(), 0, heads_v, bb.data_ptr(), 0, heads_v, state.data_ptr(), out.data_ptr(), 0, nv,
            steps, 1, heads_k, heads_v, dim, float(scale), float(eps), _stream(),
        )
        return out

    def argmax(self, x: torch.Tensor) -> torch.Tensor:
        """First-index argmax of each row (graph.py:88-91) as int32."""
        xf = self._f32(x)
        n = x.shape[-1]
        rows = xf.numel() // n
        out = torch.empty(rows, dtype=torch.int32, device=self.device)
        ws = self._workspace(("argmax", rows), int(self._lib.bt_argmax_workspace_bytes(rows)))
        N.call("bt_argmax", xf.data_ptr(), rows, n, out.data_ptr(), ws.data_ptr(), _stream())
        return out

    def close(self) -> None:
        self._ws.clear()

    def __repr__(self) -> str:
        return f"B200Backend(device={self.device!r}, dtype={self.weight_dtype})"


def make_backend(kind: str = "auto", device: str = "auto", dtype: str | torch.dtype | None = None) -> B200Backend:
    """Build the B200 backend from CLI-friendly strings (backends.py:860-903).

    ``kind`` is "auto" or "b200"; anything else is a ``ValueError`` like the
    reference's factory.  ``dtype`` names the dense-weight dtype ("bfloat16"
    default, or "float32"); the decode step itself keeps Q8_0 weights.
    """
    kind = kind.lower()
    if kind not in ("auto", "b200"):
        raise ValueError(f"unknown backend {kind!r}")
    aliases = {None: torch.bfloat16, "auto": torch.bfloat16, "bfloat16": torch.bfloat16, "bf16": torch.bfloat16,
               "float32": torch.float32, "fp32": torch.float32}
    if isinstance(dtype, torch.dtype):
        wd = dtype
    else:
        try:
            wd = aliases[dtype.lower() if isinstance(dtype, str) else dtype]
        except KeyError as exc:
            raise ValueError(f"unknown dtype {dtype!r}") from exc
    return B200Backend(resolve_device(device), wd)


__all__ = ["B200Backend", "Q8Weight", "make_backend", "resolve_device"]
_ = C  # ctypes is re-exported through _native

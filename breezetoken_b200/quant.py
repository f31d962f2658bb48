"""Host-side quantisers for the synthetic checkpoints: Q8_0 and IQ3_S.

Parity in this project is defined on the stored bytes (every decoder,
reference and CUDA, must agree bit for bit on ``dequantize(bytes)``), so the
quantisers only have to be deterministic and reasonable, not optimal.

* Q8_0 (GGML type 8): per 32 weights, d = max|x| / 127 stored as fp16 and
  q = round(x / d) as int8 -- the block layout decoded by the reference at
  breezetoken/gguf.py:184-212 and quant/dequant.py:72-75.
* IQ3_S (GGML type 21): 110 bytes per 256 weights decoded as
  ``d * (1 + 2*scale_nibble) * grid[idx] * sign`` (quant/dequant.py:164-185).
  The reference cannot encode IQ3_S; this encoder picks the block scale from
  the largest sub-block, a 4-bit scale per 32 weights, the nearest odd
  magnitude per weight and then the codebook entry nearest to that 4-tuple
  (a 4096-entry lookup built once from the codebook), with sign bits taken
  from the weights.
"""

from __future__ import annotations

import re
from functools import cache
from pathlib import Path

import numpy as np

QK8_0 = 32
QK_K = 256
IQ3S_BLOCK_BYTES = 110
_GRID_INC = Path(__file__).resolve().parent / "csrc" / "iq3s_grid.inc"


@cache
def iq3s_grid() -> np.ndarray:
    """The (512, 4) int8 IQ3_S codebook, read from the kernels' include file."""
    words = [int(w, 16) for w in re.findall(r"0x([0-9a-fA-F]{8})u", _GRID_INC.read_text())]
    if len(words) != 512:
        raise RuntimeError(f"{_GRID_INC} holds {len(words)} codebook words, expected 512")
    arr = np.array(words, dtype="<u4").view(np.uint8).reshape(512, 4)
    return arr.astype(np.int8)


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    """(rows, K) float32 -> (rows, K/32 * 34) uint8 GGUF Q8_0 bytes."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, k = x.shape
    if k % QK8_0:
        raise ValueError(f"Q8_0 needs K % 32 == 0, got {k}")
    b = x.reshape(rows, k // QK8_0, QK8_0)
    d = (np.abs(b).max(axis=-1) / 127.0).astype(np.float32)
    inv = np.divide(1.0, d, out=np.zeros_like(d), where=d > 0).astype(np.float32)
    q = np.clip(np.rint(b * inv[..., None]), -127, 127).astype(np.int8)
    out = np.empty((rows, k // QK8_0, 34), dtype=np.uint8)
    out[..., 0:2] = d.astype("<f2").view(np.uint8).reshape(rows, k // QK8_0, 2)
    out[..., 2:] = q.view(np.uint8)
    return out.reshape(rows, -1)


@cache
def _iq3s_lut() -> np.ndarray:
    """For every 4-tuple of odd magnitudes (8^4 codes), the nearest codebook row."""
    grid = iq3s_grid().astype(np.float32)  # (512, 4)
    odd = np.arange(1, 16, 2, dtype=np.float32)
    codes = np.stack(np.meshgrid(odd, odd, odd, odd, indexing="ij"), axis=-1).reshape(-1, 4)
    # code index = o0*512 + o1*64 + o2*8 + o3 with o_j in 0..7 (meshgrid "ij" order)
    dist = ((codes[:, None, :] - grid[None, :, :]) ** 2).sum(-1)  # (4096, 512)
    return dist.argmin(axis=1).astype(np.int32)


def quantize_iq3_s(x: np.ndarray) -> np.ndarray:
    """(rows, K) float32 -> (rows, K/256 * 110) uint8 GGUF IQ3_S bytes."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, k = x.shape
    if k % QK_K:
        raise ValueError(f"IQ3_S needs K % 256 == 0, got {k}")
    nb = rows * (k // QK_K)
    b = x.reshape(nb, 4, 2, 4, 2, 4)  # block, p, s, l, gsel, j
    sub_max = np.abs(b).reshape(nb, 4, 2, 32).max(axis=-1)  # (nb, 4, 2)
    sub_scale = sub_max / 15.0
    d = (sub_scale.max(axis=(1, 2)) / 31.0).astype(np.float16)
    d32 = d.astype(np.float32)
    safe_d = np.where(d32 > 0, d32, 1.0)[:, None, None]
    nib = np.clip(np.rint((sub_scale / safe_d - 1.0) / 2.0), 0, 15).astype(np.int32)
    nib = np.where(d32[:, None, None] > 0, nib, 0)
    db = d32[:, None, None] * (1 + 2 * nib).astype(np.float32)  # (nb, 4, 2)
    mag = np.abs(b) / np.where(db > 0, db, 1.0)[:, :, :, None, None, None]
    o = np.clip(np.rint((mag - 1.0) / 2.0), 0, 7).astype(np.int32)  # odd index 0..7
    code = ((o[..., 0] * 8 + o[..., 1]) * 8 + o[..., 2]) * 8 + o[..., 3]  # (nb,4,2,4,2)
    gidx = _iq3s_lut()[code]  # (nb, 4, 2, 4, 2)
    neg = (b < 0).astype(np.uint8)  # (nb, 4, 2, 4, 2, 4)

    out = np.zeros((nb, IQ3S_BLOCK_BYTES), dtype=np.uint8)
    out[:, 0:2] = d.astype("<f2").view(np.uint8).reshape(nb, 2)
    # qs: byte 2 + 16p + 8s + 2l + gsel
    out[:, 2:66] = (gidx & 0xFF).astype(np.uint8).reshape(nb, 64)
    # qh: byte 66 + 2p + s, bit 2l + gsel
    hi = (gidx >> 8).astype(np.uint8).reshape(nb, 4, 2, 8)
    out[:, 66:74] = (hi << np.arange(8, dtype=np.uint8)).sum(axis=-1, dtype=np.uint8).reshape(nb, 8)
    # signs: byte 74 + 8p + 4s + l, bit 4*gsel + j
    sb = neg.reshape(nb, 4, 2, 4, 8)
    out[:, 74:106] = (sb << np.arange(8, dtype=np.uint8)).sum(axis=-1, dtype=np.uint8).reshape(nb, 32)
    # scales: byte 106 + p, low nibble s=0, high nibble s=1
    out[:, 106:110] = (nib[:, :, 0] | (nib[:, :, 1] << 4)).astype(np.uint8)
    return out.reshape(rows, -1)


def dequantize_q8_0(raw: np.ndarray, shape: tuple[int, int]) -> np.ndarray:
    """GGUF Q8_0 bytes -> float32 (d * q, exact)."""
    rows, k = shape
    blk = np.ascontiguousarray(raw).reshape(rows, k // QK8_0, 34)
    d = blk[..., 0:2].copy().view("<f2").astype(np.float32)
    q = blk[..., 2:].view(np.int8).astype(np.float32)
    return (q * d).reshape(rows, k)

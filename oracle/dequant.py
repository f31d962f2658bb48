"""Oracle dequantisation (breezetoken/quant/dequant.py), numpy, exact.

* Q8_0 (dequant.py:72-75, gguf.py:184-212): y = d * q with d the fp16 block
  scale and q the int8 quant; the f32 product is exact.
* IQ3_S (dequant.py:164-185): per 256-weight block of 110 bytes
  (d fp16 | qs 64 | qh 8 | signs 32 | scales 4), weight
  e = 64p + 32s + 8l + 4g + j is
  d * (1 + 2*nibble_s(scales[p])) * grid[qs[16p+8s+2l+g] | bit_{2l+g}(qh[2p+s]) << 8][j]
  * (-1 if bit_{4g+j}(signs[8p+4s+l]) else 1); every product is exact in f32.
The IQ3_S codebook is the format's table (quant/_tables.py:1042), stored
beside this file as iq3s_grid.npy.
"""

from __future__ import annotations

from functools import cache
from pathlib import Path

import numpy as np


@cache
def iq3s_grid() -> np.ndarray:
    return np.load(Path(__file__).with_name("iq3s_grid.npy"))


def dequant_q8_0(raw: np.ndarray, rows: int, k: int) -> np.ndarray:
    blk = np.ascontiguousarray(raw).reshape(rows, k // 32, 34)
    d = blk[..., 0:2].copy().view("<f2").astype(np.float32)
    q = blk[..., 2:].copy().view(np.int8).astype(np.float32)
    return (q * d).reshape(rows, k)


def dequant_iq3_s(raw: np.ndarray, rows: int, cols: int) -> np.ndarray:
    nb = rows * cols // 256
    b = np.ascontiguousarray(raw).reshape(nb, 110)
    d = b[:, 0:2].copy().view("<f2").astype(np.float32).reshape(nb)
    qs = b[:, 2:66].reshape(nb, 4, 2, 4, 2).astype(np.int32)  # p, s, l, g
    qh = b[:, 66:74].reshape(nb, 4, 2).astype(np.int32)  # p, s
    signs = b[:, 74:106].reshape(nb, 4, 2, 4).astype(np.int32)  # p, s, l
    scales = b[:, 106:110].astype(np.int32)  # p
    l_idx = np.arange(4).reshape(1, 1, 1, 4)
    g_idx = np.arange(2).reshape(1, 1, 1, 1, 2)
    hbit = (qh[:, :, :, None, None] >> (2 * l_idx[..., None] + g_idx)) & 1  # (nb,4,2,4,2)
    idx = qs | (hbit << 8)
    grid = iq3s_grid().astype(np.float32)[idx]  # (nb,4,2,4,2,4)
    nib = np.stack([scales & 0xF, scales >> 4], axis=-1)  # (nb,4,2)
    db = d[:, None, None] * (1 + 2 * nib).astype(np.float32)
    bit = (signs[..., None, None] >> (4 * np.arange(2).reshape(2, 1) + np.arange(4).reshape(1, 4))) & 1
    sign = np.where(bit == 1, np.float32(-1.0), np.float32(1.0))  # (nb,4,2,4,2,4)
    y = db[:, :, :, None, None, None] * grid * sign
    return y.astype(np.float32).reshape(rows, cols)

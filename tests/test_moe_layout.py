"""CPU checks of the IQ3_S expert tile layout and the decode rules the
expert kernels apply to it (moe.cu: decode_word, sub_scale, block_steps),
restated here lane by lane: the layout re-encodes every weight losslessly
(the GGUF blocks can be rebuilt from it), and the decode reproduces the
oracle's dequantisation (quant/dequant.py:164-185) bit for bit."""

from __future__ import annotations

import numpy as np

from breezetoken_b200.quant import quantize_iq3_s
from oracle.dequant import dequant_iq3_s, iq3s_grid
from tests.test_gpu_moe import CODE_BIT, pack_iq3s_tiles

ROWS, K = 32, 512
CHUNK = 2176


def _u32(b: np.ndarray) -> int:
    return int(np.frombuffer(b.tobytes(), np.uint32)[0])


def _weights() -> np.ndarray:
    rng = np.random.default_rng(21)
    return quantize_iq3_s(rng.standard_normal((ROWS, K)).astype(np.float32) * np.float32(0.02)).reshape(ROWS, -1)


def _lane_words(c: np.ndarray, lane: int) -> dict:
    """(row half r, sub-block s) -> the lane's code word in chunk c."""
    out = {}
    for j in range(4):
        part = c[512 * j + 16 * lane:512 * j + 16 * lane + 16]
        for S in range(2):
            for r in range(2):
                out[r, 2 * j + S] = _u32(part[4 * (2 * S + r):4 * (2 * S + r) + 4])
    return out


def test_tile_layout_rebuilds_every_gguf_byte() -> None:
    """From the codes and scale records alone, the GGUF blocks come back:
    codebook index (qs byte + qh bit) from the 4 magnitudes of each group,
    signs from the code signs, scales and d from the records."""
    raw = _weights()
    dev = pack_iq3s_tiles(raw, ROWS, K).reshape(ROWS // 16, K // 256, CHUNK)
    grid = iq3s_grid().astype(np.int64) & 255
    index_of = {tuple(grid[i]): i for i in range(512)}
    assert len(index_of) == 512  # the codebook's entries are distinct
    out = np.zeros((ROWS, K // 256, 110), np.uint8)
    for tile in range(ROWS // 16):
        for kb in range(K // 256):
            c = dev[tile, kb]
            for lane in range(32):
                g, t = lane >> 2, lane & 3
                words = _lane_words(c, lane)
                for r in range(2):
                    row = 16 * tile + g + 8 * r
                    for s in range(8):
                        wd = words[r, s]
                        v = []
                        for i in range(8):
                            code = 0
                            for bit in range(4):
                                code |= ((wd >> ((CODE_BIT[i] + bit) % 32)) & 1) << bit
                            v.append(2 * code - 15)
                        signs = sum(1 << i for i in range(8) if v[i] < 0)
                        out[row, kb, 74 + 4 * s + t] = signs
                        for h in range(2):
                            idx = index_of[tuple(abs(x) for x in v[4 * h:4 * h + 4])]
                            q = 8 * s + 2 * t + h
                            out[row, kb, 2 + q] = idx & 255
                            out[row, kb, 66 + s] |= (idx >> 8) << (2 * t + h)
            for rr in range(16):
                rec = c[2048 + 8 * rr:2056 + 8 * rr]
                out[16 * tile + rr, kb, 106:110] = rec[:4]
                out[16 * tile + rr, kb, 0:2] = rec[4:6]
                assert (rec[6:] == 0).all()
    assert (out == raw.reshape(ROWS, K // 256, 110)).all()


def _f16x2(u: int) -> np.ndarray:
    return np.frombuffer(np.uint32(u).tobytes(), np.float16)


def test_kernel_decode_rules_reproduce_the_dequantisation() -> None:
    """decode_word's mask-or into an fp16 of exponent 1024 and one f16x2 add
    or fma per register, and sub_scale's exact fma, give every weight's
    dequantised f32 value bit for bit."""
    raw = _weights()
    want = dequant_iq3_s(raw, ROWS, K)
    dev = pack_iq3s_tiles(raw, ROWS, K).reshape(ROWS // 16, K // 256, CHUNK)
    magic = 0x64006400
    h1039, h16, h79 = _f16x2(0xE40FE40F), _f16x2(0x2C002C00), _f16x2(0xD4F0D4F0)
    assert (h1039 == -1039).all() and (h16 == 1 / 16).all() and (h79 == -79).all()
    got = np.zeros((ROWS, K), np.float32)
    for tile in range(ROWS // 16):
        for kb in range(K // 256):
            c = dev[tile, kb]
            for lane in range(32):
                g, t = lane >> 2, lane & 3
                words = _lane_words(c, lane)
                for r in range(2):
                    row = 16 * tile + g + 8 * r
                    rec = c[2048 + 8 * (g + 8 * r):2056 + 8 * (g + 8 * r)]
                    sc = _u32(rec[:4])
                    d = np.frombuffer(rec[4:6].tobytes(), np.float16)[0].astype(np.float32)
                    for s in range(8):
                        w = words[r, s]
                        rot = ((w >> 12) | (w << 20)) & 0xFFFFFFFF
                        regs = [
                            _f16x2((w & 0x001E001E) | magic).astype(np.float64) + h1039,  # exact sums
                            _f16x2((w & 0x01E001E0) | magic).astype(np.float64) * h16 + h79,
                            _f16x2(((w >> 8) & 0x001E001E) | magic).astype(np.float64) + h1039,
                            _f16x2((rot & 0x001E001E) | magic).astype(np.float64) + h1039,
                        ]
                        vals = np.concatenate(regs)
                        assert (vals == np.round(vals)).all() and (np.abs(vals) <= 15).all()
                        vals16 = vals.astype(np.float16)  # exact: small odd integers
                        two_n = ((sc << 1) if s == 0 else (sc >> (4 * s - 1))) & 0x1E
                        m = np.frombuffer(np.uint32(0x4B000001 | two_n).tobytes(), np.float32)[0]
                        # fma(m, d, -2^23 d), restated exactly in f64, rounded once to f32
                        scale = np.float32(np.float64(m) * np.float64(d) + np.float64(np.float32(-8388608.0) * d))
                        assert scale == d * np.float32(1 + 2 * ((sc >> (4 * s)) & 15))
                        base = kb * 256 + 32 * s + 8 * t
                        got[row, base:base + 8] = scale * vals16.astype(np.float32)
    assert np.array_equal(got, want)

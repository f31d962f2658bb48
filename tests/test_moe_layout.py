"""CPU checks of the IQ3_S expert tile layout and the decode rules the
expert kernels apply to it (moe.cu: tile_word, row_scale, cursor_next,
block_steps),
restated here lane by lane: the layout keeps every GGUF byte, and the decode
reproduces the oracle's dequantisation (quant/dequant.py:164-185) bit for
bit."""

from __future__ import annotations

import numpy as np

from breezetoken_b200.quant import quantize_iq3_s
from oracle.dequant import dequant_iq3_s, iq3s_grid
from tests.test_gpu_moe import pack_iq3s_tiles

ROWS, K = 32, 512


def _u32(b: np.ndarray) -> int:
    return int(np.frombuffer(b.tobytes(), np.uint32)[0])


def _weights() -> np.ndarray:
    rng = np.random.default_rng(21)
    return quantize_iq3_s(rng.standard_normal((ROWS, K)).astype(np.float32) * np.float32(0.02)).reshape(ROWS, -1)


def test_tile_layout_keeps_every_gguf_byte() -> None:
    raw = _weights()
    dev = pack_iq3s_tiles(raw, ROWS, K).reshape(ROWS // 16, K // 256, 1792)
    out = np.zeros((ROWS, K // 256, 110), np.uint8)
    for tile in range(ROWS // 16):
        for kb in range(K // 256):
            c = dev[tile, kb]
            for lane in range(32):
                g, t = lane >> 2, lane & 3
                qh = _u32(c[1536 + 4 * lane:1540 + 4 * lane])
                for r in range(2):
                    row = 16 * tile + g + 8 * r
                    qs = c[512 * r + 16 * lane:512 * r + 16 * lane + 16]
                    s01 = _u32(c[1024 + 16 * lane + 8 * r:1028 + 16 * lane + 8 * r])
                    s23 = _u32(c[1028 + 16 * lane + 8 * r:1032 + 16 * lane + 8 * r])
                    for s in range(8):
                        for h in range(2):
                            q = 2 * s + h
                            out[row, kb, 2 + 8 * s + 2 * t + h] = qs[4 * (q & 3) + (q >> 2)]
                            nib = ((s01 >> (15 - q)) & 1) | (((s01 >> (31 - q)) & 1) << 1)
                            nib |= (((s23 >> (15 - q)) & 1) << 2) | (((s23 >> (31 - q)) & 1) << 3)
                            out[row, kb, 74 + 4 * s + t] |= nib << (4 * h)
                            out[row, kb, 66 + s] |= ((qh >> (16 * r + q)) & 1) << (2 * t + h)
            for rr in range(16):
                rec = c[1664 + 8 * rr:1672 + 8 * rr]
                out[16 * tile + rr, kb, 106:110] = rec[:4]
                out[16 * tile + rr, kb, 0:2] = rec[4:6]
    assert (out == raw.reshape(ROWS, K // 256, 110)).all()


def test_kernel_decode_rules_reproduce_the_dequantisation() -> None:
    raw = _weights()
    want = dequant_iq3_s(raw, ROWS, K)
    grid = iq3s_grid().astype(np.int64) & 255
    lut = np.zeros(65536, np.uint8)  # the shared-memory codebook: row (b, qh), 16 copies of 4 fp16
    for b in range(256):
        for qh in range(2):
            e = np.frombuffer(grid[qh * 256 + b].astype(np.float16).tobytes(), np.uint8)
            for c in range(16):
                lut[b * 256 + qh * 128 + 8 * c:b * 256 + qh * 128 + 8 * c + 8] = e
    dev = pack_iq3s_tiles(raw, ROWS, K).reshape(ROWS // 16, K // 256, 1792)
    mask = 0xFFFFFFFF
    got = np.zeros((ROWS, K), np.float32)
    for tile in range(ROWS // 16):
        for kb in range(K // 256):
            c = dev[tile, kb]
            for lane in range(32):
                g, t = lane >> 2, lane & 3
                words = [_u32(c[o + 4 * i:o + 4 * i + 4]) for o in (16 * lane, 512 + 16 * lane) for i in range(4)]
                sg = [_u32(c[1024 + 16 * lane + 4 * i:1028 + 16 * lane + 4 * i]) for i in range(4)]
                cur = {"qa": words[:4], "qb": words[4:], "s0a": sg[0], "s1a": sg[1], "s0b": sg[2], "s1b": sg[3],
                       "qh": _u32(c[1536 + 4 * lane:1540 + 4 * lane])}
                rec = [c[1664 + 8 * g:1672 + 8 * g], c[1664 + 8 * (g + 8):1672 + 8 * (g + 8)]]
                sc = [_u32(x[:4]) for x in rec]
                d = [np.frombuffer(x[4:6].tobytes(), np.float16)[0].astype(np.float32) for x in rec]
                dneg = [np.float32(-8388608.0) * x for x in d]
                lane_off = (lane & 15) * 8
                for p in range(4):
                    sel = 0x5504 + 16 * p
                    for S in range(2):
                        for R in range(2):
                            for H in range(2):
                                qw = (cur["qb"] if R else cur["qa"])[(S << 1) | H]
                                src = qw | (lane_off << 32)  # prmt: bytes 0-3 of a, 4-7 of b
                                off = 0
                                for i in range(4):
                                    off |= ((src >> (8 * ((sel >> (4 * i)) & 7))) & 255) << (8 * i)
                                assert off == (((qw >> (8 * p)) & 255) << 8) | lane_off
                                qb = 16 * R + 2 * S + H
                                hb = (cur["qh"] >> (qb - 7)) if qb >= 7 else ((cur["qh"] << (7 - qb)) & mask)
                                off |= hb & 0x80
                                wx, wy = _u32(lut[off:off + 4]), _u32(lut[off + 4:off + 8])
                                sh = 2 * S + H
                                wx ^= ((cur["s0b"] if R else cur["s0a"]) << sh) & 0x80008000
                                wy ^= ((cur["s1b"] if R else cur["s1a"]) << sh) & 0x80008000
                                w4 = np.frombuffer(np.array([wx, wy], np.uint32).tobytes(), np.float16)
                                two_n = ((sc[R] << 1) if S == 0 else (sc[R] >> 3)) & 0x1E
                                m = np.frombuffer(np.uint32(0x4B000001 | two_n).tobytes(), np.float32)[0]
                                # fma(m, d, -2^23 d), restated exactly in f64, rounded once to f32
                                db = np.float32(np.float64(m) * np.float64(d[R]) + np.float64(dneg[R]))
                                nib = (sc[R] >> (4 * S)) & 15
                                assert db == np.float32(d[R]) * np.float32(1 + 2 * nib)
                                base = kb * 256 + 32 * (2 * p + S) + 8 * t + 4 * H
                                got[16 * tile + g + 8 * R, base:base + 4] = db * w4.astype(np.float32)
                    for key in ("s0a", "s1a", "s0b", "s1b"):
                        cur[key] = (cur[key] << 4) & mask
                    cur["qh"] >>= 4
                    sc = [x >> 8 for x in sc]
    assert np.array_equal(got, want)

"""Minimal GGUF v3 reading for the oracle (breezetoken/gguf.py:46-212).

Independent of the product's reader on purpose: shapes are reversed from the
fastest-first dims (gguf.py:114), data starts at the 32-byte aligned end of
the header (gguf.py:100,116), F32 tensors are read as-is and Q8_0 tensors are
dequantised as ``q * d`` (gguf.py:184-212).
"""

from __future__ import annotations

import struct

import numpy as np

from oracle.dequant import dequant_q8_0

_FMT = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}


class OracleGGUF:
    def __init__(self, path) -> None:
        self.buf = np.memmap(path, dtype=np.uint8, mode="r")
        self.metadata: dict = {}
        self.tensors: dict[str, tuple[tuple[int, ...], int, int]] = {}
        b = self.buf
        assert bytes(b[:4]) == b"GGUF"
        version, n_t, n_kv = struct.unpack_from("<IQQ", b, 4)
        assert version == 3
        pos = 24
        for _ in range(n_kv):
            (n,) = struct.unpack_from("<Q", b, pos)
            key = bytes(b[pos + 8 : pos + 8 + n]).decode()
            pos += 8 + n
            (vt,) = struct.unpack_from("<I", b, pos)
            self.metadata[key], pos = self._val(pos + 4, vt)
        infos = []
        for _ in range(n_t):
            (n,) = struct.unpack_from("<Q", b, pos)
            name = bytes(b[pos + 8 : pos + 8 + n]).decode()
            pos += 8 + n
            (nd,) = struct.unpack_from("<I", b, pos)
            dims = struct.unpack_from(f"<{nd}Q", b, pos + 4)
            pos += 4 + 8 * nd
            tt, off = struct.unpack_from("<IQ", b, pos)
            pos += 12
            infos.append((name, tuple(reversed(dims)), tt, off))
        align = int(self.metadata.get("general.alignment", 32))
        data = (pos + align - 1) // align * align
        for name, shape, tt, off in infos:
            self.tensors[name] = (shape, tt, data + off)

    def _val(self, pos, vt):
        b = self.buf
        if vt == 8:
            (n,) = struct.unpack_from("<Q", b, pos)
            return bytes(b[pos + 8 : pos + 8 + n]).decode(), pos + 8 + n
        if vt == 9:
            et, cnt = struct.unpack_from("<IQ", b, pos)
            pos += 12
            out = []
            for _ in range(cnt):
                v, pos = self._val(pos, et)
                out.append(v)
            return out, pos
        (v,) = struct.unpack_from(_FMT[vt], b, pos)
        return v, pos + struct.calcsize(_FMT[vt])

    def get(self, name: str) -> np.ndarray:
        """Tensor as float32 in its logical (row-major) shape."""
        shape, tt, off = self.tensors[name]
        n = int(np.prod(shape))
        if tt == 0:
            return np.frombuffer(self.buf, dtype="<f4", count=n, offset=off).reshape(shape).astype(np.float32)
        if tt == 8:
            rows, k = shape
            raw = np.frombuffer(self.buf, dtype=np.uint8, count=rows * k // 32 * 34, offset=off)
            return dequant_q8_0(raw, rows, k)
        raise NotImplementedError(f"oracle reads f32/q8_0 only, {name} is type {tt}")

    def raw(self, name: str) -> np.ndarray:
        shape, tt, off = self.tensors[name]
        per, nb = {0: (1, 4), 8: (32, 34), 21: (256, 110), 30: (1, 2)}[tt]
        rows = int(np.prod(shape[:-1])) if len(shape) > 1 else 1
        return np.frombuffer(self.buf, dtype=np.uint8, count=rows * shape[-1] // per * nb, offset=off)

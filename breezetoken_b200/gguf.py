"""GGUF v3 reader and writer for the B200 backend.

The reader follows the contract of breezetoken's ``GGUFFile``
(breezetoken/gguf.py:46-235): memory-mapped file, metadata dictionary,
logical shapes reversed from GGUF's fastest-first dims (gguf.py:114), a
default data alignment of 32 bytes (gguf.py:100), and errors of the same
kinds (``ValueError`` for a non-GGUF or wrong-version file, ``KeyError`` for
a missing tensor, ``NotImplementedError`` for an unsupported type).  Unlike
the reference it hands out the raw quantised bytes, which the repacker
uploads and rearranges on the device instead of dequantising on the host.

The writer produces files the reference reader parses; it is used to build
the seeded synthetic checkpoints the benchmarks and parity tests run on.
"""

from __future__ import annotations

import struct
from pathlib import Path
from typing import Any

import numpy as np

GGML_F32 = 0
GGML_Q8_0 = 8
GGML_IQ3_S = 21
GGML_BF16 = 30

#: (elements per block, bytes per block) of each supported GGML type
TYPE_LAYOUT: dict[int, tuple[int, int]] = {
    GGML_F32: (1, 4),
    GGML_Q8_0: (32, 34),
    GGML_IQ3_S: (256, 110),
    GGML_BF16: (1, 2),
}
TYPE_NAMES = {GGML_F32: "f32", GGML_Q8_0: "q8_0", GGML_IQ3_S: "iq3_s", GGML_BF16: "bf16"}

# GGUF metadata value types
_U8, _I8, _U16, _I16, _U32, _I32, _F32, _BOOL, _STR, _ARR, _U64, _I64, _F64 = range(13)
_SCALAR = {
    _U8: "<B",
    _I8: "<b",
    _U16: "<H",
    _I16: "<h",
    _U32: "<I",
    _I32: "<i",
    _F32: "<f",
    _BOOL: "<?",
    _U64: "<Q",
    _I64: "<q",
    _F64: "<d",
}


def row_bytes(ggml_type: int, columns: int) -> int:
    """Bytes of one row of ``columns`` elements (quant/formats.py:39-44)."""
    try:
        per, nbytes = TYPE_LAYOUT[ggml_type]
    except KeyError as exc:
        raise NotImplementedError(f"GGML type {ggml_type} is not supported") from exc
    if columns % per:
        raise ValueError(f"{TYPE_NAMES[ggml_type]} needs a row divisible by {per}, got {columns}")
    return columns // per * nbytes


class GGUFFile:
    """A read-only, memory-mapped GGUF v3 file."""

    def __init__(self, path: str | Path) -> None:
        self.path = Path(path)
        self._buf: np.memmap | None = np.memmap(self.path, dtype=np.uint8, mode="r")
        self.metadata: dict[str, Any] = {}
        self._tensors: dict[str, tuple[tuple[int, ...], int, int]] = {}
        self._parse()

    # ------------------------------------------------------------------ parse
    def _value(self, pos: int, vtype: int) -> tuple[Any, int]:
        buf = self._require()
        if vtype == _STR:
            (n,) = struct.unpack_from("<Q", buf, pos)
            return bytes(buf[pos + 8 : pos + 8 + n]).decode("utf-8"), pos + 8 + n
        if vtype == _ARR:
            etype, count = struct.unpack_from("<IQ", buf, pos)
            pos += 12
            if etype == _STR:
                out = []
                for _ in range(count):
                    item, pos = self._value(pos, _STR)
                    out.append(item)
                return out, pos
            fmt = _SCALAR[etype]
            size = struct.calcsize(fmt)
            arr = np.frombuffer(buf, dtype=fmt, count=count, offset=pos).copy()
            return arr, pos + size * count
        fmt = _SCALAR[vtype]
        (value,) = struct.unpack_from(fmt, buf, pos)
        return value, pos + struct.calcsize(fmt)

    def _parse(self) -> None:
        buf = self._require()
        if buf.nbytes < 24 or bytes(buf[:4]) != b"GGUF":
            raise ValueError(f"{self.path} is not a GGUF file")
        version, n_tensors, n_kv = struct.unpack_from("<IQQ", buf, 4)
        if version != 3:
            raise ValueError(f"unsupported GGUF version {version}")
        pos = 24
        try:
            for _ in range(n_kv):
                (klen,) = struct.unpack_from("<Q", buf, pos)
                key = bytes(buf[pos + 8 : pos + 8 + klen]).decode("utf-8")
                pos += 8 + klen
                (vtype,) = struct.unpack_from("<I", buf, pos)
                self.metadata[key], pos = self._value(pos + 4, vtype)
            infos = []
            for _ in range(n_tensors):
                (nlen,) = struct.unpack_from("<Q", buf, pos)
                name = bytes(buf[pos + 8 : pos + 8 + nlen]).decode("utf-8")
                pos += 8 + nlen
                (ndim,) = struct.unpack_from("<I", buf, pos)
                dims = struct.unpack_from(f"<{ndim}Q", buf, pos + 4)
                pos += 4 + 8 * ndim
                ttype, toff = struct.unpack_from("<IQ", buf, pos)
                pos += 12
                infos.append((name, tuple(reversed(dims)), ttype, toff))
        except (struct.error, KeyError, UnicodeDecodeError) as exc:
            raise ValueError(f"{self.path}: truncated or corrupt GGUF header ({exc})") from exc
        align = int(self.metadata.get("general.alignment", 32))
        data = (pos + align - 1) // align * align
        for name, shape, ttype, toff in infos:
            start = data + toff
            nbytes = self._nbytes(shape, ttype)
            if nbytes is not None and start + nbytes > buf.nbytes:
                raise ValueError(f"{self.path}: tensor {name!r} runs past the end of the file")
            self._tensors[name] = (shape, ttype, start)

    @staticmethod
    def _nbytes(shape: tuple[int, ...], ttype: int) -> int | None:
        if ttype not in TYPE_LAYOUT or not shape:
            return None
        rows = int(np.prod(shape[:-1])) if len(shape) > 1 else 1
        return rows * row_bytes(ttype, shape[-1])

    # ------------------------------------------------------------------ query
    @property
    def arch(self) -> str:
        return str(self.metadata["general.architecture"])

    def tensor_names(self) -> list[str]:
        return list(self._tensors)

    def tensor_layout(self, name: str) -> tuple[tuple[int, ...], int, int]:
        """(logical shape, GGML type id, absolute byte offset)."""
        try:
            return self._tensors[name]
        except KeyError as exc:
            raise KeyError(f"tensor {name!r} not found in {self.path.name}") from exc

    def tensor_info(self, name: str) -> tuple[tuple[int, ...], str]:
        shape, ttype, _ = self.tensor_layout(name)
        return shape, TYPE_NAMES.get(ttype, f"type_{ttype}")

    def raw(self, name: str) -> np.ndarray:
        """Zero-copy uint8 view of a tensor's stored bytes."""
        shape, ttype, offset = self.tensor_layout(name)
        nbytes = self._nbytes(shape, ttype)
        if nbytes is None:
            raise NotImplementedError(f"GGML type {ttype} of {name} is not supported")
        return self._require()[offset : offset + nbytes]

    def f32(self, name: str) -> np.ndarray:
        """An F32 tensor as a float32 array of its logical shape."""
        shape, ttype, _ = self.tensor_layout(name)
        if ttype != GGML_F32:
            raise NotImplementedError(f"{name} is {TYPE_NAMES.get(ttype, ttype)}, expected f32")
        return self.raw(name).view("<f4").reshape(shape)

    # ------------------------------------------------------------- lifecycle
    def _require(self) -> np.memmap:
        if self._buf is None:
            raise ValueError(f"GGUF file {self.path} is closed")
        return self._buf

    def close(self) -> None:
        buf, self._buf = self._buf, None
        if buf is not None and getattr(buf, "_mmap", None) is not None:
            buf._mmap.close()

    def __enter__(self) -> GGUFFile:
        return self

    def __exit__(self, *exc: object) -> None:
        self.close()


class GGUFWriter:
    """Minimal GGUF v3 writer (metadata + tensors, 32-byte data alignment)."""

    ALIGN = 32

    def __init__(self) -> None:
        self._kv: list[tuple[str, int, Any]] = []
        self._tensors: list[tuple[str, tuple[int, ...], int, np.ndarray]] = []

    def add(self, key: str, value: Any) -> None:
        if isinstance(value, str):
            self._kv.append((key, _STR, value))
        elif isinstance(value, bool):
            self._kv.append((key, _BOOL, value))
        elif isinstance(value, int):
            self._kv.append((key, _U32 if 0 <= value < 2**32 else _I64, value))
        elif isinstance(value, float):
            self._kv.append((key, _F32, value))
        else:
            raise TypeError(f"unsupported metadata value for {key}: {type(value)}")

    @staticmethod
    def _blob(name: str, shape: tuple[int, ...], ggml_type: int, data: np.ndarray) -> np.ndarray:
        blob = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        rows = int(np.prod(shape[:-1])) if len(shape) > 1 else 1
        want = rows * row_bytes(ggml_type, shape[-1])
        if blob.nbytes != want:
            raise ValueError(f"{name}: {blob.nbytes} bytes, expected {want}")
        return blob

    def add_tensor(self, name: str, shape: tuple[int, ...], ggml_type: int, data) -> None:
        """``data``: the stored bytes (uint8) or a float32 array for F32, or a
        callable returning them, called once while the file is written (so a
        large file never holds all its tensors in memory at once)."""
        shape = tuple(int(s) for s in shape)
        if not callable(data):
            data = self._blob(name, shape, ggml_type, data)
        self._tensors.append((name, shape, ggml_type, data))

    def _nbytes(self, shape: tuple[int, ...], ggml_type: int) -> int:
        rows = int(np.prod(shape[:-1])) if len(shape) > 1 else 1
        return rows * row_bytes(ggml_type, shape[-1])

    @staticmethod
    def _str(s: str) -> bytes:
        b = s.encode("utf-8")
        return struct.pack("<Q", len(b)) + b

    def write(self, path: str | Path) -> Path:
        path = Path(path)
        head = [b"GGUF", struct.pack("<IQQ", 3, len(self._tensors), len(self._kv))]
        for key, vtype, value in self._kv:
            head.append(self._str(key) + struct.pack("<I", vtype))
            head.append(self._str(value) if vtype == _STR else struct.pack(_SCALAR[vtype], value))
        offset = 0
        for name, shape, ttype, _ in self._tensors:
            dims = tuple(reversed(shape))
            head.append(self._str(name) + struct.pack(f"<I{len(dims)}Q", len(dims), *dims))
            head.append(struct.pack("<IQ", ttype, offset))
            offset += (self._nbytes(shape, ttype) + self.ALIGN - 1) // self.ALIGN * self.ALIGN
        header = b"".join(head)
        with open(path, "wb") as f:
            f.write(header)
            f.write(b"\0" * ((-len(header)) % self.ALIGN))
            for name, shape, ttype, data in self._tensors:
                blob = self._blob(name, shape, ttype, data()) if callable(data) else data
                f.write(memoryview(blob))
                f.write(b"\0" * ((-blob.nbytes) % self.ALIGN))
                del blob
        return path

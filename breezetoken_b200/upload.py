"""Host -> device upload of checkpoint bytes.

Loading the 35B-A3B-shaped checkpoint is bound by moving ~18 GB of mapped
GGUF bytes to the device: the repack into the device layout runs on the GPU
at HBM speed (breezetoken/gguf.py:184-212 re-decodes on the host instead).  A
plain ``tensor.to("cuda")`` of a pageable (memory-mapped) array goes through
the driver's own small staging copies, one at a time.  `Uploader` stages the
bytes itself through two pinned buffers: while the copy engine moves one
chunk to the device on a side stream, host threads copy the next chunk out of
the page cache into the other buffer.  The bytes arrive unchanged; the
returned tensor is ordered before later work on the caller's current stream.
"""

from __future__ import annotations

from concurrent.futures import ThreadPoolExecutor

import numpy as np
import torch


class Uploader:
    """Double-buffered pinned staging for host -> device copies of raw bytes.

    ``to_device(arr)`` returns a uint8 device tensor holding ``arr``'s bytes
    (any dtype, C-contiguous, e.g. a slice of a memory-mapped GGUF).  On a
    CPU device it returns a copy on the host.  One instance serves one
    device; its buffers are freed with it (``close()``).
    """

    def __init__(self, device: str | torch.device, chunk_bytes: int = 64 << 20, threads: int = 8) -> None:
        self.device = torch.device(device)
        self.cuda = self.device.type == "cuda"
        self.chunk = int(chunk_bytes)
        self.threads = max(1, int(threads))
        self._bufs: list[torch.Tensor] = []
        self._views: list[np.ndarray] = []
        self._done: list[torch.cuda.Event | None] = [None, None]
        self._pool: ThreadPoolExecutor | None = None
        self._stream: torch.cuda.Stream | None = None
        if self.cuda:
            self._stream = torch.cuda.Stream(self.device)
            for _ in range(2):
                b = torch.empty(self.chunk, dtype=torch.uint8).pin_memory()
                self._bufs.append(b)
                self._views.append(b.numpy())
            self._pool = ThreadPoolExecutor(self.threads)

    def _fill(self, dst: np.ndarray, src: np.ndarray) -> None:
        """dst[:] = src, split over the host threads (np.copyto releases the GIL)."""
        n = src.size
        if n < (4 << 20) or self._pool is None:
            np.copyto(dst, src)
            return
        step = -(-n // self.threads)
        step = -(-step // 4096) * 4096  # page-sized pieces
        futs = [self._pool.submit(np.copyto, dst[o:o + step], src[o:o + step]) for o in range(0, n, step)]
        for f in futs:
            f.result()

    def to_device(self, arr) -> torch.Tensor:
        src = np.ascontiguousarray(arr)
        src = src.reshape(-1).view(np.uint8)
        n = src.size
        if not self.cuda:
            return torch.from_numpy(src.copy())
        out = torch.empty(n, dtype=torch.uint8, device=self.device)
        stream = self._stream
        stream.wait_stream(torch.cuda.current_stream(self.device))  # `out` is allocated before the copies
        for i, off in enumerate(range(0, n, self.chunk)):
            b = i & 1
            if self._done[b] is not None:
                self._done[b].synchronize()  # the copy engine is done reading this buffer
            m = min(self.chunk, n - off)
            self._fill(self._views[b][:m], src[off:off + m])
            with torch.cuda.stream(stream):
                out[off:off + m].copy_(self._bufs[b][:m], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(stream)
            self._done[b] = ev
        out.record_stream(stream)
        torch.cuda.current_stream(self.device).wait_stream(stream)
        return out

    def close(self) -> None:
        for ev in self._done:
            if ev is not None:
                ev.synchronize()
        self._done = [None, None]
        if self._pool is not None:
            self._pool.shutdown(wait=True)
            self._pool = None
        self._bufs, self._views = [], []


__all__ = ["Uploader"]

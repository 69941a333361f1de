"""Per-video feature cache reader (libeacs_b200.so eacs_fc_*).

Reads the layout the reference writes and memory-maps (<vid>.npy features,
float16/float32, shape (L, P, d) or (L, d), plus <vid>.ts.npy timestamps;
README section 3.2, data_pipeline/src/npz_to_npy.py, cst_ssm/data/dataset.py:
58-67).  `FeatureCache.read` copies frames out of the read-only mapping with
several threads; `FeatureCache.chunks` streams a video to the GPU in chunks
through two pinned staging buffers, so the upload of chunk k+1 overlaps the
caller's work on chunk k.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib

_DTYPES = {_lib.DTYPE_CODES[torch.float16]: torch.float16, _lib.DTYPE_CODES[torch.float32]: torch.float32}


class FeatureCache:
    """One video's cached features: frames (L, P, d) and timestamps (L,)."""

    def __init__(self, path: str):
        self._h = ctypes.c_void_p()
        _lib.check(_lib.lib().eacs_fc_open(path.encode(), ctypes.byref(self._h)), "eacs_fc_open")
        L, P, d, dt = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int()
        _lib.check(_lib.lib().eacs_fc_info(self._h, ctypes.byref(L), ctypes.byref(P), ctypes.byref(d),
                                           ctypes.byref(dt)), "eacs_fc_info")
        self.L, self.P, self.d = L.value, P.value, d.value
        self.dtype = _DTYPES[dt.value]
        self.path = path

    def close(self) -> None:
        if self._h:
            _lib.lib().eacs_fc_close(self._h)
            self._h = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def frame_shape(self) -> tuple:
        return (self.P, self.d)

    def timestamps(self) -> torch.Tensor:
        out = torch.empty(self.L, dtype=torch.float32)
        _lib.check(_lib.lib().eacs_fc_timestamps(self._h, out.data_ptr()), "eacs_fc_timestamps")
        return out

    def read(self, l0: int = 0, n: int | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
        """Frames [l0, l0+n) as a host tensor (n, P, d) of the file's dtype."""
        n = self.L - l0 if n is None else n
        if out is None:
            out = torch.empty(n, self.P, self.d, dtype=self.dtype)
        if out.numel() < n * self.P * self.d or out.dtype != self.dtype or not out.is_contiguous():
            raise RuntimeError("FeatureCache.read: out must be a contiguous buffer of the file's dtype")
        _lib.check(_lib.lib().eacs_fc_read(self._h, l0, n, out.data_ptr()), "eacs_fc_read")
        return out[:n] if out.dim() == 3 else out

    def chunks(self, chunk: int, device="cuda"):
        """Yield (l0, frames on `device` (n, P, d), timestamps (n,) on `device`).

        Two pinned staging buffers and a side stream: the copy of chunk k+1
        is issued before chunk k is yielded, and the caller's current stream
        waits for a chunk's copy before it uses it."""
        dev = torch.device(device)
        side = torch.cuda.Stream(dev)
        ts = self.timestamps().to(dev)
        nb = chunk * self.P * self.d * torch.finfo(self.dtype).bits // 8
        stage = [torch.empty(nb, dtype=torch.uint8).pin_memory() for _ in range(2)]
        bufs = [torch.empty(chunk, self.P, self.d, dtype=self.dtype, device=dev) for _ in range(2)]
        done = [torch.cuda.Event() for _ in range(2)]
        used = [None, None]  # event after the caller's use of each device buffer

        def issue(k):
            sl = k & 1
            l0 = k * chunk
            n = min(chunk, self.L - l0)
            with torch.cuda.stream(side):
                if used[sl] is not None:
                    side.wait_event(used[sl])
                done[sl].synchronize()  # the staging buffer's previous copy has finished
                _lib.check(_lib.lib().eacs_fc_upload(self._h, l0, n, stage[sl].data_ptr(), nb,
                                                     bufs[sl].data_ptr(), side.cuda_stream),
                           "eacs_fc_upload")
                done[sl].record(side)
            return l0, n

        nchunks = (self.L + chunk - 1) // chunk
        pending = issue(0) if nchunks else None
        for k in range(nchunks):
            l0, n = pending
            if k + 1 < nchunks:
                pending = issue(k + 1)
            sl = k & 1
            cur = torch.cuda.current_stream(dev)
            cur.wait_event(done[sl])
            yield l0, bufs[sl][:n], ts[l0:l0 + n]
            ev = torch.cuda.Event()
            ev.record(cur)
            used[sl] = ev


def write_npy_pair(stem: str, features: np.ndarray, timestamps: np.ndarray) -> str:
    """Write <stem>.npy and <stem>.ts.npy the way the reference's converter does."""
    np.save(stem + ".npy", np.ascontiguousarray(features))
    np.save(stem + ".ts.npy", np.ascontiguousarray(timestamps).astype(np.float32))
    return stem + ".npy"

"""Caller-side device workspace for libabkv entry points.

The C ABI never allocates: every call receives a workspace whose first four
bytes hold the device error word.  This helper keeps one zero-initialised,
256-byte aligned buffer per device and grows it on demand (growth happens
outside any kernel; a grown buffer starts with a clean error word).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib


class Workspace:
    def __init__(self, device: torch.device | int | str | None = None, nbytes: int = 1 << 20):
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self._buf = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=self.device)

    @property
    def nbytes(self) -> int:
        return self._buf.numel()

    def ensure(self, nbytes: int) -> "Workspace":
        if nbytes > self._buf.numel():
            # keep the error word of the old buffer visible to the caller
            old_err = self._buf[:4].clone()
            self._buf = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
            self._buf[:4].copy_(old_err)
        return self

    def ptr(self) -> int:
        return self._buf.data_ptr()

    def read_error(self, stream: torch.cuda.Stream | None = None) -> int:
        """Device error word (ABKV_DEVERR_* bits); clears it.  Synchronises."""
        s = torch.cuda.current_stream(self.device) if stream is None else stream
        v = C.c_int32(0)
        _lib.check("abkv_workspace_error", _lib.lib().abkv_workspace_error(
            C.c_void_p(self.ptr()), C.c_void_p(s.cuda_stream), C.byref(v)))
        return int(v.value)


_per_device: dict[int, Workspace] = {}


def default_workspace(device: torch.device) -> Workspace:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _per_device.get(idx)
    if ws is None:
        ws = _per_device[idx] = Workspace(torch.device("cuda", idx))
    return ws

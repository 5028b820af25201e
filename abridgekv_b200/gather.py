"""KV-head-sharded decode with the all-gather fused into the kernel (host side).

In the optional KV-head-sharded layout rank r of a
node-local process group holds KV heads [r*Hkv/W, (r+1)*Hkv/W) of every
sequence and computes the matching query heads; every rank then needs the full
[B, Hq, D] attention output of each layer.  Instead of a decode launch followed
by an NCCL all-gather (``parallel.gather_head_outputs``), ``HeadGather.decode``
runs ``abkv_decode_gather``: the decode epilogue stores each rank's head rows
straight into every rank's gather buffer (CUDA IPC mappings of plain
cudaMalloc memory, stores over NVLink / NVSwitch), and the kernel's last CTA
completes a flag barrier with the other ranks, so when the launch finishes
every rank holds the whole output.

All ranks must call ``decode`` with the same layers and shapes in the same
order (it is a collective).  ``close`` is collective too.
"""
from __future__ import annotations

import ctypes as C
import math
from typing import Sequence

import torch
import torch.distributed as dist

from . import _lib
from .decode import _validate
from .workspace import Workspace, default_workspace


class _DeviceArray:
    """Zero-copy torch view of raw device memory (__cuda_array_interface__)."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


def _view(ptr: int, shape: tuple[int, ...], device: torch.device) -> torch.Tensor:
    t = torch.as_tensor(_DeviceArray(ptr, shape, "<i2"), device=device)
    return t.view(torch.bfloat16)


class HeadGather:
    """Gather buffers of one process group: `num_layers` output slots of
    [num_seqs, hq_total, head_dim] bf16 on every rank.

    With ``group=None`` and no initialised process group the gather is
    single-rank (world 1): the same kernel path, barrier with itself."""

    def __init__(self, num_layers: int, num_seqs: int, hq_total: int, *, head_dim: int = 128,
                 group=None, device: torch.device | str | None = None, timeout_us: int = 0):
        self.device = torch.device(device) if device is not None else torch.device("cuda",
                                                                                   torch.cuda.current_device())
        self.group = group
        distributed = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if distributed else 1
        self.rank = dist.get_rank(group) if distributed else 0
        if self.world > _lib.MAX_PEERS:
            raise ValueError(f"at most {_lib.MAX_PEERS} ranks")
        if hq_total % self.world:
            raise ValueError("query heads do not split over the ranks")
        self.num_layers, self.num_seqs, self.hq_total, self.head_dim = num_layers, num_seqs, hq_total, head_dim
        self.slot_elems = num_seqs * hq_total * head_dim
        self.nbytes = _lib.GATHER_FLAG_BYTES + num_layers * self.slot_elems * 2
        lib = _lib.lib()
        ptr = C.c_void_p()
        handle = (C.c_ubyte * _lib.PEER_HANDLE_BYTES)()
        with torch.cuda.device(self.device):
            _lib.check("abkv_peer_alloc", lib.abkv_peer_alloc(self.nbytes, C.byref(ptr), handle))
        self._local = int(ptr.value)
        self._opened: list[int] = []
        bufs = [0] * self.world
        bufs[self.rank] = self._local
        if self.world > 1:
            handles: list = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
            with torch.cuda.device(self.device):
                for r in range(self.world):
                    if r == self.rank:
                        continue
                    h = (C.c_ubyte * _lib.PEER_HANDLE_BYTES).from_buffer_copy(handles[r])
                    p = C.c_void_p()
                    _lib.check("abkv_peer_open", lib.abkv_peer_open(h, C.byref(p)))
                    bufs[r] = int(p.value)
                    self._opened.append(bufs[r])
        self._bufs = bufs
        self.epoch = 0
        self.timeout_us = int(timeout_us)  # barrier wait limit per launch (0: the library's 5 s)
        self.outputs = _view(self._local + _lib.GATHER_FLAG_BYTES, (num_layers, num_seqs, hq_total, head_dim),
                             self.device)

    def layer_output(self, layer: int) -> torch.Tensor:
        """[num_seqs, hq_total, head_dim] output slot of `layer` on this rank."""
        return self.outputs[layer]

    def decode(self, layers: Sequence[int], queries: Sequence[torch.Tensor], kv_caches: Sequence[torch.Tensor],
               block_tables: Sequence[torch.Tensor], seq_lens: Sequence[torch.Tensor], *,
               scale: float | None = None, max_pages_per_seq: int | None = None, chunk_tokens: int = 0,
               workspace: Workspace | None = None, stream: torch.cuda.Stream | None = None) -> list[torch.Tensor]:
        """This rank's decode of `layers` (its KV-head shard: queries[i] [B, hq_total/W, D]) with
        the all-gather fused: returns the full [B, hq_total, D] outputs (views of the slots)."""
        if self._local == 0:
            raise RuntimeError("HeadGather is closed")
        L = len(layers)
        if L != len(queries):
            raise ValueError("one query tensor per layer")
        if any(not 0 <= l < self.num_layers for l in layers):
            raise ValueError("layer slot out of range")
        B, Hq, Hkv, D, page, _ = _validate(queries, kv_caches, block_tables, seq_lens, None, alloc=False)
        if B != self.num_seqs or D != self.head_dim or Hq * self.world != self.hq_total:
            raise ValueError(f"shard shape [{B}, {Hq}, {D}] does not match the gather buffers "
                             f"([{self.num_seqs}, {self.hq_total}/{self.world}, {self.head_dim}])")
        if max_pages_per_seq is None:
            max_pages_per_seq = max(int(bt.shape[1]) for bt in block_tables)
        scale = 1.0 / math.sqrt(D) if scale is None else float(scale)
        lib = _lib.lib()
        need = lib.abkv_decode_workspace_size(L, B, Hq, D, page, max_pages_per_seq, chunk_tokens)
        if need == 0:
            raise _lib.AbkvError("abkv_decode_workspace_size", 3, f"unsupported shape (B={B}, Hq={Hq}, D={D})")
        ws = (workspace or default_workspace(self.device)).ensure(need)
        s = torch.cuda.current_stream(self.device) if stream is None else stream
        self.epoch += 1
        g = _lib.GatherT()
        for r, b in enumerate(self._bufs):
            g.rank_buffers[r] = b
        g.buffer_bytes = self.nbytes
        g.world, g.rank, g.hq_total, g.epoch = self.world, self.rank, self.hq_total, self.epoch
        g.timeout_us = self.timeout_us
        outs = [self.outputs[l] for l in layers]
        with torch.cuda.device(self.device):
            st = lib.abkv_decode_gather(
                _lib.ptr_array([q.data_ptr() for q in queries]),
                _lib.ptr_array([kv.data_ptr() for kv in kv_caches]),
                _lib.ptr_array([bt.data_ptr() for bt in block_tables]),
                _lib.i64_array([bt.stride(0) for bt in block_tables]),
                _lib.ptr_array([sl.data_ptr() for sl in seq_lens]),
                _lib.i64_array([kv.shape[0] for kv in kv_caches]),
                _lib.ptr_array([o.data_ptr() for o in outs]),
                L, B, Hq, Hkv, D, page, max_pages_per_seq, scale, chunk_tokens, C.byref(g),
                ws.ptr(), ws.nbytes, s.cuda_stream)
        _lib.check("abkv_decode_gather", st)
        return outs

    def close(self) -> None:
        """Collective: unmap the peers' buffers and free this rank's (after every rank is done
        writing into it)."""
        if self._local == 0:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        lib = _lib.lib()
        with torch.cuda.device(self.device):
            for p in self._opened:
                lib.abkv_peer_close(p)
            if self.world > 1:
                dist.barrier(group=self.group)
            lib.abkv_peer_free(self._local)
        self._opened, self._local, self._bufs = [], 0, []
        self.outputs = None

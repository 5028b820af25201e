"""KV-head-sharded decode with the fused all-gather (abkv_decode_gather) on B200s.

* one rank (no process group): the gather path writes exactly what the plain
  decode writes, over repeated epochs;
* a barrier flag that no rank ever sets: the kernel gives up after its time
  limit, reports ABKV_DEVERR_TIMEOUT and the context stays usable;
* two ranks on two GPUs (skipped with fewer): each rank decodes its half of the
  KV heads and ends up with every head's output, which matches the float64
  oracle within the decode tolerances.
"""
import ctypes as C
import os
import socket

import numpy as np
import pytest
import torch

from abridgekv_b200 import _lib, decode
from abridgekv_b200.gather import HeadGather
from abridgekv_b200.workspace import Workspace
from oracle.decode_ref import decode_exact
from oracle.synth import paged_case

pytestmark = pytest.mark.gpu
ATOL_EXACT, MEAN_EXACT = 1.5e-2, 2e-3


def _case(seed=5, hq=8, hkv=2, lens=(300, 17, 1000, 64)):
    c = paged_case(seed, list(lens), num_q_heads=hq, num_kv_heads=hkv)
    dev = lambda x, dt=None: torch.from_numpy(x).to(dt).cuda() if dt else torch.from_numpy(x).cuda()  # noqa: E731
    return c, dev(c.q, torch.bfloat16), dev(c.kv, torch.bfloat16), dev(c.block_table), dev(c.seq_lens)


def test_gather_single_rank_equals_plain_decode():
    c, q, kv, bt, sl = _case()
    ref = decode.paged_decode([q, q], [kv, kv], [bt, bt], [sl, sl])
    g = HeadGather(num_layers=3, num_seqs=q.shape[0], hq_total=q.shape[1])
    ws = Workspace()
    try:
        for _ in range(4):
            outs = g.decode([2, 0], [q, q], [kv, kv], [bt, bt], [sl, sl], workspace=ws)
        torch.cuda.synchronize()
        assert ws.read_error() == 0
        assert g.epoch == 4
        assert torch.equal(outs[0], ref[0]) and torch.equal(outs[1], ref[1])
        assert torch.equal(g.layer_output(2), ref[0]) and torch.equal(g.layer_output(0), ref[0])
        assert torch.all(g.layer_output(1) == 0)  # untouched slot stays zero
    finally:
        g.close()


def test_gather_barrier_times_out_when_a_flag_never_arrives():
    """world=2 with a second local buffer standing in for a peer that never launches: the
    last CTA's wait runs out (100 ms), the error word says TIMEOUT, the next call works."""
    c, q, kv, bt, sl = _case()
    lib = _lib.lib()
    B, Hq, D = q.shape
    nbytes = _lib.GATHER_FLAG_BYTES + B * 2 * Hq * D * 2
    bufs = []
    for _ in range(2):
        p = C.c_void_p()
        h = (C.c_ubyte * _lib.PEER_HANDLE_BYTES)()
        _lib.check("abkv_peer_alloc", lib.abkv_peer_alloc(nbytes, C.byref(p), h))
        bufs.append(p.value)
    try:
        g = _lib.GatherT()
        g.rank_buffers[0], g.rank_buffers[1] = bufs
        g.buffer_bytes, g.world, g.rank, g.hq_total, g.epoch, g.timeout_us = nbytes, 2, 0, 2 * Hq, 1, 100000
        ws = Workspace()
        need = lib.abkv_decode_workspace_size(1, B, Hq, D, c.page, bt.shape[1], 0)
        ws.ensure(need)
        st = lib.abkv_decode_gather(
            _lib.ptr_array([q.data_ptr()]), _lib.ptr_array([kv.data_ptr()]), _lib.ptr_array([bt.data_ptr()]),
            _lib.i64_array([bt.stride(0)]), _lib.ptr_array([sl.data_ptr()]), _lib.i64_array([kv.shape[0]]),
            _lib.ptr_array([bufs[0] + _lib.GATHER_FLAG_BYTES]), 1, B, Hq, 2, D, c.page, bt.shape[1],
            float(c.scale), 0, C.byref(g), ws.ptr(), ws.nbytes, torch.cuda.current_stream().cuda_stream)
        assert st == 0
        torch.cuda.synchronize()
        assert ws.read_error() & 0x4
        # the context is still usable
        out = decode.paged_decode([q], [kv], [bt], [sl], workspace=ws)
        torch.cuda.synchronize()
        assert ws.read_error() == 0 and torch.isfinite(out[0].float()).all()
    finally:
        for b in bufs:
            lib.abkv_peer_free(b)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _two_rank_worker(rank, world, port):
    import datetime

    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        c = paged_case(11, [700, 33, 1500, 16, 250, 901], num_q_heads=32, num_kv_heads=8)
        hk = 8 // world
        sl_heads = slice(rank * hk, (rank + 1) * hk)
        q = torch.from_numpy(c.q[:, rank * hk * 4:(rank + 1) * hk * 4].copy()).to(torch.bfloat16).cuda()
        kv = torch.from_numpy(c.kv[:, :, :, sl_heads].copy()).to(torch.bfloat16).cuda()
        bt = torch.from_numpy(c.block_table).cuda()
        sl = torch.from_numpy(c.seq_lens).cuda()
        g = HeadGather(num_layers=2, num_seqs=q.shape[0], hq_total=32)
        ws = Workspace()
        try:
            for _ in range(3):
                out = g.decode([1], [q], [kv], [bt], [sl], workspace=ws)[0]
            torch.cuda.synchronize()
            assert ws.read_error() == 0
            exact = decode_exact(c.q, c.kv, c.block_table, c.seq_lens, c.scale, c.page)
            err = np.abs(out.float().cpu().numpy() - exact)
            assert err.max() <= ATOL_EXACT and err.mean() <= MEAN_EXACT, (rank, err.max(), err.mean())
        finally:
            g.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_gather_two_ranks_assemble_all_heads():
    import torch.multiprocessing as mp

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_two_rank_worker, args=(2, _free_port()), nprocs=2, join=True)

"""abkv_decode_noalloc: decode for callers that cannot allocate device memory.

Engines that reserve all of HBM for their KV cache up front, or that must not
call into an allocator from the decode thread, cannot hand libabkv a
workspace.  This entry point keeps its split-KV scratch in a fixed 32 MiB
device array inside the library instead.  The test calls it through the C ABI
(ctypes, raw pointers) and requires its output to be bit-identical to the
workspace-based abkv_decode (same kernel, same chunk plan): on a first call,
then after a call with a larger plan has left its partials and counters in
the shared array, then once more.  It also checks that a request needing more
than the fixed scratch is refused before anything runs.  This file sorts last
so that a run stopping at the first failure has already run every other test.
"""
import ctypes as C

import pytest
import torch

from abridgekv_b200 import _lib, decode
from oracle.synth import paged_case

pytestmark = pytest.mark.gpu

ABKV_ERR_SCRATCH_LIMIT = 10


def _case(seed, lens):
    # long enough for several split-KV chunks, so the scratch partials and the
    # per-(layer, sequence) counters are used
    case = paged_case(seed, lens, num_q_heads=32, num_kv_heads=8, head_dim=128, page=16)
    q = torch.from_numpy(case.q).to(torch.bfloat16).cuda()
    kv = torch.from_numpy(case.kv).to(torch.bfloat16).cuda()
    bt = torch.from_numpy(case.block_table).cuda()
    sl = torch.from_numpy(case.seq_lens).cuda()
    return case, q, kv, bt, sl


def _noalloc(q, kv, bt, sl, out, max_pages, chunk_tokens, scale, err):
    lib = _lib.lib()
    B, Hq, D = q.shape
    return lib.abkv_decode_noalloc(
        _lib.ptr_array([q.data_ptr()]), _lib.ptr_array([kv.data_ptr()]), _lib.ptr_array([bt.data_ptr()]),
        _lib.i64_array([bt.stride(0)]), _lib.ptr_array([sl.data_ptr()]), _lib.i64_array([kv.shape[0]]),
        _lib.ptr_array([out.data_ptr()]), 1, B, Hq, kv.shape[3], D, kv.shape[2], max_pages, C.c_float(scale),
        chunk_tokens, C.c_void_p(err.data_ptr() if err is not None else 0),
        C.c_void_p(torch.cuda.current_stream().cuda_stream))


def _check_call(tag, case, q, kv, bt, sl, ref, chunk_tokens, err):
    out = torch.full_like(ref, float("nan"))
    st = _noalloc(q, kv, bt, sl, out, bt.shape[1], chunk_tokens, case.scale, err)
    assert st == 0, _lib.status_string(st)
    torch.cuda.synchronize()
    assert int(err.item()) == 0, f"{tag}: device error bits {int(err.item())}"
    assert torch.equal(out, ref), (tag, (out.float() - ref.float()).abs().max().item())


@pytest.mark.parametrize("chunk_tokens", [256, 0])
def test_noalloc_equals_workspace_decode_across_calls(chunk_tokens):
    small = _case(21, [3000, 17, 1025, 4096, 1, 700])
    # more sequences and longer ones: a larger split-KV plan, whose partials and
    # counters stay in the shared array after it returns
    large = _case(22, [6000, 4100, 33, 5000, 2048, 7777, 129, 4600, 3333, 6100, 2, 5555])
    refs = []
    for case, q, kv, bt, sl in (small, large):
        refs.append(decode.paged_decode([q], [kv], [bt], [sl], scale=case.scale, chunk_tokens=chunk_tokens,
                                        max_pages_per_seq=bt.shape[1])[0])
    err = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    _check_call("first call", *small, refs[0], chunk_tokens, err)
    _check_call("larger plan", *large, refs[1], chunk_tokens, err)
    _check_call("after the larger plan", *small, refs[0], chunk_tokens, err)


def test_noalloc_refuses_requests_beyond_its_scratch():
    lib = _lib.lib()
    need = lib.abkv_decode_workspace_size(36, 64, 32, 128, 16, 544, 256)
    assert need > (32 << 20)
    fake = 1 << 20  # never dereferenced: the size check comes first
    arr = _lib.ptr_array([fake] * 36)
    st = lib.abkv_decode_noalloc(arr, arr, arr, _lib.i64_array([544] * 36), arr, _lib.i64_array([1 << 20] * 36),
                                 arr, 36, 64, 32, 8, 128, 16, 544, C.c_float(0.088), 256, None,
                                 C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == ABKV_ERR_SCRATCH_LIMIT
    assert "32 MiB" in _lib.status_string(st)

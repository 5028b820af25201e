"""libabkv.so loads, exports every entry point declared in include/*.h, and its
host-side validation rejects bad arguments before any launch (CPU-only test)."""
import ctypes as C
import re
from pathlib import Path

import pytest

from abridgekv_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]


def declared_functions() -> list[str]:
    names = []
    for h in sorted((ROOT / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names += re.findall(r"^\s*(?:[\w\s\*]+?)\b(abkv_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    names = declared_functions()
    assert len(names) >= 4
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/ but not exported"
    # and the ctypes binding covers exactly what the header declares
    assert sorted(_lib.SIGNATURES) == names


def test_status_strings_and_version():
    assert _lib.status_string(0) == "ok"
    assert "workspace" in _lib.status_string(2)
    assert _lib.lib().abkv_version().decode().startswith("abkv")


def test_decode_workspace_size():
    lib = _lib.lib()
    n = lib.abkv_decode_workspace_size(36, 64, 32, 128, 16, 544, 0)
    assert n > 0 and n % 256 == 0
    assert lib.abkv_decode_workspace_size(36, 64, 32, 96, 16, 544, 0) == 0   # head_dim 96 unsupported
    assert lib.abkv_decode_workspace_size(2, 1, 4, 64, 16, 128, 0) > 0      # head_dim 64 (config 1)
    assert lib.abkv_decode_workspace_size(36, 64, 32, 128, 8, 544, 0) == 0   # page 8 unsupported
    assert lib.abkv_decode_workspace_size(1, 1, 8, 128, 16, 1, 0) == 256     # single chunk: header only


@pytest.mark.parametrize("bad", ["null_q", "kv_heads", "group", "scale", "workspace", "chunk"])
def test_decode_validation_rejects_before_launch(bad):
    lib = _lib.lib()
    fake = 1 << 20  # never dereferenced: validation fails first
    q = _lib.ptr_array([0 if bad == "null_q" else fake])
    kv = _lib.ptr_array([fake])
    bt = _lib.ptr_array([fake])
    sl = _lib.ptr_array([fake])
    out = _lib.ptr_array([fake])
    strides = _lib.i64_array([4])
    nblk = _lib.i64_array([16])
    hq, hkv = 8, 2
    if bad == "kv_heads":
        hq, hkv = 6, 3
    if bad == "group":
        hq, hkv = 32, 2
    scale = -1.0 if bad == "scale" else 0.088
    ws, ws_bytes = (0, 0) if bad == "workspace" else (fake, 1 << 30)
    chunk = 24 if bad == "chunk" else 0
    st = lib.abkv_decode(q, kv, bt, strides, sl, nblk, out, 1, 2, hq, hkv, 128, 16, 4, scale, chunk,
                         ws, ws_bytes, None)
    assert st in (1, 2, 3), st


@pytest.mark.parametrize("bad", ["no_gather", "epoch", "world", "rank", "hq_total", "unaligned", "out_in_flags",
                                 "out_past_end"])
def test_decode_gather_validation_rejects_before_launch(bad):
    """abkv_decode_gather checks its gather descriptor (and that every output slot lies in
    this rank's buffer past the flag area) before touching the GPU."""
    lib = _lib.lib()
    fake = 1 << 20
    base = 1 << 30
    B, hq, hkv, D = 2, 4, 1, 128
    world = 2
    slot = B * hq * world * D * 2
    g = _lib.GatherT()
    g.rank_buffers[0], g.rank_buffers[1] = base, base + (1 << 28)
    g.buffer_bytes = _lib.GATHER_FLAG_BYTES + slot
    g.world, g.rank, g.hq_total, g.epoch = world, 0, hq * world, 1
    out_ptr = base + _lib.GATHER_FLAG_BYTES
    if bad == "epoch":
        g.epoch = 0
    if bad == "world":
        g.world = 9
    if bad == "rank":
        g.rank = 2
    if bad == "hq_total":
        g.hq_total = hq
    if bad == "unaligned":
        g.rank_buffers[1] = base + 64
    if bad == "out_in_flags":
        out_ptr = base + 16
    if bad == "out_past_end":
        out_ptr = base + _lib.GATHER_FLAG_BYTES + 256
    st = lib.abkv_decode_gather(
        _lib.ptr_array([fake]), _lib.ptr_array([fake]), _lib.ptr_array([fake]), _lib.i64_array([4]),
        _lib.ptr_array([fake]), _lib.i64_array([16]), _lib.ptr_array([out_ptr]), 1, B, hq, hkv, D, 16, 4,
        0.088, 0, None if bad == "no_gather" else C.byref(g), fake, 1 << 30, None)
    assert st == 1, st


def test_gather_struct_layout():
    # abkv_gather_t: 8 pointers, size_t, 3 ints, 2 uint32 (natural alignment, no packing)
    assert C.sizeof(_lib.GatherT) == 8 * 8 + 8 + 4 * 5 + 4
    assert _lib.GatherT.epoch.offset == 84


def test_prefill_backward_workspace_size():
    lib = _lib.lib()
    n = lib.abkv_prefill_masked_backward_workspace_size(16, 32, 12288, 128)
    rows = 16 * 32 * 12288
    assert n >= rows * 128 * 4 + rows * 4 and n % 256 == 0   # fp32 dQ accumulator + rowsum(dO * O)
    assert lib.abkv_prefill_masked_backward_workspace_size(1, 4, 512, 96) == 0   # head_dim 96 unsupported
    assert lib.abkv_prefill_masked_backward_workspace_size(0, 4, 512, 128) == 0


@pytest.mark.parametrize("bad", ["null_dout", "heads", "scale", "head_dim", "layout", "unaligned", "stride",
                                 "workspace"])
def test_prefill_backward_validation_rejects_before_launch(bad):
    """abkv_prefill_masked_backward checks pointers, shapes, alignment, strides and the workspace before
    it encodes a tensor map or launches anything."""
    lib = _lib.lib()
    fake = 1 << 20  # never dereferenced: validation fails first
    ptr = {n: fake for n in ("q", "k", "v", "out", "dout", "lse", "dq", "dk", "dv")}
    if bad == "null_dout":
        ptr["dout"] = 0
    if bad == "unaligned":
        ptr["dq"] = fake + 8
    B, H, Hkv, S, D, Cc, K = 1, 4, 2, 512, 128, 128, 128
    if bad == "heads":
        H, Hkv = 6, 4
    if bad == "head_dim":
        D = 96
    if bad == "layout":
        S = 500
    scale = -1.0 if bad == "scale" else 0.088
    st_q = _lib.i64_array([H * S * D, S * D, D])
    st_kv = _lib.i64_array([Hkv * S * D, S * D, D])
    st_dq = _lib.i64_array([H * S * D, S * D, D + 4]) if bad == "stride" else st_q
    ws, ws_bytes = (0, 0) if bad == "workspace" else (fake, 1 << 30)
    st = lib.abkv_prefill_masked_backward(
        ptr["q"], st_q, ptr["k"], st_kv, ptr["v"], st_kv, ptr["out"], st_q, ptr["dout"], st_q, ptr["lse"],
        ptr["dq"], st_dq, ptr["dk"], st_kv, ptr["dv"], st_kv, None, None, B, H, Hkv, S, D, Cc, K, scale, ws,
        ws_bytes, None)
    expect = {"null_dout": 1, "heads": 1, "scale": 1, "head_dim": 3, "layout": 3, "unaligned": 1, "stride": 1,
              "workspace": 2}[bad]
    assert st == expect, (bad, st)


def test_code_step_compact_workspace_size():
    lib = _lib.lib()
    n = lib.abkv_code_step_compact_workspace_size(64, 8192)
    assert n >= 256 + 64 * 4 + 65 * 4 + 8192 * 16 and n % 256 == 0
    assert lib.abkv_code_step_compact_workspace_size(0, 10) == 0
    assert lib.abkv_code_step_compact_workspace_size(4, -1) == 0


@pytest.mark.parametrize("bad", ["offsets_start", "offsets_end", "offsets_order", "block_oob", "offset_oob",
                                 "dst_repeats", "dst_is_src", "workspace"])
def test_code_step_compact_rejects_ops_before_launch(bad):
    """abkv_code_step_attention_compact checks the copy ops (offsets, bounds, a destination that repeats
    or is also a source) and the workspace before any upload or launch."""
    lib = _lib.lib()
    fake = 1 << 20  # never dereferenced: validation fails first
    R, nb, page = 2, 10, 16
    ops = [[1, 0, 2, 0], [1, 1, 2, 1], [3, 0, 4, 0], [3, 1, 4, 1]]
    off = [0, 2, 4]
    if bad == "offsets_start":
        off = [1, 2, 4]
    if bad == "offsets_end":
        off = [0, 2, 3]
    if bad == "offsets_order":
        off = [0, 3, 2]
    if bad == "block_oob":
        ops[2][0] = nb
    if bad == "offset_oob":
        ops[3][3] = page
    if bad == "dst_repeats":
        ops[3][2:] = ops[2][2:]
    if bad == "dst_is_src":
        ops[3][2:] = ops[0][:2]
    flat = (C.c_int32 * 16)(*[x for op in ops for x in op])
    offs = _lib.i64_array(off)
    ws, ws_bytes = (fake, 64) if bad == "workspace" else (fake, 1 << 30)
    st = lib.abkv_code_step_attention_compact(
        fake, 32 * 128, 128, fake, 32 * 128, 128, fake, fake, 0, nb, page, fake, 8, fake, None,
        _lib.i32_array([128] * 8), R, 32, 8, 128, 256, 512, 0.088, flat, offs, len(ops), ws, ws_bytes, None)
    expect = {"offsets_start": 1, "offsets_end": 1, "offsets_order": 1, "block_oob": 1, "offset_oob": 1,
              "dst_repeats": 3, "dst_is_src": 3, "workspace": 2}[bad]
    assert st == expect, (bad, st)

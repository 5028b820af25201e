"""Decode kernel parity through the C ABI (libabkv.so) on a B200.

Tolerances (bf16 outputs): the kernel computes scores in fp32 while the
reference rounds them to bf16, so its results sit closer to the float64 truth
than the reference's; both must stay within
  |gpu - reference| <= 3e-2 and |gpu - float64| <= 1.5e-2 (max abs),
with mean abs error vs float64 below 2e-3; relative error (max |gpu - float64|
/ max |float64| and the per-element median, tests/errstats.py) is reported and
bounded as well.
"""
import numpy as np
import pytest
import torch

from abridgekv_b200 import decode
from abridgekv_b200.workspace import Workspace
from oracle.decode_ref import decode_exact
from tests.errstats import assert_relative, report
from tests.goldens import decode_cases, load_decode

pytestmark = pytest.mark.gpu

ATOL_REF = 3e-2
ATOL_EXACT = 1.5e-2
MEAN_EXACT = 2e-3


def _dev(case):
    q = torch.from_numpy(case.q).to(torch.bfloat16).cuda()
    kv = torch.from_numpy(case.kv).to(torch.bfloat16).cuda()
    bt = torch.from_numpy(case.block_table).cuda()
    sl = torch.from_numpy(case.seq_lens).cuda()
    return q, kv, bt, sl


@pytest.mark.parametrize("chunk_tokens", [0, 32, 256])
@pytest.mark.parametrize("name", decode_cases())
def test_decode_matches_reference_golden(name, chunk_tokens):
    case, ref = load_decode(name)
    if chunk_tokens and chunk_tokens % case.page:
        pytest.skip("chunk must be a multiple of the page size")
    q, kv, bt, sl = _dev(case)
    ws = Workspace()
    out = decode.paged_decode([q], [kv], [bt], [sl], scale=case.scale, chunk_tokens=chunk_tokens,
                              workspace=ws)[0]
    got = out.float().cpu().numpy()
    assert ws.read_error() == 0
    assert np.isfinite(got).all(), "kernel read a poisoned row or page"
    exact = decode_exact(case.q, case.kv, case.block_table, case.seq_lens, case.scale, case.page)
    se, sr = report(f"{name} chunk={chunk_tokens}", got, exact, ref)
    assert sr["max_abs"] <= ATOL_REF
    assert se["max_abs"] <= ATOL_EXACT
    assert se["mean_abs"] <= MEAN_EXACT
    assert_relative(se, name)


def test_multi_layer_launch_equals_single_layer_calls():
    """One launch over several layers (different tables, lengths, caches) gives
    bit-identical rows to per-layer calls."""
    cases = [load_decode(n)[0] for n in ("g4_ragged", "g4_ragged", "g4_ragged")]
    devs = [_dev(c) for c in cases]
    # vary the per-layer seq_lens (shorter prefixes of the same tables)
    devs[1] = (devs[1][0], devs[1][1], devs[1][2], torch.clamp(devs[1][3] - 7, min=0))
    devs[2] = (devs[2][0] * 0.5, devs[2][1], devs[2][2], devs[2][3] // 2)
    qs, kvs, bts, sls = [list(x) for x in zip(*devs)]
    qs = [q.contiguous() for q in qs]
    multi = decode.paged_decode(qs, kvs, bts, sls, chunk_tokens=32)
    for l in range(3):
        single = decode.paged_decode([qs[l]], [kvs[l]], [bts[l]], [sls[l]], chunk_tokens=32)[0]
        assert torch.equal(multi[l], single)


def test_empty_sequence_gives_zero_row():
    case, _ = load_decode("g4_ragged")
    q, kv, bt, sl = _dev(case)
    sl = sl.clone()
    sl[2] = 0
    out = decode.paged_decode([q], [kv], [bt], [sl])[0]
    assert torch.count_nonzero(out[2]) == 0
    assert torch.isfinite(out.float()).all()


def test_out_of_range_page_is_flagged_not_read():
    case, _ = load_decode("g4_ragged")
    q, kv, bt, sl = _dev(case)
    bt = bt.clone()
    bt[4, 1] = kv.shape[0] + 1000  # inside seq_len 100 -> must be rejected by the kernel
    ws = Workspace()
    out = decode.paged_decode([q], [kv], [bt], [sl], workspace=ws)[0]
    err = ws.read_error()
    assert err & 0x1, err  # ABKV_DEVERR_PAGE_OOB
    assert torch.isfinite(out.float()).all()
    assert ws.read_error() == 0  # reading clears the word


def test_seq_len_beyond_table_is_flagged():
    case, _ = load_decode("g4_ragged")
    q, kv, bt, sl = _dev(case)
    sl = sl.clone()
    sl[0] = bt.shape[1] * case.page + 5
    ws = Workspace()
    out = decode.paged_decode([q], [kv], [bt], [sl], workspace=ws)[0]
    assert ws.read_error() & 0x2  # ABKV_DEVERR_SEQ_OOB
    assert torch.isfinite(out[1:].float()).all()


def _torch_fp32_decode(q, kv, bt, sl, page, scale):
    """Plain PyTorch fp32 reference on the GPU (for full-size checks)."""
    B, Hq, D = q.shape
    Hkv = kv.shape[3]
    out = torch.empty((B, Hq, D), dtype=torch.float32, device=q.device)
    for b in range(B):
        n = int(sl[b])
        r = torch.arange(n, device=q.device)
        pages = bt[b, r // page].long()
        k = kv[pages, 0, r % page].float()  # [n, Hkv, D]
        v = kv[pages, 1, r % page].float()
        k = k.repeat_interleave(Hq // Hkv, dim=1)
        v = v.repeat_interleave(Hq // Hkv, dim=1)
        s = torch.einsum("hd,thd->ht", q[b].float(), k) * scale
        w = torch.softmax(s, dim=-1)
        out[b] = torch.einsum("ht,thd->hd", w, v)
    return out


def test_config2_full_size_sampled_rows_and_page_permutation():
    """BASELINE config 2 at full size (B=64, 36 layers, ~42 GB of KV): sampled
    (layer, sequence) rows against a PyTorch fp32 reference, and bit-identical
    outputs after physically permuting every page (a size-independent property)."""
    from abridgekv_b200.workloads import qwen3_decode_workload

    wl = qwen3_decode_workload(2)
    outs = decode.paged_decode(wl.queries, wl.kv_caches, wl.block_tables, wl.seq_lens, chunk_tokens=1024)
    scale = 1.0 / np.sqrt(wl.head_dim)
    rng = np.random.default_rng(0)
    for l in rng.choice(wl.num_layers, 4, replace=False):
        seqs = rng.choice(wl.num_seqs, 3, replace=False)
        sel = torch.as_tensor(seqs, device="cuda")
        ref = _torch_fp32_decode(wl.queries[l][sel], wl.kv_caches[l], wl.block_tables[l][sel],
                                 wl.seq_lens[l][sel], wl.page, scale)
        err = (outs[l][sel].float() - ref).abs()
        assert err.max().item() <= ATOL_EXACT, (l, err.max().item())
    # page permutation invariance, on three layers (one per quota)
    for l in (0, 1, 7):
        kv = wl.kv_caches[l]
        perm = torch.randperm(kv.shape[0], device="cuda", generator=torch.Generator("cuda").manual_seed(l))
        inv = torch.empty_like(perm)
        inv[perm] = torch.arange(kv.shape[0], device="cuda")
        kv2 = kv[perm].contiguous()          # new page i holds old page perm[i]
        bt2 = inv[wl.block_tables[l].long()].to(torch.int32)
        o2 = decode.paged_decode([wl.queries[l]], [kv2], [bt2], [wl.seq_lens[l]],
                                 max_pages_per_seq=wl.max_pages, chunk_tokens=1024)[0]
        o1 = decode.paged_decode([wl.queries[l]], [kv], [wl.block_tables[l]], [wl.seq_lens[l]],
                                 max_pages_per_seq=wl.max_pages, chunk_tokens=1024)[0]
        assert torch.equal(o1, o2)
        del kv2
    # the all-layer launch and per-layer launches agree bitwise
    for l in (3, 20):
        o1 = decode.paged_decode([wl.queries[l]], [wl.kv_caches[l]], [wl.block_tables[l]],
                                 [wl.seq_lens[l]], max_pages_per_seq=wl.max_pages, chunk_tokens=1024)[0]
        assert torch.equal(o1, outs[l])
    # with all 8 KV heads the automatic chunk stays at 2048 rows
    auto = decode.paged_decode(wl.queries, wl.kv_caches, wl.block_tables, wl.seq_lens,
                               max_pages_per_seq=wl.max_pages)
    fixed = decode.paged_decode(wl.queries, wl.kv_caches, wl.block_tables, wl.seq_lens,
                                max_pages_per_seq=wl.max_pages, chunk_tokens=2048)
    assert all(torch.equal(a, b) for a, b in zip(auto, fixed))


def test_config5_one_kv_head_shard_auto_chunk():
    """Config 5's KV-head shard at full size (1 KV head, 256 sequences, 36 layers): the
    automatic chunk grows to 6144 rows for a 1-head launch (bitwise equal to an explicit
    6144-row chunk), workspace sized without the head count still fits, and sampled rows
    match a PyTorch fp32 reference."""
    from abridgekv_b200.workloads import qwen3_decode_workload

    wl = qwen3_decode_workload(5, num_seqs=256, kv_heads=slice(0, 1))
    ws = Workspace()
    auto = decode.paged_decode(wl.queries, wl.kv_caches, wl.block_tables, wl.seq_lens,
                               max_pages_per_seq=wl.max_pages, workspace=ws)
    assert ws.read_error() == 0
    fixed = decode.paged_decode(wl.queries, wl.kv_caches, wl.block_tables, wl.seq_lens,
                                max_pages_per_seq=wl.max_pages, chunk_tokens=6144)
    assert all(torch.equal(a, b) for a, b in zip(auto, fixed))
    # one layer per launch (the KV-head-sharded mode): >= 4 items per SM gives 2048-row chunks
    one = decode.paged_decode(wl.queries[:1], wl.kv_caches[:1], wl.block_tables[:1], wl.seq_lens[:1],
                              max_pages_per_seq=wl.max_pages, workspace=ws)[0]
    assert ws.read_error() == 0
    one_fixed = decode.paged_decode(wl.queries[:1], wl.kv_caches[:1], wl.block_tables[:1], wl.seq_lens[:1],
                                    max_pages_per_seq=wl.max_pages, chunk_tokens=2048)[0]
    assert torch.equal(one, one_fixed)
    scale = 1.0 / np.sqrt(wl.head_dim)
    rng = np.random.default_rng(5)
    for l in rng.choice(wl.num_layers, 3, replace=False):
        sel = torch.as_tensor(rng.choice(wl.num_seqs, 3, replace=False), device="cuda")
        ref = _torch_fp32_decode(wl.queries[l][sel], wl.kv_caches[l], wl.block_tables[l][sel],
                                 wl.seq_lens[l][sel], wl.page, scale)
        err = (auto[l][sel].float() - ref).abs()
        assert err.max().item() <= ATOL_EXACT, (l, err.max().item())


def _random_layers(L, B=48, Hq=32, Hkv=8, D=128, page=16, max_pages=64, seed=0):
    g = torch.Generator("cuda").manual_seed(seed)
    qs, kvs, bts, sls = [], [], [], []
    for _ in range(L):
        nb = B * max_pages
        kvs.append(torch.randn((nb, 2, page, Hkv, D), generator=g, device="cuda").to(torch.bfloat16))
        qs.append(torch.randn((B, Hq, D), generator=g, device="cuda").to(torch.bfloat16))
        bts.append(torch.randperm(nb, generator=g, device="cuda").to(torch.int32).view(B, max_pages).contiguous())
        sls.append(torch.randint(0, max_pages * page + 1, (B,), generator=g, device="cuda", dtype=torch.int32))
    return qs, kvs, bts, sls


def test_workspace_reuse_across_plans():
    """A workspace used by a small split launch (its partials land where a larger plan keeps
    its chunk counters) gives the larger plan the same rows as a fresh workspace."""
    qs, kvs, bts, sls = _random_layers(4)
    ws = Workspace()
    fresh = decode.paged_decode(qs, kvs, bts, sls, chunk_tokens=64, workspace=Workspace())
    for _ in range(2):
        decode.paged_decode(qs[:1], kvs[:1], bts[:1], sls[:1], chunk_tokens=64, workspace=ws)
        again = decode.paged_decode(qs, kvs, bts, sls, chunk_tokens=64, workspace=ws)
        assert ws.read_error() == 0
        for a, b in zip(again, fresh):
            assert torch.equal(a, b)


@pytest.mark.parametrize("name", ["g4_ragged", "qwen3_heads", "config1_d64"])
def test_dropin_attend_decode_batched_and_forward_decode(name):
    """The two functions a maintainer binds (decode.attend_decode_batched in place of
    PackedKVSidecar._attend_decode_batched, decode.forward_decode in AttentionImpl.forward's
    shape) on the golden inputs: host seq_lens (vLLM's _seq_lens_cpu), a [T, Hq*D] output that
    is written in place for the first n rows only, and a block table with extra rows."""
    case, ref = load_decode(name)
    q, kv, bt, _ = _dev(case)
    n, Hq, D = q.shape
    Hkv = kv.shape[3]
    exact = decode_exact(case.q, case.kv, case.block_table, case.seq_lens, case.scale, case.page)
    sl_host = torch.from_numpy(case.seq_lens.astype(np.int32))
    # vLLM pads the batch: two extra query rows and block-table rows that must stay untouched
    q_pad = torch.cat([q, torch.randn((2, Hq, D), device="cuda").to(torch.bfloat16)])
    bt_pad = torch.cat([bt, torch.zeros((2, bt.shape[1]), dtype=torch.int32, device="cuda")])
    output = torch.full((n + 2, Hq * D), 7.0, dtype=torch.bfloat16, device="cuda")
    decode.attend_decode_batched(query=q_pad, kv_cache=kv, output=output, seq_lens=sl_host, block_table=bt_pad,
                                 num_kv_heads=Hkv, groups=Hq // Hkv, scale=case.scale, num_requests=n)
    got = output[:n].view(n, Hq, D).float().cpu().numpy()
    assert torch.all(output[n:] == 7.0), "rows past the active requests were written"
    se, sr = report(f"attend_decode_batched {name}", got, exact, ref)
    assert se["max_abs"] <= ATOL_EXACT and se["mean_abs"] <= MEAN_EXACT and sr["max_abs"] <= ATOL_REF
    assert_relative(se, name)
    # the same rows through the direct launch
    direct = decode.paged_decode([q], [kv], [bt], [torch.from_numpy(case.seq_lens).cuda()], scale=case.scale)[0]
    assert torch.equal(output[:n].view(n, Hq, D), direct)
    # AttentionImpl.forward shape: [T, Hq, D] query, [T, Hq*D] output (allocated or given)
    out2 = decode.forward_decode(q, kv, bt, sl_host, case.scale)
    assert out2.shape == (n, Hq * D) and torch.equal(out2.view(n, Hq, D), direct)
    given = torch.empty((n, Hq * D), dtype=torch.bfloat16, device="cuda")
    assert decode.forward_decode(q, kv, bt, sl_host, case.scale, output=given) is given
    assert torch.equal(given, out2)

"""The vLLM-shaped attention boundary on a B200 (abridgekv_b200.attention), driven with fake
metadata objects the way the reference's own vLLM-state tests drive the overlay
(scripts/test_compresslm_vllm_state.py:16-58):

* AbkvAttentionImpl.forward(layer, query, key, value, kv_cache, attn_metadata, output) of a KV-cache
  group: the step's K/V rows written through slot_mapping (abkv_store_kv), then
  - a decode step (causal, one row per request) against the reference decode goldens,
  - prompt / chunked-prefill steps (causal, ragged rows) against the reference's causal goldens,
  - a code step with the group's CodeStepMask against float64 attention under the reference's own
    build_layer_quota_masks output;
* maybe_override_attention(layer, query, kv_cache, attn_metadata, output), the packed per-head-quota
  hook: decode with and without sidecar pages, and the code step with per-KV-head quotas and
  exclusion ranges, against the goldens the reference's PackedKVSidecar produced.

Tolerances: those of the kernel tests (tests/test_decode_gpu.py, tests/test_codestep_gpu.py), with
relative error reported and bounded (tests/errstats.py).
"""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from abridgekv_b200 import attention
from abridgekv_b200.sidecar import PackedKVLayout
from abridgekv_b200.workspace import Workspace
from oracle.decode_ref import codestep_exact, decode_exact, packed_decode_exact, paged_causal_exact
from tests.errstats import assert_relative, report
from tests.goldens import (causal_cases, codestep_cases, load_causal, load_codestep, load_decode, load_packed,
                           load_qmask, packed_cases)

pytestmark = pytest.mark.gpu
ATOL_EXACT, MEAN_EXACT, ATOL_REF = 2.5e-2, 2e-3, 3e-2


def _bf(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(torch.bfloat16).cuda()


def _common(qlens, case, causal=True, mask=None, slots=None):
    qsl = torch.tensor(np.concatenate([[0], np.cumsum(qlens)]), dtype=torch.int32)
    T = int(sum(qlens))
    return SimpleNamespace(
        query_start_loc=qsl.cuda(), query_start_loc_cpu=qsl, seq_lens=torch.from_numpy(case.seq_lens).cuda(),
        _seq_lens_cpu=torch.from_numpy(case.seq_lens), num_reqs=len(qlens), num_actual_tokens=T,
        max_query_len=int(max(qlens)), block_table_tensor=torch.from_numpy(case.block_table).cuda(),
        slot_mapping=(slots if slots is not None else torch.full((T,), -1, dtype=torch.int64)).cuda(),
        causal=causal, compresslm_custom_mask=mask)


def _new_row_slots(case, qlens):
    """Slots of each request's last qlen rows (the rows the step brings), request after request."""
    slots = []
    for r, (qlen, s_len) in enumerate(zip(qlens, case.seq_lens)):
        for pos in range(int(s_len) - qlen, int(s_len)):
            slots.append(int(case.block_table[r, pos // case.page]) * case.page + pos % case.page)
    return torch.tensor(slots, dtype=torch.int64)


def _take_rows(kv, slots, page):
    """[T, 2, Hkv, D] rows of a FlashInfer-layout cache at the given slots."""
    return kv[slots // page, :, slots % page]


def _impl(Hq, Hkv, D, scale, ws):
    return attention.AbkvAttentionBackend.get_impl_cls()(Hq, D, scale, Hkv, workspace=ws)


def test_impl_decode_step_writes_the_new_rows_then_attends():
    case, ref = load_decode("qwen3_heads")
    Hq, Hkv, D = case.q.shape[1], case.kv.shape[3], case.q.shape[2]
    R = len(case.seq_lens)
    slots = _new_row_slots(case, [1] * R)
    kv = _bf(case.kv)
    new = _take_rows(kv, slots.cuda(), case.page).clone()           # the step's K/V rows
    kv[slots.cuda() // case.page, :, slots.cuda() % case.page] = 0  # not yet in the cache
    ws = Workspace()
    md = attention.AbkvMetadataBuilder().build(0, _common([1] * R, case, slots=slots))
    assert md.decode_only
    query = _bf(case.q).view(R, Hq * D)
    output = torch.full((R + 3, Hq * D), 5.0, dtype=torch.bfloat16, device="cuda")
    got = _impl(Hq, Hkv, D, case.scale, ws).forward(None, query, new[:, 0].contiguous(), new[:, 1].contiguous(),
                                                     kv, md, output)
    torch.cuda.synchronize()
    assert got is output and ws.read_error() == 0
    assert torch.equal(kv.view(torch.int16), _bf(case.kv).view(torch.int16))  # bitwise (NaN poison)
    assert torch.all(output[R:] == 5.0)
    exact = decode_exact(case.q, case.kv, case.block_table, case.seq_lens, case.scale, case.page)
    se, sr = report("impl decode", output[:R].view(R, Hq, D).float().cpu().numpy(), exact, ref)
    assert se["max_abs"] <= 1.5e-2 and sr["max_abs"] <= ATOL_REF
    assert_relative(se)


@pytest.mark.parametrize("name", causal_cases())
def test_impl_prefill_step(name):
    case, qrows, qstart, rows, ref = load_causal(name)
    qlens = np.diff(qstart).tolist()
    Hq, Hkv, D = qrows.shape[1], case.kv.shape[3], qrows.shape[2]
    slots = _new_row_slots(case, qlens).cuda()
    kv = _bf(case.kv)
    new = _take_rows(kv, slots, case.page).clone()
    kv[slots // case.page, :, slots % case.page] = 0
    ws = Workspace()
    md = attention.AbkvMetadataBuilder().build(0, _common(qlens, case, slots=slots.cpu()))
    T = qrows.shape[0]
    # key / value as strided views of a fused [T, Hq + 2 Hkv, D] projection, as vLLM hands them over
    qkv = torch.zeros((T, Hq + 2 * Hkv, D), dtype=torch.bfloat16, device="cuda")
    qkv[:, :Hq] = _bf(qrows)
    qkv[:, Hq:Hq + Hkv] = new[:, 0]
    qkv[:, Hq + Hkv:] = new[:, 1]
    out = _impl(Hq, Hkv, D, case.scale, ws).forward(None, qkv[:, :Hq], qkv[:, Hq:Hq + Hkv], qkv[:, Hq + Hkv:],
                                                    kv, md)
    torch.cuda.synchronize()
    assert ws.read_error() == 0
    assert torch.equal(kv.view(torch.int16), _bf(case.kv).view(torch.int16))  # bitwise (NaN poison)
    got = out.view(T, Hq, D).float().cpu().numpy()
    exact = paged_causal_exact(qrows, case.kv, case.block_table, case.seq_lens, qstart, case.scale, case.page)
    se, sr = report(f"impl prefill {name}", got, exact, None)
    assert se["max_abs"] <= ATOL_EXACT and se["mean_abs"] <= MEAN_EXACT
    assert_relative(se)
    _, sr = report(f"impl prefill {name} (reference rows)", got[rows], exact[rows], ref)
    assert sr["max_abs"] <= ATOL_REF


@pytest.mark.parametrize("name", ["k128_excl", "k256_groups"])
def test_impl_code_step_with_group_masks(name):
    """The code step of each physical quota group: CodeStepMask from build_layer_quota_masks, against
    float64 attention under the reference's own boolean mask for that group."""
    from oracle.synth import paged_case

    K, quotas, requests, ref_masks = load_qmask(name)
    seq_lens = [s for _, s, _, _ in requests]
    Hq, Hkv, D = 32, 8, 128
    case = paged_case(71, seq_lens, num_q_heads=Hq, num_kv_heads=Hkv, head_dim=D, page=16)
    T = K * len(requests)
    qrows = np.asarray(torch.randn((T, Hq, D), generator=torch.Generator().manual_seed(7)).to(torch.bfloat16).float())
    masks = attention.build_layer_quota_masks(requests, quotas, K, causal=False, device="cuda")
    ws = Workspace()
    impl = _impl(Hq, Hkv, D, case.scale, ws)
    for q in quotas:
        md = attention.AbkvMetadataBuilder().build(0, _common([K] * len(requests), case, causal=False,
                                                              mask=masks[q]))
        out = impl.forward(None, _bf(qrows), None, None, _bf(case.kv), md)
        torch.cuda.synchronize()
        assert ws.read_error() == 0
        got = out.view(T, Hq, D).float().cpu().numpy()
        # float64 under the reference's mask: per request [K, seq_len] rows of the ragged mask
        exact = np.zeros_like(got, dtype=np.float64)
        off = 0
        for r, (qlen, s_len, _, _) in enumerate(requests):
            vis = ref_masks[q][off:off + qlen * s_len].reshape(qlen, s_len)
            off += qlen * s_len
            pos = np.arange(s_len)
            k = case.kv[case.block_table[r, pos // 16], 0, pos % 16].astype(np.float64)
            v = case.kv[case.block_table[r, pos // 16], 1, pos % 16].astype(np.float64)
            for h in range(Hq):
                s = qrows[r * K:(r + 1) * K, h].astype(np.float64) @ k[:, h // 4].T * case.scale
                s[~vis] = -np.inf
                e = np.exp(s - s.max(axis=1, keepdims=True))
                exact[r * K:(r + 1) * K, h] = (e / e.sum(axis=1, keepdims=True)) @ v[:, h // 4]
        se, _ = report(f"impl code step {name} quota {q}", got, exact)
        assert se["max_abs"] <= ATOL_EXACT and se["mean_abs"] <= MEAN_EXACT
        assert_relative(se)


# ---------------------------------------------------------------------------
def _layers(n, Hq, Hkv, scale):
    return [SimpleNamespace(num_heads=Hq, num_kv_heads=Hkv, impl=SimpleNamespace(scale=scale)) for _ in range(n)]


@pytest.mark.parametrize("name", sorted(packed_cases()) + ["no_pages"])
def test_override_attention_decode(name):
    """maybe_override_attention on a decode step: sidecar pages + the paged cache (packed goldens of
    the reference's PackedKVSidecar), or no pages (the plain decode goldens)."""
    if name == "no_pages":
        case, ref = load_decode("g2_hkv4")
        side, counts, quotas, k_max = None, [0] * len(case.seq_lens), [16] * case.kv.shape[3], 16
        exact = decode_exact(case.q, case.kv, case.block_table, case.seq_lens, case.scale, case.page)
    else:
        case, side, counts, quotas, k_max, ref = load_packed(name)
        exact = packed_decode_exact(case.q, case.kv, case.block_table, case.seq_lens, side, counts, quotas,
                                    case.scale, case.page)
    R, Hq, D = case.q.shape
    Hkv = case.kv.shape[3]
    layout = PackedKVLayout.from_schedule([list(quotas)], num_layers=1, num_kv_heads=Hkv, k_max=k_max)
    layers = _layers(1, Hq, Hkv, case.scale)
    sc = attention.CompressedKVSidecar(layout, layers, block_size=case.page, max_requests=R + 2,
                                       max_pages_per_request=max(1, int(max(counts))) + 1, head_dim=D)
    attention.install_sidecar(layers, sc)
    rids = [f"req{r}" for r in range(R)]
    first = 0
    for r, cnt in enumerate(counts):
        if cnt:
            sc.pages[rids[r]] = [[_bf(side[first + i]) for i in range(int(cnt))]]
        first += int(cnt)
    sc.set_active_request_ids(rids)
    sc.set_common_attn_metadata(_common([1] * R, case))
    out = torch.zeros((R, Hq * D), dtype=torch.bfloat16, device="cuda")
    attention.maybe_override_attention(layers[0], _bf(case.q).view(R, Hq * D), _bf(case.kv), object(), out)
    got = out.view(R, Hq, D).float().cpu().numpy()
    se, sr = report(f"override decode {name}", got, exact, ref)
    assert se["max_abs"] <= 1.5e-2 and sr["max_abs"] <= ATOL_REF
    assert_relative(se)
    # no metadata (vLLM's profiling run) or no sidecar: nothing is written
    out2 = torch.zeros_like(out)
    attention.maybe_override_attention(layers[0], _bf(case.q).view(R, Hq * D), _bf(case.kv), None, out2)
    attention.maybe_override_attention(SimpleNamespace(), _bf(case.q).view(R, Hq * D), _bf(case.kv), object(), out2)
    assert torch.count_nonzero(out2) == 0


@pytest.mark.parametrize("name", codestep_cases())
def test_override_attention_code_step(name):
    """maybe_override_attention on a code step (causal=False): the layer's per-KV-head quotas and the
    requests' exclusion ranges, against the reference sidecar's own outputs."""
    case, qrows, K, quotas, ref, excl = load_codestep(name)
    R = len(case.seq_lens)
    Hq, Hkv, D = qrows.shape[1], case.kv.shape[3], qrows.shape[2]
    layout = PackedKVLayout.from_schedule([[int(x) for x in quotas]], num_layers=1, num_kv_heads=Hkv, k_max=K)
    layers = _layers(1, Hq, Hkv, case.scale)
    sc = attention.CompressedKVSidecar(layout, layers, block_size=case.page, max_requests=R, head_dim=D,
                                       max_pages_per_request=2)
    attention.install_sidecar(layers, sc)
    rids = [f"r{r}" for r in range(R)]
    sc.set_active_request_ids(rids)
    sc.set_code_excluded_ranges({rid: tuple(int(x) for x in excl[r]) for r, rid in enumerate(rids)}
                                if excl is not None else None)
    sc.set_common_attn_metadata(_common([K] * R, case, causal=False))
    out = torch.zeros((R * K, Hq * D), dtype=torch.bfloat16, device="cuda")
    attention.maybe_override_attention(layers[0], _bf(qrows).view(R * K, Hq * D), _bf(case.kv), object(), out)
    got = out.view(R * K, Hq, D).float().cpu().numpy()
    exact = codestep_exact(qrows, case.kv, case.block_table, case.seq_lens, K, quotas, case.scale, case.page, excl)
    se, sr = report(f"override code step {name}", got, exact, ref)
    assert se["max_abs"] <= ATOL_EXACT and se["mean_abs"] <= MEAN_EXACT and sr["max_abs"] <= ATOL_REF
    assert_relative(se)


def test_store_kv_skips_padding_and_takes_both_layouts():
    from abridgekv_b200.attention import store_kv

    g = torch.Generator(device="cuda").manual_seed(3)
    nb, page, Hkv, D, T = 12, 16, 8, 128, 40
    kv = torch.randn((nb, 2, page, Hkv, D), generator=g, device="cuda").to(torch.bfloat16)
    key = torch.randn((T, Hkv, D), generator=g, device="cuda").to(torch.bfloat16)
    value = torch.randn((T, Hkv, D), generator=g, device="cuda").to(torch.bfloat16)
    slots = torch.randperm(nb * page, generator=g, device="cuda")[:T].to(torch.int64)
    slots[5] = -1
    want = kv.clone()
    keep = slots >= 0
    want[slots[keep] // page, 0, slots[keep] % page] = key[keep]
    want[slots[keep] // page, 1, slots[keep] % page] = value[keep]
    ws = Workspace()
    fa = kv.transpose(0, 1).contiguous()
    store_kv(key, value, kv, slots, workspace=ws)
    store_kv(key, value, fa, slots, workspace=ws)
    torch.cuda.synchronize()
    assert ws.read_error() == 0
    assert torch.equal(kv, want) and torch.equal(fa, want.transpose(0, 1))
    bad = slots.clone()
    bad[0] = nb * page  # past the cache: flagged, skipped
    store_kv(key, value, kv, bad, workspace=ws)
    assert ws.read_error() & 0x8  # ABKV_DEVERR_ROW_OOB


@pytest.mark.parametrize("name", ["code_qwen", "causal_g4"])
def test_override_attention_steps_with_sidecar_pages(name):
    """maybe_override_attention on a code step and on causal chunks of requests that already hold
    packed pages (captured through CompressedKVSidecar's page store): the reference sidecar's outputs."""
    from oracle.decode_ref import packed_step_exact
    from tests.goldens import load_packedstep

    g = load_packedstep(name)
    c = g["case"]
    quotas = [int(x) for x in g["quotas"]]
    Hq, Hkv, D = g["qrows"].shape[1], len(quotas), 128
    R = len(c.seq_lens)
    layout = PackedKVLayout.from_schedule([quotas], num_layers=1, num_kv_heads=Hkv, k_max=g["k_max"])
    layers = _layers(1, Hq, Hkv, c.scale)
    sc = attention.CompressedKVSidecar(layout, layers, block_size=c.page, max_requests=R, head_dim=D,
                                       max_pages_per_request=int(max(g["counts"])) + 1)
    attention.install_sidecar(layers, sc)
    rids = [f"r{r}" for r in range(R)]
    first = 0
    for r, cnt in enumerate(g["counts"]):
        if cnt:
            sc.pages[rids[r]] = [[_bf(g["side"][first + i]) for i in range(int(cnt))]]
        first += int(cnt)
    sc.set_active_request_ids(rids)
    qlens = np.diff(g["qstart"]).tolist()
    sc.set_common_attn_metadata(_common(qlens, c, causal=g["causal"]))
    T = g["qrows"].shape[0]
    out = torch.zeros((T, Hq * D), dtype=torch.bfloat16, device="cuda")
    attention.maybe_override_attention(layers[0], _bf(g["qrows"]).view(T, Hq * D), _bf(c.kv), object(), out)
    got = out.view(T, Hq, D).float().cpu().numpy()
    exact = packed_step_exact(g["qrows"], c.kv, c.block_table, c.seq_lens, g["qstart"], g["side"], g["counts"],
                              g["quotas"], g["causal"], c.scale, c.page, g["excluded"])
    se, _ = report(f"override packed step {name}", got, exact)
    assert se["max_abs"] <= ATOL_EXACT and se["mean_abs"] <= MEAN_EXACT
    assert_relative(se)
    _, sr = report(f"override packed step {name} (reference rows)", got[g["rows"]], exact[g["rows"]], g["ref"])
    assert sr["max_abs"] <= ATOL_REF

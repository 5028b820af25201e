"""Code-step attention (tcgen05, paged K/V) through the C ABI on a B200.

Tolerances (bf16 outputs; scores in fp32, P rounded to bf16 for the P.V MMA):
|gpu - float64 oracle| <= 2.5e-2 max and 2e-3 mean; |gpu - reference| <= 3e-2
(the reference rounds scores and weights to bf16); relative error
(tests/errstats.py) reported and bounded.
"""
import numpy as np
import pytest
import torch

from abridgekv_b200 import codestep
from abridgekv_b200._lib import AbkvError
from abridgekv_b200.workspace import Workspace
from oracle.decode_ref import codestep_exact
from tests.errstats import assert_relative, report
from tests.goldens import codestep_cases, load_codestep

pytestmark = pytest.mark.gpu
ATOL_EXACT, MEAN_EXACT, ATOL_REF = 2.5e-2, 2e-3, 3e-2


def _inputs(name):
    case, qrows, K, quotas, ref, excl = load_codestep(name)
    R = len(case.seq_lens)
    dev = dict(device="cuda")
    q = torch.from_numpy(qrows).to(torch.bfloat16).cuda()
    kv = torch.from_numpy(case.kv).to(torch.bfloat16).cuda()
    bt = torch.from_numpy(case.block_table).cuda()
    sl = torch.from_numpy(case.seq_lens).cuda()
    qs = torch.arange(R + 1, dtype=torch.int32, **dev) * K
    ex = torch.from_numpy(excl).cuda() if excl is not None else None
    return case, qrows, K, quotas, ref, excl, q, kv, bt, sl, qs, ex


@pytest.mark.parametrize("name", codestep_cases())
def test_codestep_matches_reference_golden(name):
    case, qrows, K, quotas, ref, excl, q, kv, bt, sl, qs, ex = _inputs(name)
    ws = Workspace()
    out = codestep.code_step_attention(q, kv, bt, sl, qs, quota_per_kv_head=[int(x) for x in quotas], k_max=K,
                                       scale=case.scale, excluded=ex, workspace=ws)
    torch.cuda.synchronize()
    assert ws.read_error() == 0
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    exact = codestep_exact(qrows, case.kv, case.block_table, case.seq_lens, K, quotas, case.scale, case.page, excl)
    se, sr = report(name, got, exact, ref)
    assert se["max_abs"] <= ATOL_EXACT and se["mean_abs"] <= MEAN_EXACT
    assert sr["max_abs"] <= ATOL_REF
    assert_relative(se, name)


def test_codestep_flashattention_layout_and_strided_query_equal():
    """[2, nb, page, Hkv, D] caches and query views with a padded row stride give the same bits."""
    case, qrows, K, quotas, ref, excl, q, kv, bt, sl, qs, ex = _inputs("k128_excl_g3")
    quot = [int(x) for x in quotas]
    a = codestep.code_step_attention(q, kv, bt, sl, qs, quota_per_kv_head=quot, k_max=K, scale=case.scale,
                                     excluded=ex)
    kv_fa = kv.transpose(0, 1).contiguous()
    T, Hq, D = q.shape
    wide = torch.zeros((T, Hq + 3, D), dtype=torch.bfloat16, device="cuda")
    wide[:, 1:Hq + 1] = q
    out_wide = torch.full((T, Hq + 2, D), 7.0, dtype=torch.bfloat16, device="cuda")
    b = codestep.code_step_attention(wide[:, 1:Hq + 1], kv_fa, bt, sl, qs, quota_per_kv_head=quot, k_max=K,
                                     scale=case.scale, excluded=ex, out=out_wide[:, :Hq])
    assert torch.equal(a, b)
    assert torch.all(out_wide[:, Hq:] == 7.0)


def test_codestep_query_start_loc_permuted_and_padded():
    """Requests' code rows at arbitrary starts (out of order, with gaps): each lands at its rows,
    rows of no request are left untouched."""
    case, qrows, K, quotas, ref, excl, q, kv, bt, sl, qs, ex = _inputs("k128_q64")
    R = len(case.seq_lens)
    starts = [2 * K + 5, 0, K + 3][:R]
    T = 3 * K + 9
    qp = torch.zeros((T, q.shape[1], q.shape[2]), dtype=torch.bfloat16, device="cuda")
    for r, s0 in enumerate(starts):
        qp[s0:s0 + K] = q[r * K:(r + 1) * K]
    out = torch.full_like(qp, -3.0)
    quot = [int(x) for x in quotas]
    codestep.code_step_attention(qp, kv, bt, sl, torch.tensor(starts, dtype=torch.int32, device="cuda"),
                                 quota_per_kv_head=quot, k_max=K, scale=case.scale, out=out, num_requests=R)
    base = codestep.code_step_attention(q, kv, bt, sl, qs, quota_per_kv_head=quot, k_max=K, scale=case.scale)
    covered = torch.zeros(T, dtype=torch.bool, device="cuda")
    for r, s0 in enumerate(starts):
        assert torch.equal(out[s0:s0 + K], base[r * K:(r + 1) * K])
        covered[s0:s0 + K] = True
    assert torch.all(out[~covered] == -3.0)


def test_codestep_device_errors_are_reported():
    """seq_len below k_max, a page id outside the cache and an invalid exclusion range set the
    workspace error bits (the kernel clamps / skips instead of reading out of bounds)."""
    case, qrows, K, quotas, ref, excl, q, kv, bt, sl, qs, ex = _inputs("k128_q64")
    quot = [int(x) for x in quotas]
    ws = Workspace()
    bad = sl.clone()
    bad[0] = K - 1
    codestep.code_step_attention(q, kv, bt, bad, qs, quota_per_kv_head=quot, k_max=K, workspace=ws)
    assert ws.read_error() & 0x2
    bt2 = bt.clone()
    bt2[1, 0] = kv.shape[0] + 5
    codestep.code_step_attention(q, kv, bt2, sl, qs, quota_per_kv_head=quot, k_max=K, workspace=ws)
    assert ws.read_error() & 0x1
    exb = torch.tensor([[0, 0], [10, 5], [0, 0]], dtype=torch.int32, device="cuda")
    codestep.code_step_attention(q, kv, bt, sl, qs, quota_per_kv_head=quot, k_max=K, excluded=exb, workspace=ws)
    assert ws.read_error() & 0x10
    qs_bad = qs.clone()
    qs_bad[2] = q.shape[0] - K + 1
    codestep.code_step_attention(q, kv, bt, sl, qs_bad, quota_per_kv_head=quot, k_max=K, workspace=ws)
    assert ws.read_error() & 0x10
    torch.cuda.synchronize()


def test_codestep_host_validation():
    case, qrows, K, quotas, ref, excl, q, kv, bt, sl, qs, ex = _inputs("k128_q64")
    with pytest.raises(AbkvError):
        codestep.code_step_attention(q[:, :, :64].contiguous(), kv[..., :64].contiguous(), bt, sl, qs,
                                     quota_per_kv_head=[64, 64], k_max=K)
    with pytest.raises(AbkvError):
        codestep.code_step_attention(q, kv, bt, sl, qs, quota_per_kv_head=[K + 1, 0], k_max=K)
    with pytest.raises(AbkvError):
        codestep.code_step_attention(q, kv, bt, sl, qs, quota_per_kv_head=[64, 64], k_max=96)


def test_codestep_qwen_scale_sampled_requests():
    """Qwen3-4B code step at serving scale (64 requests, seq 3-5K, K=256, 32/8 heads, quotas
    256/128/64): sampled requests against a PyTorch fp32 reference on the GPU."""
    torch.manual_seed(3)
    R, K, Hq, Hkv, D, page = 64, 256, 32, 8, 128, 16
    quotas = [256, 128, 64, 128, 256, 64, 128, 128]
    lens = torch.randint(3000, 5000, (R,)) + K
    pages = (lens + page - 1) // page
    nb = int(pages.sum()) + 1
    kv = torch.randn((nb, 2, page, Hkv, D), device="cuda", dtype=torch.bfloat16)
    perm = torch.randperm(nb - 1) + 1
    maxp = int(pages.max())
    bt = torch.zeros((R, maxp), dtype=torch.int32)
    off = 0
    for r in range(R):
        bt[r, :pages[r]] = perm[off:off + pages[r]]
        off += int(pages[r])
    bt, sl = bt.cuda(), lens.to(torch.int32).cuda()
    q = torch.randn((R * K, Hq, D), device="cuda", dtype=torch.bfloat16)
    qs = (torch.arange(R + 1) * K).to(torch.int32).cuda()
    ws = Workspace()
    out = codestep.code_step_attention(q, kv, bt, sl, qs, quota_per_kv_head=quotas, k_max=K, workspace=ws)
    torch.cuda.synchronize()
    assert ws.read_error() == 0
    G = Hq // Hkv
    for r in (0, 17, 63):
        L = int(lens[r])
        rows = torch.arange(L, device="cuda")
        blk = bt[r].long()[rows // page]
        k = kv[blk, 0, rows % page].float()     # [L, Hkv, D]
        v = kv[blk, 1, rows % page].float()
        qq = q[r * K:(r + 1) * K].float()
        for h in range(Hq):
            lim = L - K + quotas[h // G]
            s = (qq[:, h] @ k[:lim, h // G].T) / D ** 0.5
            ref = torch.softmax(s, dim=-1) @ v[:lim, h // G]
            err = (out[r * K:(r + 1) * K, h].float() - ref).abs()
            assert err.max().item() <= ATOL_EXACT and err.mean().item() <= MEAN_EXACT


def test_codestep_rows_with_no_visible_key_are_zero():
    """quota 0 with the whole prefix excluded leaves a head nothing to attend to: zeros, no error
    (the reference's softmax over an all -inf row would give NaN)."""
    K, Hq, Hkv, D, page = 128, 4, 2, 128, 16
    L = K + 64
    kv = torch.randn((L // page + 1, 2, page, Hkv, D), device="cuda", dtype=torch.bfloat16)
    bt = torch.arange(1, L // page + 1, dtype=torch.int32, device="cuda").view(1, -1)
    sl = torch.tensor([L], dtype=torch.int32, device="cuda")
    q = torch.randn((K, Hq, D), device="cuda", dtype=torch.bfloat16)
    qs = torch.tensor([0, K], dtype=torch.int32, device="cuda")
    ex = torch.tensor([[0, 64]], dtype=torch.int32, device="cuda")
    ws = Workspace()
    out = codestep.code_step_attention(q, kv, bt, sl, qs, quota_per_kv_head=[0, 1], k_max=K, excluded=ex,
                                       workspace=ws)
    torch.cuda.synchronize()
    assert ws.read_error() == 0
    assert torch.all(out[:, :2] == 0)
    ref = kv[bt[0].long()[64 // page], 1, 0, 1].float()   # heads 2, 3: only code slot 0 (row 64) visible
    assert torch.allclose(out[:, 2:].float(), ref.expand(K, 2, D), atol=1e-2)


def _finished_block_ops(bt, lens, K, C, q):
    """Each request's compaction of its last finished block: code rows [L - K, L - K + q) move over
    the start of the block's content rows [L - K - C, L - K - C + q) (its own pages)."""
    ops, off = [], [0]
    page = 16
    for r in range(len(lens)):
        L = int(lens[r])
        for j in range(q):
            s_row, d_row = L - K + j, L - K - C + j
            ops.append((int(bt[r, s_row // page]), s_row % page, int(bt[r, d_row // page]), d_row % page))
        off.append(len(ops))
    return ops, off


def test_codestep_fused_compaction_equals_code_step_then_executor():
    """abkv_code_step_attention_compact equals abkv_code_step_attention followed by abkv_compact of
    the same ops, bit for bit: the outputs and the whole cache.  Also the host checks of the ops."""
    from abridgekv_b200 import compaction

    torch.manual_seed(5)
    R, K, C, Hq, Hkv, D, page = 16, 256, 512, 32, 8, 128, 16
    quotas = [128] * Hkv
    lens = torch.randint(1500, 3000, (R,)) + K
    pages = (lens + page - 1) // page
    nb = int(pages.sum()) + 1
    kv = torch.randn((nb, 2, page, Hkv, D), device="cuda", dtype=torch.bfloat16)
    perm = torch.randperm(nb - 1) + 1
    bt = torch.zeros((R, int(pages.max())), dtype=torch.int32)
    o = 0
    for r in range(R):
        bt[r, :pages[r]] = perm[o:o + pages[r]]
        o += int(pages[r])
    ops, off = _finished_block_ops(bt, lens, K, C, 128)
    btd, sl = bt.cuda(), lens.to(torch.int32).cuda()
    q = torch.randn((R * K, Hq, D), device="cuda", dtype=torch.bfloat16)
    qs = (torch.arange(R + 1) * K).to(torch.int32).cuda()
    kv_a, kv_b = kv.clone(), kv.clone()
    ws = Workspace()
    out_a = codestep.code_step_attention(q, kv_a, btd, sl, qs, quota_per_kv_head=quotas, k_max=K, workspace=ws)
    compaction.execute_kv_copy_group(ops, [kv_a], workspace=ws)
    out_b = codestep.code_step_attention_compact(q, kv_b, btd, sl, qs, ops=ops, op_offsets=off,
                                                 quota_per_kv_head=quotas, k_max=K, replay_tail=0, workspace=ws)
    torch.cuda.synchronize()
    assert ws.read_error() == 0
    assert torch.equal(out_a, out_b)
    assert torch.equal(kv_a, kv_b)
    assert not torch.equal(kv_a, kv)
    # a second call on the same workspace (counters cleared per call) keeps the same result
    kv_c = kv.clone()
    out_c = codestep.code_step_attention_compact(q, kv_c, btd, sl, qs, ops=ops, op_offsets=off,
                                                 quota_per_kv_head=quotas, k_max=K, replay_tail=0, workspace=ws)
    torch.cuda.synchronize()
    assert torch.equal(out_c, out_a) and torch.equal(kv_c, kv_a)
    # host checks: a destination that is also a source, a block out of range, bad offsets
    bad = list(ops)
    bad[0] = (ops[1][2], ops[1][3], ops[0][2], ops[0][3])
    with pytest.raises(AbkvError):
        codestep.code_step_attention_compact(q, kv.clone(), btd, sl, qs, ops=bad, op_offsets=off,
                                             quota_per_kv_head=quotas, k_max=K, replay_tail=0, workspace=ws)
    bad = list(ops)
    bad[3] = (nb, 0, ops[3][2], ops[3][3])
    with pytest.raises(AbkvError):
        codestep.code_step_attention_compact(q, kv.clone(), btd, sl, qs, ops=bad, op_offsets=off,
                                             quota_per_kv_head=quotas, k_max=K, replay_tail=0, workspace=ws)
    with pytest.raises(AbkvError):
        codestep.code_step_attention_compact(q, kv.clone(), btd, sl, qs, ops=ops, op_offsets=off[:-1] + [0],
                                             quota_per_kv_head=quotas, k_max=K, replay_tail=0, workspace=ws)


from oracle.decode_ref import paged_causal_exact  # noqa: E402
from tests.goldens import causal_cases, load_causal  # noqa: E402


@pytest.mark.parametrize("name", causal_cases())
def test_paged_prefill_matches_reference_golden(name):
    """abkv_paged_prefill (the code-step kernel's causal mode) on ragged requests -- fresh prompts,
    chunks after a prefix, a single decode row -- against the reference's causal
    _attend_request_vectorized rows and the float64 oracle; both paged layouts give the same bits;
    padding rows of no request stay untouched."""
    case, qrows, qstart, rows, ref = load_causal(name)
    Hkv = case.kv.shape[3]
    T = qrows.shape[0]
    q = torch.zeros((T + 5, qrows.shape[1], 128), dtype=torch.bfloat16, device="cuda")
    q[:T] = torch.from_numpy(qrows).to(torch.bfloat16).cuda()
    kv = torch.from_numpy(case.kv).to(torch.bfloat16).cuda()
    bt = torch.from_numpy(case.block_table).cuda()
    sl = torch.from_numpy(case.seq_lens).cuda()
    qs = torch.from_numpy(qstart).cuda()
    max_q = int(np.diff(qstart).max())
    ws = Workspace()
    out = torch.full_like(q, float("nan"))
    codestep.paged_prefill(q, kv, bt, sl, qs, max_query_len=max_q, num_kv_heads=Hkv, scale=case.scale, out=out,
                           workspace=ws)
    torch.cuda.synchronize()
    assert ws.read_error() == 0
    assert torch.isnan(out[T:].float()).all(), "rows of no request were written"
    got = out[:T].float().cpu().numpy()
    assert np.isfinite(got).all()
    exact = paged_causal_exact(qrows, case.kv, case.block_table, case.seq_lens, qstart, case.scale, case.page)
    se, _ = report(name, got, exact)
    assert se["max_abs"] <= ATOL_EXACT and se["mean_abs"] <= MEAN_EXACT
    assert_relative(se, name)
    _, sr = report(f"{name} (reference rows)", got[rows], exact[rows], ref)
    assert sr["max_abs"] <= ATOL_REF
    out_fa = codestep.paged_prefill(q, kv.transpose(0, 1).contiguous(), bt, sl, qs, max_query_len=max_q,
                                    num_kv_heads=Hkv, scale=case.scale)
    assert torch.equal(out_fa[:T], out[:T])


def test_paged_prefill_understated_max_query_len_is_flagged():
    """A request longer than max_query_len sets ABKV_DEVERR_RANGE; the rows the grid covers are still
    right and the rows past it are left unwritten."""
    case, qrows, qstart, rows, ref = load_causal("g3_page32")
    q = torch.from_numpy(qrows).to(torch.bfloat16).cuda()
    kv = torch.from_numpy(case.kv).to(torch.bfloat16).cuda()
    args = (kv, torch.from_numpy(case.block_table).cuda(), torch.from_numpy(case.seq_lens).cuda(),
            torch.from_numpy(qstart).cuda())
    ws = Workspace()
    full = codestep.paged_prefill(q, *args, max_query_len=250, num_kv_heads=2, scale=case.scale, workspace=ws)
    assert ws.read_error() == 0
    short = torch.full_like(q, float("nan"))
    codestep.paged_prefill(q, *args, max_query_len=128, num_kv_heads=2, scale=case.scale, out=short, workspace=ws)
    assert ws.read_error() & 0x10  # ABKV_DEVERR_RANGE
    last = int(qstart[2])  # request 2 has 250 rows: its first 128 are computed, the rest are not
    assert torch.equal(short[:last + 128], full[:last + 128])
    assert torch.isnan(short[last + 128:].float()).all()


from oracle.decode_ref import packed_step_exact  # noqa: E402
from tests.goldens import load_packedstep, packedstep_cases  # noqa: E402


def _packed_pool(g, spare=3):
    """SidecarPool of the golden's packed pages (request slot r = request r), spare pages poisoned."""
    from abridgekv_b200.sidecar import PackedKVLayout, SidecarPool

    quotas = [int(x) for x in g["quotas"]]
    layout = PackedKVLayout.from_schedule([quotas], num_layers=1, num_kv_heads=len(quotas), k_max=g["k_max"])
    counts = [int(c) for c in g["counts"]]
    pool = SidecarPool(layout, 0, capacity=sum(counts) + spare, num_requests=len(counts),
                       max_pages=max(1, max(counts)) + 1, head_dim=128)
    pool.pages.fill_(float("nan"))
    first = 0
    for r, cnt in enumerate(counts):
        for i in range(cnt):
            pool.append(r, torch.from_numpy(g["side"][first + i]).to(torch.bfloat16).cuda())
        first += cnt
    return layout, pool


@pytest.mark.parametrize("name", packedstep_cases())
def test_packed_step_matches_reference_golden(name):
    """Code steps and causal chunks of requests holding packed sidecar pages
    (abkv_code_step_attention_packed / abkv_paged_prefill_packed) against the reference's
    _attend_request_vectorized with layer_pages and the float64 oracle; the pool's spare pages are
    poisoned, so a read outside the requests' pages shows up as NaN."""
    g = load_packedstep(name)
    c = g["case"]
    layout, pool = _packed_pool(g)
    quotas = [int(x) for x in g["quotas"]]
    q = torch.from_numpy(g["qrows"]).to(torch.bfloat16).cuda()
    kv = torch.from_numpy(c.kv).to(torch.bfloat16).cuda()
    bt, sl = torch.from_numpy(c.block_table).cuda(), torch.from_numpy(c.seq_lens).cuda()
    qs = torch.from_numpy(g["qstart"]).cuda()
    ws = Workspace()
    if g["causal"]:
        out = codestep.paged_prefill(q, kv, bt, sl, qs, max_query_len=int(np.diff(g["qstart"]).max()),
                                     num_kv_heads=len(quotas), scale=c.scale, workspace=ws, sidecar=pool)
    else:
        ex = torch.from_numpy(g["excluded"]).cuda() if g["excluded"] is not None else None
        out = codestep.code_step_attention(q, kv, bt, sl, qs, quota_per_kv_head=quotas, k_max=g["k_max"],
                                           scale=c.scale, excluded=ex, workspace=ws, sidecar=pool)
    torch.cuda.synchronize()
    assert ws.read_error() == 0
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    exact = packed_step_exact(g["qrows"], c.kv, c.block_table, c.seq_lens, g["qstart"], g["side"], g["counts"],
                              g["quotas"], g["causal"], c.scale, c.page, g["excluded"])
    se, _ = report(f"packed step {name}", got, exact)
    assert se["max_abs"] <= ATOL_EXACT and se["mean_abs"] <= MEAN_EXACT
    assert_relative(se, name)
    _, sr = report(f"packed step {name} (reference rows)", got[g["rows"]], exact[g["rows"]], g["ref"])
    assert sr["max_abs"] <= ATOL_REF

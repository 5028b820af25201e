"""The CPU oracle reproduces the reference's own outputs (golden fixtures)."""
import numpy as np
import pytest

from oracle.decode_ref import decode_exact, decode_reference
from tests.goldens import decode_cases, load_decode


@pytest.mark.parametrize("name", decode_cases())
def test_decode_oracle_matches_reference(name):
    case, ref = load_decode(name)
    ours = decode_reference(case.q, case.kv, case.block_table, case.seq_lens, case.scale, case.page)
    assert np.isfinite(ref).all()
    diff = np.abs(ours - ref)
    # Same roundings as the reference; only fp32 summation order differs, which
    # can move a bf16 result by a unit or two in the last place.
    # two bf16 ulps, plus a floor for results that cancel to near zero
    ulp = np.maximum(np.abs(ref), np.abs(ours)) * 2.0 ** -6 + 1e-5
    assert (diff <= ulp).all(), float(diff.max())
    assert (diff == 0).mean() > 0.97


@pytest.mark.parametrize("name", decode_cases())
def test_decode_torch_port_matches_reference(name):
    """The torch CPU port that bench.py times as the decode CPU baseline and as the reference arm
    (oracle/decode_ref.sidecar_decode_torch) reproduces the reference's own
    _attend_decode_batched outputs on every golden case: within two bf16 ulps, as the numpy
    restatement above."""
    import torch

    from oracle.decode_ref import sidecar_decode_torch

    case, ref = load_decode(name)
    Hq, Hkv = case.q.shape[1], case.kv.shape[3]
    got = sidecar_decode_torch(torch.from_numpy(case.q).to(torch.bfloat16),
                               torch.from_numpy(case.kv).to(torch.bfloat16),
                               torch.from_numpy(case.seq_lens), torch.from_numpy(case.block_table),
                               Hkv, Hq // Hkv, case.scale, case.page).float().numpy()
    live = case.seq_lens > 0  # the reference leaves rows of empty requests untouched
    diff = np.abs(got[live] - ref[live])
    ulp = np.maximum(np.abs(ref[live]), np.abs(got[live])) * 2.0 ** -6 + 1e-5
    assert (diff <= ulp).all(), float(diff.max())
    assert (diff == 0).mean() > 0.97


@pytest.mark.parametrize("name", decode_cases())
def test_reference_rounding_error_is_small(name):
    """Bound on the reference's own bf16-score error vs float64 (the budget our
    kernel's tolerance is set against)."""
    case, ref = load_decode(name)
    exact = decode_exact(case.q, case.kv, case.block_table, case.seq_lens, case.scale, case.page)
    assert np.abs(ref - exact).max() < 3e-2


from oracle.decode_ref import codestep_exact  # noqa: E402
from tests.goldens import codestep_cases, load_codestep  # noqa: E402


@pytest.mark.parametrize("name", codestep_cases())
def test_codestep_oracle_matches_reference(name):
    case, qrows, K, quotas, ref, excl = load_codestep(name)
    ex = codestep_exact(qrows, case.kv, case.block_table, case.seq_lens, K, quotas, case.scale, case.page, excl)
    assert np.isfinite(ref).all()
    # the reference rounds scores and weights to bf16; float64 stays within its error budget
    assert np.abs(ex - ref).max() < 3e-2
    assert np.abs(ex - ref).mean() < 2e-3


@pytest.mark.parametrize("name", codestep_cases())
def test_codestep_torch_port_matches_reference(name):
    """The torch CPU port timed as the code step's CPU baseline reproduces the reference's
    outputs (same op sequence and roundings) on the golden cases."""
    import torch

    from oracle.decode_ref import sidecar_codestep_torch

    case, qrows, K, quotas, ref, excl = load_codestep(name)
    kv = torch.from_numpy(case.kv).to(torch.bfloat16)
    Hq, Hkv = qrows.shape[1], case.kv.shape[3]
    outs = []
    for r, s_len in enumerate(case.seq_lens):
        q = torch.from_numpy(qrows[r * K:(r + 1) * K]).to(torch.bfloat16)
        outs.append(sidecar_codestep_torch(q, kv, int(s_len), torch.from_numpy(case.block_table[r]), quotas, K,
                                           Hkv, Hq // Hkv, case.scale, case.page,
                                           None if excl is None else excl[r]).float().numpy())
    got = np.concatenate(outs)
    assert np.abs(got - ref).max() <= 1e-2


from oracle.decode_ref import packed_decode_exact  # noqa: E402
from tests.goldens import load_packed, packed_cases  # noqa: E402


@pytest.mark.parametrize("name", packed_cases())
def test_packed_oracle_matches_reference(name):
    case, side, counts, quotas, k_max, ref = load_packed(name)
    ex = packed_decode_exact(case.q, case.kv, case.block_table, case.seq_lens, side, counts, quotas, case.scale,
                             case.page)
    assert np.isfinite(ref).all()
    assert np.abs(ex - ref).max() < 3e-2
    assert np.abs(ex - ref).mean() < 2e-3


@pytest.mark.parametrize("name", ["c128k128_quota_prompt", "c256k128_g4"])
def test_prefill_backward_oracle_matches_reference(name):
    """The float64 gradient oracle (hand-derived dQ / dK / dV of masked softmax attention with GQA)
    against torch autograd through the reference's mask (tests/golden/prefillbwd_*)."""
    from oracle.mask_ref import masked_attention_grad
    from tests.goldens import load_prefill_bwd

    g, dout, rows, dq_r, dk_r, dv_r = load_prefill_bwd(name)
    dq, dk, dv = masked_attention_grad(g["q"], g["k"], g["v"], g["mask"], 1.0 / np.sqrt(g["D"]), dout)
    for got, ref in ((dq[:, :, rows], dq_r), (dk[:, :, rows], dk_r), (dv[:, :, rows], dv_r)):
        assert np.abs(got - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max())


from oracle.decode_ref import paged_causal_exact  # noqa: E402
from tests.goldens import causal_cases, load_causal  # noqa: E402


@pytest.mark.parametrize("name", causal_cases())
def test_paged_causal_oracle_matches_reference(name):
    """The float64 restatement of the causal branch of _attend_request_vectorized against the
    reference's own outputs (bf16 scores and weights there): within its rounding budget."""
    case, qrows, qstart, rows, ref = load_causal(name)
    ex = paged_causal_exact(qrows, case.kv, case.block_table, case.seq_lens, qstart, case.scale, case.page)
    assert np.isfinite(ref).all()
    assert np.abs(ex[rows] - ref).max() < 3e-2
    assert np.abs(ex[rows] - ref).mean() < 2e-3



from oracle.decode_ref import packed_step_exact  # noqa: E402
from tests.goldens import load_packedstep, packedstep_cases  # noqa: E402


@pytest.mark.parametrize("name", packedstep_cases())
def test_packed_step_oracle_matches_reference(name):
    """The float64 restatement of _attend_request_vectorized with packed sidecar pages (code steps and
    causal chunks) against the reference's own outputs, within its bf16 rounding budget."""
    g = load_packedstep(name)
    c = g["case"]
    ex = packed_step_exact(g["qrows"], c.kv, c.block_table, c.seq_lens, g["qstart"], g["side"], g["counts"],
                           g["quotas"], g["causal"], c.scale, c.page, g["excluded"])
    assert np.isfinite(g["ref"]).all()
    assert np.abs(ex[g["rows"]] - g["ref"]).max() < 3e-2
    assert np.abs(ex[g["rows"]] - g["ref"]).mean() < 2e-3

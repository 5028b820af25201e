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

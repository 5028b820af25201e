"""The prefill-mask oracle equals the reference's own mask_mod and FlexAttention outputs (CPU)."""
import numpy as np
import pytest

from oracle.mask_ref import arith_mask, bitrev_code_offsets, masked_attention
from tests.goldens import load_prefill, prefill_cases


@pytest.mark.parametrize("name", prefill_cases())
def test_oracle_mask_matches_reference(name):
    g = load_prefill(name)
    m = arith_mask(g["S0"], g["C"], g["K"], g["quota"], g["prompt_len"], batch=g["B"])
    assert np.array_equal(m, g["mask"])


@pytest.mark.parametrize("name", prefill_cases())
def test_oracle_attention_matches_reference_flex(name):
    g = load_prefill(name)
    out, lse = masked_attention(g["q"], g["k"], g["v"], g["mask"], 1.0 / np.sqrt(g["D"]))
    assert np.abs(out[:, :, g["rows"], :] - g["out_rows"]).max() < 1e-4
    assert np.abs(lse - g["lse"]).max() < 1e-4


def test_bitrev_offsets_nested_prefix():
    """_bitrev_code_offsets (compress_forward.py:46-60): any 2^m prefix is evenly spread,
    and the first K' offsets are the same for every K >= K'."""
    o256 = bitrev_code_offsets(256, 512)
    o128 = bitrev_code_offsets(128, 512)
    assert np.array_equal(o256[:128], o128)
    assert sorted(o256[:64].tolist()) == list(range(0, 512, 8))

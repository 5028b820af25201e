"""BASELINE config 1 through the reference's own model flow (tests/golden/config1_reference.npz):
the oracle restatements reproduce the reference's attention of every captured layer and step.

* prefill: CompressLM.forward's FlexAttention output (per-layer quotas 128 / 64, C=512, K_max=128,
  4 blocks) equals the float64 masked attention under oracle/mask_ref.arith_mask on the same inputs;
* decode: CompressGen's content attention equals the float64 decode over the visible store columns
  laid into a shuffled paged cache (the layout the decode kernel reads).
The golden keeps q / K / V in bf16 (what the kernels read) and the reference's fp32 outputs, so the
bound is the bf16 rounding of the inputs (measured: at most 2.7e-3 max abs and 2.9e-3 relative):
max |f64 - reference| <= 1e-2 and relative (max |diff| / max |ref|) <= 1e-2.
"""
import numpy as np
import pytest

from oracle.decode_ref import decode_exact
from oracle.mask_ref import arith_mask, masked_attention
from tests.errstats import err_stats
from tests.goldens import config1_paged, load_config1

G = load_config1()


@pytest.mark.parametrize("layer", [0, 1])
def test_config1_prefill_oracle_matches_reference(layer):
    q_rows, k, v, out = G["prefill"][layer]
    H, n, D = q_rows.shape
    S0 = G["N"] * (G["C"] + G["K"])
    q = np.zeros((1, H, S0, D), dtype=np.float32)
    q[0, :, G["rows"]] = q_rows.transpose(1, 0, 2)
    mask = arith_mask(S0, G["C"], G["K"], quota_per_head=[G["quotas"][layer]] * H)
    ref64, _ = masked_attention(q, k[None], v[None], mask, 1.0 / np.sqrt(D))
    got = ref64[0][:, G["rows"]].transpose(1, 0, 2)   # [n, H, D]
    s = err_stats(got, out)
    assert s["max_abs"] <= 1e-2 and s["rel_max"] <= 1e-2, s


@pytest.mark.parametrize("layer", [0, 1])
def test_config1_decode_oracle_matches_reference(layer):
    q, kv, bt, lens, out, steps = config1_paged(G["decode"][layer])
    # quota-layer geometry: 4 compressed blocks x quota code rows, then the live content rows
    assert [int(x) for x in lens] == [4 * G["quotas"][layer] + s + 1 for s in steps]
    got = decode_exact(q, kv, bt, lens, 1.0 / np.sqrt(q.shape[-1]), 16)
    s = err_stats(got, out)
    assert s["max_abs"] <= 1e-2 and s["rel_max"] <= 1e-2, s

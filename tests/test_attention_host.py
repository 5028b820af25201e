"""The vLLM-shaped boundary's host logic (abridgekv_b200.attention), no GPU needed.

* build_layer_quota_masks returns a CodeStepMask descriptor where the reference returns FlashInfer's
  boolean mask; expanded by the kernel's rule (a code query sees rows [0, seq_len - (K - quota)) minus
  the request's excluded range) it equals, bit for bit, the reference's own masks for the code step
  of physical quota groups (tests/golden/qmask_*.npz, made by compresslm_masks.py:165-239).
* What the kernels do not serve is refused: causal (masked-mode) quota masks, spans other than the
  block's own code rows.
* AbkvMetadataBuilder reads vLLM's CommonAttentionMetadata fields and refuses dense masks.
"""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from abridgekv_b200.attention import (AbkvAttentionBackend, AbkvMetadataBuilder, CodeStepMask,
                                      build_layer_quota_masks)
from tests.goldens import load_qmask, qmask_cases


def expand(mask: CodeStepMask, requests) -> np.ndarray:
    """The ragged row-major boolean mask a CodeStepMask stands for (what the code-step kernel evaluates)."""
    parts = []
    for r, (qlen, s_len, _, _) in enumerate(requests):
        cols = np.arange(s_len)
        vis = cols < s_len - (mask.num_code_tokens - mask.quota)
        if mask.excluded is not None and mask.excluded[r][1] > mask.excluded[r][0]:
            vis &= ~((cols >= mask.excluded[r][0]) & (cols < mask.excluded[r][1]))
        parts.append(np.broadcast_to(vis, (qlen, s_len)).reshape(-1))
    return np.concatenate(parts)


@pytest.mark.parametrize("name", qmask_cases())
def test_code_step_masks_equal_the_reference_masks(name):
    K, quotas, requests, ref = load_qmask(name)
    ours = build_layer_quota_masks(requests, quotas, K, causal=False)
    assert sorted(ours) == sorted(quotas)
    for q in quotas:
        got = expand(ours[q], requests)
        assert got.shape == ref[q].shape and np.array_equal(got, ref[q]), (name, q)


def test_unserved_masks_are_refused():
    reqs = [(128, 500, [(372, 500)], None)]
    with pytest.raises(NotImplementedError, match="physical_layer_quotas"):
        build_layer_quota_masks(reqs, [64], 128, causal=True)
    with pytest.raises(NotImplementedError, match="own 128 code rows"):
        build_layer_quota_masks([(128, 500, [(100, 228)], None)], [64], 128, causal=False)
    with pytest.raises(ValueError, match="invalid query_len/seq_len"):
        build_layer_quota_masks([(600, 500, [], None)], [64], 128, causal=False)
    assert build_layer_quota_masks([], [64], 128, causal=False) == {}
    # quota >= K hides no code row: spans need not be present
    m = build_layer_quota_masks([(128, 500, [], (3, 9))], [128], 128, causal=False)[128]
    assert m.quota == 128 and m.excluded.tolist() == [[3, 9]]


def _common(qlens, seq_lens, causal=True, mask=None):
    qsl = torch.tensor(np.concatenate([[0], np.cumsum(qlens)]), dtype=torch.int32)
    return SimpleNamespace(
        query_start_loc=qsl.clone(), query_start_loc_cpu=qsl, seq_lens=torch.tensor(seq_lens, dtype=torch.int32),
        _seq_lens_cpu=torch.tensor(seq_lens, dtype=torch.int32), num_reqs=len(qlens),
        num_actual_tokens=int(sum(qlens)), max_query_len=int(max(qlens)),
        block_table_tensor=torch.zeros((len(qlens), 4), dtype=torch.int64),
        slot_mapping=torch.arange(int(sum(qlens))), causal=causal, compresslm_custom_mask=mask)


def test_metadata_builder_reads_common_metadata():
    md = AbkvMetadataBuilder().build(0, _common([1, 1, 1], [40, 7, 100]))
    assert md.decode_only and md.causal and md.num_reqs == 3 and md.max_query_len == 1
    assert md.block_table.dtype == torch.int32 and md.block_table.is_contiguous()
    md = AbkvMetadataBuilder().build(0, _common([5, 1, 30], [40, 7, 100]))
    assert not md.decode_only and md.max_query_len == 30 and md.num_actual_tokens == 36
    mask = build_layer_quota_masks([(128, 500, [(372, 500)], None)], [64], 128, causal=False)[64]
    md = AbkvMetadataBuilder().build(0, _common([128], [500], causal=False, mask=mask))
    assert md.code_mask is mask and not md.causal
    with pytest.raises(TypeError, match="CodeStepMask"):
        AbkvMetadataBuilder().build(0, _common([128], [500], causal=False, mask=torch.ones(64000, dtype=torch.bool)))


def test_backend_names_and_cache_shape():
    assert AbkvAttentionBackend.get_name() == "ABKV_SM100"
    assert AbkvAttentionBackend.get_kv_cache_shape(10, 16, 8, 128) == (10, 2, 16, 8, 128)
    assert AbkvAttentionBackend.get_impl_cls().__name__ == "AbkvAttentionImpl"
    assert AbkvAttentionBackend.get_builder_cls() is AbkvMetadataBuilder

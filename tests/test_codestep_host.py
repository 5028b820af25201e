"""Host-side checks of the fused code-step + compaction entry (no GPU needed).

* The reference plans a block's compaction right after its code step only without a replay tail
  (CompressLMProcessor.update_after_step calls _finish_block at the end of the code role only when
  the block has no replay positions, third_party/vllm_overlay/vllm/v1/core/compresslm/
  processor.py:236-255), so code_step_attention_compact refuses any other replay_tail before it
  touches a device.
* Ownership: the copy ops the planner's finish_block produces for a request stay inside that
  request's own pages; ops that reach another request's pages, or write pages another request
  also reads (prefix sharing), are refused.
"""
import numpy as np
import pytest
import torch

from abridgekv_b200 import codestep
from abridgekv_b200.planner import BlockPlanner


def _planned(num_requests=3, C=64, K=32, quota=16, page=16):
    pl = BlockPlanner(num_blocks=64, block_size=page, num_groups=1)
    for r in range(num_requests):
        pl.add_request(r)
        assert pl.allocate_slots(r, C + K)
        pl.set_num_computed_tokens(r, C + K)
    tables = [pl.block_table(r) for r in range(num_requests)]
    width = max(len(t) for t in tables)
    bt = np.zeros((num_requests, width), dtype=np.int32)
    for r, t in enumerate(tables):
        bt[r, :len(t)] = t
    sl = np.full(num_requests, C + K, dtype=np.int32)
    # every request finishes its block: content [0, C) goes, then code slots >= quota
    for r in range(num_requests):
        pl.finish_block(r, (0, C), (C, C + K), [quota], K)
    ops, _ = pl.take_pending()
    flat, off = [], [0]
    for r in range(num_requests):
        for batch in ops.get(r, [[]])[0]:
            flat.extend(np.asarray(getattr(batch, "array", batch), dtype=np.int32).reshape(-1, 4).tolist())
        off.append(len(flat))
    return np.asarray(flat, dtype=np.int32).reshape(-1, 4), np.asarray(off, dtype=np.int64), bt, sl, page


def test_fused_entry_refuses_a_replay_tail():
    q = torch.zeros((256, 8, 128), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="replay_tail == 0"):
        codestep.code_step_attention_compact(q, q, q, q, q, ops=[], op_offsets=[0, 0], quota_per_kv_head=[256],
                                             k_max=256, replay_tail=16)


def test_planner_ops_stay_in_their_own_pages():
    ops, off, bt, sl, page = _planned()
    assert len(ops) > 0 and off[-1] == len(ops)
    codestep.check_op_ownership(ops, off, bt, sl, page)


def test_ops_reaching_another_requests_page_are_refused():
    ops, off, bt, sl, page = _planned()
    bad = ops.copy()
    bad[off[0], 2] = bt[1, 0]  # request 0 writes into request 1's first page
    with pytest.raises(ValueError, match="outside its own block-table row"):
        codestep.check_op_ownership(bad, off, bt, sl, page)


def test_shared_pages_are_refused():
    ops, off, bt, sl, page = _planned()
    shared = bt.copy()
    dst_page = int(ops[off[0], 2])
    shared[2, 0] = dst_page  # request 2 also reads the page request 0 writes (prefix sharing)
    with pytest.raises(ValueError, match="shared pages"):
        codestep.check_op_ownership(ops, off, shared, sl, page)

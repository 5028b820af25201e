"""The executor's group merge (host logic, no GPU): groups over the same layer tensors whose ops touch
disjoint blocks go to abkv_compact in one call per batch index; anything else keeps one call per group,
in group order (the reference applies the groups one after another, gpu_model_runner.py:1147-1220)."""
import numpy as np
import pytest
import torch

from abridgekv_b200 import compaction
from abridgekv_b200.compaction import CopyOps


@pytest.fixture
def calls(monkeypatch):
    rec = []

    def fake_compact(layer_caches, batches, workspace, stream):
        rec.append(([t.data_ptr() for t in layer_caches], [[tuple(op) for op in b] for b in batches]))

    monkeypatch.setattr(compaction, "_compact", fake_compact)
    return rec


def _ops(*rows):
    return CopyOps(np.array(rows, dtype=np.int32))


def test_disjoint_groups_over_shared_tensors_merge(calls):
    tensors = [torch.zeros(4, 2, 16, 1, 8) for _ in range(3)]
    ops = {"r0": [[_ops((1, 0, 1, 5)), _ops((1, 2, 1, 3))], [_ops((7, 1, 7, 0))]],
           "r1": [[_ops((2, 4, 2, 0))], [_ops((8, 3, 8, 1)), _ops((8, 9, 8, 2))]]}
    compaction.execute_kv_copy_operations(ops, [tensors, tensors])
    assert len(calls) == 1
    ptrs, batches = calls[0]
    assert ptrs == [t.data_ptr() for t in tensors]
    # batch b of group 0 (requests in order), then batch b of group 1
    assert batches == [[(1, 0, 1, 5), (2, 4, 2, 0), (7, 1, 7, 0), (8, 3, 8, 1)], [(1, 2, 1, 3), (8, 9, 8, 2)]]


def test_groups_sharing_a_block_stay_separate(calls):
    tensors = [torch.zeros(4, 2, 16, 1, 8)]
    ops = {"r0": [[_ops((1, 0, 1, 5))], [_ops((1, 7, 2, 3))]]}  # block 1 in both groups
    compaction.execute_kv_copy_operations(ops, [tensors, tensors])
    assert [b for _, b in calls] == [[[(1, 0, 1, 5)]], [[(1, 7, 2, 3)]]]


def test_groups_over_different_tensors_stay_separate(calls):
    a, b = [torch.zeros(4, 2, 16, 1, 8)], [torch.zeros(4, 2, 16, 1, 8)]
    ops = {"r0": [[[(1, 0, 1, 5)]], [[(2, 1, 2, 0)]]]}  # plain lists of tuples, as the reference passes them
    compaction.execute_kv_copy_operations(ops, [a, b])
    assert [(p, bt) for p, bt in calls] == [([a[0].data_ptr()], [[(1, 0, 1, 5)]]), ([b[0].data_ptr()], [[(2, 1, 2, 0)]])]


def test_single_group_and_empty_groups(calls):
    tensors = [torch.zeros(4, 2, 16, 1, 8)]
    compaction.execute_kv_copy_operations({"r0": [[], [_ops((3, 0, 3, 1))]]}, [tensors, tensors])
    assert [b for _, b in calls] == [[[(3, 0, 3, 1)]]]
    calls.clear()
    compaction.execute_kv_copy_operations({}, [tensors, tensors])
    assert calls == []


def test_block_ids_outside_the_pool_keep_groups_separate(calls):
    """Ids outside [0, num_blocks) are not compared one by one: two groups holding such ids take the
    per-group path (in group order), so the kernel reports them exactly as the unmerged executor would."""
    tensors = [torch.zeros(4, 2, 16, 1, 8)]  # 4 blocks
    ops = {"r0": [[_ops((1, 0, 9, 5))], [_ops((2, 7, 11, 3))]]}
    compaction.execute_kv_copy_operations(ops, [tensors, tensors])
    assert [b for _, b in calls] == [[[(1, 0, 9, 5)]], [[(2, 7, 11, 3)]]]


def test_disjoint_check_matches_set_intersection():
    rng = np.random.default_rng(3)
    for _ in range(200):
        n = int(rng.integers(1, 5))
        sets = [rng.integers(-2, 40, size=int(rng.integers(0, 12))) for _ in range(n)]
        inside = [set(int(x) for x in s if 0 <= x < 32) for s in sets]
        outside = [any(not (0 <= x < 32) for x in s) for s in sets]
        expect = all(not (inside[i] & inside[j]) and not (outside[i] and outside[j])
                     for i in range(n) for j in range(i + 1, n))
        assert compaction._disjoint(sets, 32) == expect

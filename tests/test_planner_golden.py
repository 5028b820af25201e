"""The C++ compaction planner replays the reference's own serving traces
bit-exactly: copy-op batches, block-table truncations, page tables, removed
spans, free-queue order and rejection messages (tests/golden/compaction_*.json,
made by tests/golden/make_golden.py from the reference's processor, scheduler,
block pool and managers)."""
import json
from pathlib import Path

import pytest

from abridgekv_b200.planner import BlockPlanner

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = sorted(p.name for p in GOLDEN.glob("compaction_*.json"))


def _as_lists(ops):
    return {str(r): [[[list(op) for op in b] for b in per_g] for per_g in groups] for r, groups in ops.items()}


@pytest.mark.parametrize("fname", CASES)
def test_planner_replays_reference_trace(fname):
    t = json.loads((GOLDEN / fname).read_text())
    G = len(t["quotas"])
    p = BlockPlanner(t["pool_blocks"], t["page"], G)
    reqs = [100 + i for i in range(len(t["prompts"]))]
    for r in reqs:
        p.add_request(r)
    n_finish = n_mask = 0
    for e in t["events"]:
        op, r = e["op"], e["req"]
        if op == "alloc":
            assert p.allocate_slots(r, e["num_tokens"])
            p.set_num_computed_tokens(r, e["num_tokens"])
        elif op == "mask":
            before = (p.free_queue(), [p.block_table(x, g) for x in reqs for g in range(G)])
            res = p.mask_token_span(r, e["start"], e["end"], e["groups"])
            assert [res.success, res.tokens_removed, res.blocks_freed, res.error_message] == e["result"]
            after = (p.free_queue(), [p.block_table(x, g) for x in reqs for g in range(G)])
            assert before == after  # a rejected span changes nothing
            n_mask += 1
        elif op == "finish":
            p.finish_block(r, tuple(e["resp"]) if e["resp"] else None, tuple(e["code"]), t["quotas"], t["K"])
            ops, trunc = p.take_pending()
            assert _as_lists(ops) == e["ops"]
            assert {str(k): list(v) for k, v in trunc.items()} == e["trunc"]
            for rid, tables in e["tables"].items():
                assert [p.block_table(int(rid), g) for g in range(G)] == tables
            for rid, spans in e["spans"].items():
                assert [[list(s) for s in p.compacted_spans(int(rid), g)] for g in range(G)] == spans
            assert p.free_queue() == e["free_queue"]
            n_finish += 1
        elif op == "free":
            p.free(r)
            assert p.free_queue() == e["free_queue"]
    assert n_finish >= 4


def test_span_index_maps_match_brute_force():
    """CompactedSpanIndex property of the reference test (test_compresslm_physical_quotas.py:28-49):
    logical<->physical maps equal a brute force over random layouts."""
    import random

    rng = random.Random(0)
    for trial in range(300):
        n = rng.randint(2, 60)
        p = BlockPlanner(64, 4, 1)
        p.add_request(1)
        p.set_num_computed_tokens(1, n)
        assert p.allocate_slots(1, n)
        removed = set()
        for _ in range(rng.randint(0, 4)):
            s = rng.randrange(n)
            e = min(n, s + rng.randint(1, 6))
            if any(x in removed for x in range(s, e)) or len(removed) + (e - s) >= n:
                continue
            res = p.mask_token_span(1, s, e)
            assert res.success, res.error_message
            removed.update(range(s, e))
            p.take_pending()
        active = [x for x in range(n) if x not in removed]
        for phys, logical in enumerate(active):
            assert p.logical_to_physical(1, logical) == phys
            assert p.physical_to_logical(1, phys) == logical

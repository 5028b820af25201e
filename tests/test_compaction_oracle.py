"""Compaction oracle pinned to the reference's own traces, and the C++ planner
checked against the oracle on larger randomized serving scenarios (CPU only)."""
import hashlib
import json
import random
from pathlib import Path

import numpy as np
import pytest

from abridgekv_b200.planner import BlockPlanner
from oracle.compaction_ref import Planner, execute_kv_copy_operations, labelled_cache

GOLDEN = Path(__file__).resolve().parent / "golden"
TRACES = sorted(p.name for p in GOLDEN.glob("compaction_*.json"))


def _norm_ops(ops):
    return {str(r): [[[list(op) for op in b] for b in per_g] for per_g in g] for r, g in ops.items()}


@pytest.mark.parametrize("fname", TRACES)
def test_oracle_planner_replays_reference_trace(fname):
    t = json.loads((GOLDEN / fname).read_text())
    G = len(t["quotas"])
    p = Planner(t["pool_blocks"], t["page"], G)
    for i in range(len(t["prompts"])):
        p.add_request(100 + i)
    for e in t["events"]:
        r = e["req"]
        if e["op"] == "alloc":
            assert p.allocate_slots(r, e["num_tokens"])
            p.computed[r] = e["num_tokens"]
        elif e["op"] == "mask":
            assert list(p.mask_token_span(r, e["start"], e["end"], e["groups"])) == e["result"]
        elif e["op"] == "finish":
            p.finish_block(r, e["resp"], e["code"], t["quotas"], t["K"])
            ops, trunc = p.take_pending()
            assert _norm_ops(ops) == e["ops"]
            assert {str(k): list(v) for k, v in trunc.items()} == e["trunc"]
            assert p.pool.q.order == e["free_queue"]
        elif e["op"] == "free":
            p.free(r)
            assert p.pool.q.order == e["free_queue"]


@pytest.mark.parametrize("fname", sorted(p.name for p in GOLDEN.glob("executor_*.json")))
def test_oracle_executor_matches_reference(fname):
    gold = json.loads((GOLDEN / fname).read_text())
    t = json.loads((GOLDEN / gold["source"]).read_text())
    G = len(t["quotas"])
    for case in gold["cases"]:
        caches = [labelled_cache(case["layout"], t["pool_blocks"], t["page"], i) for i in range(2)]
        for e in t["events"]:
            if e["op"] == "finish" and e["ops"]:
                execute_kv_copy_operations(e["ops"], [caches] * G)
        assert [hashlib.sha256(c.tobytes()).hexdigest() for c in caches] == case["sha256"]


def _random_serving(seed, G=3, K=16, C=32, page=4, pool=600, n_req=5):
    """Random interleaving of prefill/decode/code steps, block finishes, early
    frees and rejected spans; every planner call is mirrored on the oracle."""
    rng = random.Random(seed)
    quotas = tuple(sorted(rng.choice([K, K // 2, K // 4]) for _ in range(G)))
    a, b = BlockPlanner(pool, page, G), Planner(pool, page, G)
    state = {}
    next_id = 1
    for step in range(1500):
        if len(state) < n_req and rng.random() < 0.05:
            r = next_id
            next_id += 1
            a.add_request(r)
            b.add_request(r)
            state[r] = {"P": rng.randint(1, 2 * C), "blk": 0, "c": 0, "n": 0}
            continue
        if not state:
            continue
        r = rng.choice(sorted(state))
        st = state[r]
        if rng.random() < 0.01:  # request finishes early / is preempted
            a.free(r)
            b.free(r)
            assert a.free_queue() == b.pool.q.order
            del state[r]
            continue
        if rng.random() < 0.03:  # arbitrary span probe (valid or not)
            s0 = rng.randint(-2, st["n"] + 2)
            e0 = s0 + rng.randint(0, 5)
            groups = None if rng.random() < 0.5 else [rng.randint(-1, G) for _ in range(rng.randint(0, 2))]
            ra = a.mask_token_span(r, s0, e0, groups)
            rb = b.mask_token_span(r, s0, e0, groups)
            assert [ra.success, ra.tokens_removed, ra.blocks_freed, ra.error_message] == list(rb)
            oa, ta = a.take_pending()
            ob, tb = b.take_pending()
            assert _norm_ops(oa) == _norm_ops(ob) and ta == tb
            continue
        if st["c"] < C:
            first = st["blk"] == 0 and st["c"] == 0
            k = min(C, st["P"]) if first else 1
            ok_a = a.allocate_slots(r, st["n"] + k)
            ok_b = b.allocate_slots(r, st["n"] + k)
            assert ok_a == ok_b
            if not ok_a:
                continue
            st["n"] += k
            st["c"] += k
            a.set_num_computed_tokens(r, st["n"])
            b.computed[r] = st["n"]
            continue
        ok_a, ok_b = a.allocate_slots(r, st["n"] + K), b.allocate_slots(r, st["n"] + K)
        assert ok_a == ok_b
        if not ok_a:
            continue
        st["n"] += K
        a.set_num_computed_tokens(r, st["n"])
        b.computed[r] = st["n"]
        base = st["blk"] * (C + K)
        resp = [base + j for j in range(C) if st["blk"] * C + j >= st["P"]]
        span = (resp[0], resp[-1] + 1) if resp else None
        err_a = err_b = None
        try:
            a.finish_block(r, span, (base + C, base + C + K), quotas, K)
        except RuntimeError as e:
            err_a = str(e)
        try:
            b.finish_block(r, span, (base + C, base + C + K), quotas, K)
        except RuntimeError as e:
            err_b = str(e)
        assert (err_a is None) == (err_b is None)
        oa, ta = a.take_pending()
        ob, tb = b.take_pending()
        assert _norm_ops(oa) == _norm_ops(ob) and ta == tb
        for g in range(G):
            assert a.block_table(r, g) == b.blocks[g].get(r, [])
        assert a.free_queue() == b.pool.q.order
        st["blk"] += 1
        st["c"] = 0
    for r in list(state):
        a.free(r)
        b.free(r)
    assert a.free_queue() == b.pool.q.order


@pytest.mark.parametrize("seed", range(6))
def test_cpp_planner_matches_oracle_random_serving(seed):
    _random_serving(seed)


def test_copy_ops_reads_like_reference_lists_and_flattens_identically():
    """take_pending batches (CopyOps) compare, index and iterate like the reference's lists of
    (src_block, src_off, dst_block, dst_off) tuples, and the executor flattens them to the same
    int32 buffer as the plain-list form."""
    import numpy as np
    from abridgekv_b200.compaction import CopyOps, _flatten

    rng = np.random.default_rng(0)
    arrays = [rng.integers(0, 5000, size=(n, 4)).astype(np.int32) for n in (3, 0, 17)]
    ops = [CopyOps(a) for a in arrays]
    lists = [[tuple(int(v) for v in row) for row in a] for a in arrays]
    for o, l in zip(ops, lists):
        assert o == l and list(o) == l and len(o) == len(l)
        if l:
            assert o[0] == l[0] and o[-1] == l[-1] and list(o[1:]) == l[1:]
    f_fast, c_fast = _flatten(ops)
    f_list, c_list = _flatten(lists)
    assert c_fast == c_list and np.array_equal(f_fast, f_list)

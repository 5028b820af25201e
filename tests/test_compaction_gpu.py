"""Compaction executor kernels through the C ABI on a B200 (bit-exact).

* the reference's own executor results (tests/golden/executor_*.json) in both
  paged layouts;
* adversarial batches (overlapping left shifts = long chains, swap cycles,
  duplicate destinations, rows read twice, rows copied onto themselves,
  hazard-free moves) against the numpy oracle;
* BASELINE config 4 at full size: 16 sequences x 16 blocks (C=512, K=256),
  quotas 256/128/64, all 36 layers; after every block's compaction, each
  surviving logical row's checksum equals its pre-compaction checksum
  (checksum of checksums) and freed pages are the planner's.
"""
import hashlib
import json
import random
from pathlib import Path

import numpy as np
import pytest
import torch

from abridgekv_b200 import compaction
from abridgekv_b200.planner import BlockPlanner
from abridgekv_b200.workspace import Workspace
from oracle.compaction_ref import execute_kv_copy_group, execute_kv_copy_operations, labelled_cache

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("fname", sorted(p.name for p in GOLDEN.glob("executor_*.json")))
def test_executor_matches_reference(fname):
    gold = json.loads((GOLDEN / fname).read_text())
    t = json.loads((GOLDEN / gold["source"]).read_text())
    G = len(t["quotas"])
    for case in gold["cases"]:
        caches = [torch.from_numpy(labelled_cache(case["layout"], t["pool_blocks"], t["page"], i)).cuda()
                  for i in range(2)]
        ws = Workspace()
        for e in t["events"]:
            if e["op"] == "finish" and e["ops"]:
                compaction.execute_kv_copy_operations(e["ops"], [caches] * G, workspace=ws)
        assert ws.read_error() == 0
        got = [hashlib.sha256(c.cpu().numpy().tobytes()).hexdigest() for c in caches]
        assert got == case["sha256"], case["layout"]


def _random_batch(rng, nb, page, kind):
    slots = nb * page
    if kind == "shift":  # one request's left shift: src s -> s - R
        start = rng.randrange(slots // 2)
        R = rng.choice([1, 2, 3, 7, 16, 100])
        end = min(slots - 1, start + R)
        n_active = rng.randint(end + 1, slots)
        ops = [(s, s - (end - start)) for s in range(end, n_active)]
    elif kind == "swap":
        a = rng.sample(range(slots), 8)
        ops = [(a[i], a[(i + 1) % 8]) for i in range(8)]  # a cycle
    elif kind == "dup":
        ops = [(rng.randrange(slots), rng.randrange(slots)) for _ in range(60)]
        ops += [(rng.randrange(slots), ops[0][1])]  # duplicate destination, last wins
    elif kind == "read_twice":
        s = rng.randrange(slots)
        ops = [(s, rng.randrange(slots)) for _ in range(5)]
        ops = list({d: (x, d) for x, d in ops}.values())
    elif kind == "self":  # rows copied onto themselves among disjoint moves
        pool = rng.sample(range(slots), 300)
        ops = [(pool[i], pool[100 + i]) for i in range(100)] + [(pool[200 + i], pool[200 + i]) for i in range(100)]
        rng.shuffle(ops)
    else:  # disjoint
        pool = rng.sample(range(slots), 400)
        ops = [(pool[i], pool[200 + i]) for i in range(200)]
    perm = list(range(nb))
    rng.shuffle(perm)  # slot -> (block id, offset) through a random table
    return [(perm[s // page], s % page, perm[d // page], d % page) for s, d in ops]


@pytest.mark.parametrize("layout", [0, 1])
@pytest.mark.parametrize("kind", ["shift", "swap", "dup", "read_twice", "self", "disjoint"])
def test_executor_hazards_match_oracle(layout, kind):
    rng = random.Random(hash((layout, kind)) & 0xFFFF)
    nb, page, hkv, d, L = 48, 16, 8, 128, 5
    gen = torch.Generator().manual_seed(3)
    shape = (nb, 2, page, hkv, d) if layout == 0 else (2, nb, page, hkv, d)
    host = [torch.randn(shape, generator=gen).to(torch.bfloat16) for _ in range(L)]
    dev = [h.cuda() for h in host]
    ref = [h.view(torch.int16).numpy().copy() for h in host]
    ws = Workspace()
    batches = [_random_batch(rng, nb, page, kind) for _ in range(3)]
    for b in batches:
        if kind == "dup":
            # the reference's index_put with repeated destinations has no defined
            # winner; the oracle applies "last listed op wins" like libabkv
            last = {}
            for op in b:
                last[(op[2], op[3])] = op
            execute_kv_copy_group(list(last.values()), ref)
        else:
            execute_kv_copy_group(b, ref)
        compaction.execute_kv_copy_group(b, dev, workspace=ws)
    assert ws.read_error() == 0
    for r, dv in zip(ref, dev):
        assert np.array_equal(r, dv.cpu().view(torch.int16).numpy())


def test_evict_columns_matches_torch_index():
    gen = torch.Generator(device="cuda").manual_seed(0)
    K = [torch.randn((1, 8, 700, 128), device="cuda", generator=gen, dtype=torch.bfloat16) for _ in range(3)]
    V = [torch.randn((1, 8, 700, 128), device="cuda", generator=gen, dtype=torch.bfloat16) for _ in range(3)]
    keep = torch.tensor(sorted(random.Random(1).sample(range(700), 300)), device="cuda")
    k2, v2 = compaction.evict_columns(K, V, keep)
    for a, b in zip(K + V, k2 + v2):
        assert torch.equal(a[:, :, keep, :], b)


def test_config4_full_size_compaction_preserves_rows():
    """BASELINE config 4's compaction at full size, in serving order: each block's
    K code rows are computed, then the block's content and its code slots >= q
    are removed (finish_block) and the copy ops executed before the next block.
    Layer i of every quota group shares physical tensor i (vLLM's grouping)."""
    C, K, page = 512, 256, 16
    quotas = (256, 128, 64)
    G = len(quotas)
    B, blocks, L = 16, 16, 36
    per = C + K
    n_tensors = L // G  # 12 physical tensors, each used by one layer of every group
    nb = 1 + B * (blocks * per // page) * G
    planner = BlockPlanner(nb, page, G)
    gen = torch.Generator(device="cuda").manual_seed(4)
    caches = [torch.randn((nb, 2, page, 8, 128), device="cuda", generator=gen, dtype=torch.bfloat16)
              for _ in range(n_tensors)]
    w = torch.randint(1, 1 << 20, (2 * 8 * 128,), device="cuda", generator=gen, dtype=torch.int64)
    groups = [caches] * G  # group g's layers -> tensors 0..11
    ws = Workspace()
    before = {}
    for b in range(B):
        planner.add_request(b)
    n_ops = 0
    for blk in range(blocks):
        for b in range(B):
            n = (blk + 1) * per
            assert planner.allocate_slots(b, n)
            planner.set_num_computed_tokens(b, n)
            for g in range(G):
                table = planner.block_table(b, g)
                first = planner.logical_to_physical(b, blk * per, g)
                rows = _row_checksums_range(caches, table, first, first + per, page, w)
                for t in range(n_tensors):
                    before[(t, g, b, blk)] = rows[t][C:]  # the code rows that survive
            planner.finish_block(b, (blk * per, blk * per + C), (blk * per + C, (blk + 1) * per), quotas, K)
        ops, _ = planner.take_pending()
        n_ops += sum(len(x) for per_g in ops.values() for bl in per_g for x in bl)
        compaction.execute_kv_copy_operations(ops, groups, workspace=ws)
    torch.cuda.synchronize()
    assert ws.read_error() == 0
    assert n_ops > 0
    for g, q in enumerate(quotas):
        for b in range(B):
            table = planner.block_table(b, g)
            assert len(table) == -(-blocks * q // page)
            assert planner.logical_to_physical(b, (blocks - 1) * per + C, g) == (blocks - 1) * q
            after = _row_checksums_range(caches, table, 0, blocks * q, page, w)
            for t in range(n_tensors):
                exp = torch.cat([before[(t, g, b, blk)][:q] for blk in range(blocks)])
                assert torch.equal(after[t], exp), (g, b, t)


def _row_checksums_range(caches, table, lo, hi, page, w):
    r = torch.arange(lo, hi, device="cuda")
    pages = torch.as_tensor(table, device="cuda", dtype=torch.long)[r // page]
    out = []
    for kv in caches:
        rows = kv[pages, :, r % page].reshape(hi - lo, -1).view(torch.int16).to(torch.int64)
        out.append((rows * w).sum(dim=1))
    return out

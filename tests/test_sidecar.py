"""Packed per-head-quota sidecar: PackedKVLayout on CPU; decode over sidecar pages + the paged
main cache through abkv_decode_packed on a B200 against the reference goldens and the float64
oracle (tolerances as the plain decode: |gpu - reference| <= 3e-2, |gpu - float64| <= 1.5e-2 max
and <= 2e-3 mean; relative error reported and bounded as in tests/errstats.py)."""
import numpy as np
import pytest
import torch

from abridgekv_b200.sidecar import PackedKVLayout

ATOL_REF, ATOL_EXACT, MEAN_EXACT = 3e-2, 1.5e-2, 2e-3


def test_layout_pack_unpack_roundtrip_and_slot_order():
    layout = PackedKVLayout.from_schedule([[4, 2, 3], [1, 4, 4]], num_layers=2, num_kv_heads=3, k_max=4)
    assert layout.offsets == ((0, 4, 6, 9), (0, 1, 5, 9))
    assert layout.packed_slots_per_layer == (9, 9)
    dense = torch.arange(2 * 4 * 3 * 5, dtype=torch.float32).reshape(2, 4, 3, 5)
    for layer in range(2):
        packed = layout.pack_layer(layer, dense)
        assert packed.shape == (2, 9, 5)
        for h, q in enumerate(layout.quotas[layer]):
            o = layout.offsets[layer][h]
            assert torch.equal(packed[:, o:o + q], dense[:, :q, h])
        back = layout.unpack_layer(layer, packed, fill_value=-1.0)
        for h, q in enumerate(layout.quotas[layer]):
            assert torch.equal(back[:, :q, h], dense[:, :q, h])
            assert torch.all(back[:, q:, h] == -1.0)


@pytest.mark.parametrize("bad", [[[0, 2]], [[5, 2]], [[2, 2], [2]]])
def test_layout_rejects_bad_quotas(bad):
    with pytest.raises(ValueError):
        PackedKVLayout(quotas=tuple(tuple(r) for r in bad), k_max=4)


def _pool(layout, side, counts, head_dim, spare=3):
    """SidecarPool holding each request's pages (request after request), with spare pages
    poisoned with NaN that no request references."""
    from abridgekv_b200.sidecar import SidecarPool

    pool = SidecarPool(layout, 0, capacity=int(sum(counts)) + spare, num_requests=len(counts),
                       max_pages=max(1, int(max(counts))) + 1, head_dim=head_dim)
    pool.pages.fill_(float("nan"))
    first = 0
    for r, cnt in enumerate(counts):
        for i in range(int(cnt)):
            pool.append(r, torch.from_numpy(side[first + i]).to(torch.bfloat16).cuda())
        first += int(cnt)
    return pool


@pytest.mark.gpu
@pytest.mark.parametrize("chunk_tokens", [0, 32, 256])
def test_packed_decode_matches_reference_golden(chunk_tokens):
    from abridgekv_b200.sidecar import attend_decode_batched_packed
    from abridgekv_b200.workspace import Workspace
    from oracle.decode_ref import packed_decode_exact
    from tests.errstats import assert_relative, report
    from tests.goldens import load_packed, packed_cases

    for name in packed_cases():
        case, side, counts, quotas, k_max, ref = load_packed(name)
        if chunk_tokens and chunk_tokens % case.page:
            continue
        layout = PackedKVLayout.from_schedule([list(quotas)], num_layers=1, num_kv_heads=len(quotas), k_max=k_max)
        pool = _pool(layout, side, counts, case.q.shape[-1])
        q = torch.from_numpy(case.q).to(torch.bfloat16).cuda()
        kv = torch.from_numpy(case.kv).to(torch.bfloat16).cuda()
        out = torch.full_like(q, float("nan"))
        ws = Workspace()
        from abridgekv_b200 import sidecar as sc
        sc.packed_decode([q], [kv], [torch.from_numpy(case.block_table).cuda()],
                         [torch.from_numpy(case.seq_lens).cuda()], [pool], scale=case.scale, outputs=[out],
                         chunk_tokens=chunk_tokens, workspace=ws)
        torch.cuda.synchronize()
        assert ws.read_error() == 0, name
        got = out.float().cpu().numpy()
        ex = packed_decode_exact(case.q, case.kv, case.block_table, case.seq_lens, side, counts, quotas,
                                 case.scale, case.page)
        se, sr = report(f"{name} chunk={chunk_tokens}", got, ex, ref)
        assert sr["max_abs"] <= ATOL_REF, name
        assert se["max_abs"] <= ATOL_EXACT and se["mean_abs"] <= MEAN_EXACT, name
        assert_relative(se, name)
        # the drop-in form writes the same rows
        out2 = torch.zeros((q.shape[0], q.shape[1] * q.shape[2]), dtype=torch.bfloat16, device="cuda")
        attend_decode_batched_packed(query=q, kv_cache=kv, output=out2,
                                     seq_lens=torch.from_numpy(case.seq_lens), block_table=torch.from_numpy(
                                         case.block_table).cuda(), num_kv_heads=len(quotas),
                                     groups=q.shape[1] // len(quotas), scale=case.scale, sidecar=pool)
        if chunk_tokens == 0:
            assert torch.equal(out2.view_as(out), out)


@pytest.mark.gpu
def test_packed_decode_without_sidecar_equals_plain_decode():
    """Layers with no sidecar in a packed launch give exactly the plain decode's rows."""
    from abridgekv_b200 import decode
    from abridgekv_b200.sidecar import packed_decode
    from tests.goldens import load_packed

    case, side, counts, quotas, k_max, ref = load_packed("h2_small")
    layout = PackedKVLayout.from_schedule([list(quotas)], num_layers=1, num_kv_heads=len(quotas), k_max=k_max)
    pool = _pool(layout, side, counts, case.q.shape[-1])
    q = torch.from_numpy(case.q).to(torch.bfloat16).cuda()
    kv = torch.from_numpy(case.kv).to(torch.bfloat16).cuda()
    bt, sl = torch.from_numpy(case.block_table).cuda(), torch.from_numpy(case.seq_lens).cuda()
    plain = decode.paged_decode([q], [kv], [bt], [sl], scale=case.scale)[0]
    both = packed_decode([q, q], [kv, kv], [bt, bt], [sl, sl], [None, pool], scale=case.scale)
    assert torch.equal(both[0], plain)
    assert not torch.equal(both[1], plain)


@pytest.mark.gpu
@pytest.mark.parametrize("chunk_tokens", [0, 32])
def test_packed_decode_repeat_calls_on_one_workspace_are_identical(chunk_tokens):
    """Work items past a request's last chunk are claimed and skipped; a skipped item must not
    change the chunking of the next one, and every call leaves the workspace counters at zero,
    so repeated launches on one workspace give bit-identical rows with no device error."""
    from abridgekv_b200.sidecar import packed_decode
    from abridgekv_b200.workspace import Workspace
    from tests.goldens import load_packed, packed_cases

    for name in packed_cases():
        case, side, counts, quotas, k_max, _ = load_packed(name)
        if chunk_tokens and chunk_tokens % case.page:
            continue
        layout = PackedKVLayout.from_schedule([list(quotas)], num_layers=1, num_kv_heads=len(quotas), k_max=k_max)
        pool = _pool(layout, side, counts, case.q.shape[-1])
        q = torch.from_numpy(case.q).to(torch.bfloat16).cuda()
        kv = torch.from_numpy(case.kv).to(torch.bfloat16).cuda()
        bt, sl = torch.from_numpy(case.block_table).cuda(), torch.from_numpy(case.seq_lens).cuda()
        ws = Workspace()
        outs = [packed_decode([q, q], [kv, kv], [bt, bt], [sl, sl], [pool, pool], scale=case.scale,
                              chunk_tokens=chunk_tokens, workspace=ws) for _ in range(4)]
        torch.cuda.synchronize()
        assert ws.read_error() == 0, name
        for o in outs[1:]:
            assert torch.equal(o[0], outs[0][0]) and torch.equal(o[1], outs[0][0]), name


def test_layout_matches_the_reference_class():
    """PackedKVLayout against the reference's own class on the same inputs
    (tests/golden/packed_layout_reference.json, made by make_golden.py --only layout): the same
    validation messages, offsets and packed slot counts."""
    import json
    from pathlib import Path

    gold = json.loads((Path(__file__).resolve().parent / "golden" / "packed_layout_reference.json").read_text())

    def describe(fn):
        try:
            x = fn()
            return {"quotas": [list(r) for r in x.quotas], "offsets": [list(r) for r in x.offsets],
                    "slots": list(x.packed_slots_per_layer), "k_max": x.k_max}
        except ValueError as e:
            return {"error": str(e)}

    for case in gold["layouts"]:
        quotas = tuple(tuple(r) for r in case["quotas"])
        assert describe(lambda: PackedKVLayout(quotas=quotas, k_max=case["k_max"])) == case["result"], case
    for case in gold["schedules"]:
        got = describe(lambda: PackedKVLayout.from_schedule(case["schedule"], num_layers=case["num_layers"],
                                                            num_kv_heads=case["num_kv_heads"], k_max=case["k_max"]))
        assert got == case["result"], case

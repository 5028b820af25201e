"""HostDecode: decode with pinned host queries/outputs, copies overlapped with the launches of
layer groups.  CPU: the group split.  GPU: rows bit-identical to paged_decode launched with the
same layer groups from device tensors, for several splits, across repeated calls."""
import pytest
import torch

from abridgekv_b200.hostdecode import split_layers


@pytest.mark.parametrize("L,max_group,edge,expect", [
    (1, 12, 1, [(0, 1)]),
    (2, 12, 1, [(0, 1), (1, 2)]),
    (5, 12, 1, [(0, 1), (1, 4), (4, 5)]),
    (36, 12, 1, [(0, 1), (1, 13), (13, 24), (24, 35), (35, 36)]),
    (36, 16, 2, [(0, 2), (2, 18), (18, 34), (34, 36)]),
    (36, 6, 0, [(0, 6), (6, 12), (12, 18), (18, 24), (24, 30), (30, 36)]),
])
def test_split_layers(L, max_group, edge, expect):
    groups = split_layers(L, max_group, edge)
    assert [(g.start, g.stop) for g in groups] == expect
    assert [l for g in groups for l in g] == list(range(L))


def test_split_layers_rejects_bad_arguments():
    with pytest.raises(ValueError):
        split_layers(0)
    with pytest.raises(ValueError):
        split_layers(4, max_group=0)


@pytest.mark.gpu
@pytest.mark.parametrize("groups", [None, "one", "per_layer"])
def test_host_decode_matches_device_decode_by_group(groups):
    from abridgekv_b200 import decode
    from abridgekv_b200.hostdecode import HostDecode
    from abridgekv_b200.workspace import Workspace
    from tests.test_decode_gpu import _random_layers

    L = 5
    qs, kvs, bts, sls = _random_layers(L, B=16, max_pages=32, seed=3)
    # two layers share one block table / seq_lens pair (one quota group): uploaded once
    bts[3], sls[3] = bts[2], sls[2]
    grp = {None: None, "one": [range(0, L)], "per_layer": [range(l, l + 1) for l in range(L)]}[groups]
    hd = HostDecode(kvs, groups=grp, chunk_tokens=64, workspace=Workspace())
    ref = []
    for g in hd.groups:
        ls = list(g)
        ref += decode.paged_decode([qs[l] for l in ls], [kvs[l] for l in ls], [bts[l] for l in ls],
                                   [sls[l] for l in ls], chunk_tokens=64, workspace=Workspace())
    pin = lambda t: t.cpu().pin_memory()
    host_bt = {id(t): pin(t) for t in bts}
    host_sl = {id(t): pin(t) for t in sls}
    q_h = [pin(q) for q in qs]
    out_h = [torch.full(q.shape, float("nan"), dtype=q.dtype).pin_memory() for q in qs]
    for rep in range(3):
        hd.run(q_h, [host_bt[id(t)] for t in bts], [host_sl[id(t)] for t in sls], out_h)
        torch.cuda.current_stream().synchronize()
        for l in range(L):
            assert torch.equal(out_h[l], ref[l].cpu()), (rep, l)
    assert hd.workspace.read_error() == 0


@pytest.mark.gpu
def test_host_decode_rejects_device_or_unpinned_tensors():
    from abridgekv_b200.hostdecode import HostDecode
    from tests.test_decode_gpu import _random_layers

    qs, kvs, bts, sls = _random_layers(1, B=4, max_pages=4)
    hd = HostDecode(kvs)
    with pytest.raises(ValueError):
        hd.run(qs, bts, sls, [torch.empty_like(qs[0])])
    with pytest.raises(ValueError):
        hd.run([qs[0].cpu()], [bts[0].cpu()], [sls[0].cpu()], [qs[0].cpu()])

"""BASELINE config 1 on a B200: the kernels reproduce the attention of the reference's own model flow
(tests/golden/config1_reference.npz, made by running CompressLM.forward and CompressGen on the tiny
Qwen3 of config 1: 2 layers, 4 q / 2 kv heads, head_dim 64, quotas [128, 64], C=512, K_max=128).

* decode: six of the 256 greedy steps of both layers, their visible store columns (4 compressed blocks x
  the layer's quota code rows + the live content rows) laid into shuffled paged caches, one abkv_decode
  launch over both layers;
* prefill: CompressLM.forward's per-layer attention (FlexAttention with the quota masks) through
  abkv_prefill_masked with C=512, K_layout=128 and each layer's quota.
Tolerances: against float64 on the same bf16 inputs, those of the kernel tests (decode 1.5e-2 max abs,
prefill 2.5e-2); against the reference's fp32 outputs, 2e-2 max abs (bf16 input rounding: the float64
oracle itself sits within 2.7e-3 of them); relative error reported and bounded (tests/errstats.py).
"""
import numpy as np
import pytest
import torch

from abridgekv_b200 import decode, prefill
from abridgekv_b200.workspace import Workspace
from oracle.decode_ref import decode_exact
from oracle.mask_ref import arith_mask, masked_attention
from tests.errstats import assert_relative, report
from tests.goldens import config1_paged, load_config1

pytestmark = pytest.mark.gpu
G = load_config1()


def _bf(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(torch.bfloat16).cuda()


def test_config1_decode_steps_both_layers_one_launch():
    per_layer = [config1_paged(G["decode"][l], seed=l) for l in range(2)]
    # both layers' batches share B (the same six steps); the tables are padded to one width
    width = max(p[2].shape[1] for p in per_layer)
    qs, kvs, bts, sls = [], [], [], []
    for q, kv, bt, lens, _, _ in per_layer:
        qs.append(_bf(q))
        kvs.append(_bf(kv))
        pad = np.zeros((bt.shape[0], width), np.int32)
        pad[:, :bt.shape[1]] = bt
        bts.append(torch.from_numpy(pad).cuda())
        sls.append(torch.from_numpy(lens).cuda())
    ws = Workspace()
    outs = decode.paged_decode(qs, kvs, bts, sls, scale=1.0 / np.sqrt(64), workspace=ws)
    torch.cuda.synchronize()
    assert ws.read_error() == 0
    for l, (q, kv, bt, lens, ref, steps) in enumerate(per_layer):
        got = outs[l].float().cpu().numpy()
        exact = decode_exact(q, kv, bt, lens, 1.0 / np.sqrt(64), 16)
        se, sr = report(f"config1 decode layer {l} (quota {G['quotas'][l]}, steps {steps})", got, exact, ref)
        assert se["max_abs"] <= 1.5e-2 and sr["max_abs"] <= 2e-2
        assert_relative(se)
        assert_relative(sr)


@pytest.mark.parametrize("layer", [0, 1])
def test_config1_prefill_layer(layer):
    q_rows, k, v, ref = G["prefill"][layer]
    H, n, D = q_rows.shape
    S0 = G["N"] * (G["C"] + G["K"])
    q = np.zeros((1, H, S0, D), dtype=np.float32)
    q[0, :, G["rows"]] = q_rows.transpose(1, 0, 2)
    quota = [G["quotas"][layer]] * H
    ws = Workspace()
    out = prefill.prefill_masked(_bf(q), _bf(k[None]), _bf(v[None]), C=G["C"], K_layout=G["K"], quota_per_head=quota,
                                 workspace=ws)
    torch.cuda.synchronize()
    assert ws.read_error() == 0
    got = out[0][:, G["rows"]].float().cpu().numpy().transpose(1, 0, 2)     # [n, H, D]
    mask = arith_mask(S0, G["C"], G["K"], quota_per_head=quota)
    ex, _ = masked_attention(q, k[None], v[None], mask, 1.0 / np.sqrt(D))
    exact = ex[0][:, G["rows"]].transpose(1, 0, 2)
    se, sr = report(f"config1 prefill layer {layer} (quota {G['quotas'][layer]})", got, exact, ref)
    assert se["max_abs"] <= 2.5e-2 and se["mean_abs"] <= 2e-3 and sr["max_abs"] <= 2e-2
    assert_relative(se)
    assert_relative(sr)

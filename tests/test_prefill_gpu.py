"""tcgen05 prefill-mask attention through the C ABI on a B200.

Tolerances (bf16 output; P rounded to bf16 before P.V as FlexAttention's
kernels do): max |gpu - float64 oracle| <= 2.5e-2, mean <= 2e-3; the same
bounds against the reference's FlexAttention rows; lse within 1e-2; relative
error (tests/errstats.py) reported and bounded.
"""
import numpy as np
import pytest
import torch

from abridgekv_b200 import prefill
from abridgekv_b200.workspace import Workspace
from oracle.mask_ref import arith_mask, masked_attention
from tests.errstats import assert_relative, report
from tests.goldens import load_prefill, prefill_cases

pytestmark = pytest.mark.gpu
ATOL, MEAN = 2.5e-2, 2e-3


def _dev(x):
    return torch.from_numpy(x).to(torch.bfloat16).cuda()


@pytest.mark.parametrize("name", prefill_cases())
def test_prefill_matches_reference_flex_and_oracle(name):
    g = load_prefill(name)
    q, k, v = _dev(g["q"]), _dev(g["k"]), _dev(g["v"])
    pl = torch.as_tensor(g["prompt_len"], device="cuda") if g["prompt_len"] is not None else None
    ws = Workspace()
    out, lse = prefill.prefill_masked(q, k, v, C=g["C"], K_layout=g["K"], quota_per_head=list(g["quota"]),
                                      prompt_len=pl, return_lse=True, workspace=ws)
    torch.cuda.synchronize()
    assert ws.read_error() == 0
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    ref64, lse64 = masked_attention(g["q"], g["k"], g["v"], g["mask"], 1.0 / np.sqrt(g["D"]))
    se, _ = report(name, got, ref64)
    assert se["max_abs"] <= ATOL and se["mean_abs"] <= MEAN
    assert_relative(se, name)
    _, sr = report(f"{name} (reference FlexAttention rows)", got[:, :, g["rows"], :],
                   ref64[:, :, g["rows"], :], g["out_rows"])
    assert sr["max_abs"] <= ATOL
    assert np.abs(lse.cpu().numpy() - g["lse"]).max() <= 1e-2


def test_prefill_strided_views_equal_contiguous():
    """HF hands [B, H, S, D] views of [B, S, H, D] projections: same results as contiguous inputs."""
    g = load_prefill("c128k128_quota_prompt")
    B, H, Hkv, S0 = g["B"], g["H"], g["Hkv"], g["S0"]
    q, k, v = _dev(g["q"]), _dev(g["k"]), _dev(g["v"])
    qs = q.transpose(1, 2).contiguous().transpose(1, 2)
    ks = k.transpose(1, 2).contiguous().transpose(1, 2)
    vs = v.transpose(1, 2).contiguous().transpose(1, 2)
    pl = torch.as_tensor(g["prompt_len"], device="cuda")
    a = prefill.prefill_masked(q, k, v, C=g["C"], K_layout=g["K"], quota_per_head=list(g["quota"]), prompt_len=pl)
    b = prefill.prefill_masked(qs, ks, vs, C=g["C"], K_layout=g["K"], quota_per_head=list(g["quota"]),
                               prompt_len=pl)
    assert torch.equal(a, b)


def test_attention_interface_shim():
    g = load_prefill("c128k128_layer1")
    q, k, v = _dev(g["q"]), _dev(g["k"]), _dev(g["v"])
    mask = prefill.CompressMask(C=g["C"], K_layout=g["K"], quota_per_head=tuple(int(x) for x in g["quota"]))
    out, none = prefill.abkv_attention_forward(None, q, k, v, mask, scaling=1.0 / np.sqrt(128))
    assert none is None and out.shape == (g["B"], g["S0"], g["H"], 128)
    ref = prefill.prefill_masked(q, k, v, C=g["C"], K_layout=g["K"], quota_per_head=list(g["quota"]))
    assert torch.equal(out, ref.transpose(1, 2))


def test_config4_full_size_sampled_rows():
    """BASELINE config 4 shape: B=16, 16 blocks of 512 + 256 code rows (S0=12288), 32/8 heads,
    quotas 256/128/64 over the heads' groups; sampled query rows against a PyTorch fp32
    reference of the same mask on the GPU."""
    B, H, Hkv, C, K, N = 16, 32, 8, 512, 256, 16
    S0 = N * (C + K)
    gen = torch.Generator(device="cuda").manual_seed(7)
    q = torch.randn((B, S0, H, 128), device="cuda", generator=gen, dtype=torch.bfloat16).transpose(1, 2)
    k = torch.randn((B, S0, Hkv, 128), device="cuda", generator=gen, dtype=torch.bfloat16).transpose(1, 2)
    v = torch.randn((B, S0, Hkv, 128), device="cuda", generator=gen, dtype=torch.bfloat16).transpose(1, 2)
    quota = [256, 128, 64, 256, 128, 64, 128, 128]
    qph = [quota[h // 4] for h in range(H)]
    pl = torch.tensor([0, 300, 1000, 5000] * 4, device="cuda", dtype=torch.int32)
    ws = Workspace()
    out = prefill.prefill_masked(q, k, v, C=C, K_layout=K, quota_per_head=qph, prompt_len=pl, workspace=ws)
    torch.cuda.synchronize()
    assert ws.read_error() == 0
    rng = np.random.default_rng(0)
    kv = torch.arange(S0, device="cuda")
    per = C + K
    for b in (0, 1, 2, 3, 9):
        for h in rng.choice(H, 3, replace=False):
            rows = torch.as_tensor(np.sort(rng.choice(S0, 24, replace=False)), device="cuda")
            qb, qw = rows[:, None] // per, rows[:, None] % per
            kb, kw = kv[None, :] // per, kv[None, :] % per
            kc = kw < C
            same = kb == qb
            vis = (kc & same) | (~kc & (kb < qb))
            vis = vis | (kc & (kb * C + kw < int(pl[b])))
            vis = vis & (kv[None, :] <= rows[:, None])
            vis = vis | ((qw >= C) & ~kc & same)
            vis = vis & (kc | ((kw - C) < qph[h]))
            s = (q[b, h, rows].float() @ k[b, h // 4].float().T) / np.sqrt(128)
            s = s.masked_fill(~vis, float("-inf"))
            ref = torch.softmax(s, dim=-1) @ v[b, h // 4].float()
            err = (out[b, h, rows].float() - ref).abs()
            assert err.max().item() <= ATOL, (b, h, err.max().item())


def test_prefill_accepts_any_stride_on_an_extent_one_batch():
    """A batch of one may carry any stride on that dimension (numpy / torch give 0 after unsqueeze or
    expand); the stride addresses nothing and the result equals the contiguous call's."""
    g = load_prefill("config1_d64")
    q, k, v = _dev(g["q"]), _dev(g["k"]), _dev(g["v"])
    assert q.shape[0] == 1
    zero = [torch.as_strided(t, t.shape, (0,) + t.stride()[1:]) for t in (q, k, v)]
    kw = dict(C=g["C"], K_layout=g["K"], quota_per_head=list(g["quota"]))
    assert torch.equal(prefill.prefill_masked(*zero, **kw), prefill.prefill_masked(q, k, v, **kw))

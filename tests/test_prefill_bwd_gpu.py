"""Backward of the tcgen05 prefill-mask attention (abkv_prefill_masked_backward) on a B200: dQ, dK,
dV against the float64 gradient oracle and the reference goldens (torch autograd through the
reference's mask, tests/golden/prefillbwd_*), then the autograd function and the AttentionInterface
training path.

Tolerance: P and dS enter the tensor-core products as bf16 (as in FlexAttention's kernels) and the
outputs are bf16, so each gradient is compared relative to its largest magnitude:
max |gpu - ref| <= 1e-2 x max |ref| and mean |gpu - ref| <= 5e-4 x max |ref| (measured: <= 5e-3 and
<= 1.2e-4 on every golden case)."""
import numpy as np
import pytest
import torch

from abridgekv_b200 import prefill
from abridgekv_b200.workspace import Workspace
from oracle.mask_ref import masked_attention_grad
from tests.goldens import load_prefill_bwd, prefill_bwd_cases

pytestmark = pytest.mark.gpu
REL_MAX, REL_MEAN = 1e-2, 5e-4


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(torch.bfloat16).cuda()


def _close(name, got, ref):
    scale = np.abs(ref).max()
    err = np.abs(got - ref)
    print(f"{name}: max {err.max() / scale:.3e} mean {err.mean() / scale:.3e} (relative to max |ref| {scale:.3f})")
    assert np.isfinite(got).all(), name
    assert err.max() <= REL_MAX * scale and err.mean() <= REL_MEAN * scale, name


def _run(g, dout):
    q, k, v = _dev(g["q"]), _dev(g["k"]), _dev(g["v"])
    pl = torch.as_tensor(g["prompt_len"], device="cuda") if g["prompt_len"] is not None else None
    ws = Workspace()
    out, lse = prefill.prefill_masked(q, k, v, C=g["C"], K_layout=g["K"], quota_per_head=list(g["quota"]),
                                      prompt_len=pl, return_lse=True, workspace=ws)
    dq, dk, dv = prefill.prefill_masked_backward(q, k, v, out, _dev(dout), lse, C=g["C"], K_layout=g["K"],
                                                 quota_per_head=list(g["quota"]), prompt_len=pl, workspace=ws)
    torch.cuda.synchronize()
    assert ws.read_error() == 0
    return (q, k, v, pl), [t.float().cpu().numpy() for t in (dq, dk, dv)]


@pytest.mark.parametrize("name", prefill_bwd_cases())
def test_backward_matches_oracle_and_reference(name):
    g, dout, rows, dq_r, dk_r, dv_r = load_prefill_bwd(name)
    _, (dq, dk, dv) = _run(g, dout)
    ref = masked_attention_grad(g["q"], g["k"], g["v"], g["mask"], 1.0 / np.sqrt(g["D"]), dout)
    for label, got, r, gold in (("dq", dq, ref[0], dq_r), ("dk", dk, ref[1], dk_r), ("dv", dv, ref[2], dv_r)):
        _close(f"{name} {label} vs f64", got, r)
        _close(f"{name} {label} vs reference", got[:, :, rows], gold)


def test_autograd_function_and_attention_interface():
    """prefill_masked_attention's gradients equal prefill_masked_backward's, and the
    AttentionInterface shim takes the same path when its inputs require grad."""
    g, dout, *_ = load_prefill_bwd("c128k128_quota_prompt")
    (q, k, v, pl), direct = _run(g, dout)
    qs, ks, vs = (t.detach().clone().requires_grad_(True) for t in (q, k, v))
    out = prefill.prefill_masked_attention(qs, ks, vs, C=g["C"], K_layout=g["K"], quota_per_head=list(g["quota"]),
                                           prompt_len=pl)
    out.backward(_dev(dout))
    for t, d in zip((qs, ks, vs), direct):
        assert np.array_equal(t.grad.float().cpu().numpy(), d)
    # transformers layout: [B, S, H, D] projections viewed as [B, H, S, D]
    qt, kt, vt = (t.detach().transpose(1, 2).contiguous().transpose(1, 2).requires_grad_(True) for t in (q, k, v))
    mask = prefill.CompressMask(C=g["C"], K_layout=g["K"], quota_per_head=tuple(g["quota"]), prompt_len=pl)
    o, _ = prefill.abkv_attention_forward(None, qt, kt, vt, mask)
    o.backward(_dev(dout).transpose(1, 2))
    for t, d in zip((qt, kt, vt), direct):
        assert np.array_equal(t.grad.float().cpu().numpy(), d)


def test_forward_and_backward_from_a_fresh_thread():
    """Tensor-map encoding is a driver call: a thread that made no CUDA runtime call yet (autograd's
    device thread, a worker pool) must still get results equal to the calling thread's."""
    import threading

    g, dout, *_ = load_prefill_bwd("c256k128_g4")
    (q, k, v, pl), direct = _run(g, dout)
    box = {}

    def work():
        try:
            out, lse = prefill.prefill_masked(q, k, v, C=g["C"], K_layout=g["K"], quota_per_head=list(g["quota"]),
                                              prompt_len=pl, return_lse=True)
            box["grads"] = prefill.prefill_masked_backward(q, k, v, out, _dev(dout), lse, C=g["C"], K_layout=g["K"],
                                                           quota_per_head=list(g["quota"]), prompt_len=pl)
            torch.cuda.current_stream().synchronize()
        except Exception as e:  # reported below, in the test thread
            box["error"] = e

    t = threading.Thread(target=work)
    t.start()
    t.join()
    assert "error" not in box, box.get("error")
    for got, d in zip(box["grads"], direct):
        np.testing.assert_allclose(got.float().cpu().numpy(), d, atol=2e-3 * float(np.abs(d).max()))


def test_gradients_are_linear_in_dout():
    """A size-independent property at a larger shape than the goldens (B = 2, 4 blocks of 512 + 256
    rows, 8 / 2 heads, head_dim 128, mixed quotas, a prompt on one sequence): doubling dO (exact in
    bf16) doubles every gradient.  dK and dV accumulate in a fixed order, so they double bit for bit;
    dQ is summed by unordered fp32 reductions, so it doubles to within fp32 rounding."""
    B, H, Hkv, D, C, K, N = 2, 8, 2, 128, 512, 256, 4
    S = N * (C + K)
    g = torch.Generator(device="cuda").manual_seed(7)
    mk = lambda h: torch.randn((B, S, h, D), device="cuda", generator=g, dtype=torch.bfloat16).transpose(1, 2)
    q, k, v, dout = mk(H), mk(Hkv), mk(Hkv), mk(H)
    quotas = [256, 128, 64, 192, 256, 32, 64, 128]
    pl = torch.tensor([300, 0], dtype=torch.int32, device="cuda")
    ws = Workspace()
    out, lse = prefill.prefill_masked(q, k, v, C=C, K_layout=K, quota_per_head=quotas, prompt_len=pl,
                                      return_lse=True, workspace=ws)
    g1 = prefill.prefill_masked_backward(q, k, v, out, dout, lse, C=C, K_layout=K, quota_per_head=quotas,
                                         prompt_len=pl, workspace=ws)
    g2 = prefill.prefill_masked_backward(q, k, v, out, dout * 2, lse, C=C, K_layout=K, quota_per_head=quotas,
                                         prompt_len=pl, workspace=ws)
    torch.cuda.synchronize()
    assert ws.read_error() == 0
    dq1, dk1, dv1 = (t.float() for t in g1)
    dq2, dk2, dv2 = (t.float() for t in g2)
    assert torch.isfinite(dq1).all() and dk1.abs().max() > 0 and dv1.abs().max() > 0
    assert torch.equal(dk2, 2 * dk1)
    assert torch.equal(dv2, 2 * dv1)
    assert ((dq2 - 2 * dq1).abs().max() <= 1e-2 * dq1.abs().max()).item()

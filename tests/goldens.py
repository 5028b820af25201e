"""Loaders for the committed golden fixtures (tests/golden/*)."""
from __future__ import annotations

from pathlib import Path

import numpy as np

from oracle.bf16 import from_bits
from oracle.synth import paged_case

GOLDEN = Path(__file__).resolve().parent / "golden"


def decode_cases():
    return sorted(p.stem[len("decode_"):] for p in GOLDEN.glob("decode_*.npz"))


def load_decode(name: str):
    z = np.load(GOLDEN / f"decode_{name}.npz")
    case = paged_case(int(z["seed"]), z["seq_lens"], num_q_heads=int(z["num_q_heads"]),
                      num_kv_heads=int(z["num_kv_heads"]), head_dim=int(z["head_dim"]),
                      page=int(z["page"]))
    return case, from_bits(z["out_bits"])


def prefill_cases():
    return sorted(p.stem[len("prefill_"):] for p in GOLDEN.glob("prefill_*.npz"))


def load_prefill(name: str):
    """-> dict(case params, q, k, v, mask [B,H,S,S], rows, out_rows, lse) from the reference goldens."""
    from tests.golden.make_golden import prefill_inputs

    z = dict(np.load(GOLDEN / f"prefill_{name}.npz"))
    B, H, Hkv = int(z["B"]), int(z["H"]), int(z["Hkv"])
    S0 = int(z["N"]) * (int(z["C"]) + int(z["K"]))
    D = int(z["D"]) if "D" in z else 128
    q, k, v = prefill_inputs(int(z["seed"]), B, H, Hkv, S0, D)
    mask = np.unpackbits(z["mask_bits"])[: B * H * S0 * S0].reshape(B, H, S0, S0).astype(bool)
    pl = z["prompt_len"] if z["prompt_len"].size else None
    return dict(B=B, H=H, Hkv=Hkv, S0=S0, D=D, C=int(z["C"]), K=int(z["K"]), quota=z["quota_per_head"], prompt_len=pl,
                q=q, k=k, v=v, mask=mask, rows=z["rows"], out_rows=z["out_rows"], lse=z["lse"])


def codestep_cases():
    return sorted(p.stem[len("codestep_"):] for p in GOLDEN.glob("codestep_*.npz"))


def load_codestep(name: str):
    """-> (case, qrows [T,Hq,D], K, quotas per kv head, reference output [T,Hq,D],
    exclusion ranges [R,2] or None)."""
    from oracle.bf16 import round_bf16

    z = np.load(GOLDEN / f"codestep_{name}.npz")
    K = int(z["K"])
    case = paged_case(int(z["seed"]), z["seq_lens"], num_q_heads=int(z["num_q_heads"]),
                      num_kv_heads=int(z["num_kv_heads"]), head_dim=128, page=int(z["page"]))
    rng = np.random.default_rng(int(z["seed"]) + 1000)
    qrows = round_bf16(rng.standard_normal((len(z["seq_lens"]) * K, int(z["num_q_heads"]), 128)).astype(np.float32))
    excl = z["excluded"] if "excluded" in z.files and len(z["excluded"]) else None
    return case, qrows, K, z["quotas"], from_bits(z["out_bits"]), excl


def packed_cases():
    return sorted(p.stem[len("packed_"):] for p in GOLDEN.glob("packed_*.npz"))


def load_packed(name: str):
    """-> (main case, side pages [sum(counts), 2, slots, D], counts, quotas per kv head, k_max,
    reference output [B, Hq, D])."""
    from tests.golden.make_golden import packed_side_pages

    z = np.load(GOLDEN / f"packed_{name}.npz")
    case = paged_case(int(z["seed"]), z["seq_lens"], num_q_heads=int(z["num_q_heads"]),
                      num_kv_heads=int(z["num_kv_heads"]), head_dim=int(z["head_dim"]), page=int(z["page"]))
    side = packed_side_pages(int(z["seed"]), z["counts"], int(z["quotas"].sum()), int(z["head_dim"]))
    return case, side, z["counts"], z["quotas"], int(z["k_max"]), from_bits(z["out_bits"])


def prefill_bwd_cases():
    return sorted(p.stem[len("prefillbwd_"):] for p in GOLDEN.glob("prefillbwd_*.npz"))


def load_prefill_bwd(name: str):
    """-> (load_prefill(name) dict, dout [B,H,S,D], rows, dq_rows, dk_rows, dv_rows) of the reference goldens."""
    from tests.golden.make_golden import prefill_dout

    g = load_prefill(name)
    z = np.load(GOLDEN / f"prefillbwd_{name}.npz")
    z0 = np.load(GOLDEN / f"prefill_{name}.npz")
    dout = prefill_dout(int(z0["seed"]), g["B"], g["H"], g["S0"], g["D"])
    return g, dout, z["rows"], z["dq_rows"], z["dk_rows"], z["dv_rows"]


def causal_cases():
    return sorted(p.stem[len("causal_"):] for p in GOLDEN.glob("causal_*.npz"))


def load_causal(name: str):
    """-> (case, qrows [T,Hq,D], query_start [R+1], rows kept, reference output at those rows)."""
    from tests.golden.make_golden import causal_query_rows

    z = np.load(GOLDEN / f"causal_{name}.npz")
    case = paged_case(int(z["seed"]), z["seq_lens"], num_q_heads=int(z["num_q_heads"]),
                      num_kv_heads=int(z["num_kv_heads"]), head_dim=128, page=int(z["page"]))
    qlens = z["query_lens"].astype(np.int64)
    qstart = np.concatenate([[0], np.cumsum(qlens)]).astype(np.int32)
    qrows = causal_query_rows(int(z["seed"]), int(qlens.sum()), int(z["num_q_heads"]))
    return case, qrows, qstart, z["rows"], from_bits(z["out_bits"])


def qmask_cases():
    return sorted(p.stem[len("qmask_"):] for p in GOLDEN.glob("qmask_*.npz"))


def load_qmask(name: str):
    """-> (K, quotas, requests [(query_len, seq_len, spans, excluded)], {quota: reference ragged mask})
    of the reference's build_layer_quota_masks (tests/golden/qmask_*.npz)."""
    z = np.load(GOLDEN / f"qmask_{name}.npz")
    K = int(z["K"])
    reqs = []
    for q, s_, own, ex in zip(z["query_lens"], z["seq_lens"], z["own_span"], z["excluded"]):
        q, s_ = int(q), int(s_)
        reqs.append((q, s_, [(s_ - K, s_)] if own else [], (int(ex[0]), int(ex[1])) if ex[1] > ex[0] else None))
    masks = {int(q): np.unpackbits(z[f"mask_{int(q)}"])[: int(z[f"size_{int(q)}"])].astype(bool)
             for q in z["quotas"]}
    return K, [int(q) for q in z["quotas"]], reqs, masks


def load_config1():
    """BASELINE config 1 through the reference's own CompressLM.forward and CompressGen
    (tests/golden/config1_reference.npz, make_golden.py --only config1) -> dict with
    prefill[l] = (q_rows [H, n, D], k [Hkv, S0, D], v [Hkv, S0, D], out_rows [n, H, D] fp32) and the row
    indices; decode[l] = (k_store [Hkv, T, D], v_store, {step: (q [H, D], cols [m], out [H, D] fp32)})."""
    z = np.load(GOLDEN / "config1_reference.npz")
    prefill = {l: (from_bits(z[f"prefill{l}_q_bits"]), from_bits(z[f"prefill{l}_k_bits"]),
                   from_bits(z[f"prefill{l}_v_bits"]), z[f"prefill{l}_out"]) for l in range(2)}
    decode = {}
    for l in range(2):
        steps = {int(s): (from_bits(z[f"decode{l}_s{int(s)}_q_bits"]), z[f"decode{l}_s{int(s)}_cols"],
                          z[f"decode{l}_s{int(s)}_out"]) for s in z["decode_steps"]}
        decode[l] = (from_bits(z[f"decode{l}_k_bits"]), from_bits(z[f"decode{l}_v_bits"]), steps)
    return {"C": 512, "K": 128, "N": 4, "quotas": (128, 64), "rows": z["prefill_rows"], "prefill": prefill,
            "decode": decode, "tokens": z["tokens"]}


def config1_paged(decode_layer, page=16, seed=0):
    """The decode steps of one config-1 layer as a paged batch: sequence i = step i's visible store
    columns (in order) laid into pages of a shuffled pool.  -> (q [B, H, D], kv [pages, 2, page, Hkv, D],
    block_table [B, max_pages] int32, seq_lens [B] int32, reference out [B, H, D], steps)."""
    k_store, v_store, steps = decode_layer
    keys = sorted(steps)
    rng = np.random.default_rng(seed)
    lens = [len(steps[s][1]) for s in keys]
    pages = [(n + page - 1) // page for n in lens]
    total = sum(pages) + 1
    perm = 1 + rng.permutation(total - 1)
    Hkv, _, D = k_store.shape
    kv = np.zeros((total, 2, page, Hkv, D), dtype=np.float32)
    bt = np.zeros((len(keys), max(pages)), dtype=np.int32)
    at = 0
    for i, s in enumerate(keys):
        cols = steps[s][1]
        ids = perm[at:at + pages[i]]
        at += pages[i]
        bt[i, :pages[i]] = ids
        for r, c in enumerate(cols):
            kv[ids[r // page], 0, r % page] = k_store[:, c]
            kv[ids[r // page], 1, r % page] = v_store[:, c]
    q = np.stack([steps[s][0] for s in keys])
    out = np.stack([steps[s][2] for s in keys])
    return q, kv, bt, np.asarray(lens, np.int32), out, keys


def packedstep_cases():
    return sorted(p.stem[len("packedstep_"):] for p in GOLDEN.glob("packedstep_*.npz"))


def load_packedstep(name: str):
    """-> dict(case, qrows [T,Hq,D], qstart [R+1], side pages, counts, quotas, k_max, causal, excluded or
    None, rows kept, reference output at those rows) of tests/golden/packedstep_<name>.npz."""
    from tests.golden.make_golden import causal_query_rows, packed_side_pages

    z = np.load(GOLDEN / f"packedstep_{name}.npz")
    case = paged_case(int(z["seed"]), z["seq_lens"], num_q_heads=int(z["num_q_heads"]),
                      num_kv_heads=int(z["num_kv_heads"]), head_dim=128, page=int(z["page"]))
    qlens = z["query_lens"].astype(np.int64)
    qstart = np.concatenate([[0], np.cumsum(qlens)]).astype(np.int32)
    qrows = causal_query_rows(int(z["seed"]), int(qlens.sum()), int(z["num_q_heads"]))
    side = packed_side_pages(int(z["seed"]), z["counts"], int(z["quotas"].sum()), 128)
    excl = z["excluded"] if len(z["excluded"]) else None
    return dict(case=case, qrows=qrows, qstart=qstart, side=side, counts=z["counts"], quotas=z["quotas"],
                k_max=int(z["k_max"]), causal=bool(z["causal"]), excluded=excl, rows=z["rows"],
                ref=from_bits(z["out_bits"]))

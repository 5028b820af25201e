"""Secondary benchmarks (one JSON line each); the headline decode line is bench.py.

    python benchmarks.py prefill   [--layers 36] [--steps 3] [--flex]
    python benchmarks.py compaction [--steps 5]
    python benchmarks.py codestep   [--layers 36] [--steps 3]
    python benchmarks.py packed     [--steps 20]
    python benchmarks.py kvshard    [--kv-heads 1] [--seqs 256] [--chunk-tokens 0]
    python benchmarks.py codestep_compact [--steps 20]
    python benchmarks.py flashinfer [--steps 10]

prefill    BASELINE config 4: B=16 sequences of 16 blocks x (512 content + 256 code rows)
           = 12,288 rows, Qwen3-4B attention (32 q / 8 kv heads, head_dim 128), per-layer
           quotas from sched_trunc_perlayer_mean128, prompt_len 0, bf16 N(0,1) Q/K/V.  One
           step = all layers (one abkv_prefill_masked launch each).  Algorithmic FLOPs =
           4 x head_dim per visible (query, key) pair per head.  With --flex the same step
           is also timed with torch FlexAttention compiled on this GPU (the reference's
           prefill kernel: compress_forward.py:1229 through transformers' flex path) using
           the reference's mask formula.
compaction BASELINE config 4's block compaction for all 16 sequences and 36 layers
           (12 physical tensors shared by 3 quota groups): finish one block per sequence,
           execute the planned copy ops; algorithmic bytes = 2 x rows moved x 4 KiB per layer.
codestep   the code step at a block boundary on BASELINE config 2's caches: 64 requests,
           36 layers with per-layer quotas, each request's cache = its config-2 rows + the
           K=256 freshly written code rows; 256 code queries per request (32 q / 8 kv heads,
           head_dim 128).  One step = all layers (one abkv_code_step_attention launch each).
           Algorithmic FLOPs = 4 x head_dim x visible keys per query per head.
packed     decode with per-head code quotas in packed sidecar pages: config 2's geometry
           (64 requests, 36 layers, 256-token prompt + tail U[0,511] in the paged main
           cache, 31 compressed blocks) with per-KV-head quotas 256/128/64/64/192/64/128/128
           (mean 128, as config 2's per-layer mean): 31 sidecar pages per request and layer.
           Algorithmic bytes = every key/value row read once + Q/O.
kvshard    one GPU's share of BASELINE config 5 under KV-head sharding: --kv-heads of the 8
           KV heads (with their 4 query heads each) of --seqs sequences, 36 layers of 128-row
           quotas over a 32K-token generation, one decode launch over all layers per step.
           --chunk-tokens 0 is the automatic split-KV chunk.  Algorithmic bytes = every kept
           key/value row of the shard read once + Q/O.
codestep_compact
           one layer of the code step at a block boundary (64 requests, 3-5K cache rows + K=256
           code rows, 32 q / 8 kv heads, quota 128) followed by each request's finished-block
           compaction (its first 128 code rows moved over the start of its last content block):
           code step alone, code step + the separate executor (abkv_compact), and the fused
           abkv_code_step_attention_compact, each from the host call to completion.
flashinfer BASELINE config 2's decode step through FlashInfer's paged decode (the reference's
           production decode library) on the same caches, against abkv_decode.
"""
from __future__ import annotations

import argparse
import json
import math
import time

import numpy as np
import torch

from abridgekv_b200.workloads import SCHEDULE_PERLAYER_MEAN128


def visible_pairs(N: int, C: int, K: int, quota: int, prompt_len: int = 0) -> int:
    """Visible (query, key) pairs of one (sequence, head) under _arith_mask_mod with prompt_len 0."""
    assert prompt_len == 0
    tot = 0
    for qb in range(N):
        tot += C * (C + 1) // 2 + C * qb * quota          # content rows: causal own block + earlier codes
        tot += K * (C + quota + qb * quota)                # code rows: own content + own codes + earlier
    return tot


def _peaks() -> dict:
    from pathlib import Path

    p = Path(__file__).resolve().parent / "MEASURED_PEAKS.json"
    try:
        return json.loads(p.read_text())
    except Exception:
        return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0, "fallback": True}


def bench_prefill(args) -> dict:
    from abridgekv_b200 import prefill

    B, H, Hkv, D, C, K, N = 16, 32, 8, 128, 512, 256, 16
    S0 = N * (C + K)
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(0)
    q = torch.randn((B, S0, H, D), device=dev, generator=gen, dtype=torch.bfloat16).transpose(1, 2)
    k = torch.randn((B, S0, Hkv, D), device=dev, generator=gen, dtype=torch.bfloat16).transpose(1, 2)
    v = torch.randn((B, S0, Hkv, D), device=dev, generator=gen, dtype=torch.bfloat16).transpose(1, 2)
    out = torch.empty((B, S0, H, D), device=dev, dtype=torch.bfloat16).transpose(1, 2)
    quotas = SCHEDULE_PERLAYER_MEAN128[: args.layers]
    flops = sum(4 * D * visible_pairs(N, C, K, qq) * B * H for qq in quotas)

    def step():
        for qq in quotas:
            prefill.prefill_masked(q, k, v, C=C, K_layout=K, quota_per_head=[qq] * H, out=out)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    pk = _peaks()
    tflops = flops / (ms / 1e3) / 1e12
    line = {
        "metric": "pause-token prefill attention TFLOP/s (config 4)", "value": tflops, "unit": "TFLOP/s",
        "ms_per_step": ms, "layers": len(quotas), "algorithmic_tflop_per_step": flops / 1e12,
        "roofline": {"bound": "tensor", "achieved": tflops, "peak": pk.get("bf16_tflops_sustained"),
                     "peak_kind": "measured sustained cuBLAS bf16 (MEASURED_PEAKS.json)",
                     "frac": tflops / pk.get("bf16_tflops_sustained", 1400.0)},
        "config": {"B": B, "S0": S0, "heads": f"{H}/{Hkv}", "C": C, "K_layout": K, "quotas": "per layer",
                   "prompt_len": 0},
    }
    if args.flex:
        line["flex"] = bench_flex(q, k, v, quotas, C, K, N, args, flops)
        line["speedup_vs_flex"] = line["flex"]["ms_per_step"] / ms
        # parity on one layer: our kernel vs compiled FlexAttention on the same inputs
        line["flex"]["max_abs_diff_layer0"] = line["flex"].pop("_diff")
    return line


def bench_prefill_bwd(args) -> dict:
    """Backward of the config-4 prefill (36 layers at their quotas): abkv_prefill_masked_backward
    timed alone (the forward's output and log-sum-exp computed beforehand), and forward + backward.
    Algorithmic work: 10 x D FLOP per visible (query, key) pair per head (S recomputed, dP, dV, dK, dQ)."""
    from abridgekv_b200 import prefill

    B, H, Hkv, D, C, K, N = getattr(args, "batch", 16), 32, 8, 128, 512, 256, 16
    S0 = N * (C + K)
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(0)
    q = torch.randn((B, S0, H, D), device=dev, generator=gen, dtype=torch.bfloat16).transpose(1, 2)
    k = torch.randn((B, S0, Hkv, D), device=dev, generator=gen, dtype=torch.bfloat16).transpose(1, 2)
    v = torch.randn((B, S0, Hkv, D), device=dev, generator=gen, dtype=torch.bfloat16).transpose(1, 2)
    dout = torch.randn((B, S0, H, D), device=dev, generator=gen, dtype=torch.bfloat16).transpose(1, 2)
    quotas = SCHEDULE_PERLAYER_MEAN128[: args.layers]
    fwd = {}
    for qq in sorted(set(quotas)):
        fwd[qq] = prefill.prefill_masked(q, k, v, C=C, K_layout=K, quota_per_head=[qq] * H, return_lse=True)
    pairs = sum(visible_pairs(N, C, K, qq) for qq in quotas) * B * H
    flops_bwd, flops_fwd = 10.0 * D * pairs, 4.0 * D * pairs

    def bwd_step():
        for qq in quotas:
            out, lse = fwd[qq]
            prefill.prefill_masked_backward(q, k, v, out, dout, lse, C=C, K_layout=K, quota_per_head=[qq] * H)

    def train_step():
        for qq in quotas:
            out, lse = prefill.prefill_masked(q, k, v, C=C, K_layout=K, quota_per_head=[qq] * H, return_lse=True)
            prefill.prefill_masked_backward(q, k, v, out, dout, lse, C=C, K_layout=K, quota_per_head=[qq] * H)

    def timed(fn, steps):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    ms = timed(bwd_step, args.steps)
    ms_train = timed(train_step, max(1, args.steps // 2))
    pk = _peaks()
    tflops = flops_bwd / (ms / 1e3) / 1e12
    line = {
        "metric": "pause-token prefill attention backward TFLOP/s (config 4)", "value": tflops, "unit": "TFLOP/s",
        "ms_per_step": ms, "layers": len(quotas), "algorithmic_tflop_per_step": flops_bwd / 1e12,
        "forward_plus_backward_ms": ms_train,
        "forward_plus_backward_tflops": (flops_fwd + flops_bwd) / (ms_train / 1e3) / 1e12,
        "roofline": {"bound": "tensor", "achieved": tflops, "peak": pk.get("bf16_tflops_sustained"),
                     "peak_kind": "measured sustained cuBLAS bf16 (MEASURED_PEAKS.json)",
                     "frac": tflops / pk.get("bf16_tflops_sustained", 1400.0)},
        "config": {"B": B, "S0": S0, "heads": f"{H}/{Hkv}", "C": C, "K_layout": K, "quotas": "per layer",
                   "prompt_len": 0},
    }
    if args.flex:
        line["flex"] = bench_flex_train(q, k, v, dout, quotas, C, K, args, flops_fwd + flops_bwd)
        line["train_speedup_vs_flex"] = line["flex"]["forward_plus_backward_ms"] / ms_train
    return line


def bench_flex_train(q, k, v, dout, quotas, C, K, args, flops) -> dict:
    """Compiled FlexAttention forward + backward (the reference's training path) on the same inputs."""
    from torch.nn.attention.flex_attention import create_block_mask, flex_attention

    B, H, S0, D = q.shape
    per = C + K
    masks = {}
    for qq in sorted(set(quotas)):
        def mm(b, h, qi, kv, qq=qq):
            qb, qw = qi // per, qi % per
            kb, kw = kv // per, kv % per
            kc = kw < C
            same = kb == qb
            vis = (kc & same) | (~kc & (kb < qb))
            vis = (kv <= qi) & vis
            vis = vis | ((qw >= C) & ~kc & same)
            return vis & (kc | ((kw - C) < qq))
        masks[qq] = create_block_mask(mm, B=None, H=None, Q_LEN=S0, KV_LEN=S0, device="cuda", _compile=True)
    fa = torch.compile(flex_attention, dynamic=False)
    scale = 1.0 / math.sqrt(D)
    qg, kg, vg = (t.detach().requires_grad_(True) for t in (q, k, v))

    def step():
        for qq in quotas:
            out = fa(qg, kg, vg, block_mask=masks[qq], scale=scale, enable_gqa=True)
            out.backward(dout)
            qg.grad = kg.grad = vg.grad = None

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    steps = max(1, args.steps // 2)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    return {"forward_plus_backward_ms": ms, "tflops": flops / (ms / 1e3) / 1e12}


def bench_flex(q, k, v, quotas, C, K, N, args, flops) -> dict:
    from torch.nn.attention.flex_attention import create_block_mask, flex_attention

    from abridgekv_b200 import prefill

    B, H, S0, D = q.shape
    per = C + K
    masks = {}
    for qq in sorted(set(quotas)):
        def mm(b, h, qi, kv, qq=qq):
            qb, qw = qi // per, qi % per
            kb, kw = kv // per, kv % per
            kc = kw < C
            same = kb == qb
            vis = (kc & same) | (~kc & (kb < qb))
            vis = (kv <= qi) & vis
            vis = vis | ((qw >= C) & ~kc & same)
            return vis & (kc | ((kw - C) < qq))
        masks[qq] = create_block_mask(mm, B=None, H=None, Q_LEN=S0, KV_LEN=S0, device="cuda", _compile=True)
    fa = torch.compile(flex_attention, dynamic=False)
    opts = {"BLOCK_M": 128, "BLOCK_N": 64, "num_warps": 8}  # the reference's launch/env.sh options
    scale = 1.0 / math.sqrt(D)

    def step():
        for qq in quotas:
            fa(q, k, v, block_mask=masks[qq], scale=scale, enable_gqa=True, kernel_options=opts)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    ref = fa(q, k, v, block_mask=masks[quotas[0]], scale=scale, enable_gqa=True, kernel_options=opts)
    ours = prefill.prefill_masked(q, k, v, C=C, K_layout=K, quota_per_head=[quotas[0]] * H)
    diff = (ref.float() - ours.float()).abs().max().item()
    return {"ms_per_step": ms, "tflops": flops / (ms / 1e3) / 1e12, "kernel_options": opts, "_diff": diff}


def _torch_kv_copy_group(all_ops, layer_caches) -> None:
    """The reference's GPU executor for one batch (gpu_model_runner.py:1194-1220): upload the ops,
    then per layer tensor gather every source row with an index op and scatter it with another."""
    ops = torch.tensor(all_ops, dtype=torch.long, device=layer_caches[0].device)
    sb, so, db, do = ops[:, 0], ops[:, 1], ops[:, 2], ops[:, 3]
    for kv in layer_caches:
        src = kv[sb, :, so].clone()
        kv[db, :, do] = src


def _torch_kv_copy_operations(kv_copy_operations, caches_by_group) -> None:
    for g, layer_caches in enumerate(caches_by_group):
        per_req = [ops[g] for ops in kv_copy_operations.values() if g < len(ops)]
        for b in range(max((len(x) for x in per_req), default=0)):
            merged = [op for x in per_req if b < len(x) for op in x[b]]
            if merged:
                _torch_kv_copy_group(merged, layer_caches)


def bench_compaction(args) -> dict:
    """Per block finish: the planner (host C++) and the executor (one abkv_compact per group).
    host_ms = host time of the executor call (op flattening, chain planning, uploads, launches);
    device_ms = GPU time of its copies and kernels, measured behind a sleep kernel long enough that
    the host has enqueued everything before the GPU reaches the first event; the reference's torch
    executor (index gather + index scatter per layer tensor, ops uploaded per batch) is timed on the
    same ops and caches."""
    from abridgekv_b200 import compaction
    from abridgekv_b200.planner import BlockPlanner
    from abridgekv_b200.workspace import Workspace

    C, K, page = 512, 256, 16
    quotas = (256, 128, 64)
    G = len(quotas)
    B, L = 16, 36
    per = C + K
    blocks = args.blocks
    n_tensors = L // G
    nb = 1 + B * (blocks * per // page) * G + 64
    dev = torch.device("cuda")
    caches = [torch.zeros((nb, 2, page, 8, 128), device=dev, dtype=torch.bfloat16) for _ in range(n_tensors)]
    planner = BlockPlanner(nb, page, G)
    for b in range(B):
        planner.add_request(b)
    ws = Workspace(dev)
    rec = []
    sleep_cycles = int(2e8)  # ~0.1 s at 1.9 GHz
    launched = []
    real_compact = compaction._compact

    def counting_compact(layer_caches, batches, workspace, stream):
        launched.append(list(batches))
        real_compact(layer_caches, batches, workspace, stream)

    compaction._compact = counting_compact
    for blk in range(blocks):
        t_plan = time.perf_counter()
        for b in range(B):
            n = (blk + 1) * per
            assert planner.allocate_slots(b, n)
            planner.set_num_computed_tokens(b, n)
            planner.finish_block(b, (blk * per, blk * per + C), (blk * per + C, (blk + 1) * per), quotas, K)
        ops, _ = planner.take_pending()
        plan_ms = (time.perf_counter() - t_plan) * 1e3
        rows = sum(len(x) for per_g in ops.values() for bl in per_g for x in bl)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
        torch.cuda.synchronize()
        ev[0].record()
        torch.cuda._sleep(sleep_cycles)
        ev[1].record()
        t0 = time.perf_counter()
        compaction.execute_kv_copy_operations(ops, [caches] * G, workspace=ws)
        host_ms = (time.perf_counter() - t0) * 1e3
        # kernel launches of that call: one chain kernel per non-empty batch of each abkv_compact call
        # (a batch with a cycle or a duplicate would take two; config 4's batches have neither)
        launches = sum(1 for batches in launched for b in batches if len(b))
        launched.clear()
        ev[2].record()
        torch.cuda._sleep(sleep_cycles)
        ev[3].record()
        _torch_kv_copy_operations(ops, [caches] * G)
        ev[4].record()
        torch.cuda.synchronize()
        sleep_ms = ev[0].elapsed_time(ev[1])
        # block 0 includes one-time set-up and is not reported
        assert blk == 0 or host_ms < sleep_ms, "the sleep kernel must outlast the host enqueue"
        rec.append({"rows": rows, "plan_ms": plan_ms, "host_ms": host_ms, "device_ms": ev[1].elapsed_time(ev[2]),
                     "torch_ms": ev[3].elapsed_time(ev[4]), "launches": launches,
                     "bytes": rows * n_tensors * 2 * 2 * 8 * 128 * 2})  # rows x tensors x (K,V) x R+W x bytes
    compaction._compact = real_compact
    assert ws.read_error() == 0
    steady = rec[1:] or rec
    mean = lambda k: float(np.mean([r[k] for r in steady]))  # noqa: E731
    dev_ms, byt = mean("device_ms"), mean("bytes")
    gbs = byt / (dev_ms / 1e3) / 1e9
    pk = _peaks()
    return {"metric": "block compaction executor GB/s (config 4, 16 seqs x 36 layers)", "value": gbs,
            "unit": "GB/s", "bytes_per_block_finish": byt, "rows_per_block_finish": mean("rows"),
            "device_ms_per_block_finish": dev_ms, "host_ms_executor_call": mean("host_ms"),
            "host_ms_planner": mean("plan_ms"),
            "reference_torch_executor_ms": mean("torch_ms"),
            "speedup_vs_reference_torch_executor": mean("torch_ms") / dev_ms,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": pk.get("hbm_gbs"), "unit": "GB/s",
                         "frac": gbs / pk.get("hbm_gbs", 6650.0)},
            "gpu_launches": int(sum(r["launches"] for r in steady)),
            "config": {"sequences": B, "layers": L, "quota_groups": list(quotas), "physical_tensors": n_tensors,
                       "blocks_finished": blocks, "note": "mean over block finishes 2.."}}


def bench_codestep(args) -> dict:
    from abridgekv_b200 import codestep
    from abridgekv_b200.workloads import QWEN3_4B, build_decode_workload, config2_rows

    K = 256
    rows = {q: r + K for q, r in config2_rows(64, 0).items()}
    quotas = SCHEDULE_PERLAYER_MEAN128[: args.layers]
    wl = build_decode_workload("codestep", quotas, rows, num_q_heads=QWEN3_4B["num_q_heads"],
                               num_kv_heads=QWEN3_4B["num_kv_heads"], head_dim=QWEN3_4B["head_dim"])
    R, Hq, Hkv, D = wl.num_seqs, wl.num_q_heads, wl.num_kv_heads, wl.head_dim
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(1)
    q = torch.randn((R * K, Hq, D), device=dev, generator=gen, dtype=torch.bfloat16)
    out = torch.empty_like(q)
    qs = (torch.arange(R + 1, device=dev) * K).to(torch.int32)
    flops = sum(4.0 * D * K * Hq * float((wl.rows[l] - K + qq).sum()) for l, qq in enumerate(quotas))
    kv_bytes = float(wl.rows.sum()) * Hkv * D * 2 * 2

    def step():
        for l, qq in enumerate(quotas):
            codestep.code_step_attention(q, wl.kv_caches[l], wl.block_tables[l], wl.seq_lens[l], qs,
                                         quota_per_kv_head=[qq] * Hkv, k_max=K, out=out)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    pk = _peaks()
    tflops = flops / (ms / 1e3) / 1e12
    return {"metric": "code-step attention TFLOP/s (config 2 caches + 256 code rows)", "value": tflops,
            "unit": "TFLOP/s", "ms_per_step": ms, "layers": len(quotas), "algorithmic_tflop_per_step": flops / 1e12,
            "kv_gb_per_step": kv_bytes / 1e9,
            "roofline": {"bound": "tensor", "achieved": tflops, "peak": pk.get("bf16_tflops_sustained"),
                         "peak_kind": "measured sustained cuBLAS bf16 (MEASURED_PEAKS.json)",
                         "frac": tflops / pk.get("bf16_tflops_sustained", 1400.0)},
            "config": {"requests": R, "K": K, "heads": f"{Hq}/{Hkv}", "page": wl.page,
                       "mean_seq_len": float(wl.rows.mean())}}


def bench_packed(args) -> dict:
    from abridgekv_b200.sidecar import PackedKVLayout, SidecarPool, packed_decode
    from abridgekv_b200.workloads import BLOCK_C, build_decode_workload

    B, L, Hq, Hkv, D, blocks = 64, 36, 32, 8, 128, 31
    quotas = [256, 128, 64, 64, 192, 64, 128, 128]
    rng = np.random.default_rng(0)
    main_rows = 256 + rng.integers(0, BLOCK_C, size=B)
    wl = build_decode_workload("packed-main", (128,) * L, {128: main_rows}, num_q_heads=Hq, num_kv_heads=Hkv,
                               head_dim=D)
    layout = PackedKVLayout.from_schedule([quotas] * L, num_layers=L, num_kv_heads=Hkv, k_max=256)
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(2)
    pools = []
    for l in range(L):
        pool = SidecarPool(layout, l, capacity=B * blocks, num_requests=B, max_pages=blocks, head_dim=D)
        pool.pages.normal_(generator=gen)
        perm = torch.randperm(B * blocks, generator=torch.Generator().manual_seed(l)).to(torch.int32)
        pool.page_table.copy_(perm.view(B, blocks).to(dev))
        pool.page_count.fill_(blocks)
        pools.append(pool)
    outs = [torch.empty_like(q) for q in wl.queries]

    def step():
        packed_decode(wl.queries, wl.kv_caches, wl.block_tables, wl.seq_lens, pools, outputs=outs)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    side_bytes = L * B * blocks * sum(quotas) * D * 2 * 2
    alg = side_bytes + wl.kv_bytes + wl.qo_bytes
    gbs = alg / (ms / 1e3) / 1e9
    pk = _peaks()
    return {"metric": "packed per-head-quota decode tokens/s (config 2 geometry)", "value": B / (ms / 1e3),
            "unit": "tokens/s", "ms_per_step": ms, "algorithmic_gb_per_step": alg / 1e9,
            "sidecar_gb_per_step": side_bytes / 1e9,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": pk.get("hbm_gbs"), "unit": "GB/s",
                         "frac": gbs / pk.get("hbm_gbs", 6650.0)},
            "config": {"requests": B, "layers": L, "kv_head_quotas": quotas, "sidecar_pages_per_request": blocks,
                       "main_rows": "256 + U[0,511]"}}


def bench_hostdecode(args) -> dict:
    """Config-2 decode end to end through HostDecode (pinned host queries, tables and outputs) for
    several launch groupings of the 36 layers, in alternating rounds on one GPU (tokens/s)."""
    from abridgekv_b200.hostdecode import HostDecode, split_layers
    from abridgekv_b200.workloads import qwen3_decode_workload
    from abridgekv_b200.workspace import Workspace

    dev = torch.device("cuda", 0)
    wl = qwen3_decode_workload(2, num_seqs=64, device=dev, seed=0)
    ws = Workspace(dev)
    q_host = [q.cpu().pin_memory() for q in wl.queries]
    bt_host = {id(t): t.cpu().pin_memory() for t in wl.block_tables}
    sl_host = {id(t): t.cpu().pin_memory() for t in wl.seq_lens}
    out_host = [torch.empty(q.shape, dtype=q.dtype).pin_memory() for q in wl.queries]
    bts = [bt_host[id(t)] for t in wl.block_tables]
    sls = [sl_host[id(t)] for t in wl.seq_lens]
    L = wl.num_layers
    groupings = {"default": split_layers(L), "edge1": split_layers(L, edge=1),
                 "max32": split_layers(L, max_group=32), "max32_edge3": split_layers(L, max_group=32, edge=3)}
    runners = {k: HostDecode(wl.kv_caches, groups=g, max_pages_per_seq=wl.max_pages, workspace=ws)
               for k, g in groupings.items()}
    stream = torch.cuda.current_stream(dev)
    res = {k: [] for k in groupings}
    for _ in range(3):
        for k, hd in runners.items():
            for _ in range(args.warmup):
                hd.run(q_host, bts, sls, out_host)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.steps):
                hd.run(q_host, bts, sls, out_host)
            e1.record(stream)
            torch.cuda.synchronize()
            res[k].append(round(wl.num_seqs * args.steps / (e0.elapsed_time(e1) / 1e3)))
    if ws.read_error():
        raise RuntimeError(f"device error flag {ws.read_error():#x}")
    return {"metric": "config-2 decode end to end through HostDecode, per launch grouping", "unit": "tokens/s",
            "rounds": res, "groups": {k: [len(g) for g in v] for k, v in groupings.items()},
            "config": {"sequences": wl.num_seqs, "layers": L, "steps": args.steps, "warmup": args.warmup}}


def bench_kvshard(args) -> dict:
    from abridgekv_b200 import decode
    from abridgekv_b200.workloads import qwen3_decode_workload
    from abridgekv_b200.workspace import Workspace

    wl = qwen3_decode_workload(5, num_seqs=args.seqs, kv_heads=slice(0, args.kv_heads))
    ws = Workspace()
    outs = [torch.empty_like(q) for q in wl.queries]

    def step():
        decode.paged_decode(wl.queries, wl.kv_caches, wl.block_tables, wl.seq_lens, outputs=outs,
                            max_pages_per_seq=wl.max_pages, chunk_tokens=args.chunk_tokens, workspace=ws)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    if ws.read_error():
        raise RuntimeError(f"decode device error flag {ws.read_error():#x}")
    ms = e0.elapsed_time(e1) / args.steps
    alg = wl.kv_bytes + wl.qo_bytes
    gbs = alg / (ms / 1e3) / 1e9
    pk = _peaks()
    return {"metric": "config-5 KV-head shard decode tokens/s (one GPU's share)", "value": args.seqs / (ms / 1e3),
            "unit": "tokens/s", "ms_per_step": ms, "algorithmic_gb_per_step": alg / 1e9,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": pk.get("hbm_gbs"), "unit": "GB/s",
                         "frac": gbs / pk.get("hbm_gbs", 6650.0)},
            "config": {"kv_heads": args.kv_heads, "seqs": args.seqs, "layers": wl.num_layers,
                       "chunk_tokens": args.chunk_tokens or "auto"}}


def bench_codestep_compact(args) -> dict:
    from abridgekv_b200 import codestep, compaction
    from abridgekv_b200.workspace import Workspace

    g = torch.Generator().manual_seed(5)
    R, K, C, Hq, Hkv, D, page, qk = 64, 256, 512, 32, 8, 128, 16, 128
    quotas = [qk] * Hkv
    lens = torch.randint(3000, 5000, (R,), generator=g) + K
    pages = (lens + page - 1) // page
    nb = int(pages.sum()) + 1
    dev = torch.device("cuda")
    kv = torch.randn((nb, 2, page, Hkv, D), device=dev, dtype=torch.bfloat16)
    perm = torch.randperm(nb - 1, generator=g) + 1
    bt = torch.zeros((R, int(pages.max())), dtype=torch.int32)
    o = 0
    for r in range(R):
        bt[r, :pages[r]] = perm[o:o + pages[r]]
        o += int(pages[r])
    ops, off = [], [0]
    for r in range(R):
        L = int(lens[r])
        for j in range(qk):
            sr, dr = L - K + j, L - K - C + j
            ops.append((int(bt[r, sr // page]), sr % page, int(bt[r, dr // page]), dr % page))
        off.append(len(ops))
    ops_arr = np.asarray(ops, dtype=np.int32)
    btd, sl = bt.to(dev), lens.to(torch.int32).to(dev)
    q = torch.randn((R * K, Hq, D), device=dev, dtype=torch.bfloat16)
    qs = (torch.arange(R + 1) * K).to(torch.int32).to(dev)
    out = torch.empty_like(q)
    ws = Workspace()
    kw = dict(quota_per_kv_head=quotas, k_max=K, workspace=ws, out=out)

    def alone():
        codestep.code_step_attention(q, kv, btd, sl, qs, **kw)

    def separate():
        codestep.code_step_attention(q, kv, btd, sl, qs, **kw)
        compaction.execute_kv_copy_group(compaction.CopyOps(ops_arr), [kv], workspace=ws)

    def fused():
        codestep.code_step_attention_compact(q, kv, btd, sl, qs, ops=ops_arr, op_offsets=off, replay_tail=0,
                                             **kw)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / args.steps

    res = {name: [] for name in ("code_step", "code_step_then_executor", "fused")}
    for _ in range(2):  # the copies are idempotent: every call moves the same rows
        res["code_step"].append(round(timed(alone), 4))
        res["code_step_then_executor"].append(round(timed(separate), 4))
        res["fused"].append(round(timed(fused), 4))
    if ws.read_error():
        raise RuntimeError(f"device error flag {ws.read_error():#x}")
    moved = len(ops) * 2 * Hkv * D * 2
    return {"metric": "code step + finished-block compaction, one layer (ms per call)", "unit": "ms",
            "ms": res, "rows_moved": len(ops), "bytes_moved": moved,
            "config": {"requests": R, "K": K, "C": C, "heads": f"{Hq}/{Hkv}", "quota": qk, "steps": args.steps}}


def bench_flashinfer(args) -> dict:
    """BASELINE config 2 decode on the same caches through FlashInfer, the library the reference's
    vLLM backend runs decode with (patch_stock_flashinfer.py; FlashInfer 0.5.3 pinned by vLLM 0.13.0,
    the installed one is reported), against abkv_decode:

    * ``wrapper``: BatchDecodeWithPagedKVCacheWrapper over the NHD cache, planned once per quota
      group (indptr / indices / last_page_len from the group's block table), one run per layer;
      with ``use_tensor_cores`` False and True (its two decode paths for grouped heads);
    * ``trtllm``: trtllm_batch_decode_with_kv_cache on the NHD cache with the block tables and
      seq_lens directly (the decode kernel vLLM's FlashInfer backend selects on Blackwell).

    Each variant: ms per 36-layer step (CUDA events), GB/s of the algorithmic bytes, and the max abs
    difference of its outputs from abkv_decode's on every layer.  A variant that fails (import, JIT,
    unsupported shape) records its error instead."""
    import flashinfer

    from abridgekv_b200 import decode
    from abridgekv_b200.workloads import qwen3_decode_workload

    wl = qwen3_decode_workload(2, num_seqs=64)
    L, Hq, Hkv, D, page = wl.num_layers, wl.num_q_heads, wl.num_kv_heads, wl.head_dim, wl.page
    scale = 1.0 / math.sqrt(D)
    alg = wl.kv_bytes + wl.qo_bytes
    pk = _peaks()

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / args.steps

    ours = [torch.empty_like(q) for q in wl.queries]

    def run_ours():
        decode.paged_decode(wl.queries, wl.kv_caches, wl.block_tables, wl.seq_lens, outputs=ours,
                            max_pages_per_seq=wl.max_pages)

    ms = timed(run_ours)
    res = {"abkv_decode": {"ms_per_step": ms, "gbs": alg / (ms / 1e3) / 1e9,
                           "frac_of_hbm_peak": alg / (ms / 1e3) / 1e9 / pk["hbm_gbs"]}}

    def record(name, fn, outs):
        try:
            t = timed(fn)
            diff = max(float((o.float() - r.float()).abs().max()) for o, r in zip(outs, ours))
            res[name] = {"ms_per_step": t, "gbs": alg / (t / 1e3) / 1e9,
                         "frac_of_hbm_peak": alg / (t / 1e3) / 1e9 / pk["hbm_gbs"],
                         "abkv_speedup": t / ms, "max_abs_diff_vs_abkv": diff}
        except Exception as e:  # noqa: BLE001 -- a library path that does not run here is reported
            res[name] = {"error": f"{type(e).__name__}: {e}"[:400]}

    # one plan per quota group: layers of a group share the block-table tensor
    groups: dict[int, dict] = {}
    for l, bt in enumerate(wl.block_tables):
        g = groups.setdefault(id(bt), {"layers": [], "bt": bt, "sl": wl.seq_lens[l]})
        g["layers"].append(l)
    for tc in (False, True):
        name = f"wrapper_tensor_cores={tc}"
        try:
            wrappers = {}
            for key, g in groups.items():
                sl = g["sl"].cpu().to(torch.int64)
                pages = (sl + page - 1) // page
                bt = g["bt"].cpu()
                indptr = torch.cat([torch.zeros(1, dtype=torch.int64), pages.cumsum(0)]).to(torch.int32)
                indices = torch.cat([bt[b, :int(pages[b])] for b in range(bt.shape[0])]).to(torch.int32)
                last = ((sl - 1) % page + 1).to(torch.int32)
                w = flashinfer.BatchDecodeWithPagedKVCacheWrapper(
                    torch.zeros(128 << 20, dtype=torch.uint8, device="cuda"), "NHD", use_tensor_cores=tc)
                w.plan(indptr.cuda(), indices.cuda(), last.cuda(), Hq, Hkv, D, page, q_data_type=torch.bfloat16,
                       kv_data_type=torch.bfloat16, sm_scale=scale)
                wrappers[key] = w
            fo = [torch.empty_like(q) for q in wl.queries]
            per_layer = [wrappers[id(bt)] for bt in wl.block_tables]

            def run_wrapper(per_layer=per_layer, fo=fo):
                for l in range(L):
                    per_layer[l].run(wl.queries[l], wl.kv_caches[l], out=fo[l])
        except Exception as e:  # noqa: BLE001
            res[name] = {"error": f"{type(e).__name__}: {e}"[:400]}
            continue
        record(name, run_wrapper, fo)
    tr_ws = torch.zeros(256 << 20, dtype=torch.uint8, device="cuda")
    to = [torch.empty_like(q) for q in wl.queries]
    max_seq = int(max(int(s.max()) for s in wl.seq_lens))

    def run_trtllm():
        for l in range(L):
            flashinfer.decode.trtllm_batch_decode_with_kv_cache(
                wl.queries[l], wl.kv_caches[l], tr_ws, wl.block_tables[l], wl.seq_lens[l], max_seq,
                bmm1_scale=scale, bmm2_scale=1.0, out=to[l], kv_layout="NHD")

    record("trtllm_nhd", run_trtllm, to)
    return {"metric": "config-2 decode: abkv_decode vs FlashInfer on the same caches (ms per 36-layer step)",
            "unit": "ms", "flashinfer_version": getattr(flashinfer, "__version__", "?"),
            "algorithmic_bytes_per_step": alg, "hbm_peak_gbs": pk["hbm_gbs"], "results": res,
            "config": {"B": wl.num_seqs, "layers": L, "heads": f"{Hq}/{Hkv}", "page": page,
                       "steps": args.steps, "warmup": args.warmup}}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("which", choices=["prefill", "prefill_bwd", "compaction", "codestep", "packed", "kvshard",
                                          "codestep_compact", "flashinfer", "hostdecode"])
    ap.add_argument("--layers", type=int, default=36)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--flex", action="store_true")
    ap.add_argument("--blocks", type=int, default=6)
    ap.add_argument("--batch", type=int, default=16, help="prefill_bwd: sequences (16 = config 4)")
    ap.add_argument("--kv-heads", type=int, default=1, help="kvshard: KV heads of the shard (1, 2, 4, 8)")
    ap.add_argument("--seqs", type=int, default=256, help="kvshard: sequences")
    ap.add_argument("--chunk-tokens", type=int, default=0, help="kvshard: split-KV chunk rows (0 = auto)")
    args = ap.parse_args()
    fn = {"prefill": bench_prefill, "prefill_bwd": bench_prefill_bwd, "compaction": bench_compaction,
          "codestep": bench_codestep, "packed": bench_packed, "kvshard": bench_kvshard,
          "codestep_compact": bench_codestep_compact, "flashinfer": bench_flashinfer,
          "hostdecode": bench_hostdecode}[args.which]
    print(json.dumps(fn(args)), flush=True)


if __name__ == "__main__":
    main()

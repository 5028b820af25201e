#!/usr/bin/env python
"""Benchmark: compressed-KV decode attention on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one decode step of the whole batch through all 36 layers'
attention: a single abkv_decode launch over the Qwen3-4B-shaped compressed
cache (per-layer quotas 6x256 / 18x128 / 12x64, B=64 sequences of 256-token
prompt + 31 compressed blocks + a live tail ~U[0,511], page size 16; ~42 GB
of K/V read per step, far larger than L2, so no flush is needed).

Multi-GPU (torchrun, one rank per GPU): sequences shard across ranks with no
collective on the data path; every rank runs its own B=64 batch (weak
scaling).  Device time is the max over ranks.

Prints ONE JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "compressed-KV decode attn tokens/s/GPU + % HBM roofline at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0


# ---------------------------------------------------------------------------
def measured_hbm_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic(kernel: str) -> float | None:
    """Per-launch DRAM bytes of `kernel` from the committed ncu summary, if any."""
    p = ROOT / "profiles" / f"{kernel}.md"
    if not p.exists():
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", p.read_text())
    return float(m.group(1)) if m else None


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int | str):
        self.gpu = gpu  # nvidia-smi --id accepts an index or a GPU-<uuid>
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self._t.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ---------------------------------------------------------------------------
def cpu_baseline_decode(wl_rows: dict, budget_s: float = 20.0) -> dict:
    """Reference CPU path (oracle port of PackedKVSidecar._attend_decode_batched)
    on the host cores, over a bounded sample of config-2 sequences."""
    from abridgekv_b200.workloads import SCHEDULE_PERLAYER_MEAN128, build_decode_workload
    from oracle.decode_ref import sidecar_decode_torch

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    samples = []
    for b in range(min(4, len(next(iter(wl_rows.values()))))):
        rows = {q: r[b:b + 1] for q, r in wl_rows.items()}
        samples.append(build_decode_workload("cpu-sample", SCHEDULE_PERLAYER_MEAN128, rows, num_q_heads=32,
                                             num_kv_heads=8, head_dim=128, device="cpu", seed=100 + b))
    scale = 1.0 / np.sqrt(128)
    seqs_done, t_total = 0, 0.0
    while t_total < budget_s or seqs_done < len(samples):
        wl = samples[seqs_done % len(samples)]
        t0 = time.perf_counter()
        for l in range(wl.num_layers):
            sidecar_decode_torch(wl.queries[l], wl.kv_caches[l], wl.seq_lens[l], wl.block_tables[l],
                                 8, 4, scale, wl.page)
        t_total += time.perf_counter() - t0
        seqs_done += 1
    return {"value": seqs_done / t_total, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{seqs_done} decode steps of single config-2 sequences (4 distinct, cycled) x 36 "
                      f"layers, torch CPU (oracle/decode_ref.sidecar_decode_torch), {t_total:.1f} s"}


def run_reference(args, rank: int, world: int) -> None:
    """Reference arm: the reference's own CPU implementation of the path
    (PackedKVSidecar._attend_decode_batched restated as oracle/decode_ref.py's
    torch port; the reference itself is Python and is not installable here),
    timed on this box's host cores."""
    if rank != 0:
        return
    from abridgekv_b200.workloads import SCHEDULE_PERLAYER_MEAN128, build_decode_workload, config2_rows
    from oracle.decode_ref import sidecar_decode_torch

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    rows_all = config2_rows(64, seed=0)
    # one sampled sequence per step (bounded), cycling through the batch
    wls = []
    for b in range(min(4, args.steps + args.warmup)):
        rows = {q: r[b:b + 1] for q, r in rows_all.items()}
        wls.append(build_decode_workload("ref-sample", SCHEDULE_PERLAYER_MEAN128, rows, num_q_heads=32,
                                         num_kv_heads=8, head_dim=128, device="cpu", seed=100 + b))
    scale = 1.0 / np.sqrt(128)

    def step(i):
        wl = wls[i % len(wls)]
        for l in range(wl.num_layers):
            sidecar_decode_torch(wl.queries[l], wl.kv_caches[l], wl.seq_lens[l], wl.block_tables[l],
                                 8, 4, scale, wl.page)

    for i in range(args.warmup):
        step(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        step(i)
    dt = time.perf_counter() - t0
    value = args.steps / dt  # one sequence per step
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s (sum over GPUs)", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": config_block(world),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": "1 config-2 sequence x 36 layers per step (torch CPU port of "
                                   "compresslm_packed_kv.py:564-616)"},
        "e2e": {"value": value, "unit": "tokens/s (sum over GPUs)", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config_block(world: int, chunk_tokens: int = 0, num_seqs: int = 64) -> dict:
    return {
        "workload": "config2: Qwen3-4B decode attention over the compressed paged cache; 36 layers, "
                    "32 q / 8 kv heads, head_dim 128, per-layer quotas 6x256/18x128/12x64 "
                    f"(sched_trunc_perlayer_mean128), B={num_seqs} per GPU, 256-token prompt + 31 compressed "
                    "blocks + tail U[0,511], page 16, K/V/Q ~ N(0,1) bf16",
        "global_batch": num_seqs * world,
        "seq_len": "2496..8959 cache rows per layer",
        "parallelism": f"sequence-sharded x{world}, no collective",
        "l2": "inputs larger than L2 (~42.3 GB of K/V per step per GPU); no flush",
        "chunk_tokens": chunk_tokens or "auto",
    }


def run_ours(args, rank: int, world: int, local: int) -> None:
    from abridgekv_b200 import decode, _lib
    from abridgekv_b200.hostdecode import HostDecode
    from abridgekv_b200.workloads import qwen3_decode_workload
    from abridgekv_b200.workspace import Workspace

    dev = torch.device("cuda", local)
    wl = qwen3_decode_workload(2, num_seqs=args.num_seqs, device=dev, seed=rank)
    B, L = wl.num_seqs, wl.num_layers
    outs = [torch.empty_like(q) for q in wl.queries]
    ws = Workspace(dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        decode.paged_decode(wl.queries, wl.kv_caches, wl.block_tables, wl.seq_lens, outputs=outs,
                            max_pages_per_seq=wl.max_pages, chunk_tokens=args.chunk_tokens,
                            workspace=ws)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    assert ws.read_error() == 0, "device error word set during warm-up"

    uuid = str(getattr(torch.cuda.get_device_properties(dev), "uuid", "") or "")
    sampler = ClockSampler(("GPU-" + uuid) if uuid and not uuid.startswith("GPU-") else (uuid or local))
    sampler.start()
    time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    for e0, e1 in evs:
        e0.record(stream)
        step()
        e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    launch_ms = [e0.elapsed_time(e1) for e0, e1 in evs]
    total_ms = evs[0][0].elapsed_time(evs[-1][1])
    clocks = sampler.stop()
    total_ms_max = max_over_ranks(total_ms, world)
    mean_launch_ms = statistics.mean(launch_ms)
    tokens = B * args.steps * world
    value = tokens / (total_ms_max / 1e3)

    # ---- end to end through the public API with pinned host buffers --------
    q_host = [q.cpu().pin_memory() for q in wl.queries]
    bt_host = {id(t): t.cpu().pin_memory() for t in wl.block_tables}
    sl_host = {id(t): t.cpu().pin_memory() for t in wl.seq_lens}
    out_host = [torch.empty(o.shape, dtype=o.dtype).pin_memory() for o in outs]
    h2d = sum(q.numel() * 2 for q in q_host) + sum(t.numel() * 4 for t in bt_host.values()) + \
        sum(t.numel() * 4 for t in sl_host.values())
    d2h = sum(o.numel() * 2 for o in out_host)
    # HostDecode: every step uploads all queries and tables and downloads all outputs; the copies of
    # one layer group overlap the decode of the neighbouring groups, never those of another step
    host_decode = HostDecode(wl.kv_caches, max_pages_per_seq=wl.max_pages, chunk_tokens=args.chunk_tokens,
                             workspace=ws)
    bt_list = [bt_host[id(t)] for t in wl.block_tables]
    sl_list = [sl_host[id(t)] for t in wl.seq_lens]

    def e2e_step():
        host_decode.run(q_host, bt_list, sl_list, out_host)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = max(1, min(args.steps, 50))
    e_start.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e_end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(e_start.elapsed_time(e_end), world)
    e2e_value = B * e2e_steps * world / (e2e_ms / 1e3)
    # the e2e outputs equal device-resident launches over the same layer groups (the split-KV
    # chunking of a launch depends on its layer count, so the grouping fixes the bits)
    for g in host_decode.groups:
        ref = decode.paged_decode([wl.queries[l] for l in g], [wl.kv_caches[l] for l in g],
                                  [wl.block_tables[l] for l in g], [wl.seq_lens[l] for l in g],
                                  max_pages_per_seq=wl.max_pages, chunk_tokens=args.chunk_tokens, workspace=ws)
        assert all(torch.equal(out_host[l], r.cpu()) for l, r in zip(g, ref))
    assert ws.read_error() == 0
    alg_bytes = wl.kv_bytes + wl.qo_bytes
    headline_launches = args.steps * ((L + 55) // 56)
    del wl, outs, host_decode, ref
    torch.cuda.empty_cache()

    # ---- config 3 at this N: the fixed 512-sequence batch, sharded by bytes (strong scaling) ----
    strong = None
    if not args.no_strong:
        strong = strong_decode(3, rank=rank, world=world, local=local, steps=args.strong_steps, warmup=3,
                               mem_budget_gb=args.mem_budget_gb)
    # ---- config 5 at N >= 4 (323.7 GB: two GPUs cannot hold it): KV-head sharding with the all-gather
    # fused into the decode epilogue (peer stores over NVLink), and sequence sharding of the same batch
    kv_heads = None
    if world >= 4 and not args.no_kvshard:
        kv = strong_decode(5, rank=rank, world=world, local=local, steps=args.strong_steps, warmup=3,
                           mem_budget_gb=args.mem_budget_gb, shard="kv", gather="fused")
        seq = strong_decode(5, rank=rank, world=world, local=local, steps=args.strong_steps, warmup=3,
                            mem_budget_gb=args.mem_budget_gb, shard="seq")
        kv_heads = {"config": 5, "global_batch": kv["global_batch"], "unit": kv["unit"],
                    "kv_head_sharded": {k: kv[k] for k in ("value", "ms_per_step", "parallelism", "roofline")},
                    "sequence_sharded": {k: seq[k] for k in ("value", "ms_per_step", "parallelism", "roofline")},
                    "kv_over_sequence": kv["value"] / seq["value"]}
    # ---- the other kernels of the path, one GPU ----
    secondary = None
    if world == 1 and not args.no_secondary:
        secondary = run_secondary(args)

    if rank != 0:
        return
    peak, peak_kind = measured_hbm_peak()
    achieved = alg_bytes / (mean_launch_ms / 1e3) / 1e9
    traffic = profiled_traffic("decode_split_kernel")
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_decode(_config2_rows_for_cpu(), budget_s=args.cpu_budget)
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s (sum over GPUs)", "value_per_gpu": value / world,
        "unit_per_gpu": "tokens/s/GPU", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total_ms_max / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": config_block(world, args.chunk_tokens, args.num_seqs),
        "roofline": {"bound": "hbm", "kernel": "decode_split_kernel", "achieved": achieved, "peak": peak,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                     else "fallback 6.65 TB/s", "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic, "algorithmic_bytes_per_launch": alg_bytes,
                     "mean_launch_ms": mean_launch_ms},
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": "tokens/s (sum over GPUs)", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": e2e_steps},
        "gpu_launches": headline_launches,
        "clocks": clocks,
        "strong_scaling": strong,
        "config5_kv_heads": kv_heads,
        "secondary": secondary,
    }
    print(json.dumps(line), flush=True)


def strong_decode(cfg: int, *, rank: int, world: int, local: int, steps: int, warmup: int, chunk_tokens: int = 0,
                  mem_budget_gb: float = 130.0, shard: str = "seq", gather: str = "fused",
                  num_seqs: int | None = None) -> dict:
    """One strong-scaling decode measurement (the global batch is fixed); every rank calls it.

    config 3: 512 sequences with generated lengths log-uniform in [2K, 32K] (247.8 GB of K/V),
      sequence-sharded by bytes (parallel.shard_by_bytes: every rank reads about the same bytes per
      step); a rank whose share exceeds mem_budget_gb decodes it in waves (each wave's caches are
      built, timed and freed in turn) and one step = one decode step of every wave.
    config 5: 256 sequences, quota 128 in every layer, 63 compressed blocks + tail (323.7 GB).
      shard "seq": whole sequences per rank (by bytes), one 36-layer launch per step.  shard "kv":
      every rank holds KV heads [r*8/W, (r+1)*8/W) of all sequences; per layer one decode launch of
      its heads whose epilogue all-gathers the [B, 32, 128] outputs into every rank's buffer over
      NVLink (gather "fused", abkv_decode_gather), or the plain decode followed by an NCCL
      all-gather (gather "nccl").
    Returns (meaningful on rank 0) value = sequences / max-over-ranks ms per step, the roofline of
    the per-GPU mean bytes, the waves of rank 0 and the byte imbalance of the shards."""
    from abridgekv_b200 import decode, parallel
    from abridgekv_b200.workloads import (QWEN3_4B, SCHEDULE_PERLAYER_MEAN128, config3_rows, config5_rows,
                                          qwen3_decode_workload)
    from abridgekv_b200.workspace import Workspace

    dev = torch.device("cuda", local)
    n_global = num_seqs or (512 if cfg == 3 else 256)
    rows_all = (config3_rows if cfg == 3 else config5_rows)(n_global, 0)
    hkv, hd = QWEN3_4B["num_kv_heads"], QWEN3_4B["head_dim"]
    kv_mode = cfg == 5 and shard == "kv"
    heads = parallel.kv_head_shard(hkv, world, rank) if kv_mode else None
    quotas = (128,) * 36 if cfg == 5 else SCHEDULE_PERLAYER_MEAN128
    h_local = hkv // world if kv_mode else hkv
    per_seq = np.zeros(n_global)
    for q in quotas:
        per_seq += rows_all[q] * h_local * hd * 4
    shards = [np.arange(n_global)] * world if kv_mode else \
        [parallel.shard_by_bytes(per_seq, world, r) for r in range(world)]
    loads = np.array([per_seq[s].sum() for s in shards])
    mine = shards[rank]
    budget = mem_budget_gb * 1e9
    waves, cur, acc = [], [], 0.0
    for i in mine:
        if cur and acc + per_seq[i] > budget:
            waves.append(cur)
            cur, acc = [], 0.0
        cur.append(int(i))
        acc += per_seq[i]
    if cur:
        waves.append(cur)
    if kv_mode and len(waves) > 1:
        raise SystemExit(f"config 5 KV-head sharding needs {per_seq.sum() / 1e9:.1f} GB per rank "
                         f"(> --mem-budget-gb {mem_budget_gb}); use more GPUs")
    ws = Workspace(dev)
    stream = torch.cuda.current_stream(dev)
    wave_ms, alg_bytes, launches, waves_info = [], 0, 0, []
    head_gather = None
    for idx in waves:
        wl = qwen3_decode_workload(cfg, num_seqs=n_global, device=dev, seed=0,
                                   seq_slice=None if kv_mode else np.asarray(idx), kv_heads=heads)
        outs = [torch.empty_like(q) for q in wl.queries]
        gathered = [None] * wl.num_layers

        if kv_mode and gather == "fused":
            from abridgekv_b200.gather import HeadGather
            head_gather = HeadGather(wl.num_layers, wl.num_seqs, wl.num_q_heads * world, device=dev)

            def step():
                for l in range(wl.num_layers):
                    head_gather.decode([l], [wl.queries[l]], [wl.kv_caches[l]], [wl.block_tables[l]],
                                       [wl.seq_lens[l]], max_pages_per_seq=wl.max_pages,
                                       chunk_tokens=chunk_tokens, workspace=ws)
            per_step = wl.num_layers
        elif kv_mode:
            def step():
                for l in range(wl.num_layers):
                    decode.paged_decode([wl.queries[l]], [wl.kv_caches[l]], [wl.block_tables[l]],
                                        [wl.seq_lens[l]], outputs=[outs[l]], max_pages_per_seq=wl.max_pages,
                                        chunk_tokens=chunk_tokens, workspace=ws)
                    gathered[l] = parallel.gather_head_outputs(outs[l])
            per_step = wl.num_layers
        else:
            def step():
                decode.paged_decode(wl.queries, wl.kv_caches, wl.block_tables, wl.seq_lens, outputs=outs,
                                    max_pages_per_seq=wl.max_pages, chunk_tokens=chunk_tokens, workspace=ws)
            per_step = (wl.num_layers + 55) // 56
        for _ in range(max(warmup, 3)):
            step()
        torch.cuda.synchronize()
        assert ws.read_error() == 0, "device error word set during warm-up"
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        wave_ms.append(e0.elapsed_time(e1) / steps)
        alg_bytes += wl.kv_bytes + wl.qo_bytes
        launches += per_step * steps
        waves_info.append({"seqs": len(idx), "kv_gb": wl.kv_bytes / 1e9, "ms_per_step": wave_ms[-1]})
        if head_gather is not None:
            assert ws.read_error() == 0, "device error word set during the timed region"
            head_gather.close()
            head_gather = None
        del wl, outs, gathered
        torch.cuda.empty_cache()
    ms_step = sum(wave_ms)
    ms_max = max_over_ranks(ms_step, world)
    bytes_total = alg_bytes
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([float(alg_bytes)], dtype=torch.float64, device=dev)
        dist.all_reduce(t)
        bytes_total = float(t.item())
    peak, peak_kind = measured_hbm_peak()
    achieved = bytes_total / world / (ms_max / 1e3) / 1e9
    return {
        "config": cfg, "global_batch": n_global, "n_gpus": world, "value": n_global / (ms_max / 1e3),
        "unit": "tokens/s (sum over GPUs)", "ms_per_step": ms_max, "steps": steps,
        "parallelism": ((f"KV-head-sharded x{world}, all-gather fused into the decode epilogue (peer stores "
                         "over NVLink)" if gather == "fused" else f"KV-head-sharded x{world} + NCCL all-gather "
                         "per layer") if kv_mode else f"sequence-sharded x{world} by bytes (greedy longest-first), "
                                                      "no collective"),
        "shard_bytes_max_over_mean": float(loads.max() / loads.mean()),
        "waves_rank0": waves_info, "mem_budget_gb": mem_budget_gb, "gpu_launches_rank0": launches,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "note": "per-GPU mean: all ranks' algorithmic bytes / W / max time",
                     "peak_source": peak_kind},
    }


def run_scaling(args, rank: int, world: int, local: int) -> None:
    """--config 3 / 5: a strong-scaling decode line of its own (see strong_decode)."""
    res = strong_decode(args.config, rank=rank, world=world, local=local, steps=args.steps, warmup=args.warmup,
                        chunk_tokens=args.chunk_tokens, mem_budget_gb=args.mem_budget_gb, shard=args.shard,
                        gather=args.gather, num_seqs=args.num_seqs if args.num_seqs != 64 else None)
    if rank != 0:
        return
    cfg = args.config
    line = {
        "metric": METRIC, "value": res["value"], "unit": res["unit"], "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": res["ms_per_step"], "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"config{cfg}: Qwen3-4B decode attention, {res['global_batch']} sequences, "
                               + ("per-layer quotas 6x256/18x128/12x64, generated length log-uniform [2K,32K]"
                                  if cfg == 3 else "quota 128 in all 36 layers, 63 compressed blocks + tail"),
                   "global_batch": res["global_batch"], "parallelism": res["parallelism"],
                   "waves_rank0": res["waves_rank0"], "mem_budget_gb": res["mem_budget_gb"],
                   "shard_bytes_max_over_mean": res["shard_bytes_max_over_mean"],
                   "l2": "inputs larger than L2; no flush"},
        "roofline": res["roofline"], "gpu_launches": res["gpu_launches_rank0"],
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# Secondary paths (--path prefill | codestep | compaction): one GPU, one JSON line
# with the GPU measurement of benchmarks.py and the reference's CPU
# path timed on this box's host cores over a bounded sample.
def cpu_baseline_prefill(budget_s: float) -> dict:
    """Eager dense-mask attention (the reference's _dense_mask + matmul/softmax path) in fp32
    torch on the host cores, reduced shape; credited with the algorithmic FLOPs of its
    visible pairs, like the GPU number."""
    from oracle.mask_ref import arith_mask

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    C, K, N, D = 512, 256, 4, 128
    quota = [256, 128, 64, 128]
    S0 = N * (C + K)
    g = torch.Generator().manual_seed(0)
    q = torch.randn((len(quota), S0, D), generator=g)
    k = torch.randn((1, S0, D), generator=g)
    v = torch.randn((1, S0, D), generator=g)
    mask = torch.from_numpy(arith_mask(S0, C, K, quota_per_head=quota)[0])
    flops = 4.0 * D * float(mask.sum())
    scale = 1.0 / np.sqrt(D)
    n, t = 0, 0.0
    while t < budget_s or n == 0:
        t0 = time.perf_counter()
        s_ = (q @ k.transpose(1, 2)) * scale
        s_ = s_.masked_fill(~mask, float("-inf"))
        _ = torch.softmax(s_, dim=-1) @ v
        t += time.perf_counter() - t0
        n += 1
    return {"value": flops * n / t / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": f"{n} x (1 sequence of {N} blocks x (512 + 256), 4 query heads with quotas {quota}, "
                      f"fp32 dense-mask attention), {t:.1f} s"}


def cpu_baseline_prefill_bwd(budget_s: float) -> dict:
    """torch autograd backward of the eager dense-mask attention in fp32 on the host cores, reduced
    shape (the forward runs outside the timed part); credited with 10 x D FLOP per visible pair."""
    from oracle.mask_ref import arith_mask

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    C, K, N, D = 512, 256, 4, 128
    quota = [256, 128, 64, 128]
    S0 = N * (C + K)
    g = torch.Generator().manual_seed(0)
    q = torch.randn((len(quota), S0, D), generator=g, requires_grad=True)
    k = torch.randn((1, S0, D), generator=g, requires_grad=True)
    v = torch.randn((1, S0, D), generator=g, requires_grad=True)
    dout = torch.randn((len(quota), S0, D), generator=g)
    mask = torch.from_numpy(arith_mask(S0, C, K, quota_per_head=quota)[0])
    flops = 10.0 * D * float(mask.sum())
    scale = 1.0 / np.sqrt(D)
    n, t = 0, 0.0
    while t < budget_s or n == 0:
        s_ = (q @ k.transpose(1, 2)) * scale
        s_ = s_.masked_fill(~mask, float("-inf"))
        out = torch.softmax(s_, dim=-1) @ v
        t0 = time.perf_counter()
        out.backward(dout)
        t += time.perf_counter() - t0
        q.grad = k.grad = v.grad = None
        n += 1
    return {"value": flops * n / t / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": f"{n} x backward of (1 sequence of {N} blocks x (512 + 256), 4 query heads with quotas "
                      f"{quota}, fp32 dense-mask attention), {t:.1f} s"}


def cpu_baseline_codestep(budget_s: float) -> dict:
    """The reference's noncausal code step (_attend_request_vectorized, torch CPU port) on one
    config-2 request's caches + 256 code rows, layer after layer."""
    from abridgekv_b200.workloads import SCHEDULE_PERLAYER_MEAN128, build_decode_workload, config2_rows
    from oracle.decode_ref import sidecar_codestep_torch

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    K = 256
    rows = {q: r[:1] + K for q, r in config2_rows(64, 0).items()}
    wl = build_decode_workload("cpu-codestep", SCHEDULE_PERLAYER_MEAN128, rows, num_q_heads=32, num_kv_heads=8,
                               head_dim=128, device="cpu", seed=7)
    q = torch.randn((K, 32, 128), generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    scale = 1.0 / np.sqrt(128)
    n, t, flops = 0, 0.0, 0.0
    while t < budget_s or n == 0:
        l = n % wl.num_layers
        quota = wl.quotas[l]
        L = int(wl.seq_lens[l][0])
        t0 = time.perf_counter()
        sidecar_codestep_torch(q, wl.kv_caches[l], L, wl.block_tables[l][0], [quota] * 8, K, 8, 4, scale, wl.page)
        t += time.perf_counter() - t0
        flops += 4.0 * 128 * K * 32 * (L - K + quota)
        n += 1
    return {"value": flops / t / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": f"{n} layer code steps of one config-2 request (+256 code rows), torch CPU port of "
                      f"compresslm_packed_kv.py:648-741, {t:.1f} s"}


def cpu_baseline_compaction(budget_s: float) -> dict:
    """The reference's compaction on the host: the planner restatement (mask_token_span ->
    copy ops) and the gather-then-scatter executor on numpy caches, 2 sequences x 12 tensors."""
    from oracle.compaction_ref import Planner, execute_kv_copy_operations

    cores = 1
    C, K, page, quotas, B, T = 512, 256, 16, (256, 128, 64), 2, 12
    per = C + K
    n, t, moved = 0, 0.0, 0
    while t < budget_s or n == 0:
        blocks = 3
        nb = 1 + B * (blocks * per // page) * 3 + 8
        caches = [np.zeros((nb, 2, page, 8, 128), dtype=np.uint16) for _ in range(T)]
        pl = Planner(nb, page, 3)
        for b in range(B):
            pl.add_request(b)
        for blk in range(blocks):
            t0 = time.perf_counter()
            for b in range(B):
                m = (blk + 1) * per
                pl.allocate_slots(b, m)
                pl.computed[b] = m
                pl.finish_block(b, (blk * per, blk * per + C), (blk * per + C, (blk + 1) * per), quotas, K)
            ops = pl.take_pending()[0]
            execute_kv_copy_operations(ops, [caches] * 3)
            t += time.perf_counter() - t0
            rows = sum(len(x) for g_ in ops.values() for bl in g_ for x in bl)
            moved += rows * T * 2 * 2 * 8 * 128 * 2
        n += 1
    return {"value": moved / t / 1e9, "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"{n} x (2 sequences x 3 block finishes x 12 layer tensors: planner restatement + numpy "
                      f"gather/scatter executor), {t:.1f} s"}


def run_path(args) -> None:
    import benchmarks

    torch.cuda.set_device(0)
    ns = argparse.Namespace(layers=36, steps=args.steps, warmup=args.warmup, flex=args.flex, blocks=6)
    uuid = str(getattr(torch.cuda.get_device_properties(0), "uuid", "") or "")
    sampler = ClockSampler(("GPU-" + uuid) if uuid and not uuid.startswith("GPU-") else (uuid or 0))
    sampler.start()
    if args.path == "prefill":
        line = benchmarks.bench_prefill(ns)
        launches = 36 * args.steps
    elif args.path == "prefill_bwd":
        line = benchmarks.bench_prefill_bwd(ns)
        launches = 3 * 36 * args.steps  # per layer: row-dot, backward, dq store
    elif args.path == "codestep":
        line = benchmarks.bench_codestep(ns)
        launches = 36 * args.steps
    else:
        line = benchmarks.bench_compaction(ns)
        launches = line.get("gpu_launches")  # counted by the benchmark over its steady block finishes
    clocks = sampler.stop()
    budget = 0.0 if args.no_cpu_baseline else args.cpu_budget
    cpu = None if args.no_cpu_baseline else {"prefill": cpu_baseline_prefill, "prefill_bwd": cpu_baseline_prefill_bwd,
                                             "codestep": cpu_baseline_codestep,
                                             "compaction": cpu_baseline_compaction}[args.path](budget)
    line.update({"n_gpus": 1, "steps": args.steps if args.path != "compaction" else ns.blocks,
                 "warmup": args.warmup, "higher_is_better": True, "scaling": None, "vs_baseline": None,
                 "dtype": "bf16", "data": "synthetic", "cpu_baseline": cpu, "gpu_launches": launches,
                 "clocks": clocks, "path": args.path,
                 "e2e": None, "e2e_note": "secondary path: inputs stay in HBM (the headline e2e is the decode line)"})
    print(json.dumps(line), flush=True)


def run_secondary(args) -> dict:
    """The path's other kernels, one short measurement each on this GPU (CUDA events after 3 warm-up
    steps) with its roofline and the reference's CPU path timed on the host cores over a bounded
    sample: config-4 prefill (36 layers), its backward, the code step on config-2 caches + 256 code
    rows (36 layers), and config 4's block compaction (planner + executor, 16 sequences x 36 layers)."""
    import benchmarks

    ns = argparse.Namespace(layers=36, steps=2, warmup=3, flex=False, blocks=4, batch=16)
    budget = args.secondary_cpu_budget
    runs = (("prefill", benchmarks.bench_prefill, cpu_baseline_prefill, 36 * ns.steps),
            ("prefill_bwd", benchmarks.bench_prefill_bwd, cpu_baseline_prefill_bwd, 3 * 36 * ns.steps),
            ("codestep", benchmarks.bench_codestep, cpu_baseline_codestep, 36 * ns.steps),
            ("compaction", benchmarks.bench_compaction, cpu_baseline_compaction, None))
    out = {}
    for name, fn, cpu_fn, launches in runs:
        line = fn(ns)
        roof = dict(line["roofline"])
        roof.setdefault("unit", line["unit"])
        roof["peak_source"] = roof.pop("peak_kind", None) or (
            "measured sustained cuBLAS bf16 (MEASURED_PEAKS.json)" if roof["bound"] == "tensor"
            else "measured copy bandwidth (MEASURED_PEAKS.json hbm_gbs)")
        keep = {k: line[k] for k in ("metric", "value", "unit", "ms_per_step", "algorithmic_tflop_per_step",
                                     "device_ms_per_block_finish", "host_ms_executor_call", "host_ms_planner",
                                     "bytes_per_block_finish", "forward_plus_backward_ms") if k in line}
        keep.update({"roofline": roof, "gpu_launches": line.get("gpu_launches") if launches is None else launches,
                     "config": line.get("config"),
                     "cpu_baseline": None if args.no_cpu_baseline else cpu_fn(budget)})
        out[name] = keep
        torch.cuda.empty_cache()
    return out


def _config2_rows_for_cpu():
    from abridgekv_b200.workloads import config2_rows
    return config2_rows(64, seed=0)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--chunk-tokens", type=int, default=0)
    ap.add_argument("--num-seqs", type=int, default=64, help="sequences per GPU (config 2 uses 64)")
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config", type=int, choices=[2, 3, 5], default=2,
                    help="2 (default, headline): weak scaling; 3 / 5: strong-scaling saturation runs")
    ap.add_argument("--shard", choices=["seq", "kv"], default="seq", help="config 5: sequence or KV-head sharding")
    ap.add_argument("--path", choices=["decode", "prefill", "prefill_bwd", "codestep", "compaction"], default="decode",
                    help="decode (default, the headline) or a secondary path's line with its CPU baseline")
    ap.add_argument("--flex", action="store_true", help="--path prefill: also time compiled FlexAttention")
    ap.add_argument("--gather", choices=["fused", "nccl"], default="fused",
                    help="config 5 --shard kv: all-gather fused into the decode kernel, or NCCL after it")
    ap.add_argument("--mem-budget-gb", type=float, default=130.0,
                    help="configs 3/5: K/V bytes one wave may hold per GPU")
    ap.add_argument("--strong-steps", type=int, default=10,
                    help="timed steps of the config-3 strong-scaling block of the headline line")
    ap.add_argument("--no-strong", action="store_true", help="omit the config-3 strong-scaling block")
    ap.add_argument("--no-secondary", action="store_true", help="omit the secondary kernels' block (N=1)")
    ap.add_argument("--no-kvshard", action="store_true", help="omit the config-5 KV-head block (N >= 4)")
    ap.add_argument("--secondary-cpu-budget", type=float, default=6.0,
                    help="seconds of CPU baseline per secondary kernel")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.path != "decode":
        if args.gpus != 1 or args.impl != "ours":
            raise SystemExit("--path prefill/codestep/compaction runs on one GPU with --impl ours")
        run_path(args)
        return
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        run_reference(args, rank, world)
        return
    rank, world, local = dist_setup(args.gpus)
    try:
        if args.config == 2:
            run_ours(args, rank, world, local)
        else:
            run_scaling(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()

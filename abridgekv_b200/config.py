"""CompressLM serving configuration and quota-schedule files (host side).

The compressed-cache geometry this package serves -- block size C, code rows K,
per-layer code quotas (masked or physical), packed per-head quotas, code RoPE
layout -- comes from two files a CompressLM deployment already has:

* the HF export's ``compresslm_config.json`` (written by
  scripts/convert_compresslm_checkpoint_to_hf.py:189-208,286-288): block_size,
  num_code_tokens, num_passes, pause_xattn, raw_prompt, raw_tail, replay_tail,
  code_positions, retain_tail_kv, retain_tail_policy, code_exclude_replay_tail;
* a quota-schedule file (results/schedules/*.json): a 2D [layer][KV head] quota
  array, or an object holding it under "packed_kv_quotas" or "quotas".  Readers
  follow scripts/compresslm_schedules.py:6-27 (per-layer serving needs every row
  uniform across KV heads).

``CompressLMConfig`` restates the fields of the vLLM overlay's config class that
decide that geometry (third_party/vllm_overlay/vllm/config/compresslm.py:9-300):
the same defaults, the same validation messages for the enabled production
configuration, and the same helpers (layer_quota, distinct_layer_quotas,
kv_group_quotas, bitrev_code_offsets, bitrev_rope_positions).  Fields of the
overlay that only the evaluation harness uses (debug, tokenizer ids, selective
full-history layers) are not carried.  Adapters hand the geometry to this
package's kernels: quota groups for the decode launches, a ``PackedKVLayout``
for the packed sidecar, a ``CompressMask`` for the prefill.
"""
from __future__ import annotations

import json
from dataclasses import dataclass, field, fields
from pathlib import Path
from typing import Any, Sequence

import numpy as np

_POLICIES = ("rolling", "sticky", "static")


def load_quota_rows(path: str | Path) -> tuple[tuple[int, ...], ...]:
    """[layer][KV head] quota rows of a schedule file: a 2D array, or an object with
    "packed_kv_quotas" (preferred) or "quotas"."""
    payload = json.loads(Path(path).read_text())
    if isinstance(payload, dict):
        payload = payload.get("packed_kv_quotas", payload.get("quotas"))
    if not isinstance(payload, list) or not payload:
        raise ValueError(f"{path}: expected a non-empty 2D quota array or an object with 'quotas'")
    return tuple(tuple(int(v) for v in row) for row in payload)


def load_layer_quotas(path: str | Path) -> tuple[int, ...]:
    """One quota per layer; every layer's row must hold a single value across KV heads (a
    tensor-parallel server cannot give heads of one layer different quotas)."""
    out = []
    for layer, row in enumerate(load_quota_rows(path)):
        values = sorted(set(row))
        if len(values) != 1:
            raise ValueError(f"{path}: layer {layer} has per-head quotas {values}; "
                             "per-layer serving needs one quota per layer")
        out.append(values[0])
    return tuple(out)


def layer_index(layer_name: str) -> int | None:
    """n of an attention layer named '....layers.n....' (None when the name has no index)."""
    _, sep, rest = layer_name.partition(".layers.")
    if not sep:
        return None
    head = rest.split(".", 1)[0]
    return int(head) if head.isdigit() else None


@dataclass
class CompressLMConfig:
    enable: bool = False
    block_size: int = 512
    num_code_tokens: int = 128
    replay_tail: int = 16
    retain_tail_kv: int = 0
    retain_tail_policy: str = "rolling"
    code_exclude_replay_tail: bool = False
    raw_prompt: bool = True
    num_passes: int = 1
    pause_xattn: str = "full"
    raw_tail: int = 0
    packed_kv: bool = False
    packed_kv_k_max: int = 2048
    packed_kv_quotas: tuple[tuple[int, ...], ...] = ()
    code_positions: str = "appended"
    layer_code_quotas: tuple[int, ...] = ()
    physical_layer_quotas: bool = False
    extra: dict[str, Any] = field(default_factory=dict, repr=False)  # export keys this class does not model

    def __post_init__(self) -> None:
        self.packed_kv_quotas = tuple(tuple(int(v) for v in row) for row in self.packed_kv_quotas)
        self.layer_code_quotas = tuple(int(q) for q in self.layer_code_quotas)
        if self.retain_tail_policy not in _POLICIES:
            raise ValueError("retain_tail_policy must be one of: rolling, sticky, static")
        if self.code_positions not in ("appended", "bitrev"):
            raise ValueError("code_positions must be appended or bitrev")
        if not self.enable:
            return
        C, K = self.block_size, self.num_code_tokens
        if self.code_positions == "bitrev":
            pow2 = C > 0 and K > 0 and not (C & (C - 1)) and not (K & (K - 1))
            if not pow2 or self.replay_tail or self.raw_tail or self.num_passes != 1:
                raise ValueError("code_positions=bitrev needs power-of-two block_size and num_code_tokens, "
                                 "no replay/raw tail and num_passes=1")
        if C <= 0:
            raise ValueError("block_size must be positive")
        if K <= 0:
            raise ValueError("num_code_tokens must be positive")
        if not 0 <= self.replay_tail <= C:
            raise ValueError("replay_tail must be in [0, block_size]")
        if not 0 <= self.retain_tail_kv < C:
            raise ValueError("retain_tail_kv must be in [0, block_size)")
        if self.retain_tail_policy == "sticky" and not self.retain_tail_kv:
            raise ValueError("retain_tail_policy='sticky' requires retain_tail_kv > 0")
        if sum(1 for v in (self.raw_tail, self.replay_tail, self.retain_tail_kv) if v) > 1:
            raise ValueError("raw_tail, replay_tail, and retain_tail_kv are mutually exclusive")
        if self.code_exclude_replay_tail and not 0 < self.replay_tail < C:
            raise ValueError("code_exclude_replay_tail requires replay_tail in [1, block_size)")
        if self.num_passes != 1:
            raise ValueError("vLLM CompressLM decoding currently supports L=1 only")
        if self.pause_xattn != "full":
            raise ValueError("vLLM CompressLM decoding currently requires pause_xattn='full'")
        if self.raw_tail:
            raise ValueError("vLLM CompressLM decoding currently supports raw_tail=0 only")
        if not self.raw_prompt:
            raise ValueError("vLLM CompressLM decoding currently requires raw_prompt=True")
        for layer, quota in enumerate(self.layer_code_quotas):
            if not 0 < quota <= K:
                raise ValueError(f"layer_code_quotas[{layer}]={quota} must be in [1, {K}]")
        if self.uses_layer_quotas:
            if self.code_positions != "bitrev":
                raise ValueError("layer_code_quotas below num_code_tokens need code_positions=bitrev "
                                 "(nested-prefix code layout)")
            if self.packed_kv:
                raise ValueError("layer_code_quotas and packed KV are mutually exclusive")
        if self.physical_layer_quotas and not self.layer_code_quotas:
            raise ValueError("physical_layer_quotas needs layer_code_quotas")
        if self.packed_kv:
            if self.raw_tail or (self.retain_tail_kv and self.retain_tail_policy != "static"):
                raise ValueError("packed KV supports code/replay checkpoints and the static retained tail, "
                                 "not window (rolling/sticky) or raw tails")
            if self.code_exclude_replay_tail:
                raise ValueError("packed KV does not yet support code_exclude_replay_tail")
            if self.packed_kv_k_max != K:
                raise ValueError("packed_kv_k_max must equal num_code_tokens so the dense code pass computes "
                                 "every schedulable slot")
            for layer, row in enumerate(self.packed_kv_quotas):
                if not row:
                    raise ValueError(f"packed_kv_quotas[{layer}] must not be empty")
                for head, quota in enumerate(row):
                    if not 0 < quota <= self.packed_kv_k_max:
                        raise ValueError(f"packed_kv_quotas[{layer}][{head}]={quota} must be in "
                                         f"[1, {self.packed_kv_k_max}]")

    # ---- the overlay's helpers -------------------------------------------------
    @property
    def code_excluded_tail(self) -> int:
        return self.replay_tail if self.code_exclude_replay_tail else self.retain_tail_kv

    @property
    def uses_layer_quotas(self) -> bool:
        """Some layer sees fewer code slots than the cache holds."""
        return any(q < self.num_code_tokens for q in self.layer_code_quotas)

    @property
    def uses_physical_layer_quotas(self) -> bool:
        return bool(self.physical_layer_quotas) and self.uses_layer_quotas

    @property
    def uses_packed_kv(self) -> bool:
        return bool(self.packed_kv)

    def layer_quota(self, layer: int) -> int:
        """Code slots visible at `layer` (all K past the end of the schedule)."""
        if 0 <= layer < len(self.layer_code_quotas):
            return self.layer_code_quotas[layer]
        return self.num_code_tokens

    @property
    def distinct_layer_quotas(self) -> tuple[int, ...]:
        return tuple(sorted(set(self.layer_code_quotas)))

    def kv_group_quotas(self, group_layer_names: Sequence[Sequence[str]]) -> tuple[int, ...]:
        """The code quota of every KV-cache group; a group must hold layers of one quota."""
        out = []
        for names in group_layer_names:
            seen = set()
            for name in names:
                idx = layer_index(name)
                if idx is None:
                    raise ValueError(f"physical per-layer quotas need indexed attention layers; got {name!r}")
                seen.add(self.layer_quota(idx))
            if len(seen) != 1:
                raise ValueError(f"KV cache group mixes code quotas {sorted(seen)}: {list(names)}")
            out.append(next(iter(seen)))
        return tuple(out)

    def bitrev_code_offsets(self) -> np.ndarray:
        """In-block RoPE offset of each code row k: floor(bitreverse_{log2 K}(k) * span / K), span = C minus
        the tail the codes do not summarise."""
        K = self.num_code_tokens
        span = self.block_size - self.code_excluded_tail
        if span < K:
            raise ValueError(f"bitrev code span {span} < num_code_tokens {K}")
        bits = K.bit_length() - 1
        k = np.arange(K, dtype=np.int64)
        rev = np.zeros_like(k)
        for b in range(bits):
            rev |= ((k >> b) & 1) << (bits - 1 - b)
        return rev * span // K

    def bitrev_rope_positions(self, logical) -> np.ndarray:
        """RoPE positions of logical sequence positions (period C + K per block) under the bitrev layout:
        content row j of block b at b*C + j, code row k at b*C + bitrev offset(k)."""
        C, K = self.block_size, self.num_code_tokens
        logical = np.asarray(logical, dtype=np.int64)
        blk, within = np.divmod(logical, C + K)
        offs = self.bitrev_code_offsets()[np.clip(within - C, 0, K - 1)]
        return blk * C + np.where(within >= C, offs, within)

    # ---- adapters to this package ---------------------------------------------------
    def decode_groups(self, num_layers: int) -> dict[int, list[int]]:
        """Layers of each distinct quota (one KV-cache group, one block table and seq_lens per group in the
        physical-quota serving layout)."""
        groups: dict[int, list[int]] = {}
        for layer in range(num_layers):
            groups.setdefault(self.layer_quota(layer), []).append(layer)
        return dict(sorted(groups.items(), reverse=True))

    def packed_layout(self, *, num_layers: int, num_kv_heads: int):
        """PackedKVLayout of the packed per-head quotas (uniform K when the config has none)."""
        from .sidecar import PackedKVLayout

        return PackedKVLayout.from_schedule(self.packed_kv_quotas or None, num_layers=num_layers,
                                            num_kv_heads=num_kv_heads, k_max=self.num_code_tokens)

    def prefill_mask(self, layer: int, *, num_q_heads: int, prompt_len=None):
        """CompressMask descriptor of one layer for the prefill AttentionInterface."""
        from .prefill import CompressMask

        return CompressMask(C=self.block_size, K_layout=self.num_code_tokens,
                            quota_per_head=[self.layer_quota(layer)] * num_q_heads, prompt_len=prompt_len)

    # ---- files ----------------------------------------------------------------------
    @classmethod
    def from_dict(cls, data: dict, **overrides) -> "CompressLMConfig":
        known = {f.name for f in fields(cls)} - {"extra"}
        kw = {k: v for k, v in data.items() if k in known}
        kw.update(overrides)
        cfg = cls(**kw)
        cfg.extra = {k: v for k, v in data.items() if k not in known}
        return cfg

    @classmethod
    def from_hf_export(cls, export_dir: str | Path, schedule: str | Path | None = None, *,
                       physical: bool = True, packed: bool = False) -> "CompressLMConfig":
        """Read ``compresslm_config.json`` of an HF export; with a schedule file, per-layer quotas
        (physical quota groups by default) or, with packed=True, packed per-head quotas."""
        data = json.loads((Path(export_dir) / "compresslm_config.json").read_text())
        overrides: dict = {}
        if schedule is not None:
            if packed:
                overrides.update(packed_kv=True, packed_kv_quotas=load_quota_rows(schedule),
                                 packed_kv_k_max=int(data.get("num_code_tokens", 128)))
            else:
                overrides.update(layer_code_quotas=load_layer_quotas(schedule), physical_layer_quotas=physical)
        return cls.from_dict(data, **overrides)

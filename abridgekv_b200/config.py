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
import re
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


_LAYER_TOKEN = re.compile(r"\.layers\.([^.]*)")


def layer_index(layer_name: str) -> int | None:
    """n of an attention layer named '....layers.n....' (the token after the first '.layers.'; None
    when there is none or it is not a number)."""
    m = _LAYER_TOKEN.search(layer_name)
    return int(m.group(1)) if m and m.group(1).isdecimal() else None


def _pow2_or_zero(n: int) -> bool:
    # the power-of-two test the geometry uses: n & (n - 1) clears the lowest set bit
    return (n & (n - 1)) == 0


def _first_violation(items, bad, message) -> str | None:
    """message(index, item) of the first item for which bad(item) holds, else None."""
    for i, item in enumerate(items):
        if bad(item):
            return message(i, item)
    return None


def _packed_rows_violation(c: "CompressLMConfig") -> str | None:
    for layer, row in enumerate(c.packed_kv_quotas):
        if not row:
            return f"packed_kv_quotas[{layer}] must not be empty"
        msg = _first_violation(row, lambda q: not 0 < q <= c.packed_kv_k_max,
                               lambda h, q: f"packed_kv_quotas[{layer}][{h}]={q} must be in [1, {c.packed_kv_k_max}]")
        if msg:
            return msg
    return None


# Validation of an enabled configuration, in the order the overlay's CompressLMConfig reports the
# first problem (vllm/config/compresslm.py:76-190): each rule returns its message when violated.
# The geometry comes first, then what vLLM serving supports, then per-layer and packed quotas.
_ENABLED_RULES: tuple = (
    lambda c: None if (_pow2_or_zero(c.block_size) and _pow2_or_zero(c.num_code_tokens) and not c.replay_tail
                       and not c.raw_tail and c.num_passes == 1) or c.code_positions != "bitrev" else
    "code_positions=bitrev needs power-of-two block_size and num_code_tokens, no replay/raw tail and num_passes=1",
    lambda c: None if c.block_size > 0 else "block_size must be positive",
    lambda c: None if c.num_code_tokens > 0 else "num_code_tokens must be positive",
    lambda c: None if 0 <= c.replay_tail <= c.block_size else "replay_tail must be in [0, block_size]",
    lambda c: None if 0 <= c.retain_tail_kv < c.block_size else "retain_tail_kv must be in [0, block_size)",
    lambda c: None if c.retain_tail_policy != "sticky" or c.retain_tail_kv else
    "retain_tail_policy='sticky' requires retain_tail_kv > 0",
    lambda c: None if np.count_nonzero([c.raw_tail, c.replay_tail, c.retain_tail_kv]) <= 1 else
    "raw_tail, replay_tail, and retain_tail_kv are mutually exclusive",
    lambda c: None if not c.code_exclude_replay_tail or 0 < c.replay_tail < c.block_size else
    "code_exclude_replay_tail requires replay_tail in [1, block_size)",
    lambda c: None if c.num_passes == 1 else "vLLM CompressLM decoding currently supports L=1 only",
    lambda c: None if c.pause_xattn == "full" else "vLLM CompressLM decoding currently requires pause_xattn='full'",
    lambda c: None if not c.raw_tail else "vLLM CompressLM decoding currently supports raw_tail=0 only",
    lambda c: None if c.raw_prompt else "vLLM CompressLM decoding currently requires raw_prompt=True",
    lambda c: _first_violation(c.layer_code_quotas, lambda q: not 0 < q <= c.num_code_tokens,
                               lambda i, q: f"layer_code_quotas[{i}]={q} must be in [1, {c.num_code_tokens}]"),
    lambda c: None if not c.uses_layer_quotas or c.code_positions == "bitrev" else
    "layer_code_quotas below num_code_tokens need code_positions=bitrev (nested-prefix code layout)",
    lambda c: None if not (c.uses_layer_quotas and c.packed_kv) else
    "layer_code_quotas and packed KV are mutually exclusive",
    lambda c: None if not c.physical_layer_quotas or c.layer_code_quotas else
    "physical_layer_quotas needs layer_code_quotas",
    lambda c: None if not c.packed_kv or not (c.raw_tail or (c.retain_tail_kv and c.retain_tail_policy != "static"))
    else "packed KV supports code/replay checkpoints and the static retained tail, not window (rolling/sticky) or "
         "raw tails",
    lambda c: None if not (c.packed_kv and c.code_exclude_replay_tail) else
    "packed KV does not yet support code_exclude_replay_tail",
    lambda c: None if not c.packed_kv or c.packed_kv_k_max == c.num_code_tokens else
    "packed_kv_k_max must equal num_code_tokens so the dense code pass computes every schedulable slot",
    lambda c: None if not c.packed_kv or c.packed_kv_k_max > 0 else "packed_kv_k_max must be positive",
    lambda c: _packed_rows_violation(c) if c.packed_kv else None,
)


@dataclass
class CompressLMConfig:
    """The geometry of a CompressLM deployment (field names and defaults of the overlay's class).

    Construction normalises the quota fields to int tuples, checks the two enumerations always and,
    when ``enable`` is set, runs ``_ENABLED_RULES`` in order: the first violated rule raises
    ``ValueError`` with its message."""

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
        self.packed_kv_quotas = tuple(map(lambda row: tuple(map(int, row)), self.packed_kv_quotas))
        self.layer_code_quotas = tuple(map(int, self.layer_code_quotas))
        if self.retain_tail_policy not in _POLICIES:
            raise ValueError("retain_tail_policy must be one of: rolling, sticky, static")
        if self.code_positions not in ("appended", "bitrev"):
            raise ValueError("code_positions must be appended or bitrev")
        if self.enable:
            for rule in _ENABLED_RULES:
                msg = rule(self)
                if msg:
                    raise ValueError(msg)

    # ---- quota views -------------------------------------------------------------------
    @property
    def code_excluded_tail(self) -> int:
        """Content rows at the end of a block the codes do not summarise (and a code step hides)."""
        return self.replay_tail if self.code_exclude_replay_tail else self.retain_tail_kv

    @property
    def uses_layer_quotas(self) -> bool:
        """Some layer sees fewer code slots than the cache holds."""
        return min(self.layer_code_quotas, default=self.num_code_tokens) < self.num_code_tokens

    @property
    def uses_physical_layer_quotas(self) -> bool:
        return self.uses_layer_quotas and bool(self.physical_layer_quotas)

    @property
    def uses_packed_kv(self) -> bool:
        return bool(self.packed_kv)

    def layer_quota(self, layer: int) -> int:
        """Code slots visible at `layer` (all K past the end of the schedule)."""
        table = self.layer_code_quotas
        return table[layer] if 0 <= layer < len(table) else self.num_code_tokens

    @property
    def distinct_layer_quotas(self) -> tuple[int, ...]:
        return tuple(np.unique(np.asarray(self.layer_code_quotas, dtype=np.int64)).tolist())

    def kv_group_quotas(self, group_layer_names: Sequence[Sequence[str]]) -> tuple[int, ...]:
        """The code quota of every KV-cache group; each group must hold layers of a single quota."""
        quotas = []
        for names in group_layer_names:
            indices = [layer_index(n) for n in names]
            missing = [n for n, i in zip(names, indices) if i is None]
            if missing:
                raise ValueError(f"physical per-layer quotas need indexed attention layers; got {missing[0]!r}")
            found = sorted({self.layer_quota(i) for i in indices})
            if len(found) != 1:
                raise ValueError(f"KV cache group mixes code quotas {found}: {list(names)}")
            quotas.append(found[0])
        return tuple(quotas)

    # ---- code RoPE layout --------------------------------------------------------------
    def bitrev_code_offsets(self) -> np.ndarray:
        """In-block RoPE offset of each code row k: (k with its log2 K bits reversed) x span // K, where
        span = C minus the tail the codes do not summarise."""
        K = self.num_code_tokens
        span = self.block_size - self.code_excluded_tail
        if span < K:
            raise ValueError(f"bitrev code span {span} < num_code_tokens {K}")
        width = K.bit_length() - 1
        reversed_index = np.array([int(np.binary_repr(k, width=width)[::-1] or "0", 2) for k in range(K)],
                                  dtype=np.int64)
        return reversed_index * span // K

    def bitrev_rope_positions(self, logical) -> np.ndarray:
        """RoPE positions of logical sequence positions (period C + K per block) under the bitrev layout:
        content row j of block b at b*C + j, code row k at b*C + bitrev offset(k)."""
        C, K = self.block_size, self.num_code_tokens
        logical = np.asarray(logical, dtype=np.int64)
        blk, within = np.divmod(logical, C + K)
        code_offset = self.bitrev_code_offsets()[np.clip(within - C, 0, K - 1)]
        return blk * C + np.where(within < C, within, code_offset)

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

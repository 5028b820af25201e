"""CompressLMConfig and the schedule readers against the reference's own classes run on the same
inputs (tests/golden/config_reference.json, made by make_golden.py --only config): validation
outcomes and messages, bitrev RoPE layout, KV-group quotas, the reference's schedule files; then the
HF-export loader and the adapters to this package's kernels."""
import json
from pathlib import Path

import numpy as np
import pytest

from abridgekv_b200.config import CompressLMConfig, layer_index, load_layer_quotas, load_quota_rows

GOLD = json.loads((Path(__file__).resolve().parent / "golden" / "config_reference.json").read_text())


@pytest.mark.parametrize("i", range(len(GOLD["validation"])))
def test_validation_matches_reference(i):
    case = GOLD["validation"][i]
    kw = dict(case["kwargs"])
    if "packed_kv_quotas" in kw:
        kw["packed_kv_quotas"] = tuple(tuple(r) for r in kw["packed_kv_quotas"])
    if "layer_code_quotas" in kw:
        kw["layer_code_quotas"] = tuple(kw["layer_code_quotas"])
    if case["error"] is None:
        CompressLMConfig(**kw)
    else:
        with pytest.raises(ValueError) as e:
            CompressLMConfig(**kw)
        assert str(e.value) == case["error"]


@pytest.mark.parametrize("i", range(len(GOLD["bitrev"])))
def test_bitrev_layout_matches_reference(i):
    case = GOLD["bitrev"][i]
    c = CompressLMConfig(block_size=case["C"], num_code_tokens=case["K"], **({"replay_tail": 0} | case["kwargs"]))
    assert c.bitrev_code_offsets().tolist() == case["offsets"]
    assert c.bitrev_rope_positions(case["logical"]).tolist() == case["positions"]


@pytest.mark.parametrize("i", range(len(GOLD["groups"])))
def test_kv_group_quotas_match_reference(i):
    case = GOLD["groups"][i]
    c = CompressLMConfig(enable=True, block_size=512, num_code_tokens=case["K"], replay_tail=0,
                         code_positions="bitrev", layer_code_quotas=tuple(case["layer_code_quotas"]),
                         physical_layer_quotas=True)
    if case["error"] is None:
        assert list(c.kv_group_quotas(case["names"])) == case["result"]
    else:
        with pytest.raises(ValueError) as e:
            c.kv_group_quotas(case["names"])
        assert str(e.value) == case["error"]


@pytest.mark.parametrize("name", sorted(GOLD["schedules"]))
def test_schedule_readers_match_reference(name, tmp_path):
    rec = GOLD["schedules"][name]
    f = tmp_path / name
    f.write_text(json.dumps(rec["payload"]))
    if "rows" in rec:
        assert [list(r) for r in load_quota_rows(f)] == rec["rows"]
    else:
        with pytest.raises(ValueError) as e:
            load_quota_rows(f)
        assert str(e.value).replace(str(f), "<path>") == rec["rows_error"]
    if "layer_quotas" in rec:
        assert list(load_layer_quotas(f)) == rec["layer_quotas"]
    else:
        with pytest.raises(ValueError) as e:
            load_layer_quotas(f)
        assert str(e.value).replace(str(f), "<path>") == rec["layer_error"]


def test_layer_index():
    assert layer_index("model.layers.12.self_attn.attn") == 12
    assert layer_index("model.layers.x.attn") is None
    assert layer_index("lm_head") is None


def test_hf_export_with_schedule_to_kernel_inputs(tmp_path):
    """compresslm_config.json as the HF export writes it + the per-layer schedule -> quota groups for
    the decode launches, one CompressMask per layer for the prefill, the packed layout."""
    meta = {"enable": True, "block_size": 512, "num_code_tokens": 256, "num_passes": 1, "pause_xattn": "full",
            "raw_prompt": True, "raw_tail": 0, "replay_tail": 0, "code_positions": "bitrev", "retain_tail_kv": 0,
            "retain_tail_policy": "rolling", "code_exclude_replay_tail": False,
            "code_token_format": "<|compress_code_{:03d}|>"}
    (tmp_path / "compresslm_config.json").write_text(json.dumps(meta))
    rows = GOLD["schedules"]["sched_trunc_perlayer_mean128.json"]["rows"]
    (tmp_path / "sched.json").write_text(json.dumps(rows))
    cfg = CompressLMConfig.from_hf_export(tmp_path, tmp_path / "sched.json")
    assert cfg.uses_physical_layer_quotas and cfg.extra["code_token_format"] == meta["code_token_format"]
    groups = cfg.decode_groups(len(rows))
    assert sorted(groups) == sorted(set(r[0] for r in rows))
    assert sorted(l for ls in groups.values() for l in ls) == list(range(len(rows)))
    for q, ls in groups.items():
        assert all(rows[l][0] == q for l in ls)
    m = cfg.prefill_mask(3, num_q_heads=32)
    assert (m.C, m.K_layout) == (512, 256) and m.quota_per_head == [rows[3][0]] * 32
    packed = CompressLMConfig.from_hf_export(tmp_path, tmp_path / "sched.json", packed=True)
    layout = packed.packed_layout(num_layers=len(rows), num_kv_heads=len(rows[0]))
    assert layout.quotas == tuple(tuple(r) for r in rows) and layout.k_max == 256
    assert layout.packed_slots_per_layer == tuple(sum(r) for r in rows)

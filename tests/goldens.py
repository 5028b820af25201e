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

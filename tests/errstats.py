"""Error statistics the parity tests report and bound.

For a kernel result ``got`` against a reference ``ref`` (float64 truth or the
reference implementation's own output):

* ``max_abs``  = max |got - ref|
* ``mean_abs`` = mean |got - ref|
* ``rel_max``  = max |got - ref| / max |ref|  (error relative to the output's scale)
* ``rel_median`` = median over elements of |got - ref| / max(|ref|, 1e-2 max |ref|)
  (per-element relative error; the floor keeps outputs that cancel to ~0 from
  dominating)

Relative bounds (bf16 outputs, whose own rounding is 2^-9 relative): the
reference's bf16-score arithmetic reaches rel_max 2.2e-2 and rel_median 5.1e-3
against float64 on the golden cases, so a kernel result must satisfy
rel_max <= REL_MAX and rel_median <= REL_MEDIAN against float64.
"""
from __future__ import annotations

import numpy as np

REL_MAX = 2e-2
REL_MEDIAN = 8e-3


def err_stats(got, ref) -> dict:
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    d = np.abs(got - ref)
    scale = float(np.abs(ref).max()) if ref.size else 0.0
    if scale == 0.0:
        scale = 1.0
    rel = d / np.maximum(np.abs(ref), 1e-2 * scale)
    return {"max_abs": float(d.max()) if d.size else 0.0, "mean_abs": float(d.mean()) if d.size else 0.0,
            "rel_max": float(d.max() / scale) if d.size else 0.0,
            "rel_median": float(np.median(rel)) if d.size else 0.0}


def fmt(s: dict) -> str:
    return (f"max_abs={s['max_abs']:.3e} mean_abs={s['mean_abs']:.3e} rel_max={s['rel_max']:.3e} "
            f"rel_median={s['rel_median']:.3e}")


def report(tag: str, got, exact, ref=None) -> tuple[dict, dict | None]:
    """Print the statistics of ``got`` vs float64 ``exact`` (and vs the reference's own output
    ``ref`` when given); -> (stats vs exact, stats vs ref or None)."""
    se = err_stats(got, exact)
    sr = err_stats(got, ref) if ref is not None else None
    line = f"{tag}: vs f64 {fmt(se)}"
    if sr is not None:
        line += f" | vs reference {fmt(sr)}"
    print(line)
    return se, sr


def assert_relative(s: dict, tag: str = "") -> None:
    assert s["rel_max"] <= REL_MAX, (tag, s)
    assert s["rel_median"] <= REL_MEDIAN, (tag, s)

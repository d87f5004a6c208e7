"""Parity metrics of the reference's tests/parity.py:28-44 (relative RMS, max abs, cosine) and
its per-token top-k set comparison (:80-86)."""
from __future__ import annotations

import numpy as np


def compare(ref: np.ndarray, got: np.ndarray) -> dict:
    a = np.asarray(ref, dtype=np.float64).reshape(-1)
    b = np.asarray(got, dtype=np.float64).reshape(-1)
    d = a - b
    ref2 = float((a * a).sum())
    rel = float(np.sqrt((d * d).sum() / ref2)) if ref2 > 0 else float(np.sqrt((d * d).sum()))
    na, nb = float((a * a).sum()), float((b * b).sum())
    cos = float((a * b).sum() / np.sqrt(na * nb)) if na > 0 and nb > 0 else 1.0
    return {"elements": int(a.size), "rel_rms": rel, "max_abs": float(np.abs(d).max()) if a.size else 0.0, "cosine": cos}


def topk_sets(ref_ids: np.ndarray, got_ids: np.ndarray) -> dict:
    """Top-k compared as per-token sets: the order within the top-k is not meaningful."""
    same = sum(set(r.tolist()) == set(g.tolist()) for r, g in zip(ref_ids, got_ids))
    return {"tokens": int(len(ref_ids)), "identical_sets": int(same), "flips": int(len(ref_ids) - same)}

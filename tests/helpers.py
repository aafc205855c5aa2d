"""Shared helpers for the parity tests."""

from __future__ import annotations

import numpy as np


def rel_l2(a, b, floor: float = 0.0) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = max(float(np.linalg.norm(b)), floor, 1e-300)
    return float(np.linalg.norm(a - b) / den)


def per_tensor_rel(table, got, ref, floor_frac: float = 1e-3, trainable_only: bool = True):
    """rel-L2 per parameter tensor. The denominator is floored at
    floor_frac * ||ref|| / sqrt(#tensors): conv biases that feed an instance
    norm have an exactly-zero true gradient, so their own norm is rounding noise."""
    ents = [e for e in table if (e["trainable"] or not trainable_only)]
    tot = float(np.linalg.norm(np.asarray(ref, np.float64)))
    floor = floor_frac * tot / np.sqrt(max(len(ents), 1))
    out = {}
    for e in ents:
        s = slice(e["offset"], e["offset"] + e["numel"])
        out[e["name"]] = rel_l2(got[s], ref[s], floor)
    return out


def random_params(table, n, seed, lo=-0.3, hi=0.3):
    rng = np.random.default_rng(seed)
    p = np.zeros(n, np.float64)
    for e in table:
        s = slice(e["offset"], e["offset"] + e["numel"])
        if ".alpha" in e["name"]:
            p[s] = rng.uniform(0.5, 1.5, e["numel"])
        else:
            p[s] = rng.uniform(lo, hi, e["numel"])
    return p

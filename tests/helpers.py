"""Shared helpers for the parity tests: golden-vector loading and the
mismatch classification of the parity contract.

A GPU token that differs from an oracle token is accepted only when the
difference is explained by one of two documented causes:

* tie order -- the reference orders equal-valued candidates through
  libstdc++'s nth_element/sort (src/sampling.cc:95-104); the engine and the
  canonical oracle order them by token id.  The two tokens then have the
  same transformed value.
* draw boundary -- the uniform draw lies within 1e-6 (relative to the
  total) of a cumulative-probability boundary, or the top-p running sum lies
  within 1e-6 of top_p.
"""
from __future__ import annotations

import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
BOUNDARY_TOL = 1e-6


def load_cases():
    with open(os.path.join(GOLDEN, "reference_cases.json")) as f:
        return json.load(f)["cases"]


def load_sequences():
    with open(os.path.join(GOLDEN, "reference_sequences.json")) as f:
        return {s["name"]: s for s in json.load(f)["sequences"]}


def hex_to_bf16(h: str) -> np.ndarray:
    return np.frombuffer(bytes.fromhex(h), dtype=">u2").astype(np.uint16)


def is_boundary(res, top_p: float, tol: float = BOUNDARY_TOL) -> bool:
    """res: oracle RowResult with candidate weights.  True when the draw or
    the top-p cut sits within `tol` of a boundary."""
    w = np.asarray(res.cand_weights, dtype=np.float64)
    if res.status != 0 or w.size == 0:
        return False
    total_all = res.total_all
    if top_p < 1.0:
        cum = np.cumsum(w / total_all)
        if np.any(np.abs(cum - np.float64(np.float32(top_p))) <= tol):
            return True
    s = np.cumsum(w[: res.n_retained])
    return bool(np.any(np.abs(s - res.draw) <= tol * res.total))


def transformed_value(res, token: int):
    """Value of `token` in an oracle candidate list (None if absent)."""
    idx = np.nonzero(res.cand_tokens == token)[0]
    return None if idx.size == 0 else float(res.cand_values[idx[0]])

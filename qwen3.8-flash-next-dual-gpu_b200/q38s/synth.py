"""Seeded synthetic inputs for the five benchmark configurations.

The reference publishes no sampler dataset; its benchmark configurations
describe logit distributions only.  These generators fix every detail the
configurations leave open (seed derivation, spike placement and magnitude),
so the GPU engine, the CPU oracle and the reference build all see the same
bytes.  Generation is host-side numpy (PCG64) so a run is reproducible
without a GPU.

Distributions:
  cfg1  1 row fp32 ~N(0, 2.5^2); 32 spikes at distinct uniform indices set to
        U[8, 15]; logits regenerated from (seed + step); 4,096-token uniform
        history.
  cfg2  same row distribution in bf16; history grows from 8,192 tokens.
  cfg3  65 target rows fp32 ~N(0, 3^2) + 16 spikes U[8, 15] per row; draft
        rows = target + N(0, 0.5^2).
  cfg4  256 rows bf16 ~N(0, 2.5^2) + 32 spikes per row at distinct uniform
        indices; spike of Zipf rank r (r = 1..32) has logit 15 - 1.1 ln r,
        i.e. spike probabilities follow Zipf(s = 1.1).  Per-row parameters:
        T ~ U[0.3, 1.2]; top_k = 0 with probability 1/4 else U{1..100};
        top_p ~ U[0.5, 1.0]; min_p ~ U[0, 0.1]; repetition ~ U[1.0, 1.2];
        history length U{1..32,768} uniform tokens.
  cfg5  1,024 rows fp32 with the cfg4 row distribution (cfg5_row: each row
        from its own seed); T 0.8, top_k 64 per shard, top_p 0.9, repetition
        1.1, 1,024-token history per row.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

VOCAB = 151_936
GAMMA = 0x9E3779B97F4A7C15
MASK64 = (1 << 64) - 1


def f32_to_bf16_rne(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 words, round-to-nearest-even on the bit pattern."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_to_f32(w: np.ndarray) -> np.ndarray:
    return (np.asarray(w, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def _gauss_row(rng: np.random.Generator, n: int, sigma: float) -> np.ndarray:
    return rng.standard_normal(n, dtype=np.float32) * np.float32(sigma)


def uniform_spikes(rng, row: np.ndarray, count: int, lo: float = 8.0, hi: float = 15.0):
    idx = rng.choice(row.size, count, replace=False)
    row[idx] = rng.uniform(lo, hi, count).astype(np.float32)
    return idx


def zipf_spikes(rng, row: np.ndarray, count: int = 32, top: float = 15.0, s: float = 1.1):
    idx = rng.choice(row.size, count, replace=False)
    ranks = np.arange(1, count + 1, dtype=np.float64)
    row[idx] = (top - s * np.log(ranks)).astype(np.float32)
    return idx


# ---------------------------------------------------------------- cfg 1
CFG1 = dict(top_k=20, top_p=0.8, temperature=0.7, repetition_penalty=1.05, seed=1234)


def cfg1_history(seed: int = 1234, vocab: int = VOCAB, n: int = 4096) -> np.ndarray:
    return np.random.default_rng([seed, 0x4157]).integers(0, vocab, n).astype(np.int32)


def cfg1_logits(step: int, seed: int = 1234, vocab: int = VOCAB) -> np.ndarray:
    rng = np.random.default_rng(seed + step)
    row = _gauss_row(rng, vocab, 2.5)
    uniform_spikes(rng, row, 32)
    return row


# ---------------------------------------------------------------- cfg 2
CFG2 = dict(top_k=20, top_p=0.95, min_p=0.0, temperature=0.6, presence_penalty=0.5, seed=2)


def cfg2_history(seed: int = 2, vocab: int = VOCAB, n: int = 8192) -> np.ndarray:
    return np.random.default_rng([seed, 0x4157]).integers(0, vocab, n).astype(np.int32)


def cfg2_logits(step: int, seed: int = 2, vocab: int = VOCAB) -> np.ndarray:
    rng = np.random.default_rng([seed, step])
    row = _gauss_row(rng, vocab, 2.5)
    uniform_spikes(rng, row, 32)
    return f32_to_bf16_rne(row)


# ---------------------------------------------------------------- cfg 3
CFG3 = dict(top_k=20, top_p=0.95, temperature=0.7, seed=3)


def cfg3_rows(seed: int = 3, rows: int = 65, vocab: int = VOCAB):
    """Returns (target fp32 [rows, V], draft fp32 [rows, V])."""
    rng = np.random.default_rng([seed, 0x3])
    target = np.empty((rows, vocab), np.float32)
    for r in range(rows):
        target[r] = _gauss_row(rng, vocab, 3.0)
        uniform_spikes(rng, target[r], 16)
    draft = target + rng.standard_normal((rows, vocab), dtype=np.float32) * np.float32(0.5)
    return target, draft


# ---------------------------------------------------------------- cfg 4
@dataclass
class BatchSpec:
    rows: int
    vocab: int
    top_k: np.ndarray
    top_p: np.ndarray
    min_p: np.ndarray
    temperature: np.ndarray
    repetition_penalty: np.ndarray
    frequency_penalty: np.ndarray
    presence_penalty: np.ndarray
    seed: np.ndarray
    histories: list = field(default_factory=list)


def cfg4_spec(seed: int = 4, rows: int = 256, vocab: int = VOCAB,
              max_history: int = 32_768) -> BatchSpec:
    rng = np.random.default_rng([seed, 0x5BEC])
    top_k = rng.integers(1, 101, rows).astype(np.uint32)
    top_k[rng.random(rows) < 0.25] = 0
    spec = BatchSpec(
        rows=rows, vocab=vocab, top_k=top_k,
        top_p=rng.uniform(0.5, 1.0, rows).astype(np.float32),
        min_p=rng.uniform(0.0, 0.1, rows).astype(np.float32),
        temperature=rng.uniform(0.3, 1.2, rows).astype(np.float32),
        repetition_penalty=rng.uniform(1.0, 1.2, rows).astype(np.float32),
        frequency_penalty=np.zeros(rows, np.float32),
        presence_penalty=np.zeros(rows, np.float32),
        seed=rng.integers(1, 2**63, rows, dtype=np.uint64),
    )
    lens = rng.integers(1, max_history + 1, rows)
    spec.histories = [rng.integers(0, vocab, n).astype(np.int32) for n in lens]
    return spec


def cfg4_logits(batch: int = 0, seed: int = 4, rows: int = 256, vocab: int = VOCAB,
                dtype: str = "bf16") -> np.ndarray:
    rng = np.random.default_rng([seed, 0x10, batch])
    out = _gauss_row(rng, rows * vocab, 2.5).reshape(rows, vocab)
    for r in range(rows):
        zipf_spikes(rng, out[r])
    return f32_to_bf16_rne(out) if dtype == "bf16" else out


# ---------------------------------------------------------------- cfg 5
CFG5 = dict(top_k=64, top_p=0.9, temperature=0.8, repetition_penalty=1.1)


def cfg5_spec(seed: int = 5, rows: int = 1024, vocab: int = VOCAB, history: int = 1024):
    rng = np.random.default_rng([seed, 0x5BEC])
    spec = BatchSpec(
        rows=rows, vocab=vocab, top_k=np.full(rows, 64, np.uint32),
        top_p=np.full(rows, 0.9, np.float32), min_p=np.zeros(rows, np.float32),
        temperature=np.full(rows, 0.8, np.float32),
        repetition_penalty=np.full(rows, 1.1, np.float32),
        frequency_penalty=np.zeros(rows, np.float32),
        presence_penalty=np.zeros(rows, np.float32),
        seed=rng.integers(1, 2**63, rows, dtype=np.uint64))
    spec.histories = [rng.integers(0, vocab, history).astype(np.int32) for _ in range(rows)]
    return spec


def cfg5_logits(seed: int = 5, rows: int = 1024, vocab: int = VOCAB, batch: int = 0):
    return cfg4_logits(batch=batch, seed=seed, rows=rows, vocab=vocab, dtype="f32")


def cfg5_row(r: int, seed: int = 5, vocab: int = VOCAB) -> np.ndarray:
    """Row r of the vocab-parallel benchmark, generated on its own (so a rank
    can build its column shard and a checker any single row): fp32
    N(0, 2.5^2) with the Zipf(1.1)-ranked spikes of the cfg4 distribution."""
    rng = np.random.default_rng([seed, 0x55, r])
    row = _gauss_row(rng, vocab, 2.5)
    zipf_spikes(rng, row)
    return row

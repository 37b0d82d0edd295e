"""GPU parity for the streaming sampler's less common paths: rows whose
penalties can raise a value together with this call's extra tokens, one-row
batches split into many column segments (the segment merge), rows read
through a misaligned pointer with a padded row stride, and units too wide
to stream (the general path).  Same bar as test_gpu_parity: tokens and
candidate sets bit-exact against the canonical oracle, probabilities within
1e-6 relative, boundary draws counted.
"""
import numpy as np
import pytest

import oracle as O
import q38s
from helpers import is_boundary
from q38s import synth
from test_gpu_parity import PROB_RTOL, check_batch, oracle_params, to_torch

pytestmark = pytest.mark.gpu


def spiked_rows(rng, rows, vocab, spikes=32):
    x = rng.normal(0, 2.5, (rows, vocab)).astype(np.float32)
    for r in range(rows):
        idx = rng.choice(vocab, spikes, replace=False)
        x[r, idx] = rng.uniform(6, 14, spikes)
    return x


def test_negative_penalties_with_extra_tokens(cuda):
    """Negative presence / frequency penalties raise penalised values, so
    penalised elements below the raw bound are evaluated as well: the
    history bitmap and this call's extra tokens (duplicates, tokens already
    in the history, tokens with low logits)."""
    rng = np.random.default_rng(71)
    vocab, rows = 20000, 12
    configs = []
    for r in range(rows):
        configs.append(q38s.config_v2(
            top_k=[1, 5, 20, 64, 100, 256, 0, 20, 40, 3, 128, 10][r],
            top_p=[0.9, 1.0, 0.8, 0.95, 0.7, 0.9, 0.9, 0.5, 1.0, 0.9, 0.99, 0.6][r],
            min_p=[0.0, 0.0, 0.05, 0.0, 0.02, 0.01, 0.1, 0.0, 0.0, 0.0, 0.03, 0.0][r],
            temperature=[0.7, 1.0, 0.5, 1.3, 0.9, 0.8, 1.1, 0.6, 1.0, 0.4, 0.9, 1.2][r],
            repetition_penalty=[1.0, 1.1, 1.3, 1.0, 1.05, 1.2, 1.0, 1.1, 1.0, 1.3, 1.0, 1.1][r],
            presence_penalty=[-0.5, -1.0, 0.0, -2.0, -0.3, 0.0, -0.8, -1.5, -0.1, -3.0, -0.2, 0.5][r],
            frequency_penalty=[0.0, -0.2, -0.5, 0.0, -0.1, -0.3, 0.0, -0.4, 0.0, 0.0, -0.05, -0.6][r],
            seed=int(rng.integers(1, 2**63))))
    x = rng.normal(0, 2.5, (rows, vocab)).astype(np.float32)
    logits = synth.f32_to_bf16_rne(x)
    low = np.argsort(x, axis=1)  # ascending: the first columns have the lowest logits
    hists, extra = [], []
    for r in range(rows):
        h = np.concatenate([rng.integers(0, vocab, 200), low[r, :50]]).astype(np.int32)
        hists.append(h)
        e = np.concatenate([low[r, 40:80], low[r, 60:70], h[:5], rng.integers(0, vocab, 20)])
        extra.append(e.astype(np.int32))
    assert check_batch(configs, logits, hists, cuda, extra=extra) == 0


@pytest.mark.parametrize("k,min_p,top_p", [(1, 0.0, 1.0), (2, 0.0, 0.9), (20, 0.0, 0.95),
                                           (64, 0.0, 0.9), (100, 0.02, 0.9), (128, 0.0, 1.0),
                                           (256, 0.0, 0.8), (0, 0.05, 0.9), (0, 0.001, 1.0)])
@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_single_row_segment_merge(k, min_p, top_p, dtype, cuda):
    """A one-row batch is split into up to 64 column segments; the last one
    to finish merges the parked lists (bounds from the lists' k-th and
    first two entries, remainders read only where they can qualify)."""
    rng = np.random.default_rng(1000 + k + int(min_p * 1000) + (dtype == "f32"))
    vocab = synth.VOCAB
    x = spiked_rows(rng, 1, vocab)
    if k == 64:
        x = np.round(x * 2) / 2  # heavy ties at the cut
    logits = synth.f32_to_bf16_rne(x) if dtype == "bf16" else x
    cfg = q38s.config_v2(top_k=k, top_p=top_p, min_p=min_p, temperature=0.8,
                         repetition_penalty=1.1, presence_penalty=0.3,
                         seed=int(rng.integers(1, 2**63)))
    hists = [rng.integers(0, vocab, 5000).astype(np.int32)]
    assert check_batch([cfg], logits, hists, cuda) == 0


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_misaligned_strided_rows(dtype, cuda):
    """Logits that start one element past a 16-byte boundary, rows padded
    to a stride that is not a multiple of 16 bytes: no bulk copies, the
    consumers fill the tiles and the second reads use scalar loads."""
    import torch
    rng = np.random.default_rng(5 + (dtype == "f32"))
    rows, vocab, pad = 6, 50000, 5
    x = spiked_rows(rng, rows, vocab)
    logits = synth.f32_to_bf16_rne(x) if dtype == "bf16" else x
    configs = [q38s.config_v2(top_k=[20, 1, 100, 0, 64, 7][r], top_p=0.9,
                              min_p=[0.0, 0.0, 0.0, 0.05, 0.01, 0.0][r], temperature=0.9,
                              repetition_penalty=1.2, frequency_penalty=0.1,
                              seed=int(rng.integers(1, 2**63))) for r in range(rows)]
    hists = [rng.integers(0, vocab, 3000).astype(np.int32) for _ in range(rows)]
    stride = vocab + pad
    buf = np.zeros(1 + rows * stride, logits.dtype)
    for r in range(rows):
        buf[1 + r * stride: 1 + r * stride + vocab] = logits[r]
    t = to_torch(buf, cuda)[1:]  # one element past the allocation's alignment
    b = q38s.Batch(vocab, configs)
    assert (b.commit_tokens(hists) == 0).all()
    cap = 1024
    dist, dt = q38s.make_distribution(rows, cap, cuda)
    dec = b.decode_decisions(b.prepare(t, dist=dist, row_stride=stride))
    torch.cuda.synchronize()
    ntok = dt["n_candidates"].cpu().numpy()
    gtok = dt["tokens"].cpu().numpy().reshape(rows, cap)
    gprob = dt["probs"].cpu().numpy().reshape(rows, cap)
    nret = dt["n_retained"].cpu().numpy()
    for r in range(rows):
        counts = np.bincount(hists[r], minlength=vocab).astype(np.uint32)
        o = O.prepare_row(oracle_params(configs[r], configs[r].seed), logits[r], counts, (),
                          O.TIE_CANONICAL, cap=cap)
        assert o.status == 0 and dec["status"][r] == 0
        assert dec["token"][r] == o.token or is_boundary(o, configs[r].top_p), f"row {r}"
        n = o.n_candidates
        assert ntok[r] == n
        assert (gtok[r, :n] == o.cand_tokens[:n]).all(), f"row {r}: top-k set"
        rr = o.n_retained
        assert nret[r] == rr
        np.testing.assert_allclose(gprob[r, :rr], o.cand_weights[:rr] / o.total,
                                   rtol=PROB_RTOL, atol=0)


def test_wide_unit_takes_general_path(cuda):
    """A bf16 row of 480,000 columns has more tiles than the area holds
    bounds for, so its unit is not streamed: the general path samples it."""
    rng = np.random.default_rng(480)
    vocab = 480_000
    x = spiked_rows(rng, 2, vocab, spikes=64)
    logits = synth.f32_to_bf16_rne(x)
    configs = [q38s.config_v2(top_k=20, top_p=0.9, temperature=0.8, repetition_penalty=1.1,
                              seed=11),
               q38s.config_v2(top_k=0, top_p=0.95, min_p=0.05, temperature=1.0, seed=12)]
    hists = [rng.integers(0, vocab, 2000).astype(np.int32) for _ in range(2)]
    assert check_batch(configs, logits, hists, cuda) == 0


@pytest.mark.parametrize("rows", [42, 49, 59, 74, 98])
def test_cluster_sizes_three_to_seven(rows, cuda):
    """Batches of 42, 49, 59, 74 and 98 rows split every row into 7, 6, 5, 4
    and 3 column segments (one cluster per row): headers of 64 // S keys,
    the rank-based merge bound, the leader's reads of every segment's list.
    Mixed top-k (with and without min-p), penalties and temperatures."""
    rng = np.random.default_rng(3000 + rows)
    vocab = 20000
    x = spiked_rows(rng, rows, vocab, spikes=24)
    logits = synth.f32_to_bf16_rne(x)
    ks = [1, 3, 20, 40, 64, 100, 200, 256, 0]
    configs = []
    for r in range(rows):
        k = ks[r % len(ks)]
        configs.append(q38s.config_v2(
            top_k=k, top_p=float(rng.uniform(0.5, 1.0)),
            min_p=0.05 if k == 0 else float(rng.choice([0.0, 0.02])),
            temperature=float(rng.uniform(0.3, 1.2)),
            repetition_penalty=float(rng.uniform(1.0, 1.2)),
            presence_penalty=float(rng.choice([0.0, 0.4])),
            seed=int(rng.integers(1, 2**63))))
    hists = [rng.integers(0, vocab, int(rng.integers(1, 2000))).astype(np.int32)
             for _ in range(rows)]
    assert check_batch(configs, logits, hists, cuda) == 0

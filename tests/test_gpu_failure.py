"""Failure detection on the GPU without a GPU fault.

Every device wait of the sampling kernel is bounded.  These tests make one
run out on purpose through the library's test-only failure injection
(q38s_testing_set_fault): the first CTA of the launch issues no logit copy,
so its consumers wait on a ring barrier that nothing completes, and give up
after a short limit.  Nothing traps and no copy is in flight.  The rows of
that CTA must report Q38S_ROW_TIMEOUT (a one-session prepare returns
Q38S_TIMEOUT), the other rows must be sampled normally, and once the
injection is switched off the library samples every row again.
"""
import numpy as np
import pytest

import oracle as O
import q38s
from helpers import is_boundary
from q38s import synth

pytestmark = pytest.mark.gpu

SHORT_WAIT = 200_000  # cycles, ~0.1 ms: far beyond an arriving copy, far below the default


@pytest.fixture
def fault():
    L = q38s.lib()
    q38s._check(L.q38s_testing_set_fault(1, SHORT_WAIT))
    yield
    q38s._check(L.q38s_testing_set_fault(0, 0))


def _batch(rows, vocab, rng):
    configs = [q38s.config_v2(top_k=20, top_p=0.9, temperature=0.8, repetition_penalty=1.1,
                              seed=int(rng.integers(1, 2**63))) for _ in range(rows)]
    x = synth.f32_to_bf16_rne(rng.normal(0, 2.5, (rows, vocab)).astype(np.float32))
    return configs, x


def _to_torch(x, cuda):
    import torch
    return torch.from_numpy(x.view(np.int16)).to(cuda).view(torch.bfloat16)


def _sample(configs, x, cuda):
    import torch
    b = q38s.Batch(x.shape[1], configs)
    dec = b.decode_decisions(b.prepare(_to_torch(x, cuda)))
    torch.cuda.synchronize()
    return dec


def _check_tokens(configs, x, dec, rows):
    for r in rows:
        c = configs[r]
        p = O.make_params(top_k=c.top_k, top_p=c.top_p, temperature=c.temperature,
                          repetition_penalty=c.repetition_penalty, rng_state=c.seed)
        o = O.prepare_row(p, x[r], None, (), O.TIE_CANONICAL, cap=64)
        assert dec["token"][r] == o.token or is_boundary(o, c.top_p), f"row {r}"


def test_bounded_tile_wait_reports_timeout_then_recovers(cuda):
    """300 rows: one CTA per row slot (296 on a B200), so the first CTA owns
    rows 0 and 296; exactly those time out."""
    rng = np.random.default_rng(606)
    rows, vocab = 300, 20_000
    configs, x = _batch(rows, vocab, rng)
    L = q38s.lib()
    q38s._check(L.q38s_testing_set_fault(1, SHORT_WAIT))
    try:
        dec = _sample(configs, x, cuda)
    finally:
        q38s._check(L.q38s_testing_set_fault(0, 0))
    timed_out = np.flatnonzero(dec["status"] == q38s.ROW_TIMEOUT)
    assert 0 in timed_out
    assert ((dec["status"] == 0) | (dec["status"] == q38s.ROW_TIMEOUT)).all()
    assert (dec["token"][timed_out] == -1).all()
    ok = np.flatnonzero(dec["status"] == 0)
    assert len(ok) >= rows - 4
    _check_tokens(configs, x, dec, ok[::17])
    # the same batch again, injection off: every row is sampled
    dec2 = _sample(configs, x, cuda)
    assert (dec2["status"] == 0).all()
    assert (dec2["token"][ok] == dec["token"][ok]).all()
    _check_tokens(configs, x, dec2, timed_out)


def test_one_session_prepare_returns_timeout_then_recovers(cuda, fault):
    """One row splits over a thread-block cluster; its leader CTA (the
    first) never receives a tile: the call returns Q38S_TIMEOUT."""
    rng = np.random.default_rng(607)
    cfg = q38s.config_v1(top_k=20, top_p=0.95, temperature=0.6, seed=99)
    s = q38s.Sampler(synth.VOCAB, cfg)
    x = synth.f32_to_bf16_rne(rng.normal(0, 2.5, synth.VOCAB).astype(np.float32))
    with pytest.raises(q38s.Q38sError) as ex:
        s.prepare(x)
    assert ex.value.code == q38s.TIMEOUT
    q38s._check(q38s.lib().q38s_testing_set_fault(0, 0))
    tok, rb, ra = s.prepare(x)
    p = O.make_params(top_k=20, top_p=0.95, temperature=0.6, rng_state=99)
    o = O.prepare_row(p, x, None, (), O.TIE_CANONICAL, cap=64)
    assert tok == o.token or is_boundary(o, 0.95)
    assert (rb, ra) == (99, (99 + O.GAMMA) & O.MASK64)

"""Regression test for the speculative-verification ticket.

The verification runs in whichever CTA finishes the last of the 2n + 1
virtual rows (n target rows + the bonus row, n draft rows); it reads every
other row's decision and distribution.  Each row's CTA publishes its row
with one acquire-release ticket increment by thread 0, after a barrier of
all the threads that wrote the row's outputs.  An earlier version had each
thread fence its own writes and thread 0 increment the ticket without that
barrier, so a row's distribution could still be in flight when the
finishing CTA read it (wrong results for the rows that finished last,
depending on launch timing).

The scenarios vary the draft count and the vocabulary, so the rows split
into different numbers of segments (thread-block clusters of 1 to 8 CTAs)
and finish in different orders; each runs several times and must equal the
oracle's rejection sampler every time.
"""
import numpy as np
import pytest

import oracle as O
import q38s
from q38s import synth

pytestmark = pytest.mark.gpu


def _to_device(arr, cuda):
    import torch
    return torch.from_numpy(np.ascontiguousarray(arr)).to(cuda)


@pytest.mark.parametrize("vocab", [30_000, synth.VOCAB])
@pytest.mark.parametrize("n", [1, 7, 36, 64])
def test_verification_reads_complete_rows(n, vocab, cuda):
    import torch
    target, draft = synth.cfg3_rows(seed=700 + n, rows=n + 1, vocab=vocab)
    cfg = q38s.config_v2(top_k=20, top_p=0.95, temperature=0.7, repetition_penalty=1.05,
                         seed=900 + n)
    p = O.make_params(top_k=20, top_p=0.95, temperature=0.7, repetition_penalty=1.05,
                      rng_state=cfg.seed)
    drafts = []
    for i in range(n):
        pi = O.make_params(top_k=20, top_p=0.95, temperature=0.7, repetition_penalty=1.05,
                           rng_state=(cfg.seed * 31 + i) & O.MASK64)
        drafts.append(O.prepare_row(pi, draft[i], extra=drafts, cap=32).token)
    want_toks, want_acc, want_rng, st = O.mtp_verify(p, target, draft[:n], drafts)
    assert st == 0
    b = q38s.Batch(vocab, [cfg])
    t, d = _to_device(target, cuda), _to_device(draft[:n], cuda)
    dt = torch.tensor(drafts, dtype=torch.int32, device=cuda)
    for rep in range(5):
        res = b.decode_mtp(b.mtp_verify(0, t, d, dt))
        assert res.status == 0, f"rep {rep}: status {res.status}"
        assert res.n_accepted == want_acc, f"rep {rep}"
        assert list(res.tokens[: res.n_tokens]) == list(want_toks), f"rep {rep}"
        assert res.rng_after == want_rng

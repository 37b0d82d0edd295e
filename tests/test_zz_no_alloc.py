"""q38s_prepare_noalloc: sampling for callers that may not allocate GPU memory.

Some callers cannot call cudaMalloc at all: code running inside a memory
pool or arena it does not own, a plug-in whose host process forbids device
allocation after start-up, or a latency-critical loop in which an allocation
(and the device-wide synchronisation it may trigger) is not allowed.  For
them q38s_prepare_noalloc keeps every working buffer in one static device
array of the library.  This file checks, through the C ABI, that two calls in
a row return exactly what q38s_batch_prepare returns on a freshly created
batch with the same configurations (the same kernel runs behind both), and
that sizes beyond the static limits are rejected.

It is collected last on purpose, and it sets up everything it uses itself,
so it passes alone in a fresh process as well as after the other tests.
"""
import ctypes as C

import numpy as np
import pytest

import q38s
from q38s import synth

pytestmark = pytest.mark.gpu


def _bind():
    L = q38s.lib()
    P = C.c_void_p
    L.q38s_prepare_noalloc.argtypes = [P, C.c_uint16, C.c_uint32, C.c_uint32, C.c_uint64,
                                       P, P, P, P]
    L.q38s_prepare_noalloc.restype = C.c_int
    return L


def _noalloc(L, logits, configs, rng_states=None, stream=0):
    import torch
    rows, vocab = logits.shape
    cfg_arr = (q38s.ConfigV2 * rows)(*configs)
    st = None
    if rng_states is not None:
        st = (C.c_uint64 * rows)(*[int(x) for x in rng_states])
    dec = torch.zeros(rows * 3, dtype=torch.int64, device=logits.device)
    dtype = q38s.DTYPE_BF16 if logits.dtype == torch.bfloat16 else q38s.DTYPE_F32
    rc = L.q38s_prepare_noalloc(C.c_void_p(logits.data_ptr()), dtype, vocab, rows,
                                logits.stride(0), cfg_arr, st, C.c_void_p(dec.data_ptr()),
                                C.c_void_p(stream))
    return rc, dec


def _reference(configs, logits, rng_states=None):
    """The existing entry point, q38s_batch_prepare, on a new batch.  A row's
    RNG state before its first draw is its seed, so explicit states become
    the seeds of the reference batch."""
    if rng_states is not None:
        configs = [q38s.config_v2(top_k=c.top_k, top_p=c.top_p, temperature=c.temperature,
                                  repetition_penalty=c.repetition_penalty,
                                  frequency_penalty=c.frequency_penalty,
                                  presence_penalty=c.presence_penalty, min_p=c.min_p,
                                  seed=int(s)) for c, s in zip(configs, rng_states)]
    b = q38s.Batch(logits.shape[1], configs)
    return b.decode_decisions(b.prepare(logits))


def _configs():
    return [q38s.config_v2(top_k=20, top_p=0.9, temperature=0.7, repetition_penalty=1.1,
                           seed=11),
            q38s.config_v2(top_k=0, top_p=0.95, temperature=1.0, min_p=0.05, seed=12),
            q38s.config_v2(top_k=0, top_p=0.8, temperature=1.1, seed=13),   # general path
            q38s.config_v2(top_k=1, top_p=1.0, temperature=0.5, presence_penalty=0.3,
                           frequency_penalty=0.2, seed=14)]


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_noalloc_matches_batch_prepare_on_two_calls(dtype, cuda):
    import torch
    L = _bind()
    rng = np.random.default_rng(77)
    configs = _configs()
    for call, states in enumerate([None, [123456789, 2**63 + 5, 42, 987654321987]]):
        x = rng.normal(0, 2.5, (4, synth.VOCAB)).astype(np.float32)
        for r in range(4):
            synth.zipf_spikes(rng, x[r])
        if dtype == "bf16":
            t = torch.from_numpy(synth.f32_to_bf16_rne(x).view(np.int16)).to(cuda).view(
                torch.bfloat16)
        else:
            t = torch.from_numpy(x).to(cuda)
        rc, dec = _noalloc(L, t, configs, states)
        assert rc == 0, L.q38s_last_error().decode()
        got = q38s.Batch.decode_decisions(dec)
        want = _reference(configs, t, states)
        torch.cuda.synchronize()
        assert (got["status"] == 0).all(), f"call {call}: {got['status']}"
        assert (got["token"] == want["token"]).all(), f"call {call}"
        assert (got["rng_before"] == want["rng_before"]).all()
        assert (got["rng_after"] == want["rng_after"]).all()


def test_noalloc_rejects_sizes_beyond_its_static_memory(cuda):
    import torch
    L = _bind()
    t = torch.zeros((5, 1000), dtype=torch.float32, device=cuda)
    rc, _ = _noalloc(L, t, [q38s.config_v2(top_k=5, seed=1)] * 5)
    assert rc == q38s.INVALID_ARGUMENT
    assert "1 to 4 rows" in L.q38s_last_error().decode()
    big = torch.zeros((1, 262145), dtype=torch.float32, device=cuda)
    rc, _ = _noalloc(L, big, [q38s.config_v2(top_k=5, seed=1)])
    assert rc == q38s.INVALID_ARGUMENT
    assert "262,144" in L.q38s_last_error().decode()

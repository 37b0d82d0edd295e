"""q38s_prepare_noalloc: sampling for callers that may not allocate GPU memory.

Some callers cannot call cudaMalloc at all: code running inside a memory
pool or arena it does not own, a plug-in whose host process forbids device
allocation after start-up, or a latency-critical loop in which an allocation
(and the device-wide synchronisation it may trigger) is not allowed.  For
them q38s_prepare_noalloc keeps every working buffer in one static device
array of the library.  This file checks, through the C ABI, that two calls in
a row return what q38s_batch_prepare returns on a freshly created batch with
the same configurations, and the canonical CPU oracle's token (or a counted
draw boundary); that the calls leave the device's free memory unchanged;
that a caller's non-blocking stream orders them; and that sizes beyond the
static limits are rejected.

It is collected last on purpose, and it sets up everything it uses itself,
so it passes alone in a fresh process as well as after the other tests.
"""
import ctypes as C

import numpy as np
import pytest

import oracle as O
import q38s
from helpers import is_boundary
from q38s import synth

pytestmark = pytest.mark.gpu

MAX_VOCAB = 262_144


def _bind():
    L = q38s.lib()
    P = C.c_void_p
    L.q38s_prepare_noalloc.argtypes = [P, C.c_uint16, C.c_uint32, C.c_uint32, C.c_uint64,
                                       P, P, P, P]
    L.q38s_prepare_noalloc.restype = C.c_int
    return L


def _noalloc(L, logits, configs, rng_states=None, stream=0, dec=None):
    import torch
    rows, vocab = logits.shape
    cfg_arr = (q38s.ConfigV2 * rows)(*configs)
    st = None
    if rng_states is not None:
        st = (C.c_uint64 * rows)(*[int(x) for x in rng_states])
    if dec is None:
        dec = torch.zeros(rows * 3, dtype=torch.int64, device=logits.device)
    dtype = q38s.DTYPE_BF16 if logits.dtype == torch.bfloat16 else q38s.DTYPE_F32
    rc = L.q38s_prepare_noalloc(C.c_void_p(logits.data_ptr()), dtype, vocab, rows,
                                logits.stride(0), cfg_arr, st, C.c_void_p(dec.data_ptr()),
                                C.c_void_p(stream))
    return rc, dec


def _with_seeds(configs, rng_states):
    """A row's RNG state before its first draw is its seed, so explicit
    states become the seeds of the comparison batch."""
    if rng_states is None:
        return configs
    return [q38s.config_v2(top_k=c.top_k, top_p=c.top_p, temperature=c.temperature,
                           repetition_penalty=c.repetition_penalty,
                           frequency_penalty=c.frequency_penalty,
                           presence_penalty=c.presence_penalty, min_p=c.min_p, seed=int(s))
            for c, s in zip(configs, rng_states)]


def _batch_prepare(configs, logits, rng_states=None):
    """The existing entry point, q38s_batch_prepare, on a new batch."""
    cfgs = _with_seeds(configs, rng_states)
    b = q38s.Batch(logits.shape[1], cfgs)
    return b.decode_decisions(b.prepare(logits))


def _configs():
    # a top-k row, a min-p row, a top_k = 0 row without min-p (the general
    # path, whose keys and weights fill the static array at V = 262,144) and
    # a greedy-like top_k = 1 row with penalties that have no history to act on
    return [q38s.config_v2(top_k=20, top_p=0.9, temperature=0.7, repetition_penalty=1.1,
                           seed=11),
            q38s.config_v2(top_k=0, top_p=0.95, temperature=1.0, min_p=0.05, seed=12),
            q38s.config_v2(top_k=0, top_p=0.8, temperature=1.1, seed=13),
            q38s.config_v2(top_k=1, top_p=1.0, temperature=0.5, presence_penalty=0.3,
                           frequency_penalty=0.2, seed=14)]


def _logits(rng, rows, vocab, dtype, cuda):
    import torch
    x = rng.normal(0, 2.5, (rows, vocab)).astype(np.float32)
    for r in range(rows):
        synth.zipf_spikes(rng, x[r])
    if dtype == "bf16":
        host = synth.f32_to_bf16_rne(x)
        return host, torch.from_numpy(host.view(np.int16)).to(cuda).view(torch.bfloat16)
    return x, torch.from_numpy(x).to(cuda)


def _check_oracle(configs, host, got, rng_states):
    boundary = 0
    for r, c in enumerate(configs):
        state = c.seed if rng_states is None else int(rng_states[r])
        p = O.make_params(top_k=c.top_k, top_p=c.top_p, min_p=c.min_p,
                          temperature=c.temperature, repetition_penalty=c.repetition_penalty,
                          frequency_penalty=c.frequency_penalty,
                          presence_penalty=c.presence_penalty, rng_state=state)
        o = O.prepare_row(p, host[r], None, (), O.TIE_CANONICAL, cap=64)
        assert got["rng_before"][r] == state
        if got["token"][r] != o.token:
            o = O.prepare_row(p, host[r], None, (), O.TIE_CANONICAL)  # every weight
            assert is_boundary(o, c.top_p), f"row {r}: {got['token'][r]} vs oracle {o.token}"
            boundary += 1
    return boundary


@pytest.mark.parametrize("vocab", [synth.VOCAB, MAX_VOCAB])
@pytest.mark.parametrize("rows", [1, 2, 4])
@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_noalloc_matches_batch_prepare_and_oracle_on_two_calls(dtype, rows, vocab, cuda):
    import torch
    L = _bind()
    rng = np.random.default_rng(77 + rows + vocab)
    configs = _configs()[:rows] if rows > 1 else [_configs()[2]]
    for call, states in enumerate([None, [123456789, 2**63 + 5, 42, 987654321987][:rows]]):
        host, t = _logits(rng, rows, vocab, dtype, cuda)
        rc, dec = _noalloc(L, t, configs, states)
        assert rc == 0, L.q38s_last_error().decode()
        got = q38s.Batch.decode_decisions(dec)
        want = _batch_prepare(configs, t, states)
        torch.cuda.synchronize()
        assert (got["status"] == 0).all(), f"call {call}: {got['status']}"
        assert (got["token"] == want["token"]).all(), f"call {call}"
        assert (got["rng_before"] == want["rng_before"]).all()
        assert (got["rng_after"] == want["rng_after"]).all()
        _check_oracle(configs, host, got, states)


def test_noalloc_leaves_device_memory_unchanged(cuda):
    """After a first call (which may load the library's device code), calls
    change neither the device's free memory nor torch's allocations."""
    import torch
    L = _bind()
    rng = np.random.default_rng(5)
    configs = _configs()
    _, t = _logits(rng, 4, synth.VOCAB, "bf16", cuda)
    dec = torch.zeros(12, dtype=torch.int64, device=cuda)
    rc, _ = _noalloc(L, t, configs, dec=dec)
    assert rc == 0, L.q38s_last_error().decode()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    alloc0 = torch.cuda.memory_allocated()
    for _ in range(3):
        rc, _ = _noalloc(L, t, configs, dec=dec)
        assert rc == 0, L.q38s_last_error().decode()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert torch.cuda.memory_allocated() == alloc0
    assert (q38s.Batch.decode_decisions(dec)["status"] == 0).all()


def test_noalloc_on_a_non_blocking_stream(cuda):
    """Two calls on a caller's non-blocking stream, the second with other
    rows and states, each compared with q38s_batch_prepare."""
    import torch
    L = _bind()
    rng = np.random.default_rng(9)
    s = torch.cuda.Stream(device=cuda)  # created with cudaStreamNonBlocking
    configs = _configs()
    for call, states in enumerate([None, [7, 8, 9, 10]]):
        host, t = _logits(rng, 4, synth.VOCAB, "f32", cuda)
        dec = torch.zeros(12, dtype=torch.int64, device=cuda)
        torch.cuda.synchronize()
        with torch.cuda.stream(s):
            rc, _ = _noalloc(L, t, configs, states, stream=s.cuda_stream, dec=dec)
        assert rc == 0, L.q38s_last_error().decode()
        s.synchronize()
        got = q38s.Batch.decode_decisions(dec)
        want = _batch_prepare(configs, t, states)
        torch.cuda.synchronize()
        assert (got["status"] == 0).all(), f"call {call}: {got['status']}"
        assert (got["token"] == want["token"]).all(), f"call {call}"
        _check_oracle(configs, host, got, states)


def test_noalloc_rejects_sizes_beyond_its_static_memory(cuda):
    import torch
    L = _bind()
    t = torch.zeros((5, 1000), dtype=torch.float32, device=cuda)
    rc, _ = _noalloc(L, t, [q38s.config_v2(top_k=5, seed=1)] * 5)
    assert rc == q38s.INVALID_ARGUMENT
    assert "1 to 4 rows" in L.q38s_last_error().decode()
    big = torch.zeros((1, MAX_VOCAB + 1), dtype=torch.float32, device=cuda)
    rc, _ = _noalloc(L, big, [q38s.config_v2(top_k=5, seed=1)])
    assert rc == q38s.INVALID_ARGUMENT
    assert "262,144" in L.q38s_last_error().decode()

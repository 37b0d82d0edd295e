"""Greedy argmax and the MoE router top-k against the reference's own kernels.

The reference's device kernels (cuda/q38_kernels.cu: argmax_bf16_kernel,
topk_router_bf16_kernel and topk_router_512_decode_kernel) are compiled
unmodified into oracle/_ref/libq38ref_kernels.so and called on the same
device buffers as q38s_argmax_bf16 / q38s_topk_router_bf16.  Results must be
bit-identical: indices, expert ids and the fp32 weights (NaN compared as NaN),
on inputs with many exact ties, -inf, +inf and NaN entries.

The router's 512-expert decode path is chosen by Q38_CUDA_DECODE_TOPK in both
implementations, read once per process; the "scalar" setting is checked in a
child process.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

import oracle as O
import q38s
from q38s import synth

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))

# (tokens, experts, top_k, normalize, specials): specials adds +-inf / NaN entries
ROUTER_CASES = [
    (1, 512, 10, True, False),     # the reference's decode shape
    (64, 512, 10, True, True),
    (257, 512, 8, True, False),
    (33, 512, 8, False, True),     # 512 experts without normalisation: general kernel
    (7, 128, 8, True, True),
    (16, 64, 32, False, False),
    (5, 40, 32, True, True),
    (3, 1, 1, True, False),
    (2, 3072, 16, False, True),
]


def _need_ref():
    if not O.ref_kernels_available():
        pytest.skip("reference kernels not built (oracle/_ref/libq38ref_kernels.so)")


def _router_logits(tokens, experts, specials, seed, nan_ok=True):
    rng = np.random.default_rng(seed)
    x = (np.round(rng.normal(0, 1.5, (tokens, experts)) * 4) / 4).astype(np.float32)
    if specials and experts > 4:
        for t in range(tokens):
            kind = t % 4
            if kind == 1:
                x[t, rng.choice(experts, max(1, experts // 8), replace=False)] = -np.inf
            elif kind == 2:
                x[t, rng.integers(experts)] = np.inf
            elif kind == 3 and nan_ok:
                x[t, rng.choice(experts, max(1, experts // 16), replace=False)] = np.nan
    return synth.f32_to_bf16_rne(x)


def _same_f32(a, b):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    return bool(np.all((a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))))


def compare_router(cases, seed0=0):
    import torch
    dev = torch.device("cuda", 0)
    stream = torch.cuda.Stream(dev)
    for i, (tokens, experts, top_k, normalize, specials) in enumerate(cases):
        # the reference's 512-expert sort orders NaN arbitrarily: no NaN there
        decode = experts == 512 and normalize and \
            os.environ.get("Q38_CUDA_DECODE_TOPK") not in ("scalar", "0", "false")
        w = _router_logits(tokens, experts, specials, seed0 + i, nan_ok=not decode)
        d = torch.from_numpy(w.view(np.int16)).to(dev)
        ids = [torch.full((tokens, top_k), -7, dtype=torch.int32, device=dev) for _ in range(2)]
        wts = [torch.full((tokens, top_k), 7.0, dtype=torch.float32, device=dev) for _ in range(2)]
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            q38s.topk_router_bf16(d, ids[0], wts[0], top_k, normalize, stream=stream)
        O.ref_topk_router_bf16(d.data_ptr(), ids[1].data_ptr(), wts[1].data_ptr(), tokens,
                               experts, top_k, normalize, stream.cuda_stream, 0)
        stream.synchronize()
        a_ids, b_ids = ids[0].cpu().numpy(), ids[1].cpu().numpy()
        assert (a_ids == b_ids).all(), f"case {cases[i]}: expert ids differ"
        assert _same_f32(wts[0].cpu().numpy(), wts[1].cpu().numpy()), \
            f"case {cases[i]}: weights differ"


def test_router_bit_exact_against_the_reference_kernels(cuda):
    _need_ref()
    compare_router(ROUTER_CASES)


def test_router_scalar_dispatch_in_a_child_process(cuda):
    """Q38_CUDA_DECODE_TOPK=scalar sends 512 experts with normalisation to
    the reference's general kernel (p order, all ties by expert id)."""
    _need_ref()
    code = ("import sys; sys.path[:0] = {paths!r}; import test_gpu_ref_kernels as t; "
            "t.compare_router([(64, 512, 10, True, True), (3, 512, 32, True, False)], 100)")
    paths = [HERE] + [p for p in sys.path if p]
    env = dict(os.environ, Q38_CUDA_DECODE_TOPK="scalar")
    r = subprocess.run([sys.executable, "-c", code.format(paths=paths)], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]


def test_router_rejects_what_the_reference_rejects(cuda):
    import torch
    dev = torch.device("cuda", 0)
    d = torch.zeros((2, 16), dtype=torch.int16, device=dev)
    ids = torch.zeros((2, 33), dtype=torch.int32, device=dev)
    wts = torch.zeros((2, 33), dtype=torch.float32, device=dev)
    for top_k in (0, 17, 33):
        with pytest.raises(q38s.Q38sError, match="invalid top-k router buffers"):
            q38s.topk_router_bf16(d, ids, wts, top_k)


def test_argmax_bit_exact_against_the_reference_kernel(cuda):
    import torch
    _need_ref()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.Stream(dev)
    rng = np.random.default_rng(52)
    cases = []
    for n in (1, 2, 255, 256, 257, 4097, 65_537, 151_936, 248_320):
        x = (np.round(rng.normal(0, 2, n) * 2) / 2).astype(np.float32)
        if n > 10:
            x[rng.choice(n, n // 10)] = np.nan
            x[rng.choice(n, n // 10)] = -np.inf
        cases.append(x)
    cases.append(np.full(300, -np.inf, np.float32))
    cases.append(np.full(1000, np.nan, np.float32))
    cases.append(np.full(151_936, 1.0, np.float32))  # every entry ties
    late = np.full(248_320, -1.0, np.float32)
    late[-1] = np.inf
    cases.append(late)
    for x in cases:
        d = torch.from_numpy(synth.f32_to_bf16_rne(x).view(np.int16)).to(dev)
        out = torch.full((2,), -7, dtype=torch.int32, device=dev)
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            q38s.argmax_bf16(d, out[0:1], stream=stream)
        O.ref_argmax_bf16(d.data_ptr(), x.size, out[1:2].data_ptr(), stream.cuda_stream, 0)
        stream.synchronize()
        a, b = out.cpu().numpy()
        assert a == b, f"n={x.size}: {a} vs reference {b}"


def test_argmax_unaligned_rows_against_the_reference_kernel(cuda):
    """Rows starting 1..7 elements past a 16-byte boundary (scalar head and
    tail around the vector loads)."""
    import torch
    _need_ref()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.Stream(dev)
    rng = np.random.default_rng(53)
    x = (np.round(rng.normal(0, 2, 70_000) * 2) / 2).astype(np.float32)
    d = torch.from_numpy(synth.f32_to_bf16_rne(x).view(np.int16)).to(dev)
    for off in range(8):
        for n in (1, 5, 9, 17, 4097, 65_000):
            sl = d[off:off + n]
            out = torch.full((2,), -7, dtype=torch.int32, device=dev)
            torch.cuda.synchronize()
            with torch.cuda.stream(stream):
                q38s.argmax_bf16(sl, out[0:1], stream=stream)
            O.ref_argmax_bf16(sl.data_ptr(), n, out[1:2].data_ptr(), stream.cuda_stream, 0)
            stream.synchronize()
            a, b = out.cpu().numpy()
            assert a == b, f"offset {off}, n={n}: {a} vs reference {b}"


def test_router_and_argmax_timed_against_the_reference(cuda):
    """Device time of both implementations at the reference's decode shapes
    (CUDA events on one stream, 200 launches each), printed; the argmax must
    not be slower than the reference's."""
    import torch
    _need_ref()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.Stream(dev)

    def timed(fn, n=200):
        for _ in range(10):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            fn()
        e1.record(stream)
        e1.synchronize()
        return e0.elapsed_time(e1) * 1e3 / n

    w = torch.from_numpy(_router_logits(1, 512, False, 9).view(np.int16)).to(dev)
    ids = torch.zeros((1, 10), dtype=torch.int32, device=dev)
    wts = torch.zeros((1, 10), dtype=torch.float32, device=dev)
    x = torch.from_numpy(synth.f32_to_bf16_rne(
        np.random.default_rng(3).normal(0, 2, 248_320).astype(np.float32)).view(np.int16)).to(dev)
    out = torch.zeros(1, dtype=torch.int32, device=dev)
    with torch.cuda.stream(stream):
        ours_r = timed(lambda: q38s.topk_router_bf16(w, ids, wts, 10, True, stream=stream))
        ref_r = timed(lambda: O.ref_topk_router_bf16(w.data_ptr(), ids.data_ptr(),
                                                     wts.data_ptr(), 1, 512, 10, True,
                                                     stream.cuda_stream, 0))
        ours_a = timed(lambda: q38s.argmax_bf16(x, out, stream=stream))
        ref_a = timed(lambda: O.ref_argmax_bf16(x.data_ptr(), 248_320, out.data_ptr(),
                                                stream.cuda_stream, 0))
    print(f"router 1x512 top10: ours {ours_r:.2f} us, reference {ref_r:.2f} us; "
          f"argmax 248,320: ours {ours_a:.2f} us, reference {ref_a:.2f} us")
    assert ours_a <= ref_a

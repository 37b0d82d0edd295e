"""Python binding of the q38s C ABI (include/q38s.h) over ctypes.

This mirrors the reference sampler's interface (q38::TransactionalSampler,
include/q38/sampling.h:52-75 of the reference) for tests and benchmarks:
``Sampler`` is one session with host bf16 logits, ``Batch`` is many sessions
resident on one GPU.  Device buffers are torch CUDA tensors; torch is only
the allocator and stream provider here.

The engine has no CPU fallback: if ``lib/libq38s.so`` is missing, loading
fails loudly.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
LIB_PATH = os.path.join(PKG, "lib", "libq38s.so")

GAMMA = 0x9E3779B97F4A7C15
MASK64 = (1 << 64) - 1

OK, INVALID_ARGUMENT, LOGIC_ERROR, RUNTIME_ERROR, CUDA_ERROR, OUT_OF_MEMORY, TIMEOUT = range(7)
ROW_OK, ROW_NO_FINITE, ROW_NORMALIZATION, ROW_STATE_MISMATCH, ROW_TIMEOUT, ROW_BAD_TOKEN = range(6)
DTYPE_BF16, DTYPE_F32 = 1, 2
MODE_GREEDY, MODE_TOP_K_TOP_P = 0, 1

# Every entry point the header declares (checked by tests/test_capi.py).
EXPORTS = (
    "q38s_last_error", "q38s_version",
    "q38s_sampler_create", "q38s_sampler_create_v2", "q38s_sampler_destroy",
    "q38s_sampler_prepare", "q38s_sampler_prepare_device", "q38s_sampler_commit",
    "q38s_sampler_commit_tokens", "q38s_sampler_reset", "q38s_sampler_state",
    "q38s_sampler_config",
    "q38s_batch_create", "q38s_batch_create_shard", "q38s_batch_destroy", "q38s_batch_rows",
    "q38s_batch_reset", "q38s_batch_states", "q38s_batch_commit_tokens", "q38s_batch_prepare",
    "q38s_batch_commit", "q38s_batch_sample_commit",
    "q38s_mtp_verify", "q38s_shard_topk", "q38s_shard_merge_sample", "q38s_argmax_bf16",
    "q38s_topk_router_bf16", "q38s_testing_set_fault", "q38s_prepare_noalloc",
)


class ConfigV1(C.Structure):
    _fields_ = [("mode", C.c_uint16), ("version", C.c_uint16), ("top_k", C.c_uint32),
                ("top_p", C.c_float), ("temperature", C.c_float),
                ("repetition_penalty", C.c_float), ("frequency_penalty", C.c_float),
                ("presence_penalty", C.c_float), ("reserved_", C.c_uint32), ("seed", C.c_uint64)]


class ConfigV2(C.Structure):
    _fields_ = [("mode", C.c_uint16), ("version", C.c_uint16), ("top_k", C.c_uint32),
                ("top_p", C.c_float), ("temperature", C.c_float),
                ("repetition_penalty", C.c_float), ("frequency_penalty", C.c_float),
                ("presence_penalty", C.c_float), ("min_p", C.c_float), ("seed", C.c_uint64)]


class StateV1(C.Structure):
    _fields_ = [("magic", C.c_uint32), ("version", C.c_uint16), ("header_bytes", C.c_uint16),
                ("rng_state", C.c_uint64), ("sampled_tokens", C.c_uint64),
                ("canonical_tokens", C.c_uint64), ("penalty_checksum", C.c_uint64)]


class Decision(C.Structure):
    _fields_ = [("token", C.c_int32), ("status", C.c_int32), ("rng_before", C.c_uint64),
                ("rng_after", C.c_uint64)]


class Candidate(C.Structure):
    _fields_ = [("value", C.c_float), ("token", C.c_int32)]


class Distribution(C.Structure):
    _fields_ = [("capacity", C.c_uint32), ("tokens", C.c_void_p), ("values", C.c_void_p),
                ("probs", C.c_void_p), ("n_candidates", C.c_void_p),
                ("n_retained", C.c_void_p), ("total", C.c_void_p), ("draw", C.c_void_p)]


class PenaltyExtra(C.Structure):
    _fields_ = [("tokens", C.c_void_p), ("offsets", C.c_void_p)]


class MtpResult(C.Structure):
    _fields_ = [("tokens", C.c_int32 * 65), ("n_tokens", C.c_uint32), ("n_accepted", C.c_uint32),
                ("status", C.c_int32), ("rng_before", C.c_uint64), ("rng_after", C.c_uint64)]


assert C.sizeof(ConfigV1) == 40 and C.sizeof(ConfigV2) == 40 and C.sizeof(StateV1) == 40
assert C.sizeof(Decision) == 24 and C.sizeof(Candidate) == 8


class Q38sError(RuntimeError):
    """A non-zero status from the C ABI.  ``kind`` names the reference's
    exception class (invalid_argument / logic_error / runtime_error)."""

    KINDS = {INVALID_ARGUMENT: "invalid_argument", LOGIC_ERROR: "logic_error",
             RUNTIME_ERROR: "runtime_error", CUDA_ERROR: "cuda_error",
             OUT_OF_MEMORY: "out_of_memory", TIMEOUT: "timeout"}

    def __init__(self, code: int, message: str):
        super().__init__(f"{self.KINDS.get(code, code)}: {message}")
        self.code = code
        self.kind = self.KINDS.get(code, str(code))
        self.message = message


_lib = None


def lib():
    """Loads lib/libq38s.so (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(
                f"{LIB_PATH} is missing; build it with `make -C {PKG}` "
                "(the sampler has no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        P, u16, u32, u64, i32 = C.c_void_p, C.c_uint16, C.c_uint32, C.c_uint64, C.c_int
        sz = C.c_size_t
        L.q38s_last_error.restype = C.c_char_p
        L.q38s_version.restype = C.c_char_p
        L.q38s_sampler_create.argtypes = [i32, u32, C.POINTER(ConfigV1), C.POINTER(P)]
        L.q38s_sampler_create_v2.argtypes = [i32, u32, C.POINTER(ConfigV2), C.POINTER(P)]
        L.q38s_sampler_destroy.argtypes = [P]
        L.q38s_sampler_destroy.restype = None
        L.q38s_sampler_prepare.argtypes = [P, P, sz, P, sz, C.POINTER(Decision)]
        L.q38s_sampler_prepare_device.argtypes = [P, P, u16, sz, P, sz, C.POINTER(Decision), P]
        L.q38s_sampler_commit.argtypes = [P, C.POINTER(Decision)]
        L.q38s_sampler_commit_tokens.argtypes = [P, P, sz]
        L.q38s_sampler_reset.argtypes = [P]
        L.q38s_sampler_state.argtypes = [P, C.POINTER(StateV1)]
        L.q38s_sampler_config.argtypes = [P, C.POINTER(ConfigV1)]
        L.q38s_batch_create.argtypes = [i32, u32, u32, P, C.POINTER(P)]
        L.q38s_batch_create_shard.argtypes = [i32, u32, u32, u32, u32, P, C.POINTER(P)]
        L.q38s_batch_destroy.argtypes = [P]
        L.q38s_batch_destroy.restype = None
        L.q38s_batch_rows.argtypes = [P]
        L.q38s_batch_rows.restype = u32
        L.q38s_batch_reset.argtypes = [P, P]
        L.q38s_batch_states.argtypes = [P, P, P]
        L.q38s_batch_commit_tokens.argtypes = [P, P, P, P, P]
        L.q38s_batch_prepare.argtypes = [P, P, u16, u64, C.POINTER(PenaltyExtra), P,
                                         C.POINTER(Distribution), P]
        L.q38s_batch_commit.argtypes = [P, P, P]
        L.q38s_batch_sample_commit.argtypes = [P, P, u16, u64, P, P]
        L.q38s_mtp_verify.argtypes = [P, u32, P, P, u16, u64, P, u32, P, P]
        L.q38s_shard_topk.argtypes = [P, P, u16, u64, u32, P, P]
        L.q38s_shard_merge_sample.argtypes = [P, P, u32, u32, P, P]
        L.q38s_argmax_bf16.argtypes = [P, u32, P, P, i32]
        L.q38s_testing_set_fault.argtypes = [u32, u64]
        L.q38s_topk_router_bf16.argtypes = [P, P, P, u32, u32, u32, i32, P, i32]
        _lib = L
    return _lib


def _check(rc: int):
    if rc != OK:
        raise Q38sError(rc, lib().q38s_last_error().decode())


def config_v1(top_k=0, top_p=1.0, temperature=1.0, repetition_penalty=1.0,
              frequency_penalty=0.0, presence_penalty=0.0, seed=1, mode=MODE_TOP_K_TOP_P,
              version=1) -> ConfigV1:
    return ConfigV1(mode, version, top_k, top_p, temperature, repetition_penalty,
                    frequency_penalty, presence_penalty, 0, seed & MASK64)


def config_v2(top_k=0, top_p=1.0, temperature=1.0, repetition_penalty=1.0,
              frequency_penalty=0.0, presence_penalty=0.0, min_p=0.0, seed=1,
              mode=MODE_TOP_K_TOP_P, version=2) -> ConfigV2:
    return ConfigV2(mode, version, top_k, top_p, temperature, repetition_penalty,
                    frequency_penalty, presence_penalty, min_p, seed & MASK64)


def _stream_ptr(stream):
    if stream is None:
        return None
    return C.c_void_p(stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream))


_DTYPES = None


def _dtype_code(t) -> int:
    global _DTYPES
    if _DTYPES is None:
        import torch
        _DTYPES = {torch.bfloat16: DTYPE_BF16, torch.float32: DTYPE_F32}
    code = _DTYPES.get(t.dtype)
    if code is None:
        raise TypeError("logits must be torch.bfloat16 or torch.float32")
    return code


class Sampler:
    """One session: q38::TransactionalSampler semantics over the C ABI."""

    def __init__(self, vocabulary: int, config, device: int = 0):
        L = lib()
        h = C.c_void_p()
        if isinstance(config, ConfigV2):
            _check(L.q38s_sampler_create_v2(device, vocabulary, C.byref(config), C.byref(h)))
        else:
            _check(L.q38s_sampler_create(device, vocabulary, C.byref(config), C.byref(h)))
        self._h = h
        self.vocabulary = vocabulary
        self.device = device
        # reused per call: the decision out-parameter, a one-token buffer
        self._dec = Decision()
        self._dec_ref = C.byref(self._dec)
        self._tok = (C.c_int32 * 1)()
        self._tok_ref = C.cast(self._tok, C.c_void_p)
        self._prepare_device = L.q38s_sampler_prepare_device
        self._commit = L.q38s_sampler_commit
        self._commit_tokens = L.q38s_sampler_commit_tokens

    def close(self):
        h = getattr(self, "_h", None)
        if h:
            self._h = None
            try:
                lib().q38s_sampler_destroy(h)
            except TypeError:  # interpreter shutdown: the module is gone already
                pass

    __del__ = close

    def prepare(self, logits_bf16: np.ndarray, extra=()) -> tuple[int, int, int]:
        """prepare() with host bf16 words (numpy uint16)."""
        l = np.ascontiguousarray(logits_bf16, dtype=np.uint16)
        e = np.ascontiguousarray(np.asarray(extra, dtype=np.int32))
        d = Decision()
        _check(lib().q38s_sampler_prepare(self._h, C.c_void_p(l.ctypes.data), l.size,
                                          C.c_void_p(e.ctypes.data), e.size, C.byref(d)))
        return d.token, d.rng_before, d.rng_after

    def prepare_device(self, logits, extra=(), stream=None) -> tuple[int, int, int]:
        # the per-token call: argument conversion kept to a minimum
        if len(extra):
            e = np.ascontiguousarray(np.asarray(extra, dtype=np.int32))
            ep, en = e.ctypes.data, e.size
        else:
            ep, en = None, 0
        d = self._dec
        rc = self._prepare_device(self._h, logits.data_ptr(), _dtype_code(logits),
                                  logits.numel(), ep, en, self._dec_ref,
                                  None if stream is None else _stream_ptr(stream))
        if rc:
            _check(rc)
        return d.token, d.rng_before, d.rng_after

    def commit(self, decision) -> None:
        d = self._dec
        d.token, d.status, d.rng_before, d.rng_after = decision[0], 0, decision[1], decision[2]
        rc = self._commit(self._h, self._dec_ref)
        if rc:
            _check(rc)

    def commit_tokens(self, tokens) -> None:
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        _check(lib().q38s_sampler_commit_tokens(self._h, C.c_void_p(t.ctypes.data), t.size))

    def commit_token(self, token: int) -> None:
        self._tok[0] = token
        rc = self._commit_tokens(self._h, self._tok_ref, 1)
        if rc:
            _check(rc)

    def reset(self) -> None:
        _check(lib().q38s_sampler_reset(self._h))

    def state(self) -> StateV1:
        s = StateV1()
        _check(lib().q38s_sampler_state(self._h, C.byref(s)))
        return s

    def config(self) -> ConfigV1:
        c = ConfigV1()
        _check(lib().q38s_sampler_config(self._h, C.byref(c)))
        return c


class Batch:
    """Many sessions on one GPU (one row each)."""

    def __init__(self, vocabulary: int, configs, device: int = 0, shard=None):
        import torch  # noqa: F401  (initialises the CUDA runtime torch shares)
        L = lib()
        rows = len(configs)
        arr = (ConfigV2 * rows)(*configs)
        h = C.c_void_p()
        if shard is None:
            _check(L.q38s_batch_create(device, vocabulary, rows, C.cast(arr, C.c_void_p),
                                       C.byref(h)))
            self.columns, self.col_begin = vocabulary, 0
        else:
            col_begin, columns = shard
            _check(L.q38s_batch_create_shard(device, vocabulary, col_begin, columns, rows,
                                             C.cast(arr, C.c_void_p), C.byref(h)))
            self.columns, self.col_begin = columns, col_begin
        self._h = h
        self.rows = rows
        self.vocabulary = vocabulary
        self.device = device
        self.configs = list(configs)

    def close(self):
        h = getattr(self, "_h", None)
        if h:
            self._h = None
            try:
                lib().q38s_batch_destroy(h)
            except TypeError:  # interpreter shutdown: the module is gone already
                pass

    __del__ = close

    @property
    def handle(self):
        return self._h

    def _dev(self):
        import torch
        return torch.device("cuda", self.device)

    def decisions_buffer(self):
        import torch
        return torch.zeros(self.rows * 3, dtype=torch.int64, device=self._dev())

    @staticmethod
    def decode_decisions(buf) -> dict:
        a = buf.cpu().numpy().view(np.uint8).reshape(-1, 24)
        tok = a[:, 0:4].copy().view(np.int32).ravel()
        st = a[:, 4:8].copy().view(np.int32).ravel()
        rb = a[:, 8:16].copy().view(np.uint64).ravel()
        ra = a[:, 16:24].copy().view(np.uint64).ravel()
        return {"token": tok, "status": st, "rng_before": rb, "rng_after": ra}

    def commit_tokens(self, histories, stream=None):
        """commit_tokens() per row; histories is a list of int arrays."""
        import torch
        offs = np.zeros(self.rows + 1, np.uint32)
        for r, h in enumerate(histories):
            offs[r + 1] = offs[r] + len(h)
        flat = np.concatenate([np.asarray(h, np.int32) for h in histories]) if offs[-1] else \
            np.zeros(1, np.int32)
        d_tok = torch.from_numpy(flat).to(self._dev())
        d_off = torch.from_numpy(offs.view(np.int32)).to(self._dev())
        status = torch.zeros(self.rows, dtype=torch.int32, device=self._dev())
        _check(lib().q38s_batch_commit_tokens(self._h, C.c_void_p(d_tok.data_ptr()),
                                              C.c_void_p(d_off.data_ptr()),
                                              C.c_void_p(status.data_ptr()),
                                              _stream_ptr(stream)))
        torch.cuda.synchronize(self._dev())
        return status.cpu().numpy()

    def prepare(self, logits, decisions=None, extra=None, dist=None, stream=None, row_stride=None):
        d = self.decisions_buffer() if decisions is None else decisions
        ex = None
        if extra is not None:
            ex = PenaltyExtra(extra[0].data_ptr(), extra[1].data_ptr())
        _check(lib().q38s_batch_prepare(
            self._h, C.c_void_p(logits.data_ptr()), _dtype_code(logits),
            row_stride or logits.shape[-1], C.byref(ex) if ex else None,
            C.c_void_p(d.data_ptr()), C.byref(dist) if dist is not None else None,
            _stream_ptr(stream)))
        return d

    def sample_commit(self, logits, decisions=None, stream=None):
        d = self.decisions_buffer() if decisions is None else decisions
        _check(lib().q38s_batch_sample_commit(
            self._h, C.c_void_p(logits.data_ptr()), _dtype_code(logits), logits.shape[-1],
            C.c_void_p(d.data_ptr()), _stream_ptr(stream)))
        return d

    def commit(self, decisions, stream=None):
        _check(lib().q38s_batch_commit(self._h, C.c_void_p(decisions.data_ptr()),
                                       _stream_ptr(stream)))

    def states(self, stream=None):
        arr = (StateV1 * self.rows)()
        _check(lib().q38s_batch_states(self._h, C.cast(arr, C.c_void_p), _stream_ptr(stream)))
        return list(arr)

    def reset(self, stream=None):
        _check(lib().q38s_batch_reset(self._h, _stream_ptr(stream)))

    def mtp_verify(self, row, target, draft, draft_tokens, result=None, stream=None):
        import torch
        res = torch.zeros(C.sizeof(MtpResult), dtype=torch.uint8, device=self._dev()) \
            if result is None else result
        _check(lib().q38s_mtp_verify(
            self._h, row, C.c_void_p(target.data_ptr()), C.c_void_p(draft.data_ptr()),
            _dtype_code(target), target.shape[-1], C.c_void_p(draft_tokens.data_ptr()),
            draft_tokens.numel(), C.c_void_p(res.data_ptr()), _stream_ptr(stream)))
        return res

    @staticmethod
    def decode_mtp(buf) -> MtpResult:
        raw = buf.cpu().numpy().tobytes()
        return MtpResult.from_buffer_copy(raw)

    def shard_topk(self, logits, k_local, out=None, stream=None):
        import torch
        o = torch.zeros(self.rows * k_local * 2, dtype=torch.int32, device=self._dev()) \
            if out is None else out
        _check(lib().q38s_shard_topk(self._h, C.c_void_p(logits.data_ptr()),
                                     _dtype_code(logits), logits.shape[-1], k_local,
                                     C.c_void_p(o.data_ptr()), _stream_ptr(stream)))
        return o

    def shard_merge_sample(self, gathered, n_shards, k_local, decisions=None, stream=None):
        d = self.decisions_buffer() if decisions is None else decisions
        _check(lib().q38s_shard_merge_sample(self._h, C.c_void_p(gathered.data_ptr()),
                                             n_shards, k_local, C.c_void_p(d.data_ptr()),
                                             _stream_ptr(stream)))
        return d


def decode_candidates(buf, rows, k):
    a = buf.cpu().numpy().view(np.uint8).reshape(rows, k, 8)
    vals = a[:, :, 0:4].copy().view(np.float32).reshape(rows, k)
    toks = a[:, :, 4:8].copy().view(np.int32).reshape(rows, k)
    return vals, toks


def make_distribution(rows: int, capacity: int, device):
    """Device buffers for Batch.prepare(dist=...); returns (struct, tensors)."""
    import torch
    t = {
        "tokens": torch.zeros(rows * capacity, dtype=torch.int32, device=device),
        "values": torch.zeros(rows * capacity, dtype=torch.float32, device=device),
        "probs": torch.zeros(rows * capacity, dtype=torch.float64, device=device),
        "n_candidates": torch.zeros(rows, dtype=torch.int32, device=device),
        "n_retained": torch.zeros(rows, dtype=torch.int32, device=device),
        "total": torch.zeros(rows, dtype=torch.float64, device=device),
        "draw": torch.zeros(rows, dtype=torch.float64, device=device),
    }
    s = Distribution(capacity, *(t[k].data_ptr() for k in
                                 ("tokens", "values", "probs", "n_candidates", "n_retained",
                                  "total", "draw")))
    return s, t


def topk_router_bf16(logits, expert_ids, expert_weights, top_k: int, normalize: bool = True,
                     stream=None, device: int = 0):
    """MoE router top-k over torch bf16 logits [tokens, experts] into int32
    ids and float32 weights [tokens, top_k]."""
    tokens, experts = logits.shape
    _check(lib().q38s_topk_router_bf16(logits.data_ptr(), expert_ids.data_ptr(),
                                       expert_weights.data_ptr(), tokens, experts, top_k,
                                       int(normalize), _stream_ptr(stream), device))


def argmax_bf16(logits, output, stream=None, device: int = 0):
    _check(lib().q38s_argmax_bf16(C.c_void_p(logits.data_ptr()), logits.numel(),
                                  C.c_void_p(output.data_ptr()), _stream_ptr(stream), device))
    return output


def version() -> str:
    return lib().q38s_version().decode()

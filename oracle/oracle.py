"""ctypes bindings for the parity checkers (TEST INFRASTRUCTURE ONLY).

Two libraries live beside this file:

* ``_ref/libq38ref.so`` -- the unmodified reference ``src/sampling.cc``
  (``TransactionalSampler``, include/q38/sampling.h:52-75) behind the C shim
  in ``ref_shim.cc``.
* ``liboracle.so`` -- the CPU restatement in ``q38_oracle.cc`` (canonical or
  libstdc++ tie order, fp32 input, min-p, speculative verification, vocab
  shards).

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` import this module.  The product
never does.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_LIB = os.path.join(HERE, "_ref", "libq38ref.so")
ORACLE_LIB = os.path.join(HERE, "liboracle.so")

GAMMA = 0x9E3779B97F4A7C15
MASK64 = (1 << 64) - 1

TIE_CANONICAL = 0
TIE_LIBSTDCXX = 1

DTYPE_BF16 = 1  # q38::DType::kBFloat16 (contracts.h:17-24)
DTYPE_F32 = 2   # q38::DType::kFloat32


# ----------------------------------------------------------------- helpers
def f32_to_bf16_rne(x: np.ndarray) -> np.ndarray:
    """Round fp32 to bf16 words with the reference test helper's rule
    (tests/test_runtime.cc:1089-1094): (bits + 0x7fff + lsb) >> 16."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_to_f32(w: np.ndarray) -> np.ndarray:
    return (np.asarray(w, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def splitmix64(x: int) -> int:
    """sampling.cc:22-27 in Python integers."""
    x &= MASK64
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & MASK64
    return x ^ (x >> 31)


def uniform01(state: int) -> float:
    """sampling.cc:33-36."""
    return float(splitmix64(state) >> 11) * (1.0 / 9007199254740992.0)


# ------------------------------------------------------- struct layouts
class SamplingConfigV1(C.Structure):
    """include/q38/sampling.h:19-29 (40 bytes)."""
    _fields_ = [("mode", C.c_uint16), ("version", C.c_uint16), ("top_k", C.c_uint32),
                ("top_p", C.c_float), ("temperature", C.c_float),
                ("repetition_penalty", C.c_float), ("frequency_penalty", C.c_float),
                ("presence_penalty", C.c_float), ("_pad", C.c_uint32),
                ("seed", C.c_uint64)]


class SamplerStateV1(C.Structure):
    """include/q38/sampling.h:31-39 (40 bytes)."""
    _fields_ = [("magic", C.c_uint32), ("version", C.c_uint16), ("header_bytes", C.c_uint16),
                ("rng_state", C.c_uint64), ("sampled_tokens", C.c_uint64),
                ("canonical_tokens", C.c_uint64), ("penalty_checksum", C.c_uint64)]


class RowParams(C.Structure):
    """q38o_row_params in q38_oracle.cc."""
    _fields_ = [("top_k", C.c_uint32), ("top_p", C.c_float), ("min_p", C.c_float),
                ("temperature", C.c_float), ("repetition_penalty", C.c_float),
                ("frequency_penalty", C.c_float), ("presence_penalty", C.c_float),
                ("reserved", C.c_uint32), ("rng_state", C.c_uint64)]


class OracleResult(C.Structure):
    _fields_ = [("token", C.c_int32), ("status", C.c_int32), ("rng_before", C.c_uint64),
                ("rng_after", C.c_uint64), ("n_candidates", C.c_uint32),
                ("n_retained", C.c_uint32), ("total_all", C.c_double), ("total", C.c_double),
                ("draw", C.c_double), ("selected", C.c_uint32), ("reserved", C.c_uint32)]


assert C.sizeof(SamplingConfigV1) == 40 and C.sizeof(SamplerStateV1) == 40
assert C.sizeof(RowParams) == 40


def make_config(top_k=0, top_p=1.0, temperature=1.0, repetition_penalty=1.0,
                frequency_penalty=0.0, presence_penalty=0.0, seed=1, mode=1,
                version=1) -> SamplingConfigV1:
    return SamplingConfigV1(mode, version, top_k, top_p, temperature, repetition_penalty,
                            frequency_penalty, presence_penalty, 0, seed)


def make_params(top_k=0, top_p=1.0, min_p=0.0, temperature=1.0, repetition_penalty=1.0,
                frequency_penalty=0.0, presence_penalty=0.0, rng_state=1) -> RowParams:
    return RowParams(top_k, top_p, min_p, temperature, repetition_penalty,
                     frequency_penalty, presence_penalty, 0, rng_state & MASK64)


class SamplerError(Exception):
    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code
        self.message = message


_P = C.c_void_p
_i32p = C.POINTER(C.c_int32)
_u16p = C.POINTER(C.c_uint16)
_u32p = C.POINTER(C.c_uint32)
_u64p = C.POINTER(C.c_uint64)


def _ptr(a: np.ndarray | None, ctype=C.c_void_p):
    if a is None:
        return None
    return a.ctypes.data_as(ctype) if ctype is not C.c_void_p else C.c_void_p(a.ctypes.data)


# ------------------------------------------------------------ reference
_ref = None


def ref_available() -> bool:
    return os.path.exists(REF_LIB)


def _load_ref():
    global _ref
    if _ref is None:
        if not os.path.exists(REF_LIB):
            raise FileNotFoundError(f"{REF_LIB} missing: run `make -C oracle`")
        lib = C.CDLL(REF_LIB)
        lib.q38ref_create.argtypes = [C.c_uint32, _P, C.POINTER(_P), C.c_char_p, C.c_size_t]
        lib.q38ref_destroy.argtypes = [_P]
        lib.q38ref_prepare.argtypes = [_P, _u16p, C.c_size_t, _i32p, C.c_size_t, _i32p,
                                       _u64p, _u64p, C.c_char_p, C.c_size_t]
        lib.q38ref_commit.argtypes = [_P, C.c_int32, C.c_uint64, C.c_uint64, C.c_char_p,
                                      C.c_size_t]
        lib.q38ref_commit_tokens.argtypes = [_P, _i32p, C.c_size_t, C.c_char_p, C.c_size_t]
        lib.q38ref_state.argtypes = [_P, _P]
        lib.q38ref_config.argtypes = [_P, _P]
        lib.q38ref_reset.argtypes = [_P]
        lib.q38ref_prepare_rows.argtypes = [C.POINTER(_P), C.c_uint32, _u16p, C.c_size_t,
                                            _i32p, _i32p, C.c_int]
        _ref = lib
    return _ref


class RefSampler:
    """The unmodified reference TransactionalSampler (sampling.h:52-75)."""

    def __init__(self, vocabulary: int, config: SamplingConfigV1):
        lib = _load_ref()
        h = _P()
        err = C.create_string_buffer(256)
        rc = lib.q38ref_create(vocabulary, C.byref(config), C.byref(h), err, 256)
        if rc:
            raise SamplerError(rc, err.value.decode())
        self._h = h
        self._lib = lib
        self.vocabulary = vocabulary

    def __del__(self):
        if getattr(self, "_h", None):
            self._lib.q38ref_destroy(self._h)
            self._h = None

    @property
    def handle(self):
        return self._h

    def prepare(self, logits_bf16: np.ndarray, extra=()) -> tuple[int, int, int]:
        l = np.ascontiguousarray(logits_bf16, dtype=np.uint16)
        e = np.ascontiguousarray(np.asarray(extra, dtype=np.int32))
        tok, rb, ra = C.c_int32(), C.c_uint64(), C.c_uint64()
        err = C.create_string_buffer(256)
        rc = self._lib.q38ref_prepare(self._h, _ptr(l, _u16p), l.size, _ptr(e, _i32p), e.size,
                                      C.byref(tok), C.byref(rb), C.byref(ra), err, 256)
        if rc:
            raise SamplerError(rc, err.value.decode())
        return tok.value, rb.value, ra.value

    def commit(self, decision: tuple[int, int, int]) -> None:
        err = C.create_string_buffer(256)
        rc = self._lib.q38ref_commit(self._h, decision[0], decision[1], decision[2], err, 256)
        if rc:
            raise SamplerError(rc, err.value.decode())

    def commit_tokens(self, tokens) -> None:
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        err = C.create_string_buffer(256)
        rc = self._lib.q38ref_commit_tokens(self._h, _ptr(t, _i32p), t.size, err, 256)
        if rc:
            raise SamplerError(rc, err.value.decode())

    def commit_token(self, token: int) -> None:
        self.commit_tokens([token])

    def state(self) -> SamplerStateV1:
        s = SamplerStateV1()
        self._lib.q38ref_state(self._h, C.byref(s))
        return s

    def reset(self) -> None:
        self._lib.q38ref_reset(self._h)


REF_KERNELS_LIB = os.path.join(HERE, "_ref", "libq38ref_kernels.so")
_refk = None


def ref_kernels_available() -> bool:
    return os.path.exists(REF_KERNELS_LIB)


def _load_ref_kernels():
    """The reference's own device kernels (cuda/q38_kernels.cu, unmodified,
    built for sm_100a): greedy argmax and the MoE router top-k."""
    global _refk
    if _refk is None:
        lib = C.CDLL(REF_KERNELS_LIB)
        lib.q38ref_argmax_bf16.argtypes = [_P, C.c_uint32, _P, _P, C.c_int, C.c_char_p,
                                           C.c_size_t]
        lib.q38ref_topk_router_bf16.argtypes = [_P, _P, _P, C.c_uint32, C.c_uint32, C.c_uint32,
                                                C.c_int, _P, C.c_int, C.c_char_p, C.c_size_t]
        _refk = lib
    return _refk


def ref_argmax_bf16(logits_ptr: int, count: int, out_ptr: int, stream_ptr: int, device: int):
    """cuda_argmax_bf16 of the reference on device buffers (stream must be a
    real stream, as the reference requires)."""
    err = C.create_string_buffer(256)
    rc = _load_ref_kernels().q38ref_argmax_bf16(logits_ptr, count, out_ptr, stream_ptr, device,
                                                err, 256)
    if rc:
        raise SamplerError(rc, err.value.decode())


def ref_topk_router_bf16(logits_ptr: int, ids_ptr: int, weights_ptr: int, tokens: int,
                         experts: int, top_k: int, normalize: bool, stream_ptr: int,
                         device: int):
    """cuda_topk_router_bf16 of the reference on device buffers."""
    err = C.create_string_buffer(256)
    rc = _load_ref_kernels().q38ref_topk_router_bf16(logits_ptr, ids_ptr, weights_ptr, tokens,
                                                     experts, top_k, int(normalize), stream_ptr,
                                                     device, err, 256)
    if rc:
        raise SamplerError(rc, err.value.decode())


def ref_prepare_rows(samplers: list[RefSampler], logits_bf16: np.ndarray, threads: int):
    """prepare() on one reference sampler per row, rows spread over threads."""
    lib = _load_ref()
    rows, vocab = logits_bf16.shape
    handles = (_P * rows)(*[s.handle for s in samplers])
    l = np.ascontiguousarray(logits_bf16, dtype=np.uint16)
    tokens = np.empty(rows, np.int32)
    status = np.empty(rows, np.int32)
    lib.q38ref_prepare_rows(handles, rows, _ptr(l, _u16p), vocab, _ptr(tokens, _i32p),
                            _ptr(status, _i32p), threads)
    return tokens, status


# -------------------------------------------------------- restatement
_orc = None


def _load_oracle():
    global _orc
    if _orc is None:
        if not os.path.exists(ORACLE_LIB):
            raise FileNotFoundError(f"{ORACLE_LIB} missing: run `make -C oracle`")
        lib = C.CDLL(ORACLE_LIB)
        lib.q38o_prepare_row.argtypes = [C.c_uint32, C.POINTER(RowParams), C.c_int, _P, _u32p,
                                         _i32p, C.c_size_t, C.c_int, C.POINTER(OracleResult),
                                         _i32p, C.POINTER(C.c_float), C.POINTER(C.c_double),
                                         C.c_uint32]
        lib.q38o_prepare_rows.argtypes = [C.c_uint32, C.c_uint32, C.POINTER(RowParams), C.c_int,
                                          _P, C.c_size_t, C.POINTER(_u32p), C.c_int, _i32p,
                                          _i32p, C.c_int]
        lib.q38o_shard_topk.argtypes = [C.c_uint32, C.c_uint32, C.c_uint32, C.POINTER(RowParams),
                                        C.c_int, _P, _u32p, C.c_uint32, C.POINTER(C.c_float),
                                        _i32p]
        lib.q38o_mtp_verify.argtypes = [C.c_uint32, C.c_uint32, C.POINTER(RowParams), C.c_int, _P,
                                        _P, _i32p, _u32p, C.c_int, _i32p, _u32p, _u32p, _u64p]
        lib.q38o_splitmix64.argtypes = [C.c_uint64]
        lib.q38o_splitmix64.restype = C.c_uint64
        lib.q38o_uniform01.argtypes = [C.c_uint64]
        lib.q38o_uniform01.restype = C.c_double
        _orc = lib
    return _orc


@dataclass
class RowResult:
    token: int
    status: int
    rng_before: int
    rng_after: int
    n_candidates: int
    n_retained: int
    total_all: float
    total: float
    draw: float
    selected: int
    cand_tokens: np.ndarray
    cand_values: np.ndarray
    cand_weights: np.ndarray


def _dtype_code(logits: np.ndarray) -> int:
    if logits.dtype == np.uint16:
        return DTYPE_BF16
    if logits.dtype == np.float32:
        return DTYPE_F32
    raise TypeError("logits must be uint16 (bf16 words) or float32")


def prepare_row(params: RowParams, logits: np.ndarray, counts: np.ndarray | None = None,
                extra=(), tie_mode: int = TIE_CANONICAL, cap: int | None = None) -> RowResult:
    lib = _load_oracle()
    l = np.ascontiguousarray(logits)
    vocab = l.size
    cap = vocab if cap is None else cap
    c = None if counts is None else np.ascontiguousarray(counts, dtype=np.uint32)
    e = np.ascontiguousarray(np.asarray(extra, dtype=np.int32))
    res = OracleResult()
    ct = np.zeros(cap, np.int32)
    cv = np.zeros(cap, np.float32)
    cw = np.zeros(cap, np.float64)
    lib.q38o_prepare_row(vocab, C.byref(params), _dtype_code(l), _ptr(l), _ptr(c, _u32p),
                         _ptr(e, _i32p), e.size, tie_mode, C.byref(res), _ptr(ct, _i32p),
                         cv.ctypes.data_as(C.POINTER(C.c_float)),
                         cw.ctypes.data_as(C.POINTER(C.c_double)), cap)
    n = min(cap, res.n_candidates) if res.status == 0 else 0
    return RowResult(res.token, res.status, res.rng_before, res.rng_after, res.n_candidates,
                     res.n_retained, res.total_all, res.total, res.draw, res.selected,
                     ct[:n].copy(), cv[:n].copy(), cw[:n].copy())


def prepare_rows(params: list[RowParams], logits: np.ndarray, counts: np.ndarray | None = None,
                 tie_mode: int = TIE_CANONICAL, threads: int = 1):
    """Tokens and statuses for many rows (row-major logits, optional per-row
    counts matrix of the same shape)."""
    lib = _load_oracle()
    l = np.ascontiguousarray(logits)
    rows, vocab = l.shape
    arr = (RowParams * rows)(*params)
    tokens = np.empty(rows, np.int32)
    status = np.empty(rows, np.int32)
    cptrs = None
    if counts is not None:
        cc = np.ascontiguousarray(counts, dtype=np.uint32)
        cptrs = (_u32p * rows)(*[C.cast(cc.ctypes.data + r * vocab * 4, _u32p)
                                 for r in range(rows)])
    lib.q38o_prepare_rows(vocab, rows, arr, _dtype_code(l), _ptr(l), vocab, cptrs, tie_mode,
                          _ptr(tokens, _i32p), _ptr(status, _i32p), threads)
    return tokens, status


def shard_topk(vocab: int, col_begin: int, params: RowParams, logits_shard: np.ndarray,
               k: int, counts_shard: np.ndarray | None = None):
    lib = _load_oracle()
    l = np.ascontiguousarray(logits_shard)
    n = l.size
    m = min(k, n)
    vals = np.zeros(m, np.float32)
    toks = np.zeros(m, np.int32)
    c = None if counts_shard is None else np.ascontiguousarray(counts_shard, dtype=np.uint32)
    rc = lib.q38o_shard_topk(vocab, col_begin, n, C.byref(params), _dtype_code(l), _ptr(l),
                             _ptr(c, _u32p), k, vals.ctypes.data_as(C.POINTER(C.c_float)),
                             _ptr(toks, _i32p))
    if rc:
        raise SamplerError(rc, "shard_topk rejected its arguments")
    return vals, toks


def mtp_verify(params: RowParams, target: np.ndarray, draft: np.ndarray, draft_tokens,
               counts: np.ndarray | None = None, tie_mode: int = TIE_CANONICAL):
    """Returns (published tokens, n_accepted, rng_after, status)."""
    lib = _load_oracle()
    t = np.ascontiguousarray(target)
    d = np.ascontiguousarray(draft)
    dt = np.ascontiguousarray(np.asarray(draft_tokens, dtype=np.int32))
    n_draft = dt.size
    vocab = t.shape[-1]
    out = np.zeros(n_draft + 1, np.int32)
    n_out, n_acc, rng_after = C.c_uint32(), C.c_uint32(), C.c_uint64()
    c = None if counts is None else np.ascontiguousarray(counts, dtype=np.uint32)
    st = lib.q38o_mtp_verify(vocab, n_draft, C.byref(params), _dtype_code(t), _ptr(t), _ptr(d),
                             _ptr(dt, _i32p), _ptr(c, _u32p), tie_mode, _ptr(out, _i32p),
                             C.byref(n_out), C.byref(n_acc), C.byref(rng_after))
    return out[: n_out.value].copy(), n_acc.value, rng_after.value, st

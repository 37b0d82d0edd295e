"""The C-ABI library without a GPU: it loads, exports every entry point that
include/q38s.h declares, and its struct layouts match the reference's
(include/q38/sampling.h:19-50).  No kernel is launched here."""
import ctypes as C
import os
import re
import subprocess

import pytest

import q38s

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
HEADER = os.path.join(ROOT, "include", "q38s.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(q38s_[a-z0-9_]+)\s*\(", text)))


def test_library_exists_and_loads():
    assert os.path.exists(q38s.LIB_PATH), "build with make -C qwen3.8-flash-next-dual-gpu_b200"
    q38s.lib()
    assert q38s.version().startswith("q38s")


def test_every_declared_symbol_is_exported():
    L = q38s.lib()
    names = declared_functions()
    assert len(names) >= 25
    for n in names:
        assert hasattr(L, n), f"{n} declared in include/q38s.h but not exported"
    assert set(names) == set(q38s.EXPORTS)


def test_exports_are_c_symbols():
    out = subprocess.run(["nm", "-D", "--defined-only", q38s.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (q38s_\w+)", out))
    assert set(declared_functions()) <= exported


def test_struct_layouts_match_reference():
    assert C.sizeof(q38s.ConfigV1) == 40
    assert C.sizeof(q38s.ConfigV2) == 40
    assert C.sizeof(q38s.StateV1) == 40
    assert C.sizeof(q38s.Decision) == 24
    assert q38s.ConfigV1.seed.offset == 32 and q38s.ConfigV2.min_p.offset == 28
    assert q38s.StateV1.rng_state.offset == 8 and q38s.Decision.rng_before.offset == 8


def test_host_validation_without_gpu():
    """Argument checks run before any CUDA call and carry the reference's
    messages (sampling.cc:43-55)."""
    L = q38s.lib()
    h = C.c_void_p()
    bad = q38s.config_v1(top_k=2, top_p=0.0, temperature=1.0)
    rc = L.q38s_sampler_create(0, 3, C.byref(bad), C.byref(h))
    assert rc == q38s.INVALID_ARGUMENT
    assert L.q38s_last_error().decode() == "invalid sampling parameters"
    rc = L.q38s_sampler_create(0, 0, C.byref(q38s.config_v1()), C.byref(h))
    assert rc == q38s.INVALID_ARGUMENT
    assert L.q38s_last_error().decode() == "invalid sampler dimensions/version"
    bad_mode = q38s.config_v1(mode=7)
    assert L.q38s_sampler_create(0, 3, C.byref(bad_mode), C.byref(h)) == q38s.INVALID_ARGUMENT
    assert L.q38s_last_error().decode() == "unsupported sampling mode"
    v2 = q38s.config_v2(min_p=1.5)
    assert L.q38s_sampler_create_v2(0, 3, C.byref(v2), C.byref(h)) == q38s.INVALID_ARGUMENT
    assert L.q38s_argmax_bf16(None, 0, None, None, 0) == q38s.INVALID_ARGUMENT
    assert L.q38s_last_error().decode() == "invalid BF16 argmax buffers"
    assert L.q38s_topk_router_bf16(None, None, None, 1, 512, 10, 1, None, 0) == \
        q38s.INVALID_ARGUMENT
    assert L.q38s_last_error().decode() == "invalid top-k router buffers"
    fake = C.c_void_p(16)  # never dereferenced: every check below fails first
    for args, msg in (((1, 512, 33, 1), "invalid top-k router buffers"),
                      ((1, 8, 9, 1), "invalid top-k router buffers"),
                      ((0, 512, 10, 1), "invalid top-k router buffers"),
                      ((1, 4000, 10, 1), "router experts above 3,072 per token")):
        tokens, experts, top_k, norm = args
        assert L.q38s_topk_router_bf16(fake, fake, fake, tokens, experts, top_k, norm, None,
                                       0) == q38s.INVALID_ARGUMENT
        assert L.q38s_last_error().decode() == msg
    assert L.q38s_topk_router_bf16(fake, fake, fake, 1, 512, 10, 1, None, -1) == \
        q38s.INVALID_ARGUMENT
    assert L.q38s_last_error().decode() == "invalid CUDA kernel launch context"
    wide = q38s.config_v1(top_k=20)
    assert L.q38s_sampler_create(0, (1 << 20) + 1, C.byref(wide), C.byref(h)) == \
        q38s.INVALID_ARGUMENT
    assert L.q38s_last_error().decode() == "more than 1,048,576 columns per batch"


def test_public_cpp_header_compiles_standalone(tmp_path):
    src = tmp_path / "t.cc"
    src.write_text('#include "q38/sampling.h"\n#include "q38s.h"\n'
                   "static_assert(sizeof(q38::SamplingConfigV1) == sizeof(q38s_sampling_config_v1));\n"
                   "int main() { return 0; }\n")
    r = subprocess.run(["g++", "-std=c++17", "-Wall", "-Wextra", "-Werror", "-pedantic",
                        "-I", os.path.join(ROOT, "include"), "-c", str(src), "-o",
                        str(tmp_path / "t.o")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr

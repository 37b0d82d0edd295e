"""The sampler as a drop-in behind the reference runtime's own executor.

oracle/executor_harness.cc drives the reference's DualStageExecutor and mock
stage backends (src/executor.cc, src/mock_backend.cc and their dependencies,
compiled unmodified) through sampled decode sessions.  oracle/Makefile links
it twice: exec_ref with the reference's src/sampling.cc, exec_q38s with this
repository's include/q38/sampling.h and lib/libq38s.so.  The executor calls
the sampler exactly as in production (executor.cc:450-469, :537-540, :643,
:663, :684, :734, :767), so identical output lines mean the GPU sampler is a
drop-in for the CPU one: same tokens, same SamplerStateV1 words after every
step, same executor counters.

The CPU test checks the reference arm against the counters that the
reference's own sampler test asserts (tests/test_runtime.cc:1088-1137); the
GPU test compares the two arms line by line.
"""
import json
import os
import subprocess

import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
EXEC_REF = os.path.join(ROOT, "oracle", "_ref", "exec_ref")
EXEC_Q38S = os.path.join(ROOT, "oracle", "_ref", "exec_q38s")


def _run(path):
    r = subprocess.run([path], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    return [json.loads(line) for line in r.stdout.splitlines() if line.strip()]


@pytest.mark.skipif(not os.path.exists(EXEC_REF), reason="executor harness not built")
def test_reference_arm_matches_the_reference_test_counters():
    lines = _run(EXEC_REF)
    by_op = {}
    for x in lines:
        assert "error" not in x or x["op"] == "stale_commit", x
        by_op.setdefault(x["op"], []).append(x)
    assert by_op["fixture_prepare"][0]["sampled"] == 0
    assert by_op["fixture_commit"][0]["sampled"] == 1
    c = by_op["fixture_commit_tokens"][0]
    assert c["canonical"] == 3 and c["checksum"] != 0
    assert by_op["stale_commit"][0]["error"] == "sampler decision does not match committed state"
    # test_runtime.cc:1124-1136: append 5 tokens, seed, decode, speculative fallback
    ap = by_op["fixture:append"][0]
    assert ap["sampled"] == 1 and ap["canonical"] == 5
    assert by_op["fixture:seed_decode"][0]["canonical"] == 6
    d1 = by_op["fixture:decode_one"][0]
    assert d1["sampled"] == 2 and d1["canonical"] == 7
    sp = by_op["fixture:speculative_step"][0]
    assert sp["spec_txn"] == 0 and sp["drafted"] == 0
    assert sp["sampled"] == by_op["fixture:decode_one"][3]["sampled"] + 1
    assert by_op["fixture:reset"][0]["sampled"] == 0
    assert len(lines) > 150


@pytest.mark.gpu
@pytest.mark.skipif(not (os.path.exists(EXEC_REF) and os.path.exists(EXEC_Q38S)),
                    reason="executor harness not built")
def test_gpu_sampler_behind_the_reference_executor_matches_the_cpu_sampler(cuda):
    ref = _run(EXEC_REF)
    ours = _run(EXEC_Q38S)
    assert len(ours) == len(ref)
    for i, (a, b) in enumerate(zip(ours, ref)):
        assert a == b, f"line {i}: {a} != {b}"
    decoded = sum(len(x.get("tokens", [])) for x in ours if ":" in x.get("op", ""))
    print(f"executor drop-in: {len(ours)} steps identical, {decoded} tokens")


DEV_REF = os.path.join(ROOT, "oracle", "_ref", "dev_ref")
DEV_Q38S = os.path.join(ROOT, "oracle", "_ref", "dev_q38s")


@pytest.mark.gpu
@pytest.mark.skipif(not (os.path.exists(DEV_REF) and os.path.exists(DEV_Q38S)),
                    reason="device decode harness not built")
def test_device_logits_decode_matches_the_cpu_sampler(cuda):
    """oracle/device_decode_harness.cc: the executor's sampled decode steps
    with the stage-1 logits resident on the device (prepare_device, no D2H
    copy of the logits) against the reference's CPU sampler on the same
    logits on the host, three sessions of 120 steps at V = 248,320: every
    token and SamplerStateV1 word identical."""
    def run(path):
        r = subprocess.run([path, "120"], capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
        lines = [json.loads(line) for line in r.stdout.splitlines() if line.strip()]
        timing = [x for x in lines if x.get("op") == "timing"]
        return [x for x in lines if x.get("op") != "timing"], timing[0]["us_per_step"]

    ref, ref_t = run(DEV_REF)
    dev, dev_t = run(DEV_Q38S)
    assert len(ref) == len(dev) == 3 * 121
    for a, b in zip(ref, dev):
        assert a == b, f"reference {a} vs device {b}"
    print(f"us per step: device logits {dev_t}, reference on host logits {ref_t}")

"""The CPU oracle against the reference's golden vectors (no GPU).

Pins the restatement in oracle/q38_oracle.cc: in libstdc++ tie mode it must
reproduce every golden decision of the unmodified reference bit for bit;
in canonical mode (the engine's order) every difference must be a tie-order
difference.  Also checks the oracle's extensions against their documented
reductions (min_p = 0, q == p speculative verification, vocab shards).
"""
import numpy as np
import pytest

import oracle as O
from helpers import hex_to_bf16, is_boundary, load_cases, load_sequences, transformed_value
from q38s import synth

CASES = load_cases()
SEQS = load_sequences()


def params_from(cfg: dict, rng_state: int, min_p: float = 0.0) -> O.RowParams:
    return O.make_params(top_k=cfg["top_k"], top_p=cfg["top_p"], min_p=min_p,
                         temperature=cfg["temperature"],
                         repetition_penalty=cfg["repetition_penalty"],
                         frequency_penalty=cfg["frequency_penalty"],
                         presence_penalty=cfg["presence_penalty"], rng_state=rng_state)


def run_oracle(case, tie_mode):
    cfg = case["config"]
    v = case["vocab"]
    logits = hex_to_bf16(case["logits_bf16_hex"])
    counts = np.bincount(np.asarray(case["history"], np.int64), minlength=v).astype(np.uint32) \
        if v else None
    return O.prepare_row(params_from(cfg, cfg["seed"]), logits, counts, case["extra"], tie_mode)


def expected_ok(case):
    return "token" in case["expect"]


@pytest.mark.parametrize("case", [c for c in CASES if expected_ok(c)], ids=lambda c: c["name"])
def test_libstdcxx_mode_matches_reference_bit_for_bit(case):
    r = run_oracle(case, O.TIE_LIBSTDCXX)
    e = case["expect"]
    assert r.status == 0
    assert (r.token, r.rng_before, r.rng_after) == (e["token"], e["rng_before"], e["rng_after"])


@pytest.mark.parametrize("case", [c for c in CASES if expected_ok(c)], ids=lambda c: c["name"])
def test_canonical_mode_differs_only_by_tie_order(case):
    r = run_oracle(case, O.TIE_CANONICAL)
    e = case["expect"]
    assert r.status == 0 and r.rng_after == e["rng_after"]
    if r.token != e["token"]:
        ref = run_oracle(case, O.TIE_LIBSTDCXX)
        # same sorted position, same transformed value: a tie-order swap
        assert r.selected == ref.selected
        assert transformed_value(r, r.token) == transformed_value(ref, e["token"])


@pytest.mark.parametrize("case", [c for c in CASES if c["expect"].get("stage") == "prepare"],
                         ids=lambda c: c["name"])
def test_oracle_reports_reference_prepare_errors(case):
    cfg = case["config"]
    if cfg["mode"] == 0 or len(hex_to_bf16(case["logits_bf16_hex"])) != case["vocab"] or \
            any(t < 0 or t >= case["vocab"] for t in case["extra"]):
        pytest.skip("checked on the host side of the engine (no arithmetic involved)")
    r = run_oracle(case, O.TIE_CANONICAL)
    assert r.status == case["expect"]["error"] == 3


def test_reference_sequence_replay():
    seq = SEQS["test_runtime_sequence"]
    cfg = seq["config"]
    v = seq["vocab"]
    logits = hex_to_bf16(seq["logits_bf16_hex"])
    counts = np.zeros(v, np.uint32)
    rng = cfg["seed"]
    canonical = 0
    checksum = 0
    for step in seq["steps"]:
        if step["op"] == "prepare":
            r = O.prepare_row(params_from(cfg, rng), logits, counts, step["extra"],
                              O.TIE_LIBSTDCXX)
            assert [r.token, r.rng_before, r.rng_after] == step["expect"]
        elif step["op"] == "commit":
            rng = step["decision"][2]
        elif step["op"] == "commit_tokens":
            for t in step["tokens"]:
                counts[t] += 1
                canonical += 1
                checksum ^= O.splitmix64(t ^ ((canonical * O.GAMMA) & O.MASK64))
        elif step["op"] == "state" and step is seq["steps"][-3]:
            st = step["expect"]
            assert st["rng_state"] == rng
            assert st["canonical_tokens"] == canonical
            assert st["penalty_checksum"] == checksum


def test_cfg1_100_steps_libstdcxx_exact_and_canonical_classified():
    seq = SEQS["cfg1_100_steps"]
    cfg = seq["config"]
    counts = np.bincount(synth.cfg1_history(), minlength=synth.VOCAB).astype(np.uint32)
    rng = cfg["seed"]
    ties = 0
    for step, expect in enumerate(seq["tokens"]):
        logits = synth.f32_to_bf16_rne(synth.cfg1_logits(step))
        p = params_from(cfg, rng)
        ref = O.prepare_row(p, logits, counts, (), O.TIE_LIBSTDCXX, cap=64)
        assert ref.token == expect
        can = O.prepare_row(p, logits, counts, (), O.TIE_CANONICAL, cap=64)
        if can.token != expect:
            ties += 1
            assert transformed_value(can, can.token) == transformed_value(ref, expect)
        counts[expect] += 1
        rng = ref.rng_after
    assert seq["final_state"]["rng_state"] == rng
    assert ties < 40


def test_min_p_zero_reduces_to_reference():
    rng = np.random.default_rng(7)
    for _ in range(20):
        v = int(rng.integers(2, 3000))
        logits = O.f32_to_bf16_rne(rng.normal(0, 2.5, v).astype(np.float32))
        p = O.make_params(top_k=int(rng.integers(0, v)), top_p=float(rng.uniform(0.3, 1.0)),
                          temperature=0.8, rng_state=int(rng.integers(1, 2**63)))
        a = O.prepare_row(p, logits, tie_mode=O.TIE_LIBSTDCXX)
        cfg = O.make_config(top_k=p.top_k, top_p=p.top_p, temperature=p.temperature,
                            seed=p.rng_state)
        if O.ref_available():
            assert O.RefSampler(v, cfg).prepare(logits)[0] == a.token


def test_min_p_filters_by_weight():
    logits = O.f32_to_bf16_rne(np.array([0.0, -1.0, -2.0, -5.0, -9.0], np.float32))
    p = O.make_params(top_k=0, top_p=1.0, min_p=0.1, temperature=1.0, rng_state=3)
    r = O.prepare_row(p, logits)
    # exp(-2) = 0.135 >= 0.1 > exp(-5)
    assert list(r.cand_tokens) == [0, 1, 2]


def test_mtp_q_equals_p_accepts_all_and_bonus_is_reference_draw():
    rng = np.random.default_rng(11)
    v, n = 5000, 8
    target = rng.normal(0, 3, (n + 1, v)).astype(np.float32)
    p = O.make_params(top_k=20, top_p=0.95, temperature=0.7, rng_state=99)
    drafts = []
    for i in range(n):
        pi = O.make_params(top_k=20, top_p=0.95, temperature=0.7,
                           rng_state=(99 + i * O.GAMMA) & O.MASK64)
        drafts.append(O.prepare_row(pi, target[i]).token)
    toks, acc, rng_after, st = O.mtp_verify(p, target, target[:n], drafts)
    assert st == 0 and acc == n and len(toks) == n + 1
    bonus = O.prepare_row(O.make_params(top_k=20, top_p=0.95, temperature=0.7,
                                        rng_state=(99 + n * O.GAMMA) & O.MASK64),
                          target[n], extra=drafts)
    assert toks[-1] == bonus.token
    assert rng_after == (99 + (n + 1) * O.GAMMA) & O.MASK64


def test_shard_topk_union_equals_global_topk():
    rng = np.random.default_rng(5)
    v, g, k = 4096, 4, 64
    x = rng.normal(0, 2.5, v).astype(np.float32)
    x[rng.choice(v, 40)] = 3.0  # ties across shards
    p = O.make_params(top_k=k, top_p=0.9, temperature=0.8, rng_state=5)
    full = O.prepare_row(p, x, cap=v)
    cands = []
    for s in range(g):
        vals, toks = O.shard_topk(v, s * v // g, p, x[s * v // g:(s + 1) * v // g], k)
        cands += list(zip(vals, toks))
    cands.sort(key=lambda c: (-c[0], c[1]))
    assert [t for _, t in cands[:k]] == list(full.cand_tokens[:k])


def test_boundary_helper_flags_exact_boundary():
    logits = O.f32_to_bf16_rne(np.array([1.0, 1.0], np.float32))
    r = O.prepare_row(O.make_params(top_k=0, top_p=0.5, temperature=1.0, rng_state=1), logits)
    assert is_boundary(r, 0.5)

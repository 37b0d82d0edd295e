"""GPU parity: the sm_100a engine (through the C ABI) against the reference
build and the canonical CPU oracle.

Bar (the north star's): token ids and top-k index sets bit-exact against the
canonical oracle (lowest-index ties); probabilities within 1e-6 relative;
a token mismatch is tolerated only at a draw / top-p boundary within 1e-6,
and every such case is counted.  Against the unmodified reference, every
difference must be a tie-order difference (same transformed value).
"""
import numpy as np
import pytest

import oracle as O
import q38s
from helpers import hex_to_bf16, is_boundary, load_cases, load_sequences, transformed_value
from q38s import synth

pytestmark = pytest.mark.gpu

PROB_RTOL = 1e-6


def oracle_params(cfg: q38s.ConfigV2, rng_state: int) -> O.RowParams:
    return O.make_params(top_k=cfg.top_k, top_p=cfg.top_p, min_p=cfg.min_p,
                         temperature=cfg.temperature, repetition_penalty=cfg.repetition_penalty,
                         frequency_penalty=cfg.frequency_penalty,
                         presence_penalty=cfg.presence_penalty, rng_state=rng_state)


def to_torch(arr, cuda):
    import torch
    if arr.dtype == np.uint16:
        return torch.from_numpy(arr.view(np.int16)).to(cuda).view(torch.bfloat16)
    return torch.from_numpy(arr).to(cuda)


# ------------------------------------------------------------------ golden
CASES = load_cases()


@pytest.mark.parametrize("case", CASES, ids=lambda c: c["name"])
def test_golden_case_through_sampler_api(case, cuda):
    cfg = case["config"]
    c1 = q38s.config_v1(top_k=cfg["top_k"], top_p=cfg["top_p"], temperature=cfg["temperature"],
                        repetition_penalty=cfg["repetition_penalty"],
                        frequency_penalty=cfg["frequency_penalty"],
                        presence_penalty=cfg["presence_penalty"], seed=cfg["seed"],
                        mode=cfg["mode"], version=cfg["version"])
    e = case["expect"]
    logits = hex_to_bf16(case["logits_bf16_hex"])
    if e.get("stage") == "ctor":
        with pytest.raises(q38s.Q38sError) as ex:
            q38s.Sampler(case["vocab"], c1)
        assert ex.value.code == e["error"] and ex.value.message == e["message"]
        return
    s = q38s.Sampler(case["vocab"], c1)
    if case["history"]:
        s.commit_tokens(case["history"])
    if e.get("stage") == "prepare":
        with pytest.raises(q38s.Q38sError) as ex:
            s.prepare(logits, case["extra"])
        assert ex.value.code == e["error"] and ex.value.message == e["message"]
        return
    tok, rb, ra = s.prepare(logits, case["extra"])
    assert (rb, ra) == (e["rng_before"], e["rng_after"])
    v = case["vocab"]
    counts = np.bincount(np.asarray(case["history"], np.int64), minlength=v).astype(np.uint32)
    p = O.make_params(top_k=cfg["top_k"], top_p=cfg["top_p"], temperature=cfg["temperature"],
                      repetition_penalty=cfg["repetition_penalty"],
                      frequency_penalty=cfg["frequency_penalty"],
                      presence_penalty=cfg["presence_penalty"], rng_state=cfg["seed"])
    can = O.prepare_row(p, logits, counts, case["extra"], O.TIE_CANONICAL)
    assert tok == can.token or is_boundary(can, cfg["top_p"])
    if tok != e["token"]:
        ref = O.prepare_row(p, logits, counts, case["extra"], O.TIE_LIBSTDCXX)
        assert transformed_value(can, tok) == transformed_value(ref, e["token"])


def test_golden_sequence_state_words(cuda):
    seq = load_sequences()["test_runtime_sequence"]
    cfg = seq["config"]
    s = q38s.Sampler(seq["vocab"], q38s.config_v1(
        top_k=cfg["top_k"], top_p=cfg["top_p"], temperature=cfg["temperature"],
        repetition_penalty=cfg["repetition_penalty"], frequency_penalty=cfg["frequency_penalty"],
        presence_penalty=cfg["presence_penalty"], seed=cfg["seed"]))
    logits = hex_to_bf16(seq["logits_bf16_hex"])
    states = [st for st in seq["steps"] if st["op"] == "state"]
    for step in seq["steps"]:
        if step["op"] == "prepare":
            d = s.prepare(logits, step["extra"])
            assert list(d) == step["expect"]   # V = 4, no ties: exact
            assert s.prepare(logits, step["extra"]) == d  # retry determinism
        elif step["op"] == "commit":
            s.commit(step["decision"])
        elif step["op"] == "commit_tokens":
            s.commit_tokens(step["tokens"])
        elif step["op"] == "reset":
            s.reset()
        elif step["op"] == "state":
            got = s.state()
            want = step["expect"]
            for k in want:
                assert getattr(got, k) == want[k], k
    assert len(states) == 2


def test_commit_rejects_mismatched_decision(cuda):
    s = q38s.Sampler(8, q38s.config_v1(top_k=2, top_p=0.9, seed=5))
    logits = synth.f32_to_bf16_rne(np.arange(8, dtype=np.float32))
    tok, rb, ra = s.prepare(logits)
    with pytest.raises(q38s.Q38sError) as ex:
        s.commit((tok, rb + 1, ra))
    assert ex.value.kind == "logic_error"
    assert ex.value.message == "sampler decision does not match committed state"
    s.commit((tok, rb, ra))
    assert s.state().sampled_tokens == 1
    with pytest.raises(q38s.Q38sError) as ex:
        s.commit_tokens([1, 2, 99, 3])
    assert ex.value.message == "committed penalty token is invalid"
    assert s.state().canonical_tokens == 2  # tokens before the invalid one stay


def test_cfg1_100_steps_against_reference_tokens(cuda):
    """Benchmark configuration 1 (bf16-rounded), 100 sequential steps.  Each
    step commits the REFERENCE's token so the two penalty histories stay
    identical; our token must equal the canonical oracle's and differ from
    the reference's only by tie order."""
    seq = load_sequences()["cfg1_100_steps"]
    cfg = seq["config"]
    c1 = q38s.config_v1(top_k=cfg["top_k"], top_p=cfg["top_p"], temperature=cfg["temperature"],
                        repetition_penalty=cfg["repetition_penalty"], seed=cfg["seed"])
    s = q38s.Sampler(synth.VOCAB, c1)
    hist = synth.cfg1_history()
    s.commit_tokens(hist)
    counts = np.bincount(hist, minlength=synth.VOCAB).astype(np.uint32)
    ties = boundary = 0
    for step, ref_tok in enumerate(seq["tokens"]):
        logits = synth.f32_to_bf16_rne(synth.cfg1_logits(step))
        tok, rb, ra = s.prepare(logits)
        p = O.make_params(top_k=cfg["top_k"], top_p=cfg["top_p"], temperature=cfg["temperature"],
                          repetition_penalty=cfg["repetition_penalty"], rng_state=rb)
        can = O.prepare_row(p, logits, counts, (), O.TIE_CANONICAL, cap=64)
        if tok != can.token:
            assert is_boundary(can, cfg["top_p"])
            boundary += 1
        if tok != ref_tok:
            ref = O.prepare_row(p, logits, counts, (), O.TIE_LIBSTDCXX, cap=64)
            assert transformed_value(can, tok) == transformed_value(ref, ref_tok)
            ties += 1
        s.commit((tok, rb, ra))
        s.commit_token(ref_tok)
        counts[ref_tok] += 1
    assert s.state().rng_state == seq["final_state"]["rng_state"]
    assert s.state().penalty_checksum == seq["final_state"]["penalty_checksum"]
    assert boundary == 0
    print(f"cfg1: tie-order differences vs sampling.cc {ties}/100, boundary 0")


# ------------------------------------------------------------- batches
def random_batch(rng, vocab, rows, dtype):
    configs = []
    for _ in range(rows):
        k = int(rng.choice([0, 1, 2, 5, 20, 64, 100, 128, min(vocab, 129), min(vocab, 300)]))
        configs.append(q38s.config_v2(
            top_k=min(k, vocab), top_p=float(rng.choice([1.0, 0.9, 0.5, float(rng.uniform(0.05, 1))])),
            temperature=float(rng.choice([0.3, 0.7, 1.0, 1.7])),
            repetition_penalty=float(rng.choice([1.0, 1.05, 1.3])),
            frequency_penalty=float(rng.choice([0.0, 0.0, 0.2, -0.1])),
            presence_penalty=float(rng.choice([0.0, 0.0, 0.5, -0.25])),
            min_p=float(rng.choice([0.0, 0.0, 0.05, float(rng.uniform(0, 0.1))])),
            seed=int(rng.integers(1, 2**63))))
    x = rng.normal(0, 2.5, (rows, vocab)).astype(np.float32)
    for r in range(rows):
        kind = r % 4
        if kind == 1:
            x[r] = np.round(x[r] * 2) / 2  # ties
        elif kind == 2:
            m = max(1, vocab // 64)
            x[r, rng.choice(vocab, m, replace=False)] = rng.uniform(8, 15, m)
        elif kind == 3:
            m = max(1, vocab // 50)
            x[r, rng.choice(vocab, m)] = rng.choice(np.array([-np.inf, np.inf, np.nan],
                                                             np.float32), m)
    logits = synth.f32_to_bf16_rne(x) if dtype == "bf16" else x
    hists = [rng.integers(0, vocab, int(rng.integers(0, 2 * vocab + 1))).astype(np.int32)
             for _ in range(rows)]
    return configs, logits, hists


def check_batch(configs, logits, hists, cuda, extra=None, cap=1024):
    import torch
    rows, vocab = logits.shape
    b = q38s.Batch(vocab, configs)
    st = b.commit_tokens(hists)
    assert (st == 0).all()
    dist, dt = q38s.make_distribution(rows, cap, cuda)
    xt = None
    if extra is not None:
        offs = np.zeros(rows + 1, np.uint32)
        for r, e in enumerate(extra):
            offs[r + 1] = offs[r] + len(e)
        flat = np.concatenate([np.asarray(e, np.int32) for e in extra] + [np.zeros(1, np.int32)])
        xt = (torch.from_numpy(flat).to(cuda), torch.from_numpy(offs.view(np.int32)).to(cuda))
    dec = b.decode_decisions(b.prepare(to_torch(logits, cuda), extra=xt, dist=dist))
    torch.cuda.synchronize()
    ntok = dt["n_candidates"].cpu().numpy()
    nret = dt["n_retained"].cpu().numpy()
    gtok = dt["tokens"].cpu().numpy().reshape(rows, cap)
    gprob = dt["probs"].cpu().numpy().reshape(rows, cap)
    boundary = 0
    for r in range(rows):
        counts = np.bincount(hists[r], minlength=vocab).astype(np.uint32)
        p = oracle_params(configs[r], configs[r].seed)
        ex = extra[r] if extra is not None else ()
        o = O.prepare_row(p, logits[r], counts, ex, O.TIE_CANONICAL, cap=cap)
        assert dec["rng_before"][r] == configs[r].seed
        if o.status != 0:
            assert dec["status"][r] != 0, f"row {r}: oracle status {o.status}"
            continue
        assert dec["status"][r] == 0, f"row {r} status {dec['status'][r]}"
        if dec["token"][r] != o.token:
            assert is_boundary(o, configs[r].top_p), f"row {r}: {dec['token'][r]} vs {o.token}"
            boundary += 1
        n = o.n_candidates
        assert ntok[r] == n, f"row {r}: {ntok[r]} candidates vs {n}"
        m = min(n, cap)
        assert (gtok[r, :m] == o.cand_tokens[:m]).all(), f"row {r}: candidate order"
        if nret[r] != o.n_retained:
            # the top-p running sum sits on top_p within the tolerance
            assert is_boundary(o, configs[r].top_p), f"row {r}: retained {nret[r]} vs {o.n_retained}"
            continue
        np.testing.assert_allclose(dt["total"].cpu().numpy()[r], o.total, rtol=PROB_RTOL)
        rr = min(o.n_retained, cap)
        want = o.cand_weights[:rr] / o.total
        np.testing.assert_allclose(gprob[r, :rr], want, rtol=PROB_RTOL, atol=0)
        assert (gprob[r, rr:m] == 0).all()
    return boundary


@pytest.mark.parametrize("vocab", [1, 2, 3, 31, 32, 33, 127, 1000, 4097])
@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_batch_small_vocab_matches_canonical_oracle(vocab, dtype, cuda):
    rng = np.random.default_rng(vocab * 7 + (dtype == "f32"))
    configs, logits, hists = random_batch(rng, vocab, 24, dtype)
    assert check_batch(configs, logits, hists, cuda) == 0


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_batch_full_vocab_matches_canonical_oracle(dtype, cuda):
    rng = np.random.default_rng(151936 + (dtype == "f32"))
    configs, logits, hists = random_batch(rng, synth.VOCAB, 16, dtype)
    assert check_batch(configs, logits, hists, cuda) == 0


def test_additional_penalty_tokens(cuda):
    rng = np.random.default_rng(3)
    vocab, rows = 5000, 8
    configs = [q38s.config_v2(top_k=20, top_p=0.9, temperature=0.8, repetition_penalty=1.3,
                              frequency_penalty=0.4, presence_penalty=0.2, seed=r + 1)
               for r in range(rows)]
    x = rng.normal(0, 2.5, (rows, vocab)).astype(np.float32)
    logits = synth.f32_to_bf16_rne(x)
    top = np.argsort(-x, axis=1)[:, :30]
    hists = [top[r, :10].astype(np.int32) for r in range(rows)]
    extra = [np.concatenate([top[r, 5:15], top[r, 5:8]]).astype(np.int32) for r in range(rows)]
    assert check_batch(configs, logits, hists, cuda, extra=extra) == 0


def test_general_paths(cuda):
    """Rows that overflow the fast path: full-vocabulary top_k = 0 without
    min-p (mass-weighted radix selection), top_k > 128 (radix cut + gather),
    an all-equal row (ties everywhere), non-finite rows."""
    vocab = synth.VOCAB
    rng = np.random.default_rng(99)
    rows = []
    cfgs = []
    for r, (k, p, mp) in enumerate([(0, 1.0, 0.0), (0, 0.9, 0.0), (0, 0.6, 0.0), (300, 0.95, 0.0),
                                    (1000, 1.0, 0.0), (0, 0.9, 1e-5), (50, 0.9, 0.0),
                                    (0, 1.0, 0.0)]):
        x = rng.normal(0, 2.5, vocab).astype(np.float32)
        if r == 6:
            x[:] = 1.0          # every logit equal
        if r == 7:
            x[:] = -np.inf
        rows.append(x)
        cfgs.append(q38s.config_v2(top_k=k, top_p=p, min_p=mp, temperature=1.1,
                                   repetition_penalty=1.1, seed=1000 + r))
    logits = synth.f32_to_bf16_rne(np.stack(rows))
    hists = [rng.integers(0, vocab, 2000).astype(np.int32) for _ in cfgs]
    assert check_batch(cfgs, logits, hists, cuda) == 0


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_general_path_full_distribution(dtype, cuda):
    """top_k = 0 rows at V = 151,936 (the reference's default configuration,
    a full sort of the vocabulary in sampling.cc:94-104): every candidate's
    token in canonical order and every probability w_i / total within 1e-6,
    with top_p 1.0, 0.95 and 0.5, penalties, ties and min-p."""
    vocab = synth.VOCAB
    rng = np.random.default_rng(1717 + (dtype == "f32"))
    cfgs, rows = [], []
    specs = [(0, 1.0, 0.0, 1.0), (0, 0.95, 0.0, 0.7), (0, 0.5, 0.0, 1.2), (0, 0.95, 0.0, 0.3),
             (0, 0.9, 1e-4, 1.0), (500, 0.95, 0.0, 1.1), (0, 0.8, 0.0, 2.0), (0, 1.0, 0.0, 0.6)]
    for r, (k, p, mp, t) in enumerate(specs):
        x = rng.normal(0, 2.5, vocab).astype(np.float32)
        synth.zipf_spikes(rng, x)
        if r == 6:
            x = np.round(x * 4) / 4  # wide tie groups
        cfgs.append(q38s.config_v2(top_k=k, top_p=p, min_p=mp, temperature=t,
                                   repetition_penalty=1.0 + 0.05 * (r % 3),
                                   presence_penalty=0.2 * (r % 2), seed=5000 + r))
        rows.append(x)
    x = np.stack(rows)
    logits = synth.f32_to_bf16_rne(x) if dtype == "bf16" else x
    hists = [rng.integers(0, vocab, int(rng.integers(0, 30000))).astype(np.int32) for _ in cfgs]
    b = check_batch(cfgs, logits, hists, cuda, cap=vocab)
    print(f"general path {dtype}: {b} boundary cases of {len(cfgs)}")
    assert b <= 1


def test_general_path_edge_rows(cuda):
    """An all-equal row (one tie group of 151,936), a row with a handful of
    finite values among -inf, huge temperatures, and a shortened capacity."""
    vocab = synth.VOCAB
    rng = np.random.default_rng(1718)
    rows, cfgs = [], []
    x = np.full(vocab, 1.5, np.float32)
    rows.append(x.copy()); cfgs.append(q38s.config_v2(top_k=0, top_p=0.37, seed=1))
    rows.append(x.copy()); cfgs.append(q38s.config_v2(top_k=0, top_p=1.0, seed=2))
    y = np.full(vocab, -np.inf, np.float32)
    y[rng.choice(vocab, 3000, replace=False)] = rng.normal(0, 1, 3000)
    rows.append(y); cfgs.append(q38s.config_v2(top_k=0, top_p=0.99, temperature=0.5, seed=3))
    z = rng.normal(0, 2.5, vocab).astype(np.float32)
    rows.append(z); cfgs.append(q38s.config_v2(top_k=0, top_p=0.999, temperature=50.0, seed=4))
    logits = synth.f32_to_bf16_rne(np.stack(rows))
    hists = [np.zeros(0, np.int32) for _ in cfgs]
    assert check_batch(cfgs, logits, hists, cuda, cap=vocab) <= 1
    assert check_batch(cfgs, logits, hists, cuda, cap=5000) <= 1


def test_sample_commit_steps_track_oracle(cuda):
    import torch
    rng = np.random.default_rng(21)
    vocab, rows, steps = 20000, 12, 6
    configs = [q38s.config_v2(top_k=int(rng.integers(1, 100)), top_p=0.9, temperature=0.8,
                              repetition_penalty=1.2, presence_penalty=0.3,
                              frequency_penalty=0.1 * (r % 2), min_p=0.01 * (r % 3),
                              seed=int(rng.integers(1, 2**63))) for r in range(rows)]
    b = q38s.Batch(vocab, configs)
    hists = [rng.integers(0, vocab, 300).astype(np.int32) for _ in range(rows)]
    b.commit_tokens(hists)
    counts = [np.bincount(h, minlength=vocab).astype(np.uint32) for h in hists]
    rngs = [c.seed for c in configs]
    for _ in range(steps):
        x = synth.f32_to_bf16_rne(rng.normal(0, 2.5, (rows, vocab)).astype(np.float32))
        dec = b.decode_decisions(b.sample_commit(to_torch(x, cuda)))
        for r in range(rows):
            o = O.prepare_row(oracle_params(configs[r], rngs[r]), x[r], counts[r], (),
                              O.TIE_CANONICAL, cap=128)
            assert dec["token"][r] == o.token or is_boundary(o, configs[r].top_p)
            counts[r][dec["token"][r]] += 1
            rngs[r] = o.rng_after
    torch.cuda.synchronize()
    for r, st in enumerate(b.states()):
        assert st.rng_state == rngs[r]
        assert st.sampled_tokens == steps
        assert st.canonical_tokens == 300 + steps


def test_batch_commit_checks_state(cuda):
    import torch
    b = q38s.Batch(100, [q38s.config_v2(top_k=5, seed=7), q38s.config_v2(top_k=5, seed=8)])
    x = torch.randn(2, 100, device=cuda)
    d = b.prepare(x)
    raw = d.clone()
    dd = raw.view(-1, 3)
    dd[1, 1] += 1  # corrupt row 1's rng_before
    b.commit(raw)
    dec = b.decode_decisions(raw)
    assert dec["status"][0] == 0 and dec["status"][1] == q38s.ROW_STATE_MISMATCH
    st = b.states()
    assert st[0].sampled_tokens == 1 and st[1].sampled_tokens == 0


# ------------------------------------------------------------- extensions
@pytest.mark.parametrize("n", [16, 20, 36])
def test_mtp_q_equals_p_accepts_every_draft(n, cuda):
    """q = p accepts every draft.  16, 20 and 36 drafts give 33, 41 and 73
    virtual rows, split into 8, 7 and 4 segments per row (a cluster each),
    more clusters than fit on the GPU at once."""
    import torch
    rng = np.random.default_rng(31)
    vocab = synth.VOCAB
    cfg = q38s.config_v2(top_k=20, top_p=0.95, temperature=0.7, seed=12345)
    target = rng.normal(0, 3, (n + 1, vocab)).astype(np.float32)
    p = oracle_params(cfg, cfg.seed)
    drafts = [O.prepare_row(p, target[i]).token for i in range(n)]
    b = q38s.Batch(vocab, [cfg])
    t = to_torch(target, cuda)
    res = b.decode_mtp(b.mtp_verify(0, t, t[:n], torch.tensor(drafts, dtype=torch.int32,
                                                               device=cuda)))
    assert res.status == 0 and res.n_accepted == n and res.n_tokens == n + 1
    bonus = O.prepare_row(oracle_params(cfg, (cfg.seed + n * O.GAMMA) & O.MASK64), target[n],
                          extra=drafts)
    assert res.tokens[n] == bonus.token
    assert list(res.tokens[:n]) == drafts
    assert res.rng_after == (cfg.seed + (n + 1) * O.GAMMA) & O.MASK64


def test_mtp_matches_oracle_verification(cuda):
    import torch
    rng = np.random.default_rng(32)
    vocab, n = 30000, 64
    target, draft = synth.cfg3_rows(seed=4, rows=n + 1, vocab=vocab)
    for seed in (1, 2, 3, 4):
        cfg = q38s.config_v2(top_k=20, top_p=0.95, temperature=0.7, seed=seed,
                             repetition_penalty=1.1)
        p = oracle_params(cfg, seed)
        drafts = []
        for i in range(n):
            pi = oracle_params(cfg, (seed * 77 + i) & O.MASK64)
            drafts.append(O.prepare_row(pi, draft[i], extra=drafts).token)
        b = q38s.Batch(vocab, [cfg])
        hist = rng.integers(0, vocab, 100).astype(np.int32)
        b.commit_tokens([hist])
        counts = np.bincount(hist, minlength=vocab).astype(np.uint32)
        res = b.decode_mtp(b.mtp_verify(0, to_torch(target, cuda), to_torch(draft[:n], cuda),
                                        torch.tensor(drafts, dtype=torch.int32, device=cuda)))
        toks, acc, rng_after, st = O.mtp_verify(p, target, draft[:n], drafts, counts)
        assert st == 0 and res.status == 0
        assert res.n_accepted == acc
        assert list(res.tokens[: res.n_tokens]) == list(toks)
        assert res.rng_after == rng_after


def test_vocab_shards_match_unsharded_row(cuda):
    import torch
    rng = np.random.default_rng(41)
    vocab, rows, k = synth.VOCAB, 32, 64
    x = synth.cfg5_logits(rows=rows, vocab=vocab)
    configs = [q38s.config_v2(top_k=64, top_p=0.9, temperature=0.8, repetition_penalty=1.1,
                              seed=int(rng.integers(1, 2**63))) for _ in range(rows)]
    hists = [rng.integers(0, vocab, 500).astype(np.int32) for _ in range(rows)]
    for g in (2, 4, 8):
        w = vocab // g
        gathered = []
        for s in range(g):
            sb = q38s.Batch(vocab, configs, shard=(s * w, w))
            sb.commit_tokens([h[(h >= s * w) & (h < (s + 1) * w)] for h in hists])
            shard = to_torch(np.ascontiguousarray(x[:, s * w:(s + 1) * w]), cuda)
            out = sb.shard_topk(shard, k)
            vals, toks = q38s.decode_candidates(out, rows, k)
            for r in range(0, rows, 7):
                counts = np.bincount(hists[r], minlength=vocab)[s * w:(s + 1) * w].astype(np.uint32)
                ov, ot = O.shard_topk(vocab, s * w, oracle_params(configs[r], 1),
                                      x[r, s * w:(s + 1) * w], k, counts)
                assert (toks[r] == ot).all() and (vals[r] == ov).all()
            gathered.append(out)
            last = sb
        allc = torch.cat(gathered)
        dec = last.decode_decisions(last.shard_merge_sample(allc, g, k))
        for r in range(rows):
            counts = np.bincount(hists[r], minlength=vocab).astype(np.uint32)
            o = O.prepare_row(oracle_params(configs[r], configs[r].seed), x[r], counts,
                              (), O.TIE_CANONICAL, cap=64)
            assert dec["token"][r] == o.token or is_boundary(o, 0.9)


def test_argmax_matches_reference_semantics(cuda):
    import torch
    rng = np.random.default_rng(51)
    for n in (1, 7, 256, 4097, 248_320):
        x = np.round(rng.normal(0, 2, n) * 4) / 4
        x = x.astype(np.float32)
        if n > 10:
            x[rng.choice(n, n // 10)] = np.nan
            x[rng.choice(n, n // 10)] = -np.inf
        w = synth.f32_to_bf16_rne(x)
        f = synth.bf16_to_f32(w)
        ok = f > np.float32(-3.402823466e38)
        want = int(np.flatnonzero(f == np.max(f[ok]))[0]) if ok.any() else -1
        out = torch.zeros(1, dtype=torch.int32, device=cuda)
        q38s.argmax_bf16(to_torch(w, cuda), out)
        assert int(out.item()) == want
    out = torch.zeros(1, dtype=torch.int32, device=cuda)
    q38s.argmax_bf16(to_torch(synth.f32_to_bf16_rne(np.full(300, -np.inf, np.float32)), cuda), out)
    assert int(out.item()) == -1


# ------------------------------------------------------- full-size config 4
def test_cfg4_batch_matches_canonical_oracle(cuda):
    """Benchmark configuration 4 at full size (256 x 151,936, heterogeneous
    rows): every token equals the canonical oracle's or is a counted
    boundary case."""
    spec = synth.cfg4_spec()
    logits = synth.cfg4_logits()
    configs = [q38s.config_v2(top_k=int(spec.top_k[r]), top_p=float(spec.top_p[r]),
                              min_p=float(spec.min_p[r]), temperature=float(spec.temperature[r]),
                              repetition_penalty=float(spec.repetition_penalty[r]),
                              seed=int(spec.seed[r])) for r in range(spec.rows)]
    b = q38s.Batch(spec.vocab, configs)
    b.commit_tokens(spec.histories)
    dec = b.decode_decisions(b.prepare(to_torch(logits, cuda)))
    params = [oracle_params(c, c.seed) for c in configs]
    counts = np.stack([np.bincount(h, minlength=spec.vocab).astype(np.uint32)
                       for h in spec.histories])
    toks, status = O.prepare_rows(params, logits, counts, O.TIE_CANONICAL, threads=8)
    assert (status == 0).all() and (dec["status"] == 0).all()
    bad = np.flatnonzero(toks != dec["token"])
    for r in bad:
        o = O.prepare_row(params[r], logits[r], counts[r], (), O.TIE_CANONICAL, cap=4096)
        assert is_boundary(o, configs[r].top_p), f"row {r}"
    print(f"cfg4: {len(bad)} boundary cases of {spec.rows}")


def test_one_session_general_rows(cuda):
    """The one-session sampler launches the general kernel itself when its
    row is deferred (top_k = 0 at full vocabulary): decisions equal the
    canonical oracle's over a few committed steps, for bf16 and fp32."""
    import torch
    rng = np.random.default_rng(808)
    vocab = synth.VOCAB
    for dtype in ("bf16", "f32"):
        cfg = q38s.config_v2(top_k=0, top_p=0.9, temperature=1.0, repetition_penalty=1.1,
                             seed=4242)
        s = q38s.Sampler(vocab, cfg)
        hist = rng.integers(0, vocab, 500).astype(np.int32)
        s.commit_tokens(hist)
        counts = np.bincount(hist, minlength=vocab).astype(np.uint32)
        for step in range(4):
            x = rng.normal(0, 2.5, vocab).astype(np.float32)
            synth.zipf_spikes(rng, x)
            logits = synth.f32_to_bf16_rne(x) if dtype == "bf16" else x
            tok, rb, ra = s.prepare_device(to_torch(logits, cuda))
            p = oracle_params(cfg, rb)
            o = O.prepare_row(p, logits, counts, (), O.TIE_CANONICAL, cap=64)
            if tok != o.token:
                full = O.prepare_row(p, logits, counts, (), O.TIE_CANONICAL)
                assert is_boundary(full, 0.9), f"{dtype} step {step}: {tok} vs {o.token}"
            assert s.prepare_device(to_torch(logits, cuda)) == (tok, rb, ra)  # retry
            s.commit((tok, rb, ra))
            s.commit_token(tok)
            counts[tok] += 1
        torch.cuda.synchronize()

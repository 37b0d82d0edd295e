"""GPU parity at the benchmark configurations' full stated sizes.

Each test runs one benchmark configuration as BASELINE.json states it, through
the C ABI, and checks every token against the canonical CPU oracle
(oracle/q38_oracle.cc, lowest-index ties) and, where the reference accepts
the input (bf16 only), against the unmodified reference (src/sampling.cc,
compiled into oracle/_ref).  The bar is the parity contract's:

* a token differs from the canonical oracle only where the uniform draw or the
  top-p running sum lies within 1e-6 of a boundary (counted, printed);
* a token differs from the reference only by tie order (the two tokens have
  the same transformed value) or at such a boundary.

cfg1  1 row, 1,000 sequential steps (logits regenerated from seed + step),
      4,096-token history, T 0.7, top-k 20, top-p 0.8, repetition 1.05:
      bf16-pinned (the reference sees the same bf16 words) and fp32-native.
cfg2  the 10,000-step decode loop, history growing from 8,192 to 18,192
      tokens, T 0.6, top-k 20, top-p 0.95, presence 0.5; final state words.
cfg3  speculative verification at V = 151,936, 64 drafts + 1 bonus row,
      8 seeds; acceptance counts printed.
cfg4  256 rows, 200 consecutive sample-commit steps, 4 parameter draws.
"""
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

import oracle as O
import q38s
from helpers import is_boundary, transformed_value
from q38s import synth

pytestmark = pytest.mark.gpu

V = synth.VOCAB
THREADS = 16


def to_device(arr, cuda):
    import torch
    if arr.dtype == np.uint16:
        return torch.from_numpy(arr.view(np.int16)).to(cuda).view(torch.bfloat16)
    return torch.from_numpy(arr).to(cuda)


def params(cfg: dict, rng_state: int, min_p: float = 0.0) -> O.RowParams:
    return O.make_params(top_k=cfg.get("top_k", 0), top_p=cfg.get("top_p", 1.0), min_p=min_p,
                         temperature=cfg.get("temperature", 1.0),
                         repetition_penalty=cfg.get("repetition_penalty", 1.0),
                         frequency_penalty=cfg.get("frequency_penalty", 0.0),
                         presence_penalty=cfg.get("presence_penalty", 0.0),
                         rng_state=rng_state)


def checksum_after(checksum: int, canonical: int, tokens) -> tuple[int, int]:
    """commit_token's state words (sampling.cc:163-172) in Python."""
    for t in tokens:
        canonical += 1
        checksum ^= O.splitmix64((int(t) & 0xFFFFFFFF) ^ ((canonical * O.GAMMA) & O.MASK64))
    return checksum, canonical


# ------------------------------------------------------------------ cfg1
def _cfg1(cuda, native_fp32: bool):
    cfg = synth.CFG1
    sampler = q38s.Sampler(V, q38s.config_v1(top_k=cfg["top_k"], top_p=cfg["top_p"],
                                             temperature=cfg["temperature"],
                                             repetition_penalty=cfg["repetition_penalty"],
                                             seed=cfg["seed"]))
    ref = None
    if not native_fp32 and O.ref_available():
        ref = O.RefSampler(V, O.make_config(top_k=cfg["top_k"], top_p=cfg["top_p"],
                                            temperature=cfg["temperature"],
                                            repetition_penalty=cfg["repetition_penalty"],
                                            seed=cfg["seed"]))
    hist = synth.cfg1_history()
    sampler.commit_tokens(hist)
    if ref is not None:
        ref.commit_tokens(hist)
    counts = np.bincount(hist, minlength=V).astype(np.uint32)
    boundary = ties = 0
    for step in range(1000):
        x = synth.cfg1_logits(step)
        logits = x if native_fp32 else synth.f32_to_bf16_rne(x)
        tok, rb, ra = sampler.prepare_device(to_device(logits, cuda))
        can = O.prepare_row(params(cfg, rb), logits, counts, (), O.TIE_CANONICAL, cap=64)
        if tok != can.token:
            full = O.prepare_row(params(cfg, rb), logits, counts, (), O.TIE_CANONICAL)
            assert is_boundary(full, cfg["top_p"]), f"step {step}: {tok} vs oracle {can.token}"
            boundary += 1
        commit_tok = tok
        if ref is not None:
            rtok, rrb, rra = ref.prepare(logits)
            assert (rrb, rra) == (rb, ra)
            if rtok != tok:
                lib = O.prepare_row(params(cfg, rb), logits, counts, (), O.TIE_LIBSTDCXX, cap=64)
                same_value = transformed_value(can, tok) == transformed_value(lib, rtok)
                assert same_value or tok != can.token, f"step {step}: {tok} vs reference {rtok}"
                ties += 1
            ref.commit((rtok, rrb, rra))
            ref.commit_token(rtok)
            commit_tok = rtok  # both histories follow the reference
        sampler.commit((tok, rb, ra))
        sampler.commit_token(commit_tok)
        counts[commit_tok] += 1
    st = sampler.state()
    assert st.sampled_tokens == 1000 and st.canonical_tokens == 4096 + 1000
    assert st.rng_state == (cfg["seed"] + 1000 * O.GAMMA) & O.MASK64
    if ref is not None:
        rs = ref.state()
        assert (rs.rng_state, rs.penalty_checksum) == (st.rng_state, st.penalty_checksum)
    return boundary, ties


def test_cfg1_1000_steps_bf16_against_reference_and_oracle(cuda):
    boundary, ties = _cfg1(cuda, native_fp32=False)
    print(f"cfg1 bf16: 1,000 steps, boundary cases {boundary}, "
          f"tie-order differences from sampling.cc {ties}")
    assert boundary <= 2


def test_cfg1_1000_steps_fp32_native(cuda):
    boundary, _ = _cfg1(cuda, native_fp32=True)
    print(f"cfg1 fp32-native: 1,000 steps, boundary cases {boundary}")
    assert boundary <= 2


# ------------------------------------------------------------------ cfg2
def test_cfg2_10000_step_decode_loop(cuda):
    """The batch-1 decode loop as the benchmark times it: prepare on device
    bf16 logits, commit, commit_token; 10,000 steps, history growing from
    8,192 tokens.  Every token is checked against the canonical oracle given
    the history so far (the checks run after the loop, in parallel)."""
    cfg = synth.CFG2
    c2 = q38s.config_v2(top_k=cfg["top_k"], top_p=cfg["top_p"], min_p=cfg["min_p"],
                        temperature=cfg["temperature"], presence_penalty=cfg["presence_penalty"],
                        seed=cfg["seed"])
    sampler = q38s.Sampler(V, c2)
    hist = synth.cfg2_history()
    sampler.commit_tokens(hist)
    steps = 10_000
    tokens = np.empty(steps, np.int32)
    for step in range(steps):
        tok, rb, ra = sampler.prepare_device(to_device(synth.cfg2_logits(step), cuda))
        assert rb == (cfg["seed"] + step * O.GAMMA) & O.MASK64
        sampler.commit((tok, rb, ra))
        sampler.commit_token(tok)
        tokens[step] = tok

    def check(chunk):
        lo, hi = chunk
        counts = np.bincount(np.concatenate([hist, tokens[:lo]]), minlength=V).astype(np.uint32)
        bad = []
        for step in range(lo, hi):
            logits = synth.cfg2_logits(step)
            p = params(cfg, (cfg["seed"] + step * O.GAMMA) & O.MASK64, cfg["min_p"])
            o = O.prepare_row(p, logits, counts, (), O.TIE_CANONICAL, cap=64)
            if o.token != tokens[step]:
                full = O.prepare_row(p, logits, counts, (), O.TIE_CANONICAL)
                bad.append((step, int(tokens[step]), o.token, is_boundary(full, cfg["top_p"])))
            counts[tokens[step]] += 1
        return bad

    edges = np.linspace(0, steps, THREADS + 1).astype(int)
    with ThreadPoolExecutor(THREADS) as ex:
        bad = [b for part in ex.map(check, zip(edges[:-1], edges[1:])) for b in part]
    assert all(b[3] for b in bad), f"non-boundary mismatches: {[b for b in bad if not b[3]][:5]}"
    st = sampler.state()
    checksum, canonical = checksum_after(0, 0, np.concatenate([hist, tokens]))
    assert st.sampled_tokens == steps and st.canonical_tokens == canonical == 8192 + steps
    assert st.rng_state == (cfg["seed"] + steps * O.GAMMA) & O.MASK64
    assert st.penalty_checksum == checksum
    print(f"cfg2: 10,000 steps, history 8,192 -> 18,192, boundary cases {len(bad)}")
    assert len(bad) <= 3


# ------------------------------------------------------------------ cfg3
def test_cfg3_speculative_verification_full_vocab_8_seeds(cuda):
    """65 rows x 151,936 fp32 target logits, draft = target + N(0, 0.5^2),
    64 drafts sampled from the draft distribution, rejection sampling with a
    residual resample; every result (accepted count, published tokens, RNG
    state) equals the oracle's rejection sampler.  Parity is unpinned beyond
    the oracle: the reference has no sampled verification."""
    import torch
    cfg = synth.CFG3
    n = 64
    accepted = []
    for seed in range(8):
        target, draft = synth.cfg3_rows(seed=100 + seed)
        state = (cfg["seed"] * 1000 + seed) & O.MASK64
        drafts = []
        for i in range(n):  # the drafter's own draws from its distribution
            pi = params(cfg, (state * 77 + i) & O.MASK64)
            drafts.append(O.prepare_row(pi, draft[i], extra=drafts, cap=32).token)
        c2 = q38s.config_v2(top_k=cfg["top_k"], top_p=cfg["top_p"],
                            temperature=cfg["temperature"], seed=state)
        b = q38s.Batch(V, [c2])
        res = b.decode_mtp(b.mtp_verify(0, to_device(target, cuda), to_device(draft[:n], cuda),
                                        torch.tensor(drafts, dtype=torch.int32, device=cuda)))
        toks, acc, rng_after, st = O.mtp_verify(params(cfg, state), target, draft[:n], drafts)
        assert st == 0 and res.status == 0, f"seed {seed}: status {res.status} / {st}"
        assert res.n_accepted == acc, f"seed {seed}: accepted {res.n_accepted} vs {acc}"
        assert list(res.tokens[: res.n_tokens]) == list(toks), f"seed {seed}"
        assert res.rng_after == rng_after
        accepted.append(acc)
    print(f"cfg3: accepted drafts per verification over 8 seeds: {accepted}")


# ------------------------------------------------------------------ cfg4
def _cfg4_configs(spec):
    return [q38s.config_v2(top_k=int(spec.top_k[r]), top_p=float(spec.top_p[r]),
                           min_p=float(spec.min_p[r]), temperature=float(spec.temperature[r]),
                           repetition_penalty=float(spec.repetition_penalty[r]),
                           seed=int(spec.seed[r])) for r in range(spec.rows)]


@pytest.mark.parametrize("draw", [4, 5, 6, 7])
def test_cfg4_200_sample_commit_steps(draw, cuda):
    """256 rows x 151,936 bf16, heterogeneous parameters of draw `draw`, 200
    consecutive q38s_batch_sample_commit steps over four rotating logit
    batches: every token equals the canonical oracle's given the history so
    far (the sampled tokens feed the repetition penalties) or is a counted
    boundary case; the final state words follow."""
    spec = synth.cfg4_spec(seed=draw)
    configs = _cfg4_configs(spec)
    b = q38s.Batch(spec.vocab, configs)
    b.commit_tokens(spec.histories)
    batches = [synth.cfg4_logits(batch=i, seed=draw) for i in range(4)]
    dev = [to_device(x, cuda) for x in batches]
    counts = np.stack([np.bincount(h, minlength=V).astype(np.uint32) for h in spec.histories])
    rngs = [int(s) for s in spec.seed]
    boundary = 0
    general = 0
    for step in range(200):
        dec = b.decode_decisions(b.sample_commit(dev[step % 4]))
        logits = batches[step % 4]
        plist = [O.make_params(top_k=c.top_k, top_p=c.top_p, min_p=c.min_p,
                               temperature=c.temperature,
                               repetition_penalty=c.repetition_penalty, rng_state=rngs[r])
                 for r, c in enumerate(configs)]
        toks, status = O.prepare_rows(plist, logits, counts, O.TIE_CANONICAL, threads=THREADS)
        assert (status == 0).all() and (dec["status"] == 0).all(), f"step {step}"
        for r in np.flatnonzero(toks != dec["token"]):
            full = O.prepare_row(plist[r], logits[r], counts[r], (), O.TIE_CANONICAL)
            assert is_boundary(full, configs[r].top_p), \
                f"draw {draw} step {step} row {r}: {dec['token'][r]} vs oracle {toks[r]}"
            boundary += 1
        for r in range(spec.rows):
            counts[r, dec["token"][r]] += 1
            rngs[r] = (rngs[r] + O.GAMMA) & O.MASK64
        if step == 199:
            general = int(sum(1 for r, c in enumerate(configs) if c.top_k == 0))
    for r, st in enumerate(b.states()):
        assert st.rng_state == rngs[r] and st.sampled_tokens == 200
        assert st.canonical_tokens == len(spec.histories[r]) + 200
    print(f"cfg4 draw {draw}: 200 steps x 256 rows, boundary cases {boundary} "
          f"({general} rows with top_k = 0)")
    assert boundary <= 4

"""Parity runs on captured logits (q38.logits.bf16.v1) through the GPU path.

* The greedy fixtures: q38s_argmax_bf16 on the capture reproduces the
  runtime's selected_token.
* The sampled fixture: a sampler session with the configuration and history
  recorded in the manifest draws the reference sampler's selected_token.
* Every capture found under $Q38S_LOGIT_CAPTURES (a directory of captures
  written by the reference's tools/q38_logit_parity.py from a live runtime;
  the committed fixtures when unset): the batch sampler under a set of
  sampling configurations must draw the canonical oracle's token on the
  captured row, or a counted boundary case.
"""
import os
from pathlib import Path

import numpy as np
import pytest

import oracle as O
import q38s
from helpers import is_boundary
from q38s import capture as cap
from q38s import synth

pytestmark = pytest.mark.gpu

FIX = Path(__file__).resolve().parent / "golden" / "logit_captures"

CONFIGS = [
    dict(top_k=0, top_p=1.0, temperature=1.0, repetition_penalty=1.0),
    dict(top_k=1, top_p=1.0, temperature=1.0, repetition_penalty=1.0),
    dict(top_k=40, top_p=0.9, temperature=0.7, repetition_penalty=1.1),
    dict(top_k=0, top_p=0.95, temperature=1.3, repetition_penalty=1.0),
    dict(top_k=100, top_p=0.5, temperature=0.5, repetition_penalty=1.2, frequency_penalty=0.1,
         presence_penalty=0.2),
]


def _captures():
    root = os.environ.get("Q38S_LOGIT_CAPTURES")
    paths = cap.find_captures(root) if root else cap.find_captures(FIX)
    return [cap.read_capture(p) for p in paths]


def test_greedy_reproduces_the_selected_token(cuda):
    caps = [cap.read_capture(FIX / f"{n}.json") for n in ("tiny", "decode_4096")]
    assert cap.greedy_tokens(caps) == [c.selected_token for c in caps]


def test_sampled_capture_reproduces_the_reference_draw(cuda):
    c = cap.read_capture(FIX / "sampled_151936.json")
    conf = dict(c.meta["q38s_sampling_config"])
    assert conf.pop("history") == "q38s.synth.cfg1_history()"
    tok = cap.sample_captures([c], q38s.config_v1(**conf), [synth.cfg1_history()])
    assert tok == [c.selected_token]


def test_capture_rows_match_the_canonical_oracle(cuda):
    caps = _captures()
    assert caps, "no captures found"
    boundary = total = 0
    for c in caps:
        vocab = c.element_count
        hist = np.random.default_rng(vocab).integers(0, vocab, min(vocab, 512)).astype(np.int32)
        counts = np.bincount(hist, minlength=vocab).astype(np.uint32)
        for j, conf in enumerate(CONFIGS):
            if conf["top_k"] > vocab:  # the sampler rejects it (sampling.cc:51)
                continue
            seed = 1000 + j
            cfg = q38s.config_v1(seed=seed, **conf)
            got = cap.sample_captures([c], cfg, [hist])[0]
            p = O.make_params(rng_state=seed, **conf)
            o = O.prepare_row(p, c.logits, counts, (), O.TIE_CANONICAL)
            total += 1
            if got != o.token:
                assert is_boundary(o, conf["top_p"]), \
                    f"{c.path.name} config {j}: {got} vs oracle {o.token}"
                boundary += 1
    print(f"capture parity: {len(caps)} captures x {len(CONFIGS)} configurations, "
          f"boundary cases {boundary} of {total}")
    assert boundary <= max(1, total // 50)

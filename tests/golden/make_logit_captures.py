"""Generate the q38.logits.bf16.v1 capture fixtures in logit_captures/.

Runs in the build container only (it needs the reference sources): the
captures are written by the reference's OWN capture tool
(tools/q38_logit_parity.py, write_capture) from snapshots laid out as the
runtime emits them (src/rpc.cc:123-166), and the comparison results come from
the same tool's compare_captures.  Run from the repository root after
``make -C oracle``:

    python tests/golden/make_logit_captures.py

Fixtures:

* tiny           the three words of the reference tool's own unit test
                 (tests/test_logit_parity.py:34), greedy.
* decode_4096    4,096 logits with exact ties, -inf and NaN; selected_token =
                 the greedy choice (largest finite value, lowest index).
* sampled_151936 a full-vocabulary decode row (benchmark configuration 1's
                 distribution, step 0); selected_token = the reference
                 sampler's prepare() with the configuration stored in the
                 manifest under "q38s_sampling_config" (an extra manifest
                 field; the reference tool keeps unknown fields) after the
                 configuration-1 history.
* comparisons.json  compare_captures of the reference tool on pairs of these
                 captures (identical, one word changed, selected token
                 changed), with paths removed.
"""
from __future__ import annotations

import importlib.util
import json
import shutil
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "oracle"))
sys.path.insert(0, str(ROOT / "qwen3.8-flash-next-dual-gpu_b200"))
import oracle as O  # noqa: E402
from q38s import synth  # noqa: E402

OUT = Path(__file__).resolve().parent / "logit_captures"
sys.path.insert(0, str(ROOT))
from __graft_entry__ import reference_root  # noqa: E402  (the reference checkout, if any)


def ref_tool():
    root = reference_root()
    if root is None:
        raise SystemExit("the reference sources are needed: set Q38S_REFERENCE_ROOT")
    tools = Path(root) / "tools"
    sys.path.insert(0, str(tools))  # the tool imports its RPC client beside it
    spec = importlib.util.spec_from_file_location("q38_logit_parity",
                                                  tools / "q38_logit_parity.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def snapshot(tool, words: np.ndarray, selected: int, epoch: int, frontier: int,
             kind: str = "decode") -> dict:
    raw = np.asarray(words, dtype="<u2").tobytes()
    return {"schema": "q38.logits.bf16.v1", "dtype": "bf16", "byte_order": "little",
            "transaction_epoch": epoch, "target_frontier": frontier,
            "transaction_kind": kind, "selected_token": int(selected),
            "element_count": len(raw) // 2, "fnv1a64": tool.fnv1a64(raw),
            "raw_bf16_le_hex": raw.hex(), "session_hash": 0x5EED}


def greedy(words: np.ndarray) -> int:
    f = synth.bf16_to_f32(words)
    ok = f > np.float32(-3.402823466e38)
    return int(np.flatnonzero(f == np.max(f[ok]))[0]) if ok.any() else -1


def main():
    tool = ref_tool()
    if OUT.exists():
        shutil.rmtree(OUT)
    OUT.mkdir()
    tiny = np.frombuffer(b"\x00\x3f\x80\x3f\x00\xc0", dtype="<u2")
    tool.write_capture(snapshot(tool, tiny, greedy(tiny), 7, 42), OUT / "tiny")

    rng = np.random.default_rng(4096)
    x = (np.round(rng.normal(0, 2, 4096) * 2) / 2).astype(np.float32)
    x[rng.choice(4096, 200, replace=False)] = -np.inf
    x[rng.choice(4096, 50, replace=False)] = np.nan
    x[[17, 900, 3001]] = 9.5  # three-way tie at the top
    w = synth.f32_to_bf16_rne(x)
    tool.write_capture(snapshot(tool, w, greedy(w), 8, 43), OUT / "decode_4096")

    w = synth.cfg1_logits(0)
    hist = synth.cfg1_history()
    cfg = dict(top_k=40, top_p=0.9, temperature=0.7, repetition_penalty=1.1, seed=1234)
    s = O.RefSampler(synth.VOCAB, O.make_config(**cfg))
    s.commit_tokens(hist)
    tok = s.prepare(w)[0]
    snap = snapshot(tool, w, tok, 9, 44)
    snap["q38s_sampling_config"] = dict(cfg, history="q38s.synth.cfg1_history()")
    tool.write_capture(snap, OUT / "sampled_151936")

    comparisons = {}
    w2 = synth.f32_to_bf16_rne(x)
    w3 = w2.copy()
    w3[1234] ^= 1
    pairs = {"same": (w2, greedy(w2)), "one_word": (w3, greedy(w3)),
             "token": (w2, greedy(w2) + 1)}
    for name, (words, sel) in pairs.items():
        tool.write_capture(snapshot(tool, words, sel, 8, 43), OUT / f"pair_{name}")
        r = tool.compare_captures(OUT / "decode_4096.json", OUT / f"pair_{name}.json")
        for side in ("left", "right"):
            r[side].pop("path")
        comparisons[name] = r
    (OUT / "comparisons.json").write_text(json.dumps(comparisons, indent=2, sort_keys=True)
                                          + "\n")
    print("wrote", sorted(p.name for p in OUT.iterdir()))


if __name__ == "__main__":
    main()

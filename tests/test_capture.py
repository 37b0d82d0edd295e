"""The q38.logits.bf16.v1 capture reader (q38s.capture) on the CPU.

The fixtures in golden/logit_captures were written by the reference's own
capture tool (tools/q38_logit_parity.py) and its compare_captures results are
in comparisons.json (golden/make_logit_captures.py).  The reader must load
them with both checksums verified, write byte-identical manifests from the
same snapshots, reproduce the tool's comparison results, and reject every
malformed input with the tool's message.
"""
import json
import shutil
from pathlib import Path

import numpy as np
import pytest

from q38s import capture as cap
from q38s import synth

FIX = Path(__file__).resolve().parent / "golden" / "logit_captures"
NAMES = ["tiny", "decode_4096", "sampled_151936", "pair_same", "pair_one_word", "pair_token"]


def _snapshot_of(c: cap.LogitCapture) -> dict:
    snap = {k: v for k, v in c.meta.items()
            if k not in ("capture_schema", "raw_file", "raw_bytes", "sha256")}
    snap["raw_bf16_le_hex"] = c.raw().hex()
    return snap


def test_fnv1a64_known_answers():
    assert cap.fnv1a64(b"") == "cbf29ce484222325"
    assert cap.fnv1a64(b"a") == "af63dc4c8601ec8c"  # published FNV-1a 64 test vector
    assert cap.fnv1a64(b"foobar") == "85944171f73967e8"


@pytest.mark.parametrize("name", NAMES)
def test_reads_reference_written_captures(name):
    c = cap.read_capture(FIX / f"{name}.json")
    assert c.logits.dtype == np.uint16 and c.logits.size == c.element_count
    assert c.raw() == (FIX / f"{name}.bf16").read_bytes()
    assert c.meta["schema"] == cap.SNAPSHOT_SCHEMA


@pytest.mark.parametrize("name", NAMES)
def test_written_manifest_is_byte_identical(name, tmp_path):
    c = cap.read_capture(FIX / f"{name}.json")
    cap.write_capture(_snapshot_of(c), tmp_path / name)
    assert (tmp_path / f"{name}.json").read_bytes() == (FIX / f"{name}.json").read_bytes()
    assert (tmp_path / f"{name}.bf16").read_bytes() == (FIX / f"{name}.bf16").read_bytes()


def test_greedy_selected_tokens_of_the_greedy_fixtures():
    for name in ("tiny", "decode_4096"):
        c = cap.read_capture(FIX / f"{name}.json")
        f = synth.bf16_to_f32(c.logits)
        ok = f > np.float32(-3.402823466e38)
        assert c.selected_token == int(np.flatnonzero(f == np.max(f[ok]))[0])
    assert cap.read_capture(FIX / "decode_4096.json").selected_token == 17  # 3-way tie


def test_comparisons_match_the_reference_tool():
    want = json.loads((FIX / "comparisons.json").read_text())
    for name, expect in want.items():
        got = cap.compare_captures(FIX / "decode_4096.json", FIX / f"pair_{name}.json")
        for side in ("left", "right"):
            got[side].pop("path")
        assert got == expect, name


def test_find_captures_lists_manifests_only():
    found = [p.name for p in cap.find_captures(FIX)]
    assert found == sorted(f"{n}.json" for n in NAMES)
    assert cap.find_captures(FIX / "tiny.json") == [FIX / "tiny.json"]


def test_cli_compare_exit_codes(capsys):
    assert cap.main(["compare", str(FIX / "decode_4096.json"),
                     str(FIX / "pair_same.json")]) == 0
    assert cap.main(["compare", str(FIX / "decode_4096.json"),
                     str(FIX / "pair_one_word.json")]) == 1
    out = capsys.readouterr().out
    assert '"first_mismatch"' in out


# ------------------------------------------------------------------ rejections
def _good_snapshot():
    return _snapshot_of(cap.read_capture(FIX / "tiny.json"))


@pytest.mark.parametrize("edit,message", [
    (lambda s: s.update(schema="q38.logits.f32.v1"), "unsupported logit snapshot schema"),
    (lambda s: s.update(dtype="f16"), "not little-endian BF16"),
    (lambda s: s.update(byte_order="big"), "not little-endian BF16"),
    (lambda s: s.update(element_count=0), "invalid element count"),
    (lambda s: s.update(element_count="3"), "invalid element count"),
    (lambda s: s.pop("raw_bf16_le_hex"), "did not include raw BF16 values"),
    (lambda s: s.update(raw_bf16_le_hex=12), "not hex text"),
    (lambda s: s.update(raw_bf16_le_hex="zz"), "malformed"),
    (lambda s: s.update(raw_bf16_le_hex="003f"), "length differs from element count"),
    (lambda s: s.update(fnv1a64="0" * 16), "checksum does not match the runtime"),
])
def test_snapshot_rejections(edit, message):
    s = _good_snapshot()
    edit(s)
    with pytest.raises(ValueError, match=message):
        cap.parse_snapshot(s)


def test_snapshot_without_payload_is_allowed_when_not_required():
    s = _good_snapshot()
    s.pop("raw_bf16_le_hex")
    assert cap.parse_snapshot(s, require_raw=False) is None
    assert cap.parse_snapshot(json.dumps(_good_snapshot())).logits.size == 3


def _copy(tmp_path, name="decode_4096"):
    for ext in (".json", ".bf16"):
        shutil.copy(FIX / f"{name}{ext}", tmp_path / f"{name}{ext}")
    return tmp_path / f"{name}.json", json.loads((FIX / f"{name}.json").read_text())


def test_manifest_rejections(tmp_path):
    path, meta = _copy(tmp_path)
    raw = (FIX / "decode_4096.bf16").read_bytes()

    def put(m):
        path.write_text(json.dumps(m))

    put(dict(meta, capture_schema="OTHER"))
    with pytest.raises(ValueError, match="is not a Q38 logit capture"):
        cap.read_capture(path)
    put({k: v for k, v in meta.items() if k != "raw_file"})
    with pytest.raises(ValueError, match="has no raw BF16 file"):
        cap.read_capture(path)
    put(dict(meta, raw_bytes=meta["raw_bytes"] - 2))
    with pytest.raises(ValueError, match="length does not match its manifest"):
        cap.read_capture(path)
    put(meta)
    bad = bytearray(raw)
    bad[10] ^= 1
    (tmp_path / "decode_4096.bf16").write_bytes(bytes(bad))
    with pytest.raises(ValueError, match="SHA-256 does not match"):
        cap.read_capture(path)
    import hashlib
    put(dict(meta, sha256=hashlib.sha256(bytes(bad)).hexdigest()))
    with pytest.raises(ValueError, match="FNV-1a does not match"):
        cap.read_capture(path)


def test_cli_check_without_captures(tmp_path, capsys):
    """`python -m q38s.capture check DIR` on a directory without captures
    reports none and exits 1 (no GPU is touched)."""
    (tmp_path / "notes.json").write_text('{"schema": "other"}')
    assert cap.main(["check", str(tmp_path)]) == 1
    assert json.loads(capsys.readouterr().out) == {"captures": 0}

"""Captured target logits (schema q38.logits.bf16.v1) as sampler input.

The reference runtime answers its RPC kLogits request (include/q38/rpc.h:35)
with one JSON snapshot of the committed target logits (src/rpc.cc:123-166):

    {"schema": "q38.logits.bf16.v1", "dtype": "bf16", "byte_order": "little",
     "transaction_epoch": E, "target_frontier": F, "transaction_kind": K,
     "selected_token": T, "element_count": N, "fnv1a64": "<16 hex>",
     "raw_bf16_le_hex": "<4 hex digits per logit: low byte, high byte>"}

and its capture tool (tools/q38_logit_parity.py:20-21, :33-100) stores a
snapshot as a manifest `<name>.json` (the snapshot fields without the hex,
plus capture_schema "Q38_LOGIT_CAPTURE_V1", raw_file, raw_bytes, sha256)
beside the raw little-endian bf16 words in `<name>.bf16`.

This module reads both forms with the same checks and messages as the
reference tool, hands the logits to the GPU sampler, and compares captures
the way the tool does.  `python -m q38s.capture check CAPTURE.json ...`
runs the greedy selection (q38s_argmax_bf16) on each capture and reports
whether it reproduces the runtime's selected_token.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

import numpy as np

SNAPSHOT_SCHEMA = "q38.logits.bf16.v1"
CAPTURE_SCHEMA = "Q38_LOGIT_CAPTURE_V1"
COMPARISON_SCHEMA = "Q38_LOGIT_COMPARISON_V1"

_FNV_OFFSET = 0xCBF29CE484222325
_FNV_PRIME = 0x100000001B3
_MASK64 = (1 << 64) - 1

# fields that must agree for two captures to describe the same logits
# (tools/q38_logit_parity.py:126-132)
CONTEXT_FIELDS = ("session_hash", "transaction_epoch", "target_frontier",
                  "transaction_kind", "element_count")


def fnv1a64(raw: bytes) -> str:
    """64-bit FNV-1a over the bytes, as 16 lower-case hex digits: the
    runtime's checksum of the little-endian bf16 words (src/rpc.cc:125-137)."""
    h = _FNV_OFFSET
    for b in raw:
        h = ((h ^ b) * _FNV_PRIME) & _MASK64
    return f"{h:016x}"


@dataclass
class LogitCapture:
    """One snapshot: its metadata and the logits as bf16 words (uint16)."""
    meta: dict[str, Any]
    logits: np.ndarray
    path: Path | None = field(default=None)

    @property
    def selected_token(self) -> int:
        return int(self.meta["selected_token"])

    @property
    def element_count(self) -> int:
        return int(self.meta["element_count"])

    @property
    def transaction_kind(self) -> str:
        return str(self.meta.get("transaction_kind", ""))

    def raw(self) -> bytes:
        return self.logits.astype("<u2", copy=False).tobytes()


def _words(raw: bytes) -> np.ndarray:
    return np.frombuffer(raw, dtype="<u2").astype(np.uint16)


def parse_snapshot(snapshot: dict[str, Any] | str, *, require_raw: bool = True
                   ) -> LogitCapture | None:
    """Check one runtime snapshot (a dict or its JSON text) and decode its
    inline hex payload.  Raises ValueError with the reference tool's
    messages (tools/q38_logit_parity.py:33-58); returns None for a snapshot
    without payload when require_raw is False."""
    if isinstance(snapshot, str):
        snapshot = json.loads(snapshot)
    if snapshot.get("schema") != SNAPSHOT_SCHEMA:
        raise ValueError("unsupported logit snapshot schema")
    if snapshot.get("dtype") != "bf16" or snapshot.get("byte_order") != "little":
        raise ValueError("logit snapshot is not little-endian BF16")
    n = snapshot.get("element_count")
    if not isinstance(n, int) or isinstance(n, bool) or n <= 0:
        raise ValueError("logit snapshot has an invalid element count")
    text = snapshot.get("raw_bf16_le_hex")
    if text is None:
        if require_raw:
            raise ValueError("logit snapshot did not include raw BF16 values")
        return None
    if not isinstance(text, str):
        raise ValueError("raw BF16 payload is not hex text")
    try:
        raw = bytes.fromhex(text)
    except ValueError as err:
        raise ValueError("raw BF16 payload is malformed") from err
    if len(raw) != 2 * n:
        raise ValueError("raw BF16 payload length differs from element count")
    if snapshot.get("fnv1a64") != fnv1a64(raw):
        raise ValueError("raw BF16 payload checksum does not match the runtime")
    meta = {k: v for k, v in snapshot.items() if k != "raw_bf16_le_hex"}
    return LogitCapture(meta, _words(raw))


def manifest_path(output: Path) -> Path:
    output = Path(output)
    return output if output.suffix == ".json" else Path(f"{output}.json")


def write_capture(snapshot: dict[str, Any], output: Path) -> dict[str, Any]:
    """Store a runtime snapshot as manifest + raw file, in the layout the
    reference tool writes (tools/q38_logit_parity.py:65-86)."""
    cap = parse_snapshot(snapshot, require_raw=True)
    raw = cap.raw()
    manifest = manifest_path(output)
    binary = manifest.with_suffix(".bf16")
    binary.parent.mkdir(parents=True, exist_ok=True)
    binary.write_bytes(raw)
    meta = dict(cap.meta)
    meta.update(capture_schema=CAPTURE_SCHEMA, raw_file=binary.name, raw_bytes=len(raw),
                sha256=hashlib.sha256(raw).hexdigest())
    manifest.write_text(json.dumps(meta, indent=2, sort_keys=True) + "\n")
    return meta


def read_capture(path: Path | str) -> LogitCapture:
    """Read a capture manifest and its raw file; every length and both
    checksums are checked (tools/q38_logit_parity.py:89-106)."""
    path = Path(path)
    meta = json.loads(path.read_text())
    if meta.get("capture_schema") != CAPTURE_SCHEMA:
        raise ValueError(f"{path} is not a Q38 logit capture")
    name = meta.get("raw_file")
    if not isinstance(name, str) or not name:
        raise ValueError(f"{path} has no raw BF16 file")
    raw = (path.parent / name).read_bytes()
    n = meta.get("element_count")
    if not isinstance(n, int) or len(raw) != meta.get("raw_bytes") or len(raw) != 2 * n:
        raise ValueError(f"{path} raw BF16 length does not match its manifest")
    if hashlib.sha256(raw).hexdigest() != meta.get("sha256"):
        raise ValueError(f"{path} raw BF16 SHA-256 does not match its manifest")
    if fnv1a64(raw) != meta.get("fnv1a64"):
        raise ValueError(f"{path} raw BF16 FNV-1a does not match its manifest")
    if meta.get("schema", SNAPSHOT_SCHEMA) != SNAPSHOT_SCHEMA:
        raise ValueError("unsupported logit snapshot schema")
    return LogitCapture(meta, _words(raw), path)


def find_captures(root: Path | str) -> list[Path]:
    """Every capture manifest under a directory (sorted), or the file itself."""
    root = Path(root)
    if root.is_file():
        return [root]
    out = []
    for p in sorted(root.rglob("*.json")):
        try:
            if json.loads(p.read_text()).get("capture_schema") == CAPTURE_SCHEMA:
                out.append(p)
        except (ValueError, UnicodeDecodeError):
            continue
    return out


def compare_captures(left: Path | str, right: Path | str) -> dict[str, Any]:
    """Bit comparison of two captures with the reference tool's result
    fields (tools/q38_logit_parity.py:109-168)."""
    a, b = read_capture(left), read_capture(right)
    n = min(a.logits.size, b.logits.size)
    diff = np.flatnonzero(a.logits[:n] != b.logits[:n])
    mismatched = int(diff.size) + abs(a.logits.size - b.logits.size)
    first = None
    if diff.size:
        i = int(diff[0])
        first = {"index": i, "left_bf16_bits": int(a.logits[i]),
                 "right_bf16_bits": int(b.logits[i])}
    exact = a.logits.size == b.logits.size and diff.size == 0
    context = all(a.meta.get(f) == b.meta.get(f) for f in CONTEXT_FIELDS)
    token = a.meta.get("selected_token") == b.meta.get("selected_token")

    def side(c: LogitCapture) -> dict[str, Any]:
        m = c.meta
        return {"path": str(c.path.resolve()), "sha256": m["sha256"],
                "element_count": m["element_count"], "selected_token": m["selected_token"],
                "transaction_epoch": m["transaction_epoch"],
                "target_frontier": m["target_frontier"],
                "transaction_kind": m["transaction_kind"],
                "session_hash": m.get("session_hash")}

    return {"schema": COMPARISON_SCHEMA, "parity_pass": exact and context and token,
            "exact_bf16_match": exact, "comparable_context": context,
            "selected_token_match": token, "mismatched_elements": mismatched,
            "first_mismatch": first, "left": side(a), "right": side(b)}


# ------------------------------------------------------------ on the GPU
def to_device(captures: list[LogitCapture], device: int = 0):
    """The captures' logits as one torch bf16 tensor [len, element_count] on
    the device (all captures must have the same element count)."""
    import torch
    n = {c.element_count for c in captures}
    if len(n) != 1:
        raise ValueError("captures differ in element count")
    host = np.stack([c.logits for c in captures]).view(np.int16)
    return torch.from_numpy(host).to(torch.device("cuda", device)).view(torch.bfloat16)


def greedy_tokens(captures: list[LogitCapture], device: int = 0) -> list[int]:
    """q38s_argmax_bf16 on each capture's logits: the token the runtime's
    greedy mode selects (largest finite value, lowest index on ties)."""
    import torch
    import q38s
    dev = torch.device("cuda", device)
    out = torch.empty(len(captures), dtype=torch.int32, device=dev)
    for i, c in enumerate(captures):
        x = torch.from_numpy(c.logits.view(np.int16)).to(dev).view(torch.bfloat16)
        q38s.argmax_bf16(x, out[i:i + 1], device=device)
    return [int(t) for t in out.cpu()]


def sample_captures(captures: list[LogitCapture], config, histories=None,
                    device: int = 0) -> list[int]:
    """One sampler session per capture (config: q38s.config_v1/v2, history
    tokens committed first), prepare() on the capture's logits in device
    memory; returns the tokens drawn."""
    import torch
    import q38s
    dev = torch.device("cuda", device)
    tokens = []
    for i, c in enumerate(captures):
        s = q38s.Sampler(c.element_count, config, device)
        if histories is not None and len(histories[i]):
            s.commit_tokens(histories[i])
        x = torch.from_numpy(c.logits.view(np.int16)).to(dev).view(torch.bfloat16)
        tokens.append(s.prepare_device(x)[0])
        s.close()
    return tokens


def _check_main(paths: list[str], device: int) -> int:
    caps = []
    for p in paths:
        for m in find_captures(p):
            caps.append(read_capture(m))
    if not caps:
        print(json.dumps({"captures": 0}))
        return 1
    greedy = greedy_tokens(caps, device)
    rows = []
    for c, g in zip(caps, greedy):
        rows.append({"path": str(c.path), "element_count": c.element_count,
                     "transaction_kind": c.transaction_kind,
                     "selected_token": c.selected_token, "greedy_token": g,
                     "greedy_matches_selected": g == c.selected_token})
    print(json.dumps({"captures": len(rows), "results": rows}, indent=2))
    return 0


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(prog="python -m q38s.capture")
    sub = ap.add_subparsers(dest="command", required=True)
    chk = sub.add_parser("check", help="greedy selection on captures vs their selected_token")
    chk.add_argument("paths", nargs="+")
    chk.add_argument("--device", type=int, default=int(os.environ.get("LOCAL_RANK", 0)))
    cmp_ = sub.add_parser("compare", help="bit comparison of two captures")
    cmp_.add_argument("left")
    cmp_.add_argument("right")
    a = ap.parse_args(argv)
    if a.command == "check":
        return _check_main(a.paths, a.device)
    res = compare_captures(a.left, a.right)
    print(json.dumps(res, indent=2, sort_keys=True))
    return 0 if res["parity_pass"] else 1


if __name__ == "__main__":
    sys.exit(main())

"""Receipts for decodes run through libcis2b, in the wire formats of the
reference's receipt server (code/cis2-llm/server/app):

* `verify2_lines` renders a run as the five stdout lines of the vendored
  verifier the server runs (code/cis2-fp/verify2/src/main.rs:489-500), and
  `parse_verify2` reads them back with the server's own patterns
  (server/app/runner.py:25-31).  `cis2b_ref --verify2` prints the same lines.
* `ReceiptLog` is an append-only JSONL log with the server's chaining rule
  (server/app/receipts.py): each record carries `prev_hash` (64 zeros for the
  first) and `log_hash` = SHA-256 of the record's fields, `prev_hash`
  included, encoded with sorted keys and no whitespace; records are stored
  with sorted keys.  A log written here verifies with the server's checker,
  and the other way round.
* `server_record` builds the fields the server stores per receipt
  (server/app/main.py:73-87) from a `Model.generate` result.
"""
from __future__ import annotations

import hashlib
import json
import os
import re
import threading
import time
import uuid
from typing import Any

GENESIS_HASH = "0" * 64

# The spec's pinned reference vector: "Once upon a time" (add_special_tokens
# false) as SmolLM2 token ids, 16 greedy tokens (verify2/src/main.rs:446-451).
CANONICAL_PROMPT = "Once upon a time"
CANONICAL_PROMPT_IDS = (6403, 1980, 253, 655)
CANONICAL_GEN = 16

_VERIFY2_PATTERNS = {
    "witness_digest": re.compile(r"^CIS2_VERIFY2 digest=([0-9a-f]+)"),
    "argmax_digest": re.compile(r"^argmax_digest=([0-9a-f]+)"),
    "table_digest": re.compile(r"^table_digest=([0-9a-f]+)"),
    "inv_freq_table_digest": re.compile(r"^inv_freq table_digest=([0-9a-f]+)"),
    "generated_token_ids": re.compile(r"^generated_token_ids=\[([0-9, ]+)\]"),
}


def verify2_lines(witness: bytes, argmax: bytes, table_digest: bytes, inv_freq_digest: bytes,
                  prompt_len: int, tokens) -> str:
    """One run's five verifier lines (trailing newline included)."""
    toks = [int(t) for t in tokens]
    return (f"CIS2_VERIFY2 digest={witness.hex()} prompt_toks={prompt_len} gen_toks={len(toks)} dtype=fp32\n"
            f"argmax_digest={argmax.hex()}\n"
            f"table_digest={table_digest.hex()}\n"
            f"inv_freq table_digest={inv_freq_digest.hex()}\n"
            f"generated_token_ids=[{', '.join(str(t) for t in toks)}]\n")


def parse_verify2(stdout: str) -> dict[str, Any]:
    """The fields the receipt server takes from the verifier's stdout; raises
    ValueError naming the missing ones, as the server refuses such output."""
    fields: dict[str, str] = {}
    for line in stdout.splitlines():
        for key, pat in _VERIFY2_PATTERNS.items():
            m = pat.match(line)
            if m:
                fields[key] = m.group(1)
    missing = [k for k in _VERIFY2_PATTERNS if k not in fields]
    if missing:
        raise ValueError(f"verifier output lacks {missing}")
    out: dict[str, Any] = dict(fields)
    out["generated_token_ids"] = [int(t) for t in fields["generated_token_ids"].split(",") if t.strip()]
    return out


def server_record(result: dict, info: dict, index: int = 0, model: str = "cis2-smollm2-135m-fp32-ref",
                  prompt: str = CANONICAL_PROMPT) -> dict[str, Any]:
    """The per-receipt fields of the server (before chaining) for sequence
    `index` of a Model.generate result; `info` is Model.info."""
    return {
        "receipt_id": uuid.uuid4().hex,
        "created": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime()),
        "model": model,
        "cis2_version": "v0.3b",
        "witness_digest": bytes(result["witness"][index]).hex(),
        "argmax_digest": bytes(result["argmax"][index]).hex(),
        "table_digest": bytes(info["table_digest"]).hex(),
        "inv_freq_table_digest": bytes(info["inv_freq_table_digest"]).hex(),
        "generated_token_ids": [int(t) for t in result["tokens"][index]],
        "prompt": prompt,
    }


def chain_hash(record: dict[str, Any]) -> str:
    """SHA-256 (hex) of a record's fields with sorted keys and no whitespace."""
    return hashlib.sha256(json.dumps(record, sort_keys=True, separators=(",", ":")).encode("utf-8")).hexdigest()


class ReceiptLog:
    """Append-only, hash-chained JSONL receipt log (one process: appends are
    serialised by a lock)."""

    def __init__(self, path: str | os.PathLike):
        self.path = os.fspath(path)
        os.makedirs(os.path.dirname(os.path.abspath(self.path)), exist_ok=True)
        if not os.path.exists(self.path):
            open(self.path, "a").close()
        self._lock = threading.Lock()

    def _records(self):
        with open(self.path) as f:
            for line in f:
                if line.strip():
                    yield json.loads(line)

    def last_hash(self) -> str:
        h = GENESIS_HASH
        for rec in self._records():
            h = rec["log_hash"]
        return h

    def append(self, fields: dict[str, Any]) -> dict[str, Any]:
        """Chains `fields` to the last record and appends it; returns the
        stored record (with prev_hash and log_hash)."""
        with self._lock:
            record = dict(fields)
            record["prev_hash"] = self.last_hash()
            record["log_hash"] = chain_hash(record)
            with open(self.path, "a") as f:
                f.write(json.dumps(record, sort_keys=True) + "\n")
            return record

    def get(self, receipt_id: str) -> dict[str, Any] | None:
        for rec in self._records():
            if rec.get("receipt_id") == receipt_id:
                return rec
        return None

    def verify_chain(self) -> tuple[bool, str]:
        """Recomputes every link; (False, reason) names the first bad record
        (0-based, in file order)."""
        prev = GENESIS_HASH
        n = 0
        for n, rec in enumerate(self._records(), 1):
            body = {k: v for k, v in rec.items() if k != "log_hash"}
            if rec.get("prev_hash") != prev:
                return False, f"record {n - 1}: prev_hash is not the previous record's log_hash"
            if chain_hash(body) != rec.get("log_hash"):
                return False, f"record {n - 1}: log_hash does not match its fields"
            prev = rec["log_hash"]
        return True, f"{n} records, chain intact"

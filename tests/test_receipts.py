"""Receipts in the reference receipt server's wire formats
(cis2-lab-archive_b200/receipts.py): the hash-chained JSONL log and the
verifier's stdout lines.  CPU only; where the reference checkout is present
its own log code and line patterns check ours, and ours check its log."""
from __future__ import annotations

import hashlib
import importlib
import importlib.util
import json
import os
import sys

import pytest

receipts = importlib.import_module("cis2-lab-archive_b200.receipts")

REF_APP = os.path.join(os.environ.get("CIS2_REFERENCE_ROOT", os.path.join(os.path.dirname(__file__), "..", "..",
                                                                        "reference")),
                       "code", "cis2-llm", "server", "app")


def _ref_module(name: str):
    path = os.path.join(REF_APP, name + ".py")
    if not os.path.exists(path):
        pytest.skip("reference receipt server sources not present")
    spec = importlib.util.spec_from_file_location("_ref_" + name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod  # the module's dataclasses look themselves up there
    spec.loader.exec_module(mod)
    return mod


def _fields(i: int) -> dict:
    return {"receipt_id": f"{i:032x}", "created": "2026-12-02T00:00:00Z", "model": "m", "cis2_version": "v0.3b",
            "witness_digest": hashlib.sha256(bytes([i])).hexdigest(), "argmax_digest": "00" * 32,
            "table_digest": "11" * 32, "inv_freq_table_digest": "22" * 32,
            "generated_token_ids": [i, i + 1, 7], "prompt": "Once upon a time"}


def test_chain_links_and_hashes(tmp_path):
    log = receipts.ReceiptLog(tmp_path / "r.jsonl")
    recs = [log.append(_fields(i)) for i in range(3)]
    assert recs[0]["prev_hash"] == receipts.GENESIS_HASH
    assert recs[1]["prev_hash"] == recs[0]["log_hash"] and recs[2]["prev_hash"] == recs[1]["log_hash"]
    body = {k: v for k, v in recs[1].items() if k != "log_hash"}
    want = hashlib.sha256(json.dumps(body, sort_keys=True, separators=(",", ":")).encode()).hexdigest()
    assert recs[1]["log_hash"] == want
    assert log.verify_chain() == (True, "3 records, chain intact")
    assert log.get(recs[2]["receipt_id"])["witness_digest"] == recs[2]["witness_digest"]
    assert log.get("nope") is None
    lines = (tmp_path / "r.jsonl").read_text().splitlines()
    assert lines[0] == json.dumps(recs[0], sort_keys=True)  # stored with sorted keys


@pytest.mark.parametrize("field,value,where", [("witness_digest", "ff" * 32, "record 1: log_hash"),
                                               ("prev_hash", "0" * 64, "record 1: prev_hash")])
def test_tampering_is_found(tmp_path, field, value, where):
    p = tmp_path / "r.jsonl"
    log = receipts.ReceiptLog(p)
    for i in range(3):
        log.append(_fields(i))
    lines = p.read_text().splitlines()
    rec = json.loads(lines[1])
    rec[field] = value
    lines[1] = json.dumps(rec, sort_keys=True)
    p.write_text("\n".join(lines) + "\n")
    ok, msg = log.verify_chain()
    assert not ok and msg.startswith(where), msg


def test_verify2_lines_round_trip():
    txt = receipts.verify2_lines(bytes(range(32)), bytes(32), b"\x11" * 32, b"\x22" * 32, 4,
                                 [1, 22, 333, 4444] * 4)
    got = receipts.parse_verify2(txt)
    assert got["witness_digest"] == bytes(range(32)).hex()
    assert got["generated_token_ids"] == [1, 22, 333, 4444] * 4
    assert txt.splitlines()[0].endswith("prompt_toks=4 gen_toks=16 dtype=fp32")
    with pytest.raises(ValueError):
        receipts.parse_verify2(txt.replace("argmax_digest", "argmax"))


def test_reference_server_reads_our_lines_and_log(tmp_path):
    runner = _ref_module("runner")
    ref_receipts = _ref_module("receipts")
    txt = receipts.verify2_lines(bytes(range(32)), b"\x05" * 32, b"\x11" * 32, b"\x22" * 32, 4, list(range(16)))
    fields = {}
    for line in txt.splitlines():
        for key, pat in runner._LINE_RE.items():
            m = pat.match(line)
            if m:
                fields[key] = m.group(1)
    assert set(fields) == set(runner._LINE_RE)
    assert fields == {k: v for k, v in receipts.parse_verify2(txt).items() if k != "generated_token_ids"} | {
        "generated_token_ids": fields["generated_token_ids"]}
    # our log, their checker; their log, our checker
    ours = receipts.ReceiptLog(tmp_path / "ours.jsonl")
    for i in range(3):
        ours.append(_fields(i))
    assert ref_receipts.ReceiptLog(tmp_path / "ours.jsonl").verify_chain()[0]
    theirs = ref_receipts.ReceiptLog(tmp_path / "theirs.jsonl")
    for i in range(3):
        theirs.append(_fields(i))
    assert receipts.ReceiptLog(tmp_path / "theirs.jsonl").verify_chain() == (True, "3 records, chain intact")
    assert (tmp_path / "ours.jsonl").read_text() == (tmp_path / "theirs.jsonl").read_text()


@pytest.mark.parametrize("extra", [["--reduction", "tree"], ["--mode", "sampled"], ["--sample", "1,0.8,40,0.95"]])
def test_cli_verify2_is_the_greedy_sequential_vector(extra, tmp_path):
    """`cis2b_ref --verify2` refuses the other modes before it loads anything."""
    import subprocess
    pkg = importlib.import_module("cis2-lab-archive_b200")
    p = subprocess.run([pkg.CLI_PATH, "--weights-dir", str(tmp_path / "absent"), "--verify2", *extra],
                       capture_output=True, text=True)
    assert p.returncode == 2 and "--verify2" in p.stderr, (p.returncode, p.stderr)

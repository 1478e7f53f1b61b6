"""`cis2b_ref --verify2` on the device: the receipt server's verifier lines for
the spec's pinned reference vector ("Once upon a time" as its token ids, 16
greedy tokens), equal to the C ABI's own run of the same ids, and a receipt
of that run chained into the server-format log."""
from __future__ import annotations

import importlib
import subprocess

import pytest

pytestmark = pytest.mark.gpu

receipts = importlib.import_module("cis2-lab-archive_b200.receipts")


def test_verify2_lines_match_the_abi_run(pkg, synth, synth_root, tmp_path):
    d = synth.ensure_model("smollm2", synth_root)
    out = subprocess.run([pkg.CLI_PATH, "--weights-dir", d, "--verify2"], capture_output=True, text=True,
                         check=True).stdout
    with pkg.Model(d) as m:
        r = m.generate([list(receipts.CANONICAL_PROMPT_IDS)], receipts.CANONICAL_GEN)
        info = m.info
    want = receipts.verify2_lines(r["witness"][0].tobytes(), r["argmax"][0].tobytes(), info["table_digest"],
                                  info["inv_freq_table_digest"], len(receipts.CANONICAL_PROMPT_IDS), r["tokens"][0])
    assert out == want
    got = receipts.parse_verify2(out)
    assert got["generated_token_ids"] == [int(t) for t in r["tokens"][0]]
    log = receipts.ReceiptLog(tmp_path / "receipts.jsonl")
    rec = log.append(receipts.server_record(r, info))
    assert rec["witness_digest"] == got["witness_digest"] and log.verify_chain()[0]


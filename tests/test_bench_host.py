"""The arithmetic behind bench.py's roofline fields, on CPU: the witness
chain's issue-bound fraction, the per-launch achieved rates from event
timings, and the step bound's label."""
from __future__ import annotations

import pytest

import bench

synth = bench.synth


def _prof(witness_ms_per_launch=None, lm_ms_per_launch=None, launches=256):
    p = {}
    if witness_ms_per_launch is not None:
        p["witness"] = {"launches": launches, "total_ms": witness_ms_per_launch * launches}
    if lm_ms_per_launch is not None:
        p["lm_head"] = {"launches": launches, "total_ms": lm_ms_per_launch * launches}
    return p


def test_witness_roofline_fields():
    m, w = synth.MODELS["smollm2"], synth.WORKLOADS["c2"]
    # 3,073 blocks per chain at 1,408 cycles each, at 1,965 MHz: the issue bound.
    blocks = (4 * m.vocab + 4) / 64.0
    t_ms = blocks * bench.CHAIN_FLOOR_CYCLES_PER_BLOCK / 1965e6 * 1e3
    r = bench.kernel_rooflines(m, w, 64, _prof(witness_ms_per_launch=t_ms), 1965.0)["witness"]
    # The witness is bound by integer issue, and its fraction is of that bound.
    assert r["bound"] == "int_issue"
    assert r["frac"] == pytest.approx(1.0, rel=1e-9)
    assert r["cycles_per_block_per_chain"] == pytest.approx(bench.CHAIN_FLOOR_CYCLES_PER_BLOCK, rel=1e-9)
    assert r["achieved"] == pytest.approx(1965e6 / bench.CHAIN_FLOOR_CYCLES_PER_BLOCK)
    assert r["frac"] == pytest.approx(r["achieved"] / r["peak"])
    # Its HBM side is reported beside it.
    assert r["algorithmic_bytes"] == 64 * (4 * m.vocab + 4)
    assert r["hbm"]["achieved"] == pytest.approx(r["algorithmic_bytes"] / (t_ms / 1e3) / 1e9)
    assert r["hbm"]["frac"] == pytest.approx(r["hbm"]["achieved"] / r["hbm"]["peak"])
    assert r["traffic"] == bench.WITNESS_TRAFFIC_C2  # the captured shape
    # Twice as slow: half the fraction.
    r2 = bench.kernel_rooflines(m, w, 64, _prof(witness_ms_per_launch=2 * t_ms), 1965.0)["witness"]
    assert r2["frac"] == pytest.approx(0.5, rel=1e-9)
    # Another shape has no captured traffic figure.
    r3 = bench.kernel_rooflines(m, w, 32, _prof(witness_ms_per_launch=t_ms), 1965.0)["witness"]
    assert r3["traffic"] is None


def test_lm_head_roofline_fields():
    m, w = synth.MODELS["smollm2"], synth.WORKLOADS["c2"]
    r = bench.kernel_rooflines(m, w, 64, _prof(lm_ms_per_launch=0.2), 1965.0)["lm_head"]
    assert r["bound"] == "fp32_pipe"
    fp32 = 148 * 128 * 1965e6
    assert r["frac"] == pytest.approx(2 * 64 * m.vocab * m.hidden / 0.2e-3 / fp32)
    byts = m.vocab * m.hidden * 2 + 64 * m.hidden * 4 + 64 * m.vocab * 4
    assert r["hbm"]["algorithmic_bytes"] == byts
    assert r["hbm"]["achieved"] == pytest.approx(byts / 0.2e-3 / 1e9)


def test_golden_check_covers_every_rank(tmp_path, monkeypatch):
    """The parity check reads every fixture of a workload and maps each
    gathered sequence to its global index, so sequences of ranks > 0 are
    checked too; a single flipped step digest fails the sequence."""
    import hashlib
    import json
    import numpy as np
    G = 3
    rows = []
    for i in range(6):
        rng = np.random.default_rng(i)
        rows.append({"tokens": rng.integers(0, 9, G).astype(np.uint32),
                     "steps": rng.integers(0, 255, (G, 32)).astype(np.uint8),
                     "witness": rng.integers(0, 255, 32).astype(np.uint8),
                     "argmax": rng.integers(0, 255, 32).astype(np.uint8)})

    def entry(r):
        return {"witness": r["witness"].tobytes().hex(), "argmax": r["argmax"].tobytes().hex(),
                "steps_sha": hashlib.sha256(r["steps"].tobytes()).hexdigest(),
                "tokens_sha": hashlib.sha256(r["tokens"].astype("<u4").tobytes()).hexdigest()}

    (tmp_path / "cx.json").write_text(json.dumps({"prompts": ["workload", "cx", 0, 2],
                                                  "sequences": [entry(r) for r in rows[:2]]}))
    (tmp_path / "cx_shards.json").write_text(json.dumps({"prompts": ["workload_idx", "cx", [3, 5]],
                                                         "sequences": [entry(rows[3]), entry(rows[5])]}))
    monkeypatch.setattr(bench, "GOLDEN_DIR", str(tmp_path))
    out = {"tokens": np.stack([r["tokens"] for r in rows]), "step_digests": np.stack([r["steps"] for r in rows]),
           "witness": np.stack([r["witness"] for r in rows]), "argmax": np.stack([r["argmax"] for r in rows])}
    g = bench.golden_check("cx", 0, out, 6)
    assert (g["checked"], g["identical"], g["unchecked"]) == (4, 4, 2)
    out["step_digests"][5, 1, 7] ^= 1
    g = bench.golden_check("cx", 0, out, 6)
    assert (g["identical"], g["differ"]) == (3, 1)


def test_step_bound_label_follows_the_longer_path():
    m, w = synth.MODELS["smollm2"], synth.WORKLOADS["c2"]
    peak, src = bench.measured_peaks()
    a = bench.step_roofline(m, w, 64, 2.8e-3, peak, src, forward_ms=2.6, witness_ms=2.76)
    b = bench.step_roofline(m, w, 64, 2.8e-3, peak, src, forward_ms=3.0, witness_ms=2.76)
    assert a["bound_actual"].startswith("witness chain")
    assert b["bound_actual"].startswith("decode forward pass")
    # The HBM side does not depend on the label: bf16 weights once, KV and logits.
    assert a["algorithmic_bytes_per_step"] == b["algorithmic_bytes_per_step"]
    assert a["weights_bytes"] == 2 * (m.layers * (m.hidden * (m.q_dim + 2 * m.kv_dim) + m.q_dim * m.hidden
                                                 + 3 * m.inter * m.hidden) + m.vocab * m.hidden)
    assert a["frac"] == pytest.approx(a["achieved"] / peak)


def test_stdout_to_stderr_redirects_native_writes(capfd):
    """Native writes to fd 1 inside the block (NCCL's banner) reach stderr;
    fd 1 is stdout again afterwards."""
    import os
    with bench.stdout_to_stderr():
        os.write(1, b"native banner\n")
    os.write(1, b"json line\n")
    out, err = capfd.readouterr()
    assert out == "json line\n" and "native banner" in err


def test_golden_entries_keep_reduction_modes_apart():
    """C1 has a sequential and a tree fixture for the same sequence; each
    mode's parity check must see only its own."""
    import json
    import os
    seq, tree = bench.golden_entries("c1", "sequential"), bench.golden_entries("c1", "tree")
    with open(os.path.join(bench.GOLDEN_DIR, "c1.json")) as f:
        want_seq = json.load(f)["sequences"][0]["witness"]
    with open(os.path.join(bench.GOLDEN_DIR, "c1_tree.json")) as f:
        want_tree = json.load(f)["sequences"][0]["witness"]
    assert seq[0]["witness"] == want_seq and tree[0]["witness"] == want_tree
    assert len(bench.golden_entries("c2", "tree")) == 64
    assert len(bench.golden_entries("c2", "sequential")) == 512
    assert bench.golden_entries("c3", "tree") == {}


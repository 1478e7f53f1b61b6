"""Per-op trace on the device (cis2b_trace, `cis2b_ref --trace F`) against the
reference's own CLI trace (`cis2_host --trace F`, code/cis2-fp/gpu/
cis2_host.cpp:76, 173-208, compiled from the reference sources into
oracle/_ref): every "pos= layer= op= sha256=" line equal, in order, so the
reference's trace-diff gate (code/cis2-fp/gpu/Makefile:160-184) runs with
this binary swapped in and a parity failure can be localised to one op."""
from __future__ import annotations

import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

CASES = [
    # (model, reduction, reference binary, prompt length, generated tokens)
    ("tiny", "sequential", "cis2_host", 6, 4),
    ("tiny", "tree", "cis2_host_tree", 6, 4),
    ("tiny_mha_untied", "sequential", "cis2_host", 9, 3),
    ("tiny_bias", "sequential", "cis2_host", 5, 3),
    ("tiny_qwen3", "sequential", "cis2_host_qwen3", 7, 3),
    ("mid", "sequential", "cis2_host", 33, 3),
]


@pytest.mark.parametrize("model,reduction,ref_exe,plen,gen", CASES)
def test_trace_matches_reference_cli(model, reduction, ref_exe, plen, gen, pkg, oracle, synth, synth_root,
                                     tmp_path):
    exe = os.path.join(oracle.REF_DIR, ref_exe)
    if not os.path.exists(exe):
        pytest.skip(f"{exe} not built")
    d = synth.ensure_model(model, synth_root)
    ids = synth.random_prompts(model, 1, plen, 4242)[0]
    idp = tmp_path / "ids.txt"
    idp.write_text(" ".join(str(int(v)) for v in ids) + "\n")
    ref = subprocess.run([exe, "--weights-dir", d, "--ids", str(idp), "--gen-toks", str(gen), "--trace",
                          str(tmp_path / "ref.txt")], capture_output=True, text=True, check=True)
    cmd = [pkg.CLI_PATH, "--weights-dir", d, "--ids", str(idp), "--gen-toks", str(gen), "--reduction", reduction,
           "--trace", str(tmp_path / "dev.txt")]
    if synth.MODELS[model].model_type == "qwen3":
        cmd += ["--arch-gate", "qwen3-port"]
    dev = subprocess.run(cmd, capture_output=True, text=True, check=True)
    want = (tmp_path / "ref.txt").read_text().splitlines()
    got = (tmp_path / "dev.txt").read_text().splitlines()
    m = synth.MODELS[model]
    per_pos = 3 + m.layers * (17 + (2 if m.qk_norm else 0))
    assert len(want) == (plen + gen) * per_pos
    for i, (a, b) in enumerate(zip(got, want)):
        assert a == b, f"first differing op, line {i}: device {a!r} vs reference {b!r}"
    assert len(got) == len(want)
    # The run traced is the run whose digest both print.
    dig = [ln.split()[1] for ln in ref.stdout.splitlines() if ln.startswith("CIS2_REF digest=")]
    assert dig and dig == [ln.split()[1] for ln in dev.stdout.splitlines() if ln.startswith("CIS2_REF digest=")]


def test_trace_rejects_bad_arguments(pkg, synth, synth_root, tmp_path):
    with pkg.Model(synth.ensure_model("tiny", synth_root)) as m:
        import ctypes
        import numpy as np
        L = pkg.lib()
        L.cis2b_trace.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_char_p]
        ids = np.array([1, 2, 600], dtype=np.uint32)  # 600 >= vocab
        assert L.cis2b_trace(m._h, ids.ctypes.data, 3, str(tmp_path / "t.txt").encode()) == 1
        assert L.cis2b_trace(m._h, ids.ctypes.data, 0, str(tmp_path / "t.txt").encode()) == 1
        ok = np.array([1, 2], dtype=np.uint32)
        assert L.cis2b_trace(m._h, ok.ctypes.data, 2, str(tmp_path / "no" / "t.txt").encode()) == 2
        assert L.cis2b_trace(m._h, ok.ctypes.data, 2, str(tmp_path / "t.txt").encode()) == 0
        assert len((tmp_path / "t.txt").read_text().splitlines()) == 2 * (3 + 2 * 17)

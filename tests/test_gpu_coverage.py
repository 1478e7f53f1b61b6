"""The constructed coverage vector on the device (labs/w1x-coverage/plans/
2026-10-16-w1x-coverage-PLAN.md:8-16): a tiny Llama-shape model whose
lm_head rows 5 and 17 are identical, so every step's logits tie exactly, and
whose row 29 gives a subnormal step-0 logit.  Random seeded weights never
reach either clause; this model reaches both on purpose.

  * argmax clause (code/cis2-fp/src/main.rs:1161-1169): strict '>' from
    index 0, so the tie must select 5, never 17;
  * FTZ/DAZ clause (spec §1.3; code/cis2-fp/gpu/cis2_fpenv.h:62-135): the
    subnormal logit is flushed to +0 (0x00000000) before the witness hashes
    it; hashing the unflushed bits gives a different digest.

Golden digests come from the reference's own compiled C++ port
(tests/golden/coverage_{seq,tree}.json, tests/golden/make_golden.py)."""
from __future__ import annotations

import hashlib

import numpy as np
import pytest

from conftest import golden_prompts, load_golden

pytestmark = pytest.mark.gpu


def witness_from_logits(info: dict, prompt, tokens, logits: np.ndarray) -> bytes:
    """CIS2_REF digest rebuilt on the host from per-step logits, with the
    byte layout of code/cis2-fp/gpu/cis2_host.cpp:179-218: the three artifact
    hashes, the table and inv_freq digests, the prompt ids (u32 LE), then per
    step every logit's bits (u32 LE) and the chosen id."""
    h = hashlib.sha256()
    for k in ("weights_sha256", "tokenizer_sha256", "config_sha256", "table_digest", "inv_freq_table_digest"):
        h.update(info[k])
    h.update(np.asarray(prompt, dtype="<u4").tobytes())
    for t, row in zip(tokens, logits):
        h.update(np.ascontiguousarray(row, dtype=np.float32).view("<u4").tobytes())
        h.update(np.array([t], dtype="<u4").tobytes())
    return h.digest()


@pytest.mark.parametrize("name", ["coverage_seq", "coverage_tree"])
def test_coverage_vector_matches_reference(name, pkg, synth, synth_root, tmp_path):
    g = load_golden(name)
    d = synth.ensure_model(g["model"], synth_root)
    prompts = golden_prompts(synth, g)
    assert np.array_equal(prompts[0], synth.coverage_prompt())
    with pkg.Model(d, reduction=g["reduction"]) as m:
        r = m.generate(prompts, g["gen"])
        e = g["sequences"][0]
        assert [int(t) for t in r["tokens"][0]] == e["tokens"]
        assert int(r["tokens"][0][0]) == synth.COVERAGE_TIE_A  # strict-first: 5, not 17
        assert [s.tobytes().hex() for s in r["step_digests"][0]] == e["step_digests"]
        assert r["witness"][0].tobytes().hex() == e["witness"]
        assert r["argmax"][0].tobytes().hex() == e["argmax"]

        # Teacher-forced logits of every step: the tie is exact at each step
        # and the subnormal row reaches the witness as +0.
        p = prompts[0]
        ids = np.concatenate([p, r["tokens"][0][:-1]]).astype(np.uint32)
        lg = m.logits(ids, len(p), g["gen"])
        bits = lg.view(np.uint32)
        assert np.array_equal(bits[:, synth.COVERAGE_TIE_A], bits[:, synth.COVERAGE_TIE_B])
        assert (lg[:, synth.COVERAGE_TIE_A] == lg.max(axis=1)).all()
        assert bits[0, synth.COVERAGE_SUB] == 0x00000000

        # The host rebuild of the witness from those logits is the reference digest ...
        wit = witness_from_logits(m.info, p, r["tokens"][0], lg)
        assert wit.hex() == e["witness"]
        # ... and the unflushed value would have moved it (the reference
        # lab's M01 mutant): the smallest normal weight times the column's
        # final-norm value x is a positive subnormal without FTZ.  x itself
        # is read exactly through a probe copy of the model whose row-29
        # weight is 1.0 (1.0 * x plus signed zeros is x).
        x = probe_column_value(d, tmp_path, p, g["reduction"], pkg, synth)
        sub = np.float32(np.float32(2.0 ** -126) * np.float32(abs(x)))
        assert 0 < sub < np.finfo(np.float32).tiny  # subnormal, non-zero
        mutant = lg.copy()
        mutant[0, synth.COVERAGE_SUB] = sub
        assert witness_from_logits(m.info, p, r["tokens"][0], mutant).hex() != e["witness"]


def probe_column_value(d, tmp_path, prompt, reduction, pkg, synth) -> float:
    """Final-norm value, at the last prompt position, of the column that
    carries row SUB's single weight."""
    import json
    import shutil
    import struct
    col = synth.coverage_column(d)
    pd = tmp_path / "probe"
    pd.mkdir()
    for fn in ("config.json", "tokenizer.json"):
        shutil.copy(f"{d}/{fn}", pd / fn)
    raw = bytearray(open(f"{d}/model.safetensors", "rb").read())
    (hl,) = struct.unpack("<Q", raw[:8])
    hdr = json.loads(raw[8:8 + hl])
    b = hdr["lm_head.weight"]["data_offsets"][0]
    H = hdr["lm_head.weight"]["shape"][1]
    o = 8 + hl + b + 2 * (synth.COVERAGE_SUB * H + col)
    raw[o:o + 2] = (0x3F80).to_bytes(2, "little")  # bf16 1.0
    (pd / "model.safetensors").write_bytes(bytes(raw))
    with pkg.Model(str(pd), reduction=reduction) as probe:
        v = probe.logits(np.asarray(prompt, dtype=np.uint32), len(prompt), 1)[0, synth.COVERAGE_SUB]
    assert 0.25 <= abs(float(v)) <= 0.75
    return float(v)

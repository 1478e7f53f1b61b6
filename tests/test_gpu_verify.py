"""Teacher-forced receipt verification on the device (cis2b_verify), the
batched form of cis2_verify_receipt_prefill (code/cis2-fp/verify3/model.c:
923-1004) and of its claim check (verify3/main.c:230-265)."""
from __future__ import annotations

import hashlib
import struct

import numpy as np
import pytest

from test_gpu_decode import model_for

pytestmark = pytest.mark.gpu


def _prompts(synth, model, lens, seed):
    return [synth.random_prompts(model, 1, L, seed, first=i)[0] for i, L in enumerate(lens)]


@pytest.mark.parametrize("model,reduction,sample", [
    ("mid", "sequential", None),
    ("tiny_qwen3", "tree", None),
    ("tiny", "sequential", {"seed": 3, "temperature": 0.8, "top_p": 0.95}),
    ("tiny_bias", "sequential", {"scheme": "gumbel", "seed": 5, "temperature": 0.7, "top_k": 20, "top_p": 0.9}),
])
def test_honest_receipt_reproduces_generation(model, reduction, sample, pkg, synth, synth_root):
    """Verifying what generate produced gives back the same tokens and the
    same per-step, witness and argmax digests, with no mismatch."""
    m = model_for(pkg, synth, synth_root, model, reduction)
    prompts = _prompts(synth, model, [1, 6, 40, 13, 2], 808)
    g = m.generate(prompts, 18, sample=sample)
    v = m.verify(prompts, g["tokens"], sample=sample)
    assert np.all(v["first_mismatch"] == -1)
    for k in ("tokens", "step_digests", "witness", "argmax"):
        assert np.array_equal(v[k], g[k]), k


def _expected_witness(oracle, d, prompt, claimed):
    """verify3/model.c:953-997 restated in Python over the oracle's
    teacher-forced logits: header, prompt ids, then per step the logits and
    the recomputed argmax."""
    o = oracle.PortOracle(d)
    ids = np.concatenate([np.asarray(prompt, np.uint32), np.asarray(claimed[:-1], np.uint32)])
    logits = o.logits(ids, len(prompt), len(claimed))
    _, inv_digest = o.inv_freq()
    h = hashlib.sha256(o.hashes + oracle.table_digest() + bytes(inv_digest))
    a = hashlib.sha256()
    for t in prompt:
        h.update(struct.pack("<I", int(t)))
        a.update(struct.pack("<I", int(t)))
    rec = []
    for row in logits:
        nxt = int(np.argmax(row))
        h.update(row.astype("<f4").tobytes())
        h.update(struct.pack("<I", nxt))
        a.update(struct.pack("<I", nxt))
        rec.append(nxt)
    return h.digest(), a.digest(), rec


def test_tampered_claim_is_localised(pkg, oracle, synth, synth_root):
    """A claim altered at step k: that sequence reports first_mismatch = k,
    its step-k token is recomputed from untouched inputs (so it equals the
    honest one), later logits follow the altered inputs, and the digests equal
    the oracle's teacher-forced restatement; the other sequences are unaffected."""
    model = "mid"
    d = synth.ensure_model(model, synth_root)
    m = model_for(pkg, synth, synth_root, model, "sequential")
    prompts = _prompts(synth, model, [5, 9, 3], 909)
    g = m.generate(prompts, 12)
    claimed = g["tokens"].copy()
    k = 4
    claimed[1, k] = (claimed[1, k] + 1) % 4096
    v = m.verify(prompts, claimed)
    assert list(v["first_mismatch"]) == [-1, k, -1]
    assert np.array_equal(v["tokens"][1, : k + 1], g["tokens"][1, : k + 1])
    for b in (0, 2):
        assert v["witness"][b].tobytes() == g["witness"][b].tobytes()
    wit, arg, rec = _expected_witness(oracle, d, prompts[1], claimed[1])
    assert list(v["tokens"][1]) == rec
    assert v["witness"][1].tobytes() == wit
    assert v["argmax"][1].tobytes() == arg
    assert v["witness"][1].tobytes() != g["witness"][1].tobytes()


def test_verify_rejects_out_of_range_claims(pkg, synth, synth_root):
    m = model_for(pkg, synth, synth_root, "tiny", "sequential")
    with pytest.raises(pkg.Cis2Error) as e:
        m.verify([[1, 2]], [[3, 600]])  # 600 >= vocab 512
    assert e.value.code == 1
    r = m.verify([[1, 2]], [[3, 4]])     # still usable
    assert r["tokens"].shape == (1, 2)


def test_cli_verifies_a_receipt(pkg, synth, synth_root, tmp_path):
    """cis2b_ref --receipt prints the verify3 lines (verify3/main.c:272-318)
    and exits 1 when a claim differs from the recomputed tokens."""
    import subprocess
    m = model_for(pkg, synth, synth_root, "tiny", "sequential")
    prompts = _prompts(synth, "tiny", [3, 7], 111)
    g = m.generate(prompts, 8)
    ids = tmp_path / "ids.txt"
    ids.write_text("\n".join(" ".join(str(int(v)) for v in p) for p in prompts) + "\n")
    rec = tmp_path / "receipt.txt"
    rec.write_text("\n".join(",".join(str(int(v)) for v in t) for t in g["tokens"]) + "\n")
    cmd = [pkg.CLI_PATH, "--weights-dir", synth.ensure_model("tiny", synth_root), "--ids", str(ids),
           "--receipt", str(rec)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    dig = [ln.split()[1].split("=")[1] for ln in r.stdout.splitlines() if ln.startswith("CIS2_VERIFY3 digest=")]
    assert dig == [w.tobytes().hex() for w in g["witness"]]
    assert r.stdout.count("CIS2_VERIFY3 first_mismatch_pos=-1") == 2
    bad = g["tokens"].copy()
    bad[0, 2] = (bad[0, 2] + 1) % 512
    rec.write_text("\n".join(",".join(str(int(v)) for v in t) for t in bad) + "\n")
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 1
    assert "CIS2_VERIFY3 first_mismatch_pos=2" in r.stdout

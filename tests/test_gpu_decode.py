"""End-to-end GPU parity through the C ABI (cis2b_generate): token streams,
every per-step witness digest, final witness and argmax digests must equal
the reference (golden fixtures made by the reference's compiled C++ port)
and the oracle, tolerance zero."""
from __future__ import annotations

import hashlib

import numpy as np
import pytest

from conftest import golden_names, golden_prompts, load_golden

pytestmark = pytest.mark.gpu

_models: dict = {}


def model_for(pkg, synth, synth_root, name: str, reduction: str, max_positions: int = 0):
    key = (name, reduction, max_positions)
    if key not in _models:
        gate = "qwen3-port" if synth.MODELS[name].model_type == "qwen3" else "reference"
        _models[key] = pkg.Model(synth.ensure_model(name, synth_root), reduction=reduction,
                                 max_positions=max_positions, arch_gate=gate)
    return _models[key]


def check_against_golden(r: dict, g: dict, first: int = 0):
    for i, e in enumerate(g["sequences"]):
        j = i + first
        assert r["witness"][j].tobytes().hex() == e["witness"], ("witness", g["case"], i)
        assert r["argmax"][j].tobytes().hex() == e["argmax"], ("argmax", g["case"], i)
        assert hashlib.sha256(r["step_digests"][j].tobytes()).hexdigest() == e["steps_sha"], ("steps", i)
    e0 = g["sequences"][0]
    assert [int(t) for t in r["tokens"][first]] == e0["tokens"]
    assert [s.tobytes().hex() for s in r["step_digests"][first]] == e0["step_digests"]


SMALL = [n for n in golden_names() if n.startswith(("tiny", "mid"))]
FULL = [n for n in golden_names() if n.startswith(("c", "tree_"))]


@pytest.mark.parametrize("name", SMALL)
def test_small_configs_match_reference(name, pkg, synth, synth_root):
    g = load_golden(name)
    m = model_for(pkg, synth, synth_root, g["model"], g["reduction"])
    r = m.generate(golden_prompts(synth, g), g["gen"], sample=g["sample"])
    check_against_golden(r, g)


@pytest.mark.parametrize("name", FULL)
def test_baseline_configs_match_reference(name, pkg, synth, synth_root):
    g = load_golden(name)
    prompts = golden_prompts(synth, g)
    maxp = max(len(p) for p in prompts) + g["gen"]
    m = model_for(pkg, synth, synth_root, g["model"], g["reduction"], max_positions=max(4096, maxp))
    r = m.generate(prompts, g["gen"], sample=g["sample"])
    check_against_golden(r, g)


@pytest.mark.parametrize("model,reduction,sampled", [("tiny", "sequential", False), ("tiny_qwen3", "tree", True),
                                                     ("tiny_mha_untied", "tree", False),
                                                     ("tiny_bias", "sequential", True)])
def test_ragged_batch_matches_oracle(model, reduction, sampled, pkg, oracle, synth, synth_root):
    d = synth.ensure_model(model, synth_root)
    lens = [1, 2, 7, 31, 64, 3, 17, 1, 50]
    prompts = [synth.random_prompts(model, 1, L, 77, first=i)[0] for i, L in enumerate(lens)]
    sample = {"seed": 5, "temperature": 0.8, "top_p": 0.95} if sampled else None
    m = model_for(pkg, synth, synth_root, model, reduction)
    r = m.generate(prompts, 20, sample=sample)
    o = oracle.PortOracle(d, tree=reduction == "tree").generate(prompts, 20, sample=sample)
    for k in ("tokens", "step_digests", "witness", "argmax"):
        assert np.array_equal(r[k], o[k]), k


@pytest.mark.parametrize("model,top_k,top_p", [("tiny", 40, 0.95), ("tiny_qwen3", 0, 0.9), ("mid", 1, 1.0),
                                               ("tiny_bias", 0, 1.0)])
def test_gumbel_sampled_decode_matches_oracle(model, top_k, top_p, pkg, oracle, synth, synth_root):
    """Sampled decode under the seeded Gumbel-max clause (CIS2-SAMPLE-1):
    tokens, per-step digests (with the clause's header after the prompt ids)
    and final digests equal the oracle's."""
    d = synth.ensure_model(model, synth_root)
    lens = [1, 9, 33, 4]
    prompts = [synth.random_prompts(model, 1, L, 404, first=i)[0] for i, L in enumerate(lens)]
    sample = {"scheme": "gumbel", "seed": 0xC0FFEE, "temperature": 0.8, "top_k": top_k, "top_p": top_p}
    m = model_for(pkg, synth, synth_root, model, "sequential")
    r = m.generate(prompts, 12, sample=sample)
    o = oracle.PortOracle(d).generate(prompts, 12, sample=sample)
    for k in ("tokens", "step_digests", "witness", "argmax"):
        assert np.array_equal(r[k], o[k]), k
    # the two schemes differ (different noise and header), as they should
    e23 = m.generate(prompts[:1], 12, sample={"seed": 0xC0FFEE, "temperature": 0.8, "top_p": top_p})
    assert e23["witness"][0].tobytes() != r["witness"][0].tobytes()


def test_batch_rows_equal_solo_runs(pkg, synth, synth_root):
    """Batch invariance (code/patches/cis2-fp__cm_gpu3-batched-full.patch:79-108):
    every row of a batched decode equals its own batch-1 decode."""
    m = model_for(pkg, synth, synth_root, "mid", "sequential")
    prompts = [synth.random_prompts("mid", 1, L, 21, first=i)[0] for i, L in enumerate([5, 40, 12, 64, 1])]
    both = m.generate(prompts, 16)
    for i, p in enumerate(prompts):
        solo = m.generate([p], 16)
        assert solo["witness"][0].tobytes() == both["witness"][i].tobytes()
        assert np.array_equal(solo["step_digests"][0], both["step_digests"][i])


def test_repeat_runs_identical(pkg, synth, synth_root):
    """The reference's run1 == run2 same-process determinism check (src/main.rs:1228-1249)."""
    m = model_for(pkg, synth, synth_root, "mid", "tree")
    prompts = [synth.random_prompts("mid", 1, 9, 3, first=i)[0] for i in range(6)]
    a = m.generate(prompts, 12)
    b = m.generate(prompts, 12)
    for k in a:
        assert np.array_equal(a[k], b[k])


def test_teacher_forced_logits_bit_exact(pkg, oracle, synth, synth_root):
    d = synth.ensure_model("mid", synth_root)
    m = model_for(pkg, synth, synth_root, "mid", "sequential")
    ids = synth.random_prompts("mid", 1, 30, 8)[0]
    got = m.logits(ids, 20, 11)
    want = oracle.PortOracle(d).logits(ids, 20, 11)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_zero_generated_tokens(pkg, oracle, synth, synth_root):
    d = synth.ensure_model("tiny", synth_root)
    m = model_for(pkg, synth, synth_root, "tiny", "sequential")
    p = [synth.random_prompts("tiny", 1, 4, 1)[0]]
    r = m.generate(p, 0)
    o = oracle.PortOracle(d).generate(p, 0)
    assert r["witness"][0].tobytes() == o["witness"][0].tobytes()
    assert r["argmax"][0].tobytes() == o["argmax"][0].tobytes()


def test_info_digests(pkg, synth, synth_root):
    m = model_for(pkg, synth, synth_root, "smollm2", "sequential", max_positions=4096)
    assert m.info["table_digest"].hex() == "23c7bfaf5cef0095fd021af2eb1808abb4928bae4219756d86bdac670a06b35d"
    assert m.info["inv_freq_table_digest"].hex() == "da9f6dcfde0425588815509e874515cdcd3d6b8818b6d0136590052e7bbf6f12"


def test_generate_rejects_bad_arguments(pkg, synth, synth_root):
    m = model_for(pkg, synth, synth_root, "tiny", "sequential")
    with pytest.raises(pkg.Cis2Error) as e:
        m.generate([[600]], 2)  # id >= vocab
    assert e.value.code == 1
    with pytest.raises(pkg.Cis2Error):
        m.generate([[1, 2]], 5000)  # exceeds max_positions
    with pytest.raises(pkg.Cis2Error):
        m.generate([[1]], 2, sample={"seed": 1, "temperature": 0.0, "top_p": 0.9})
    with pytest.raises(pkg.Cis2Error):  # top_k belongs to the Gumbel-max scheme
        m.generate([[1]], 2, sample={"seed": 1, "temperature": 0.8, "top_p": 0.9, "top_k": 5})
    with pytest.raises(pkg.Cis2Error):
        m.generate([[1]], 2, sample={"scheme": "gumbel", "seed": 1, "temperature": float("inf"), "top_p": 0.9})
    r = m.generate([[1, 2]], 2)  # still usable after errors
    assert r["tokens"].shape == (1, 2)


def test_cli_prints_reference_lines(pkg, synth, synth_root, tmp_path):
    import subprocess
    g = load_golden("tiny_seq_greedy")
    prompts = golden_prompts(synth, g)
    ids = tmp_path / "ids.txt"
    ids.write_text("\n".join(" ".join(str(int(v)) for v in p) for p in prompts) + "\n")
    out = subprocess.run([pkg.CLI_PATH, "--weights-dir", synth.ensure_model("tiny", synth_root), "--ids", str(ids),
                          "--gen-toks", str(g["gen"])], capture_output=True, text=True, check=True).stdout
    lines = [ln for ln in out.splitlines() if ln.startswith("CIS2_REF digest=")]
    assert [ln.split()[1].split("=")[1] for ln in lines] == [e["witness"] for e in g["sequences"]]
    assert "table_digest=23c7bfaf" in out

"""CPU tests of the oracle (our C restatement, oracle/cis2_oracle.c): pinned
against the reference's weight-independent golden vectors, the reference's
own unit-test cases, and the reference's compiled C++ port on seeded
synthetic models (tests/golden/*.json, written by make_golden.py)."""
from __future__ import annotations

import hashlib
import struct

import numpy as np
import pytest

from conftest import golden_names, golden_prompts, load_golden


def f2u(x: float) -> int:
    return struct.unpack("<I", struct.pack("<f", x))[0]


# ---------------------------------------------------------------- golden vectors

def test_table_digest_matches_spec(oracle):
    # code/cis2-fp/verify3/selftest.c:56 (spec §6.6)
    assert oracle.table_digest().hex() == "23c7bfaf5cef0095fd021af2eb1808abb4928bae4219756d86bdac670a06b35d"


def test_inv_freq_digest_matches_spec(oracle, synth, synth_root):
    # theta = 1e5, head_dim = 64 (verify3/selftest.c:80, spec §7.2)
    o = oracle.PortOracle(synth.ensure_model("smollm2", synth_root))
    _, d = o.inv_freq()
    assert d.hex() == "da9f6dcfde0425588815509e874515cdcd3d6b8818b6d0136590052e7bbf6f12"


def test_dot_seq_order_case(oracle):
    # src/math.rs:613-623: (((0 + 1e8) + 1) - 1e8) == +0 exactly
    a = np.array([1e8, 1.0, -1e8], dtype=np.float32)
    b = np.ones(3, dtype=np.float32)
    r = oracle.lib().cis2o_dot(a.ctypes.data, b.ctypes.data, 3, 0)
    assert f2u(r) == 0


def test_tree_sum_ragged_example(oracle):
    # src/math.rs:643-651: ((a0+a1)+(a2+a3))+a4 for n = 5
    a = np.array([1, 2, 3, 4, 5], dtype=np.float32)
    want = np.float32((np.float32(1 + 2) + np.float32(3 + 4)) + np.float32(5))
    assert oracle.lib().cis2o_sum(a.ctypes.data, 5, 1) == want
    assert oracle.lib().cis2o_sum(a.ctypes.data, 0, 1) == 0.0


def test_rsqrt_cases(oracle):
    # src/math.rs:606-609
    assert oracle.lib().cis2o_rsqrt(64.0) == 0.125


def test_widen_bf16_bits(oracle):
    # gpu/test_math.cpp:76-83: the exact <<16 widen, through a 1x1 matmul by 1.0
    W = np.array([[0x3F80], [0x0000], [0x8000]], dtype=np.uint16)
    X = np.ones((1, 1), dtype=np.float32)
    Wp = np.zeros((3, 8), dtype=np.uint16)
    Wp[:, 0] = W[:, 0]
    Xp = np.zeros((1, 8), dtype=np.float32)
    Xp[0, 0] = 1.0
    Y = oracle.matmul_bf16(Wp, Xp)
    assert [f2u(v) for v in Y[0]] == [0x3F800000, 0, 0]  # +0 acc absorbs -0


def test_sha256_kats(oracle):
    for msg in [b"", b"abc", b"a" * 55, b"a" * 56, b"a" * 64, bytes(range(256)) * 5]:
        out = np.zeros(32, dtype=np.uint8)
        buf = np.frombuffer(msg, dtype=np.uint8).copy() if msg else np.zeros(1, np.uint8)
        oracle.lib().cis2o_sha256(buf.ctypes.data, len(msg), out.ctypes.data)
        assert out.tobytes() == hashlib.sha256(msg).digest()


def test_splitmix64_kat(oracle):
    # SplitMix64 (Vigna 2015) seeded with 0 yields 0xe220a8397b1dcdaf first.
    # rng_word(s, p) = sm(s ^ sm(p)) (e23 patch :617-629); choose s = sm(p).
    M = (1 << 64) - 1

    def sm(x):
        z = (x + 0x9E3779B97F4A7C15) & M
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
        return z ^ (z >> 31)

    assert sm(0) == 0xE220A8397B1DCDAF
    for p in (0, 1, 7, 12345):
        assert oracle.lib().cis2o_rng_word(sm(p), p) == 0xE220A8397B1DCDAF
        assert oracle.lib().cis2o_rng_word(42, p) == sm(42 ^ sm(p))


# ---------------------------------------------------------------- E23 sampler cases

def _sample(oracle, logits, T, top_p, seed, pos):
    x = np.ascontiguousarray(logits, dtype=np.float32)
    return oracle.lib().cis2o_sample_pinned(x.ctypes.data, x.size, T, top_p, seed, pos)


def test_sampler_unit_cases(oracle):
    # e23 patch src/sampling.rs tests :762-805
    logits = np.arange(64, dtype=np.float32) * np.float32(0.01)
    assert _sample(oracle, logits, 0.8, 0.95, 123, 0) == _sample(oracle, logits, 0.8, 0.95, 123, 0)
    l2 = np.zeros(32, dtype=np.float32)
    l2[7] = 50.0
    assert _sample(oracle, l2, 1.0, 1e-6, 999, 3) == 7
    l3 = np.array([((i * 37) % 17) * 0.3 for i in range(128)], dtype=np.float32)
    for seed in range(16):
        assert 0 <= _sample(oracle, l3, 0.8, 1.0, seed, seed) < 128
    assert _sample(oracle, np.zeros(4, np.float32), 1.0, 1e-6, 0, 0) == 0


# ---------------------------------------------------------------- parity with the reference

SMALL = [n for n in golden_names() if n.startswith(("tiny", "mid", "coverage"))]


@pytest.mark.parametrize("name", SMALL)
def test_port_matches_reference_fixture(name, oracle, synth, synth_root):
    g = load_golden(name)
    d = synth.ensure_model(g["model"], synth_root)
    prompts = golden_prompts(synth, g)
    o = oracle.PortOracle(d, tree=g["reduction"] == "tree")
    r = o.generate(prompts, g["gen"], sample=g["sample"])
    for i, e in enumerate(g["sequences"]):
        assert r["witness"][i].tobytes().hex() == e["witness"], (name, i)
        assert r["argmax"][i].tobytes().hex() == e["argmax"], (name, i)
        steps = hashlib.sha256(r["step_digests"][i].tobytes()).hexdigest()
        assert steps == e["steps_sha"], (name, i)
    e0 = g["sequences"][0]
    assert [int(t) for t in r["tokens"][0]] == e0["tokens"]
    assert [s.tobytes().hex() for s in r["step_digests"][0]] == e0["step_digests"]


def test_port_matches_reference_binary_live(oracle, synth, synth_root):
    """Runs the reference's compiled port (oracle/_ref) next to the
    restatement on fresh prompts, when the binary is present."""
    if not oracle.have_refdrv():
        pytest.skip("oracle/_ref not built (reference sources absent)")
    d = synth.ensure_model("tiny_mha_untied", synth_root)
    prompts = [synth.random_prompts("tiny_mha_untied", 1, L, 99, first=i)[0] for i, L in enumerate([1, 2, 31])]
    for tree in (False, True):
        r = oracle.PortOracle(d, tree=tree).generate(prompts, 9)
        ref = oracle.run_refdrv(d, prompts, 9, tree=tree)
        assert [r["witness"][i].tobytes().hex() for i in range(3)] == [x["witness"] for x in ref]


def test_trace_matches_reference_cli(oracle, synth, synth_root, tmp_path):
    """Per-(pos, layer, op) SHA-256 trace equals the reference cis2_host --trace."""
    import os
    import subprocess
    exe = os.path.join(oracle.REF_DIR, "cis2_host")
    if not os.path.exists(exe):
        pytest.skip("oracle/_ref not built")
    d = synth.ensure_model("tiny", synth_root)
    ids = synth.random_prompts("tiny", 1, 6, 5)[0]
    idp = tmp_path / "ids.txt"
    idp.write_text(" ".join(str(int(v)) for v in ids))
    subprocess.run([exe, "--weights-dir", d, "--ids", str(idp), "--gen-toks", "3", "--trace",
                    str(tmp_path / "ref.txt")], check=True, capture_output=True)
    oracle.PortOracle(d).generate([ids], 3, trace_path=str(tmp_path / "port.txt"))
    ref = (tmp_path / "ref.txt").read_text().splitlines()
    port = (tmp_path / "port.txt").read_text().splitlines()
    assert len(port) > 100 and ref[:len(port)] == port


def test_logits_teacher_forced_consistent(oracle, synth, synth_root):
    """cis2o_logits rows equal the logits behind a greedy decode's choices."""
    d = synth.ensure_model("tiny", synth_root)
    o = oracle.PortOracle(d)
    p = synth.random_prompts("tiny", 1, 5, 3)[0]
    r = o.generate([p], 4)
    ids = np.concatenate([p, r["tokens"][0][:3]])
    L = o.logits(ids, 5, 4)
    assert [int(np.argmax(row)) for row in L] == [int(t) for t in r["tokens"][0]]


def test_batch_equals_solo(oracle, synth, synth_root):
    d = synth.ensure_model("tiny_qwen3", synth_root)
    o = oracle.PortOracle(d)
    ps = [synth.random_prompts("tiny_qwen3", 1, L, 4, first=i)[0] for i, L in enumerate([3, 8, 1])]
    both = o.generate(ps, 6)
    for i, p in enumerate(ps):
        solo = o.generate([p], 6)
        assert solo["witness"][0].tobytes() == both["witness"][i].tobytes()


# ---------------------------------------------------------------- seeded Gumbel-max sampler (CIS2-SAMPLE-1)

def test_murmur3_published_answers(oracle):
    # MurmurHash3_x86_32 of the empty key (seeded-sampling patch :91-93)
    assert oracle.lib().cis2o_murmur3_32(None, 0, 0) == 0x00000000
    assert oracle.lib().cis2o_murmur3_32(None, 0, 1) == 0x514E28B7


@pytest.mark.parametrize("seed,step,index,h,u,g", [
    # seeded-sampling patch :150-155 (hash seed 0x43495332)
    (0x0000000000000001, 0, 0, 0x07731EA2, 0x3CEE63E0, 0xBFA1B32B),
    (0x0000000000000001, 0, 1, 0xC832451B, 0x3F483245, 0x3FB392C7),
    (0x0000000000000001, 1, 0, 0xC0D0C4FA, 0x3F40D0C5, 0x3FA15FFE),
    (0xFFFFFFFFFFFFFFFF, 7, 49151, 0xE682298D, 0x3F668229, 0x40104F5A),
    # toy vector rows of labs/w1x-sample/reports/w1x-sample/RESULTS-hq-builder.md:31-38
    (1, 0, 2, 0x68663A0B, 0x3ED0CC76, 0x3DDEB89E),
    (1, 0, 3, 0x0F68EB80, 0x3D768EB0, 0xBF844163),
    (1, 0, 4, 0xEF1F23D1, 0x3F6F1F23, 0x402BDAE7),
    (1, 0, 5, 0x62C78D96, 0x3EC58F1A, 0x3D483F2A),
    (1, 0, 6, 0x03469A9A, 0x3C51A6C0, 0xBFBC6F8D),
    (1, 0, 7, 0xDE644043, 0x3F5E6441, 0x3FFAFD67),
])
def test_gumbel_noise_known_answers(seed, step, index, h, u, g, oracle):
    assert oracle.gumbel_noise(seed, step, index) == (h, u, g)


def test_gumbel_toy_vector(oracle):
    # seeded-sampling patch :157-164: V = 8, seed 1, step 0, T = 0.8, top_k 4, top_p 0.9
    logits = np.array([1.0, 2.0, 2.0, -1.0, 0.5, 3.0, 3.0, -4.0], dtype=np.float32)
    t = np.uint32(0x3F4CCCCD).view(np.float32)
    p = np.uint32(0x3F666666).view(np.float32)
    nxt, z = oracle.sample_gumbel(logits, float(t), 4, float(p), 1, 0)
    assert nxt == 1
    want = [0xFF800000, 0x4079C964, 0x4026F5C5, 0xFF800000, 0xFF800000, 0x407320FD, 0x4011C83A, 0xFF800000]
    assert [int(v) for v in z.view(np.uint32)] == want


def test_gumbel_candidate_set_rules(oracle):
    rng = np.random.default_rng(11)
    logits = rng.standard_normal(1000).astype(np.float32)
    logits[10] = logits[20] = 9.0          # tie at the top: rank order puts index 10 first
    # top_k = 1 keeps rank 0 only: the lowest index among the maximal logits
    assert oracle.sample_gumbel(logits, 0.7, 1, 1.0, 5, 3)[0] == 10
    # a tiny top_p keeps rank 0 only as well
    assert oracle.sample_gumbel(logits, 0.7, 0, 1e-7, 5, 3)[0] == 10
    # -0 and +0 are equal for the rank order
    z = np.zeros(6, dtype=np.float32)
    z[2] = -0.0
    nxt, zz = oracle.sample_gumbel(z, 1.0, 3, 1.0, 9, 0)
    kept = [i for i, v in enumerate(zz.view(np.uint32)) if v != 0xFF800000]
    assert kept == [0, 1, 2]


# ---------------------------------------------------------------- pinned-function sweep

def _math_fixture():
    import json
    import os
    with open(os.path.join(os.path.dirname(__file__), "golden", "math_sweep.json")) as f:
        return json.load(f)


def test_math_sweep_port_matches_reference_digests(oracle):
    """The port's six pinned functions over the 242,428-point sweep equal the
    reference's cis2_math.h (fixture written by tests/golden/make_math_golden.py)."""
    g = _math_fixture()
    x = oracle.math_sweep_inputs()
    outs = {f: oracle.pinned_map(i, x) for i, f in enumerate(oracle.MATH_FUNCS)}
    d = oracle.sweep_digests(x, outs)
    assert d["n"] == g["n"] == 242428
    assert d["inputs_sha256"] == g["inputs_sha256"]
    for f in oracle.MATH_FUNCS:
        assert d[f] == g[f], f
    # x86 SSE on both sides: the exact rows, NaN encodings included
    for i, row in zip(g["row_index"], g["rows"]):
        assert int(x.view(np.uint32)[i]) == row[0]
        assert [int(outs[f].view(np.uint32)[i]) for f in oracle.MATH_FUNCS] == row[1:], i


def test_math_sweep_port_equals_reference_binary(oracle, tmp_path):
    """Bit for bit against the reference functions run live, when oracle/_ref is built."""
    import os
    import subprocess
    exe = os.path.join(oracle.REF_DIR, "refmath")
    if not os.path.exists(exe):
        pytest.skip("oracle/_ref not built")
    subprocess.run([exe, str(tmp_path / "s.bin")], check=True, capture_output=True)
    x, ref = oracle.read_refmath(str(tmp_path / "s.bin"))
    assert np.array_equal(x.view(np.uint32), oracle.math_sweep_inputs().view(np.uint32))
    for i, f in enumerate(oracle.MATH_FUNCS):
        assert np.array_equal(oracle.pinned_map(i, x).view(np.uint32), ref[f].view(np.uint32)), f


def test_argmax_edge_rows_match_serial_scan(oracle):
    """The oracle's argmax is the reference's strict '>' scan from index 0
    (code/cis2-fp/src/main.rs:1161-1169) on the device test's edge rows."""
    from conftest import argmax_edge_rows
    for V in (32, 257):
        for r in argmax_edge_rows(V):
            best, bv = 0, r[0]
            for i in range(1, V):
                if r[i] > bv:
                    best, bv = i, r[i]
            assert int(oracle.lib().cis2o_argmax(r.ctypes.data, V)) == best

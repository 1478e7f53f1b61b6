"""GPU parity of single kernels, through the C ABI, against the oracle.
Bit-exact (tolerance zero) everywhere."""
from __future__ import annotations

import hashlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def sweep_inputs() -> np.ndarray:
    """Edge values plus a seeded sweep, following the reference's golden
    sweep recipe (code/cis2-fp/src/bin/math_dump.rs:67-180): explicit edges,
    exp clamp boundaries, k*pi/2 and k*pi/4 neighbours, then LCG bit
    patterns and uniform ranges."""
    edges = [0x00000000, 0x80000000, 0x00000001, 0x80000001, 0x007FFFFF, 0x807FFFFF, 0x00800000,
             0x80800000, 0x3F800000, 0xBF800000, 0x3F000000, 0xBF000000, 0x7F7FFFFF, 0xFF7FFFFF,
             0x7F800000, 0xFF800000, 0x7FC00000, 0x34000000, 0x4B000000, 0x5F000000]
    v = list(np.array(edges, dtype=np.uint32).view(np.float32))
    for x in [-88.0, -87.99999, -88.00001, 88.0, 87.99999, 88.00001, 1e-10, -1e-10, 0.6931472,
              -0.6931472, 0.3465736, 1e10, -1e10]:
        f = np.float32(x)
        v += [f, np.nextafter(f, np.float32(np.inf)), np.nextafter(f, np.float32(-np.inf))]
    for k in range(-64, 65):
        for base in (np.pi / 2, np.pi / 4):
            f = np.float32(k * base)
            v += [f, np.nextafter(f, np.float32(np.inf)), np.nextafter(f, np.float32(-np.inf))]
    state = np.uint64(0x243F6A8885A308D3)
    bits = []
    for _ in range(60000):
        state = np.uint64((int(state) * 6364136223846793005 + 1442695040888963407) & ((1 << 64) - 1))
        bits.append(int(state) >> 32)
    v += list(np.array(bits, dtype=np.uint32).view(np.float32))
    rng = np.random.default_rng(7)
    v += list(rng.uniform(-100, 100, 40000).astype(np.float32))
    v += list(rng.uniform(-3, 3, 40000).astype(np.float32))
    v += list((rng.uniform(0, 1, 20000) * 2048 * 0.5).astype(np.float32))  # RoPE angles
    v += list(np.exp(rng.uniform(-80, 80, 20000)).astype(np.float32))      # ln domain
    return np.array(v, dtype=np.float32)


def test_pinned_math_reference_sweep(pkg, oracle):
    """The device's six pinned functions over the reference sweep's 242,428
    points: every non-NaN output bit-identical to the reference's
    cis2_math.h (digests in tests/golden/math_sweep.json), NaN exactly where
    the reference gives NaN, and the explicit NaN returns of exp and ln
    (0x7FC00000 for a NaN input) bit for bit."""
    import json
    import os
    with open(os.path.join(os.path.dirname(__file__), "golden", "math_sweep.json")) as f:
        g = json.load(f)
    x = oracle.math_sweep_inputs()
    outs = {f: pkg.pinned_map(f, x) for f in oracle.MATH_FUNCS}
    d = oracle.sweep_digests(x, outs)
    assert d["inputs_sha256"] == g["inputs_sha256"]
    for f in oracle.MATH_FUNCS:
        assert d[f] == g[f], f
    nan_in = np.isnan(x)
    for f in ("exp", "ln"):
        assert np.all(outs[f][nan_in].view(np.uint32) == 0x7FC00000), f


@pytest.mark.parametrize("fn", ["exp", "sin", "cos", "ln", "silu", "rsqrt"])
def test_pinned_math_bit_exact(fn, pkg, oracle):
    x = sweep_inputs()
    got = pkg.pinned_map(fn, x)
    want = oracle.pinned_map(pkg.PINNED_FUNCS[fn], x)
    gb, wb = got.view(np.uint32), want.view(np.uint32)
    # NaNs made by arithmetic (inf - inf inside a polynomial fed a
    # non-finite or |x| ~ 1e38 argument) carry the hardware's own encoding:
    # x86 SSE returns its default NaN 0xFFC00000 or the quieted operand,
    # NVIDIA GPUs the canonical 0x7FFFFFFF.  Those must still be NaN; every
    # other output, and every NaN the pinned functions return explicitly
    # (0x7FC00000), must match bit for bit.
    want_nan = np.isnan(want)
    assert np.all(np.isnan(got[want_nan]))
    bad = np.nonzero((gb != wb) & ~want_nan)[0]
    assert bad.size == 0, [(hex(x.view(np.uint32)[i]), hex(gb[i]), hex(wb[i])) for i in bad[:8]]
    explicit = np.isnan(x) & (fn in ("exp", "ln"))
    assert np.array_equal(gb[explicit], wb[explicit])


SHAPES = [(1, 576, 576), (3, 192, 576), (4, 100, 96), (7, 1536, 576), (16, 64, 1536), (33, 200, 40),
          (64, 576, 1536), (64, 960, 576), (5, 4099, 64), (128, 1024, 3072), (65, 300, 8), (2, 49152, 576),
          (2048, 2560, 96), (1970, 2500, 40), (300, 20000, 32),   # the 64 x 64 prompt-pass tile
          (4096, 576, 96), (700, 9000, 16),                       # the 128 x 64 tile
          # the narrower register tiles the many-row decode steps pick (every
          # tile is some shape's choice, checked in test_abi): 64 x 32, 64 x 16
          # and 16 x 32 thread-block tiles, ragged edges and K not a multiple
          # of the 32-deep k stage included
          (300, 768, 768), (300, 2304, 96), (121, 960, 64), (256, 576, 40), (70, 40, 32),
          (300, 32000, 16), (96, 100, 24), (129, 72, 16), (96, 8192, 24), (65, 2048, 40)]

# Tile (threads along m, threads along n, rows per thread, columns per
# thread) of the register-tiled kernel, in the order the library numbers them.
BIG_TILES = [(16, 16, 8, 4), (16, 16, 4, 4), (16, 8, 4, 4), (16, 8, 4, 2), (8, 16, 2, 2)]


@pytest.mark.parametrize("form", ["sequential", "tree", "decode", "decode_tree"])
@pytest.mark.parametrize("rows,n,k", SHAPES)
def test_matmul_bit_exact(rows, n, k, form, pkg, oracle):
    """Both GEMM kernels (the panel kernels of the prompt pass in both orders,
    the few-row kernel of decode steps in both orders) against the oracle's
    dot products, bit for bit."""
    tree = form in ("tree", "decode_tree")
    decode = form.startswith("decode")
    rng = np.random.default_rng(rows * 1000003 + n * 31 + k)
    W = (rng.standard_normal((n, k)).astype(np.float32) * np.float32(0.02)).view(np.uint32)
    W = ((W + 0x7FFF + ((W >> 16) & 1)) >> 16).astype(np.uint16)
    X = rng.standard_normal((rows, k)).astype(np.float32)
    X[:, ::7] = 0.0  # signed zeros and cancellations in the chains
    X[:, 1::11] *= -0.0
    if decode and (rows > 1024 or (tree and k % 32)):  # shapes the few-row form refuses
        with pytest.raises(pkg.Cis2Error) as e:
            pkg.matmul(W, X, tree=tree, decode=True)
        assert e.value.code == 1
        return
    got = pkg.matmul(W, X, tree=tree, decode=decode)
    want = oracle.matmul_bf16(W, X, tree=tree)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("prefix_len,chunk", [(0, 17), (160, 49153), (190, 49153), (30, 1024), (2, 2),
                                              (62, 16), (64, 15), (190, 151937), (14, 100)])
def test_witness_stream_sha256(prefix_len, chunk, pkg):
    rng = np.random.default_rng(prefix_len * 7 + chunk)
    prefix = rng.integers(0, 256, prefix_len, dtype=np.uint8).tobytes()
    n_chunks = 3
    words = rng.integers(0, 2**32, chunk * n_chunks, dtype=np.uint64).astype(np.uint32)
    got = pkg.sha256_stream(prefix, words, chunk)
    h = hashlib.sha256(prefix)
    for c in range(n_chunks):
        h.update(words[c * chunk:(c + 1) * chunk].astype("<u4").tobytes())
        assert got[c].tobytes() == h.copy().digest(), c


def test_witness_stream_prefix_only(pkg):
    got = pkg.sha256_stream(b"abc", np.zeros(0, np.uint32), 0)
    assert got[0].tobytes() == hashlib.sha256(b"abc").digest()


@pytest.mark.parametrize("n,T,top_p", [(64, 0.8, 0.95), (4096, 0.8, 0.95), (151936, 0.8, 0.95),
                                       (1000, 1.0, 1e-6), (1000, 0.5, 1.0), (49152, 1.3, 0.5)])
def test_sampler_matches_oracle(n, T, top_p, pkg, oracle):
    rng = np.random.default_rng(n)
    for trial in range(3):
        logits = (rng.standard_normal(n) * (0.6 + trial)).astype(np.float32)
        if trial == 2:
            logits[::5] = logits[0]  # many exact ties -> index tie-break
        for pos in (0, 63, 300):
            seed = 1234 + trial
            want = oracle.lib().cis2o_sample_pinned(logits.ctypes.data, n, T, top_p, seed, pos)
            assert pkg.sample(logits, T, top_p, seed, pos) == want


def test_sampler_unit_cases_gpu(pkg):
    l2 = np.zeros(32, dtype=np.float32)
    l2[7] = 50.0
    assert pkg.sample(l2, 1.0, 1e-6, 999, 3) == 7
    assert pkg.sample(np.zeros(4, np.float32), 1.0, 1e-6, 0, 0) == 0


# ---------------------------------------------------------------- seeded Gumbel-max sampler (CIS2-SAMPLE-1)

def test_gumbel_toy_vector_gpu(pkg):
    # code/patches/cis2-spec__seeded-sampling.patch:157-164: next_id = 1
    logits = np.array([1.0, 2.0, 2.0, -1.0, 0.5, 3.0, 3.0, -4.0], dtype=np.float32)
    t = float(np.uint32(0x3F4CCCCD).view(np.float32))
    p = float(np.uint32(0x3F666666).view(np.float32))
    assert pkg.sample_gumbel(logits, t, 4, p, 1, 0) == 1


@pytest.mark.parametrize("n", [8, 1000, 49152, 151936])
@pytest.mark.parametrize("T,top_k,top_p", [(0.8, 40, 0.95), (1.0, 0, 1.0), (0.7, 0, 0.9), (1.3, 5, 1.0),
                                           (0.5, 100000, 0.5), (2.0, 1, 0.3)])
def test_gumbel_sampler_matches_oracle(n, T, top_k, top_p, pkg, oracle):
    rng = np.random.default_rng(n * 7 + top_k)
    for trial in range(3):
        logits = (rng.standard_normal(n) * (0.5 + trial)).astype(np.float32)
        if trial == 1:
            logits[::3] = logits[1]      # exact ties: index order decides the rank
        if trial == 2:
            logits[: n // 2] = 0.0
            logits[1: n // 2: 2] = -0.0  # -0 and +0 rank as equal values
        for seed, step in ((1, 0), (0xFFFFFFFFFFFFFFFF, 7), (12345, 255)):
            want, _ = oracle.sample_gumbel(logits, T, top_k, top_p, seed, step)
            assert pkg.sample_gumbel(logits, T, top_k, top_p, seed, step) == want, (trial, seed, step)


@pytest.mark.parametrize("V", [32, 49152, 151936])
def test_argmax_ties_zeros_and_nans(V, pkg, oracle):
    from conftest import argmax_edge_rows
    """The decode steps' argmax kernel against the oracle's serial scan and a
    plain-Python strict '>' scan, on every edge row at once (one row per
    block, as in a batched step)."""
    rows = argmax_edge_rows(V)
    X = np.stack(rows)
    got = pkg.argmax(X)
    for r, g in zip(rows, got):
        best, bv = 0, r[0]
        for i in range(1, V) if V <= 64 else ():
            if r[i] > bv:
                best, bv = i, r[i]
        want = int(oracle.lib().cis2o_argmax(r.ctypes.data, V))
        if V <= 64:
            assert want == best
        assert int(g) == want

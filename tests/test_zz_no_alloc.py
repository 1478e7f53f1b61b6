"""The sampler entry point that allocates nothing (cis2b_op_sample_static).

It serves callers that cannot call cudaMalloc: code whose device memory
belongs to its own allocator, or code that must not trigger the device
synchronisation an allocation brings.  It takes device pointers and runs in
a fixed scratch array inside the library.  Here the test itself allocates
the input row and the output slot (through torch) and checks that two calls
in a row, the second smaller than the first, draw the same index as the
allocating entry point cis2b_op_sample and as the CPU oracle's restatement
of the E23 sampler; then the same on a stream of the caller's own, and the
argument checks.  Indices are integers, so the match must be exact.

This file is named so that pytest collects it after every other test file.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_N = 262144  # CIS2B_STATIC_SAMPLE_MAX in include/cis2b.h


def _static_sample(pkg, d_logits, n, temperature, top_p, seed, position, d_out, stream=None):
    return pkg.lib().cis2b_op_sample_static(0, d_logits.data_ptr(), n, temperature, top_p, seed, position,
                                            d_out.data_ptr(), stream)


# (n, temperature, top_p, seed, position): the Qwen3 vocabulary first, then a
# smaller row that leaves stale data from the first call in the scratch array.
CASES = [(151936, 0.8, 0.95, 7, 64), (4099, 1.3, 0.5, 9, 300)]


def _row(rng, n):
    logits = (rng.standard_normal(n) * 1.5).astype(np.float32)
    logits[::7] = logits[3]  # exact ties exercise the index-ascending order
    return logits


def _want(pkg, oracle, logits, temperature, top_p, seed, position):
    want = pkg.sample(logits, temperature, top_p, seed, position)
    ref = int(oracle.lib().cis2o_sample_pinned(logits.ctypes.data, logits.size, temperature, top_p, seed,
                                               position))
    assert want == ref
    return want


def test_static_sampler_matches_allocating_entry_point(pkg, oracle):
    import torch
    rng = np.random.default_rng(20261201)
    for n, temperature, top_p, seed, position in CASES:
        logits = _row(rng, n)
        d_logits = torch.from_numpy(logits).to("cuda")
        d_out = torch.full((1,), -1, dtype=torch.int32, device="cuda")
        rc = _static_sample(pkg, d_logits, n, temperature, top_p, seed, position, d_out)
        assert rc == 0, pkg.lib().cis2b_last_error().decode()
        torch.cuda.synchronize()
        got = int(d_out.item()) & 0xFFFFFFFF
        assert got == _want(pkg, oracle, logits, temperature, top_p, seed, position), n


def test_static_sampler_on_a_caller_stream(pkg, oracle):
    """The intended use: the caller's own stream, synchronised by the caller."""
    import torch
    rng = np.random.default_rng(7)
    stream = torch.cuda.Stream()
    for n, temperature, top_p, seed, position in CASES:
        logits = _row(rng, n)
        d_logits = torch.from_numpy(logits).to("cuda")
        d_out = torch.full((1,), -1, dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()  # the inputs are ready before the caller's stream reads them
        rc = _static_sample(pkg, d_logits, n, temperature, top_p, seed + 1, position, d_out,
                            ctypes.c_void_p(stream.cuda_stream))
        assert rc == 0, pkg.lib().cis2b_last_error().decode()
        stream.synchronize()
        got = int(d_out.item()) & 0xFFFFFFFF
        assert got == _want(pkg, oracle, logits, temperature, top_p, seed + 1, position), n


def test_static_sampler_rejects_bad_arguments(pkg):
    import torch
    d_logits = torch.zeros(16, dtype=torch.float32, device="cuda")
    d_out = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = _static_sample(pkg, d_logits, MAX_N + 1, 0.8, 0.95, 1, 1, d_out)
    assert rc == 1
    assert "262144" in pkg.lib().cis2b_last_error().decode()
    assert _static_sample(pkg, d_logits, 16, 0.8, 0.95, 1, 2 ** 31, d_out) == 1
    assert "position" in pkg.lib().cis2b_last_error().decode()
    assert _static_sample(pkg, d_logits, 16, 0.8, 0.0, 1, 1, d_out) == 1
    assert _static_sample(pkg, d_logits, 16, 0.0, 0.95, 1, 1, d_out) == 1
    assert _static_sample(pkg, d_logits, 0, 0.8, 0.95, 1, 1, d_out) == 1

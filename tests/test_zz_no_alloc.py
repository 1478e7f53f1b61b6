"""The sampler entry point that allocates nothing (cis2b_op_sample_static).

It serves callers that cannot call cudaMalloc: code whose device memory
belongs to its own allocator, or code that must not trigger the device
synchronisation an allocation brings.  It takes device pointers and runs in
a fixed scratch array inside the library.  Here the test itself allocates
the input row and the output slot (through torch) and checks that two calls
in a row, the second smaller than the first, draw the same index as the
allocating entry point cis2b_op_sample.  Indices are integers, so the match
must be exact.

This file is named so that pytest collects it after every other test file.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_N = 262144  # CIS2B_STATIC_SAMPLE_MAX in include/cis2b.h


def _static_sample(pkg, d_logits, n, temperature, top_p, seed, position, d_out):
    return pkg.lib().cis2b_op_sample_static(0, d_logits.data_ptr(), n, temperature, top_p, seed, position,
                                            d_out.data_ptr(), None)


def test_static_sampler_matches_allocating_entry_point(pkg):
    import torch
    rng = np.random.default_rng(20261201)
    # (n, temperature, top_p, seed, position): the Qwen3 vocabulary first,
    # then a smaller row that leaves stale data from the first call in the
    # scratch array.
    cases = [(151936, 0.8, 0.95, 7, 64), (4099, 1.3, 0.5, 9, 300)]
    for n, temperature, top_p, seed, position in cases:
        logits = (rng.standard_normal(n) * 1.5).astype(np.float32)
        logits[::7] = logits[3]  # exact ties exercise the index-ascending order
        d_logits = torch.from_numpy(logits).to("cuda")
        d_out = torch.full((1,), -1, dtype=torch.int32, device="cuda")
        rc = _static_sample(pkg, d_logits, n, temperature, top_p, seed, position, d_out)
        assert rc == 0, pkg.lib().cis2b_last_error().decode()
        torch.cuda.synchronize()
        got = int(d_out.item()) & 0xFFFFFFFF
        want = pkg.sample(logits, temperature, top_p, seed, position)
        assert got == want, (n, got, want)


def test_static_sampler_rejects_oversize_rows(pkg):
    import torch
    d_logits = torch.zeros(16, dtype=torch.float32, device="cuda")
    d_out = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = _static_sample(pkg, d_logits, MAX_N + 1, 0.8, 0.95, 1, 1, d_out)
    assert rc == 1
    assert "262144" in pkg.lib().cis2b_last_error().decode()

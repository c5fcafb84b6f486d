"""sicu_gemv_host_noalloc, the host-buffer matvec for callers that must not
allocate device memory (an application allocator already owns the GPU's
memory, or device allocation is banned on the hot path). Its staging is a
fixed array inside the library, shared by every call, so these checks call it
twice in a row with different shapes and inputs and compare each result with
the allocating entry point, sicu_gemv_host, bit for bit (and within the 1e-5
per-element tolerance the other GPU tests state). This file sorts last so a
run that stops at the first failure has already run every other test."""

from __future__ import annotations

import numpy as np
import pytest

from siphon_b200 import lib as L
from siphon_b200 import quant as Q
from siphon_b200 import synth
from tests.gpu_util import assert_bits_equal, assert_within_tol, dev

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("wt", (Q.Q4_K, Q.Q6_K, Q.Q8_0, Q.F16), ids=lambda t: Q.NAMES[t])
def test_noalloc_matches_gemv_host_twice(sicu, wt):
    cases = [(1000, 4096, 3), (300, 2048, 4)]   # second call: fewer rows, shorter rows
    for n_out, n_in, seed in cases:
        w = dev(synth.weights(wt, n_out, n_in, seed=seed))
        x = synth.activations(n_in, 1, seed=seed + 10)[0]
        want = np.zeros(n_out, np.float32)
        sicu.gemv_host(wt, w, n_in, n_out, x, want)
        got = np.full(n_out, np.nan, np.float32)
        sicu.gemv_host_noalloc(wt, w, n_in, n_out, x, got)
        assert_bits_equal(got, want, f"{Q.NAMES[wt]} {n_out}x{n_in} no-alloc")
        assert_within_tol(got, want, "no-alloc")


def test_noalloc_rejects_shapes_beyond_its_scratch(sicu):
    x = np.zeros(65536 + 256, np.float32)
    y = np.zeros(8, np.float32)
    rc = sicu.lib.sicu_gemv_host_noalloc(Q.Q4_K, 16, 65536 + 256, 8, x.ctypes.data, y.ctypes.data, None)
    assert rc == L.SICU_EINVAL
    assert "scratch" in sicu.last_error()

"""sicu_gemv_host_noalloc, the host-buffer matvec for callers that must not
allocate device memory (an application allocator already owns the GPU's
memory, or device allocation is banned on the hot path). Its staging is a
fixed array inside the library, shared by every call, so these checks call it
twice in a row with different shapes and inputs and compare each result with
the oracle's matvec (the reference's scalar dots) and with the allocating
entry point, sicu_gemv_host, bit for bit (and within the 1e-5 per-element
tolerance the other GPU tests state). This file sorts last so a run that
stops at the first failure has already run every other test."""

from __future__ import annotations

import os
import subprocess
import sys
import textwrap
from pathlib import Path

import numpy as np
import pytest

from siphon_b200 import lib as L
from siphon_b200 import quant as Q
from siphon_b200 import synth
from tests.gpu_util import assert_bits_equal, assert_within_tol, dev

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.parametrize("wt", (Q.Q4_K, Q.Q6_K, Q.Q8_0, Q.F16), ids=lambda t: Q.NAMES[t])
def test_noalloc_matches_oracle_twice(sicu, oracle, wt):
    cases = [(1000, 4096, 3), (300, 2048, 4)]   # second call: fewer rows, shorter rows
    for n_out, n_in, seed in cases:
        wh = synth.weights(wt, n_out, n_in, seed=seed)
        w = dev(wh)
        x = synth.activations(n_in, 1, seed=seed + 10)[0]
        want = oracle.gemv(wt, wh, n_in, n_out, oracle.quantize_pair(wt, x)[0])
        got = np.full(n_out, np.nan, np.float32)
        sicu.gemv_host_noalloc(wt, w, n_in, n_out, x, got)
        assert_bits_equal(got, want, f"{Q.NAMES[wt]} {n_out}x{n_in} no-alloc vs oracle")
        assert_within_tol(got, want, "no-alloc")
        other = np.zeros(n_out, np.float32)
        sicu.gemv_host(wt, w, n_in, n_out, x, other)
        assert_bits_equal(got, other, f"{Q.NAMES[wt]} {n_out}x{n_in} no-alloc vs sicu_gemv_host")


def test_noalloc_empty_output_leaves_y_untouched(sicu):
    x = synth.activations(512, 1, seed=1)[0]
    y = np.full(4, 7.0, np.float32)
    rc = sicu.lib.sicu_gemv_host_noalloc(Q.Q4_K, None, 512, 0, x.ctypes.data, y.ctypes.data, None)
    assert rc == L.SICU_OK
    assert (y == 7.0).all()


def test_noalloc_rejects_shapes_beyond_its_scratch(sicu):
    x = np.zeros(65536 + 256, np.float32)
    y = np.zeros(8, np.float32)
    rc = sicu.lib.sicu_gemv_host_noalloc(Q.Q4_K, 16, 65536 + 256, 8, x.ctypes.data, y.ctypes.data, None)
    assert rc == L.SICU_EINVAL
    assert "scratch" in sicu.last_error()


def test_noalloc_without_init_in_a_fresh_process():
    """The entry point needs no sicu_init: a process that never calls it (the
    caller brought its own device context) gets the oracle's results, twice."""
    code = textwrap.dedent("""
        import sys
        import numpy as np
        import torch
        sys.path.insert(0, sys.argv[1])
        from oracle.oracle import Oracle
        from siphon_b200 import lib, synth
        from siphon_b200 import quant as Q
        torch.cuda.set_device(0)
        s = lib.load()                     # no s.init()
        o = Oracle()
        for n_out, n_in, seed in ((700, 2048, 5), (64, 1024, 6)):
            wh = synth.weights(Q.Q4_K, n_out, n_in, seed=seed)
            w = torch.from_numpy(wh).cuda()
            x = synth.activations(n_in, 1, seed=seed)[0]
            y = np.full(n_out, np.nan, np.float32)
            s.gemv_host_noalloc(Q.Q4_K, w, n_in, n_out, x, y)
            want = o.gemv(Q.Q4_K, wh, n_in, n_out, o.quantize_pair(Q.Q4_K, x)[0])
            assert (y.view(np.uint32) == want.view(np.uint32)).all(), (n_out, n_in)
        print("fresh ok")
    """)
    r = subprocess.run([sys.executable, "-c", code, str(ROOT)], capture_output=True, text=True, timeout=600,
                       env=dict(os.environ))
    assert r.returncode == 0, r.stdout + r.stderr
    assert "fresh ok" in r.stdout

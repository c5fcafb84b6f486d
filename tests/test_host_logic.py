"""Host-side helpers: geometry mirror, byte model, seeded synthetic inputs."""

from __future__ import annotations

import numpy as np

from siphon_b200 import quant as Q
from siphon_b200 import synth


def test_geometry_matches_oracle(oracle):
    import ctypes as C
    for t, (blck, size) in Q.GEOMETRY.items():
        b, s = C.c_uint32(), C.c_uint32()
        assert oracle.lib.orc_geometry(t, C.byref(b), C.byref(s)) == 1
        assert (b.value, s.value) == (blck, size)


def test_matvec_byte_model_configs0():
    # Q4_K 5632x2048 batch 1: weights + Q8_K activation + f32 out + f32 in
    assert Q.matvec_bytes(Q.Q4_K, 5632, 2048) == 6_521_120


def test_synthetic_weights_are_seeded_and_scaled():
    a = synth.weights(Q.Q4_K, 8, 512, seed=3)
    b = synth.weights(Q.Q4_K, 8, 512, seed=3)
    assert (a == b).all() and a.size == 8 * Q.row_bytes(Q.Q4_K, 512)
    d = a.reshape(-1, 144)[:, 0:2].copy().view(np.float16).astype(np.float32)
    assert (d >= 1e-4 * 0.999).all() and (d <= 1e-2 * 1.001).all()
    f = synth.weights(Q.F16, 4, 64, seed=1).view(np.float16)
    assert np.isfinite(f).all() and np.abs(f).max() <= 1.0

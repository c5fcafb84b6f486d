"""Randomised pin of the oracle restatement against the reference compiled
from its own sources (oracle/_ref). Skipped where that build is absent."""

from __future__ import annotations

import numpy as np
import pytest

from oracle.oracle import PAIR, row_bytes
from siphon_b200 import quant as Q
from siphon_b200 import synth


def _pair(reference, wt, x):
    if PAIR[wt] == Q.Q8_K:
        return reference.quant_q8_K(x)
    if PAIR[wt] == Q.Q8_0:
        return reference.quant_q8_0(x, "avx2")
    return reference.convert_f16(x)


@pytest.mark.parametrize("wt", Q.WEIGHT_TYPES, ids=lambda t: Q.NAMES[t])
def test_dots_bit_identical_to_reference_scalar(oracle, reference, wt):
    n_in, n_out = (768, 40) if wt != Q.F16 else (100, 20)
    if Q.GEOMETRY[wt][0] == 32:
        n_in = 96 * 7
    for seed in range(3):
        w = synth.weights(wt, n_out, n_in, seed=seed)
        x = synth.activations(n_in, 1, seed=seed + 50)[0] * (10.0 ** (seed - 1))
        xq = _pair(reference, wt, x)
        assert (oracle.quantize_pair(wt, x)[0] == xq).all()
        y_ref = reference.gemv_scalar(wt, w, n_in, n_out, xq)
        y = oracle.gemv(wt, w, n_in, n_out, xq)
        assert (y.view(np.uint32) == y_ref.view(np.uint32)).all()


def test_quantizers_bit_identical_to_reference(oracle, reference):
    rng = np.random.default_rng(7)
    for t in range(60):
        x = (rng.standard_normal(2048) * rng.choice([1e-6, 1e-2, 1, 1e3, 1e6])).astype(np.float32)
        if t % 5 == 0:
            x[rng.integers(0, 2048, 40)] = 0.0
        if t % 7 == 0:
            x[:256] = 0.0
        assert (oracle.quant_q8_K(x) == reference.quant_q8_K(x)).all()
        assert (oracle.quant_q8_0(x) == reference.quant_q8_0(x, "avx2")).all()


def test_nonfinite_inputs_match_reference(oracle, reference):
    rng = np.random.default_rng(8)
    x = rng.standard_normal(1024).astype(np.float32)
    x[5] = np.inf                                  # block 0: max is +inf
    x[300] = -np.inf                               # block 1: max is -inf
    x[600] = np.float32(np.nan)                    # block 2: a NaN among normals
    x[601:603] = np.array([0x7fc0007f, 0xffc12345], np.uint32).view(np.float32)  # payload NaNs
    assert (oracle.quant_q8_K(x) == reference.quant_q8_K(x)).all()
    assert (oracle.quant_q8_0(x) == reference.quant_q8_0(x, "avx2")).all()


@pytest.mark.parametrize("wt", Q.WEIGHT_TYPES, ids=lambda t: Q.NAMES[t])
def test_dequant_bit_identical_to_reference(oracle, reference, wt):
    n = 512
    w = synth.weights(wt, 3, n, seed=11)
    rb = row_bytes(wt, n)
    for r in range(3):
        a = oracle.dequant_row(wt, w[r * rb:(r + 1) * rb], n)
        b = reference.dequant_row(wt, w[r * rb:(r + 1) * rb], n)
        assert (a.view(np.uint32) == b.view(np.uint32)).all()


def test_f32_to_f16_random_patterns(oracle, reference):
    rng = np.random.default_rng(3)
    bits = rng.integers(0, 2 ** 32, 50000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    for v in bits:
        assert oracle.f32_to_f16(float(v)) == reference.lib.si_f32_to_f16(float(v))


def test_scalar_and_avx2_q8_0_forms_differ_rarely(oracle):
    """The reference's two Q8_0 quantizers (scalar kernels.c:542-558, AVX2
    kernels_avx2.c:594-645) disagree on a small fraction of N(0,1) blocks;
    the CUDA quantizer follows the AVX2 form that x86 hosts dispatch to."""
    rng = np.random.default_rng(0)
    x = rng.standard_normal(32 * 40000).astype(np.float32)
    a = oracle.quant_q8_0(x).reshape(-1, 34)
    b = oracle.quant_q8_0(x, scalar=True).reshape(-1, 34)
    frac = float((a != b).any(axis=1).mean())
    assert frac < 1e-3


def test_activation_steps_bit_identical_to_reference(oracle, reference):
    rng = np.random.default_rng(77)
    xs = np.concatenate([rng.standard_normal(3000) * 10, rng.uniform(-230, 230, 3000)]).astype(np.float32)
    for v in xs:
        v = float(v)
        assert np.float32(oracle.expf(v)).view(np.uint32) == np.float32(reference.expf(v)).view(np.uint32), v
        assert np.float32(oracle.silu(v)).view(np.uint32) == np.float32(reference.silu(v)).view(np.uint32), v
    for n in (256, 4096, 5120, 8192):
        for s in (1e-4, 1.0, 100.0):
            x = (rng.standard_normal(n) * s).astype(np.float32)
            for eps in (1e-5, 1e-6):
                a, b = np.float32(oracle.rms_scale(x, eps)), np.float32(reference.rms_scale(x, eps))
                assert a.view(np.uint32) == b.view(np.uint32)

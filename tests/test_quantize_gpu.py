"""Activation quantizers on the GPU, byte-for-byte against the oracle (which is
pinned to the reference: si_quant_row_q8_K and the AVX2 si_quant_row_q8_0)."""

from __future__ import annotations

import numpy as np
import pytest

from siphon_b200 import quant as Q
from tests.gpu_util import dev, empty_u8, host

pytestmark = pytest.mark.gpu


def _rows(n: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    rows = [rng.standard_normal(n) * s for s in (1.0, 1e-3, 37.0, 1e4, 1e-30, 1e30)]
    z = np.zeros(n); rows.append(z)
    tie = rng.standard_normal(n); tie[[3, 70, 200]] = 6.0; tie[[300, 301]] = [-6.0, 6.0]; rows.append(tie)
    half = rng.standard_normal(n); half[:256] = 0.0; rows.append(half)
    ints = np.round(rng.standard_normal(n) * 50); rows.append(ints)   # exact halves after scaling
    return np.stack(rows).astype(np.float32)


def test_q8_K_bytes_match(sicu, oracle):
    x = _rows(1024, 1)
    m, n = x.shape
    out = empty_u8(m * Q.row_bytes(Q.Q8_K, n))
    sicu.quantize_q8_K(dev(x), out, n, m)
    got = host(out).reshape(m, -1)
    for i in range(m):
        assert (got[i] == oracle.quant_q8_K(x[i])).all(), f"row {i}"


def test_q8_0_bytes_match_avx2_form(sicu, oracle):
    x = _rows(1024, 2)
    m, n = x.shape
    out = empty_u8(m * Q.row_bytes(Q.Q8_0, n))
    sicu.quantize_q8_0(dev(x), out, n, m)
    got = host(out).reshape(m, -1)
    for i in range(m):
        assert (got[i] == oracle.quant_q8_0(x[i])).all(), f"row {i}"


def test_f16_conversion_all_halves_and_random_bits(sicu, oracle):
    halves = np.arange(65536, dtype=np.uint16).view(np.float16).astype(np.float32)
    rng = np.random.default_rng(3)
    bits = rng.integers(0, 2 ** 32, 65536, dtype=np.uint64).astype(np.uint32).view(np.float32)
    x = np.concatenate([halves, bits]).astype(np.float32)
    out = empty_u8(2 * x.size)
    sicu.convert_f16(dev(x), out, x.size, 1)
    assert (host(out) == oracle.convert_f16(x)).all()


def test_nonfinite_inputs(sicu, oracle):
    rng = np.random.default_rng(4)
    x = rng.standard_normal(1024).astype(np.float32)
    x[5] = np.inf
    x[300] = -np.inf
    x[600] = np.float32(np.nan)
    x[601:603] = np.array([0x7fc0007f, 0xffc12345], np.uint32).view(np.float32)
    x[700] = np.inf; x[701] = np.float32(np.nan)
    for q, fn, ref in ((Q.Q8_K, sicu.quantize_q8_K, oracle.quant_q8_K), (Q.Q8_0, sicu.quantize_q8_0, oracle.quant_q8_0)):
        out = empty_u8(Q.row_bytes(q, 1024))
        fn(dev(x), out, 1024, 1)
        assert (host(out) == ref(x)).all(), Q.NAMES[q]


@pytest.mark.parametrize("wt", Q.WEIGHT_TYPES, ids=lambda t: Q.NAMES[t])
def test_quantize_pair_dispatch(sicu, oracle, wt):
    n = 4096
    x = np.random.default_rng(wt).standard_normal((3, n)).astype(np.float32)
    out = empty_u8(3 * Q.row_bytes(Q.pair_type(wt), n))
    sicu.quantize_pair(wt, dev(x), out, n, 3)
    assert (host(out).reshape(3, -1) == oracle.quantize_pair(wt, x)).all()

"""Batch decode matvec (sicu_gemv_batch): up to eight activation rows, every
weight block read once for all of them (Q4_K and Q6_K on the tensor cores),
bit-identical with the oracle's scalar dot products of the reference
(src/kernels.c:349-410 Q4_K, 480-523 Q6_K) applied row by row and token by
token, and with the per-row matvec. The north-star tolerance (1e-5 relative
per output) is asserted as well; bit equality is the stricter claim."""

from __future__ import annotations

import numpy as np
import pytest

from siphon_b200 import quant as Q
from siphon_b200 import synth
from tests.gpu_util import assert_bits_equal, assert_within_tol, dev, empty_f32, host

pytestmark = pytest.mark.gpu

BATCH_TYPES = (Q.Q4_K, Q.Q6_K)


def _check(sicu, oracle, wt, shapes, n_in, m, seed, xscale=1.0, patch=None):
    ws = [synth.weights(wt, n_out, n_in, seed=seed + i) for i, n_out in enumerate(shapes)]
    x = synth.activations(n_in, m, seed=seed + 50) * np.float32(xscale)
    if patch:
        ws, x = patch(ws, x)
    xq = oracle.quantize_pair(wt, x)
    ys = [empty_f32(m, n_out) for n_out in shapes]
    sicu.gemv_batch(wt, [dev(w) for w in ws], list(shapes), n_in, dev(x), m, ys)
    for i, (w, n_out) in enumerate(zip(ws, shapes)):
        want = oracle.gemv_batch(wt, w, n_in, n_out, xq)
        got = host(ys[i])
        what = f"{Q.NAMES[wt]} batch m={m} mat {i} {n_out}x{n_in}"
        assert_bits_equal(got, want, what)
        assert_within_tol(got, want, what)
    assert sicu.status() == 0


@pytest.mark.parametrize("wt", BATCH_TYPES, ids=lambda t: Q.NAMES[t])
@pytest.mark.parametrize("n_out,n_in,m", [
    (16, 256, 8),        # one tile, one super-block (a single-super-block stage)
    (37, 512, 3),        # ragged rows, three tokens
    (5, 768, 2),         # fewer rows than a tile; three super-blocks (odd stage count;
                         # Q6_K rows 2-byte aligned)
    (1000, 4096, 8),     # many tiles
    (264, 5120, 7),      # 20 super-blocks (the 32B model width)
    (300, 14336, 8),     # long rows: the ring wraps many times
])
def test_batch_matches_reference(sicu, oracle, wt, n_out, n_in, m):
    _check(sicu, oracle, wt, (n_out,), n_in, m, seed=n_out + n_in + m)


@pytest.mark.parametrize("wt", BATCH_TYPES, ids=lambda t: Q.NAMES[t])
def test_batch_multi_matrix(sicu, oracle, wt):
    """Wq / Wk / Wv-like launch: three matrices sharing the activation rows."""
    _check(sicu, oracle, wt, (512, 128, 130), 2048, 8, seed=3)


@pytest.mark.slow
@pytest.mark.parametrize("wt", BATCH_TYPES, ids=lambda t: Q.NAMES[t])
def test_batch_full_size(sicu, oracle, wt):
    """A 32B-class W_down shape (5120 x 27648, 108 super-blocks) with eight tokens."""
    _check(sicu, oracle, wt, (5120,), 27648, 8, seed=11)


@pytest.mark.parametrize("wt", BATCH_TYPES, ids=lambda t: Q.NAMES[t])
@pytest.mark.parametrize("xscale", [1e-20, 1e20], ids=["tiny", "huge"])
def test_batch_activation_scales(sicu, oracle, wt, xscale):
    _check(sicu, oracle, wt, (96,), 1024, 8, seed=5, xscale=xscale)


@pytest.mark.parametrize("wt", BATCH_TYPES, ids=lambda t: Q.NAMES[t])
def test_batch_zero_rows_and_zero_scales(sicu, oracle, wt):
    """An all-zero activation row, an all-zero block of another, and weight
    blocks whose f16 scales are zero."""
    bsz = Q.GEOMETRY[wt][1]

    def patch(ws, x):
        x = x.copy()
        x[1, :] = 0.0
        x[4, 256:512] = 0.0
        w = ws[0].copy().reshape(-1, bsz)
        if wt == Q.Q4_K:
            w[::3, 0:2] = 0          # d = 0
            w[1::5, 2:4] = 0         # dmin = 0
        else:
            w[::3, 208:210] = 0      # d = 0
        return [w.reshape(-1)], x
    _check(sicu, oracle, wt, (80,), 1024, 6, seed=8, patch=patch)


@pytest.mark.parametrize("wt", (Q.Q8_0, Q.F16, Q.Q5_K), ids=lambda t: Q.NAMES[t])
def test_batch_other_types_per_row(sicu, oracle, wt):
    """Types without the tensor-core batch kernel run the matvec per row."""
    _check(sicu, oracle, wt, (70, 33), 1024, 4, seed=2)


@pytest.mark.parametrize("wt", BATCH_TYPES, ids=lambda t: Q.NAMES[t])
def test_batch_one_row(sicu, oracle, wt):
    _check(sicu, oracle, wt, (200,), 2048, 1, seed=4)


@pytest.mark.parametrize("wt", BATCH_TYPES, ids=lambda t: Q.NAMES[t])
def test_prefill_few_tokens_bit_exact(sicu, oracle, wt):
    """sicu_gemm_prefill / _f32 with m <= 8 tokens take the batch kernel:
    bit-identical with the reference per token (the larger-m tensor-core path
    is held to 1e-5 of the L1 norm instead)."""
    n_out, n_in, m = 300, 4096, 8
    w = synth.weights(wt, n_out, n_in, seed=21)
    x = synth.activations(n_in, m, seed=22)
    xq = oracle.quantize_pair(wt, x)
    want = oracle.gemv_batch(wt, w, n_in, n_out, xq)
    y = empty_f32(m, n_out)
    sicu.gemm_prefill(wt, dev(w), n_in, n_out, dev(xq), m, y)
    assert_bits_equal(host(y), want, "prefill from Q8_K rows, 8 tokens")
    y2 = empty_f32(m, n_out)
    sicu.gemm_prefill_f32(wt, dev(w), n_in, n_out, dev(x), m, y2)
    assert_bits_equal(host(y2), want, "prefill from f32 rows, 8 tokens")


def test_batch_rejects_bad_arguments(sicu):
    from siphon_b200.lib import SicuError
    w = empty_f32(1000)
    x = empty_f32(9, 256)
    y = empty_f32(9, 16)
    with pytest.raises(SicuError):
        sicu.gemv_batch(Q.Q4_K, [w], [16], 256, x, 9, [y])          # more than 8 rows
    with pytest.raises(SicuError):
        sicu.gemv_batch(Q.Q4_K, [w] * 17, [16] * 17, 256, x, 2, [y] * 17)   # more than 16 matrices
    with pytest.raises(SicuError):
        sicu.gemv_batch(Q.Q4_K, [w], [16], 300, x, 2, [y])          # row length not whole super-blocks

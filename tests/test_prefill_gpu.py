"""Prefill product (sicu_gemm_prefill) against the oracle's scalar per-row
dots of the reference (src/kernels.c:349-410 for Q4_K).

The tensor-core path computes each super-block's integer sums exactly and
scales them in a different order from the reference's eight lane sums, so it
is held to a tolerance, stated here:

    |y - y_ref| <= PREFILL_TOL * L1,   L1 = sum_k |w_k| * |x_k|

with w the dequantized weight row and x the dequantized Q8_K activation row
(the products the dot adds up). Types without a tensor-core kernel run the
decode matvec per token and must match bit for bit.
"""

from __future__ import annotations

import numpy as np
import pytest

from siphon_b200 import quant as Q
from siphon_b200 import synth
from tests.gpu_util import assert_bits_equal, dev, empty_f32, host

pytestmark = pytest.mark.gpu

PREFILL_TOL = 1e-5


def _dequant_q8k(xq: np.ndarray, n_in: int) -> np.ndarray:
    """[m, n_in] float64 values d * q of Q8_K rows."""
    blk = np.ascontiguousarray(xq).reshape(-1, n_in // 256, 292)
    d = blk[:, :, 0:4].copy().view(np.float32)[..., 0].astype(np.float64)
    q = blk[:, :, 4:260].view(np.int8).astype(np.float64)
    return (q * d[..., None]).reshape(-1, n_in)


def _dequant_w(oracle, wt, w, n_in, n_out) -> np.ndarray:
    rb = Q.row_bytes(wt, n_in)
    return np.stack([oracle.dequant_row(wt, w[r * rb:(r + 1) * rb], n_in) for r in range(n_out)]).astype(np.float64)


def _check_tol(got, want, l1, what):
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    bound = PREFILL_TOL * l1
    bad = ~(err <= bound)
    assert not bad.any(), (f"{what}: {bad.sum()}/{bad.size} outputs beyond {PREFILL_TOL} * L1; "
                           f"worst err/L1 {np.max(err / np.maximum(l1, 1e-300)):.3g}")


def _run(sicu, oracle, wt, n_out, n_in, m, seed=0, xscale=1.0, patch=None):
    w = synth.weights(wt, n_out, n_in, seed=seed)
    x = synth.activations(n_in, m, seed=seed + 1) * np.float32(xscale)
    if patch:
        w, x = patch(w, x)
    xq = oracle.quantize_pair(wt, x)
    want = oracle.gemv_batch(wt, w, n_in, n_out, xq)
    y = empty_f32(m, n_out)
    sicu.gemm_prefill(wt, dev(w), n_in, n_out, dev(xq), m, y)
    got = host(y)
    return w, x, xq, want, got


@pytest.mark.parametrize("n_out,n_in,m", [
    (128, 256, 128),     # one tile, one super-block
    (256, 1024, 128),    # two row tiles
    (200, 512, 77),      # ragged rows and tokens
    (128, 2048, 300),    # three token tiles, the last one partial
    (384, 4096, 64),     # long rows: the pipeline wraps many times
])
def test_prefill_q4k_vs_reference(sicu, oracle, n_out, n_in, m):
    wt = Q.Q4_K
    w, x, xq, want, got = _run(sicu, oracle, wt, n_out, n_in, m, seed=n_out + n_in + m)
    l1 = np.abs(_dequant_q8k(xq, n_in)) @ np.abs(_dequant_w(oracle, wt, w, n_in, n_out)).T
    _check_tol(got, want, l1, f"Q4_K prefill {n_out}x{n_in} m={m}")
    assert np.isfinite(got).all()


@pytest.mark.parametrize("n_out,n_in,m", [
    (128, 256, 128),     # one super-block, one tile
    (256, 2048, 128),    # rows of 8 super-blocks: 16-byte multiple, no padding copy
    (200, 1280, 77),     # 5 super-blocks per row: rows padded to 16 bytes first
    (130, 5632, 140),    # 22 super-blocks, ragged rows and tokens
])
def test_prefill_q6k_vs_reference(sicu, oracle, n_out, n_in, m):
    wt = Q.Q6_K
    w, x, xq, want, got = _run(sicu, oracle, wt, n_out, n_in, m, seed=n_out + 3 * n_in + m)
    l1 = np.abs(_dequant_q8k(xq, n_in)) @ np.abs(_dequant_w(oracle, wt, w, n_in, n_out)).T
    _check_tol(got, want, l1, f"Q6_K prefill {n_out}x{n_in} m={m}")
    assert np.isfinite(got).all()


@pytest.mark.parametrize("wt", [Q.Q4_K, Q.Q6_K])
@pytest.mark.parametrize("n_out,n_in,m", [
    (128, 512, 1),       # one token: a 32-token tile with 31 padding tokens
    (200, 1024, 8),      # a batched-decode block
    (256, 2048, 32),     # a full 32-token tile
    (130, 1280, 20),     # ragged rows; Q6_K rows padded to 16 bytes
])
def test_prefill_small_token_blocks(sicu, oracle, wt, n_out, n_in, m):
    """Blocks of <= 32 tokens take the 32-token tile variant of the kernel."""
    w, x, xq, want, got = _run(sicu, oracle, wt, n_out, n_in, m, seed=n_out + m)
    l1 = np.abs(_dequant_q8k(xq, n_in)) @ np.abs(_dequant_w(oracle, wt, w, n_in, n_out)).T
    _check_tol(got, want, l1, f"{Q.NAMES[wt]} prefill {n_out}x{n_in} m={m}")


def test_prefill_q4k_exact_value(sicu, oracle):
    """Against the exact value of the product (float64 over the dequantized
    operands) at a larger size, where the scalar oracle would be slow."""
    wt, n_out, n_in, m = Q.Q4_K, 1024, 4096, 256
    w = synth.weights(wt, n_out, n_in, seed=7)
    x = synth.activations(n_in, m, seed=8)
    xq = oracle.quantize_pair(wt, x)
    xd = _dequant_q8k(xq, n_in)
    wd = _dequant_w(oracle, wt, w, n_in, n_out)
    exact = xd @ wd.T
    l1 = np.abs(xd) @ np.abs(wd).T
    y = empty_f32(m, n_out)
    sicu.gemm_prefill(wt, dev(w), n_in, n_out, dev(xq), m, y)
    _check_tol(host(y), exact, l1, "Q4_K prefill vs exact")


def test_prefill_q4k_edge_rows(sicu, oracle):
    """Zero activation rows (d = 0), weight blocks with d = 0 or dmin = 0, and
    large activations."""
    wt, n_out, n_in, m = Q.Q4_K, 160, 768, 96

    def patch(w, x):
        w = w.copy()
        blocks = w.reshape(-1, 144)
        blocks[::5, 0:2] = 0            # d = 0
        blocks[1::7, 2:4] = 0           # dmin = 0
        x = x.copy()
        x[3] = 0.0
        x[10] *= 1e4
        return w, x

    w, x, xq, want, got = _run(sicu, oracle, wt, n_out, n_in, m, seed=3, patch=patch)
    l1 = np.abs(_dequant_q8k(xq, n_in)) @ np.abs(_dequant_w(oracle, wt, w, n_in, n_out)).T
    _check_tol(got, want, l1, "Q4_K prefill edge rows")
    assert (got[3] == 0).all()


@pytest.mark.parametrize("wt,n_out,n_in,m,packed", [
    (Q.Q4_K, 256, 1024, 100, False),    # converter kernel
    (Q.Q6_K, 200, 1280, 50, False),
    (Q.Q4_K, 128, 512, 40, True),       # one row tile: one-CTA kernel from the copy
    (Q.Q4_K, 640, 2048, 300, True),     # CTA pairs, 256-token tiles
    (Q.Q6_K, 384, 1280, 77, True),      # CTA pairs, two planes per quarter
])
def test_prefill_f32_entry_matches_quantized(sicu, oracle, wt, n_out, n_in, m, packed):
    """The f32 entries quantize inside the launch, straight into the token
    operand: the same bits as quantizing with the reference's quantizer first
    (zero rows and very large rows included)."""
    w = synth.weights(wt, n_out, n_in, seed=11)
    x = synth.activations(n_in, m, seed=12)
    x[1] = 0.0
    x[2] *= 3e4
    xq = oracle.quantize_pair(wt, x)
    dw = dev(w)
    dp = None
    if packed:
        import torch
        nb = sicu.prefill_pack_bytes(wt, n_in, n_out)
        dp = torch.zeros(nb, dtype=torch.uint8, device="cuda")
        sicu.prefill_pack(wt, dw, n_in, n_out, dp, nb)
    y1 = empty_f32(m, n_out)
    sicu.gemm_prefill_packed(wt, dw, dp, n_in, n_out, dev(xq), m, y1)
    y2 = empty_f32(m, n_out)
    sicu.gemm_prefill_packed_f32(wt, dw, dp, n_in, n_out, dev(x), m, y2)
    assert_bits_equal(host(y2), host(y1), "prefill f32 entry vs pre-quantized")


@pytest.mark.parametrize("wt", [Q.Q8_0, Q.Q5_K, Q.F16])
def test_prefill_other_types_bit_exact(sicu, oracle, wt):
    """Types without a tensor-core kernel: the decode matvec per token."""
    n_out, n_in, m = 96, 512, 5
    w = synth.weights(wt, n_out, n_in, seed=21)
    x = synth.activations(n_in, m, seed=22)
    xq = oracle.quantize_pair(wt, x)
    want = oracle.gemv_batch(wt, w, n_in, n_out, xq)
    y = empty_f32(m, n_out)
    sicu.gemm_prefill_f32(wt, dev(w), n_in, n_out, dev(x), m, y)
    assert_bits_equal(host(y), want, f"{Q.NAMES[wt]} prefill fallback")


def test_prefill_empty_and_errors(sicu):
    import torch
    from siphon_b200.lib import SicuError
    w = dev(synth.weights(Q.Q4_K, 128, 256, seed=1))
    x = torch.zeros(256, dtype=torch.float32, device="cuda")
    y = empty_f32(1, 128)
    sicu.gemm_prefill_f32(Q.Q4_K, w, 256, 128, x, 0, y)       # m = 0: nothing
    sicu.gemm_prefill_f32(Q.Q4_K, w, 256, 0, x, 1, y)         # no rows: nothing
    with pytest.raises(SicuError):
        sicu.gemm_prefill_f32(Q.Q4_K, w, 200, 128, x, 1, y)   # not a multiple of 256
    with pytest.raises(SicuError):
        sicu.gemm_prefill_f32(Q.Q4_K, w, 256, 128, x, 70000, y)
    assert sicu.status() == 0


@pytest.mark.parametrize("wt,n_out,n_in,m", [
    (Q.Q4_K, 256, 8192, 8),      # two row tiles, 32 super-blocks: the row split into ranges
    (Q.Q6_K, 200, 5632, 5),      # 22 super-blocks, ragged rows, padded Q6_K rows
    (Q.Q4_K, 640, 4096, 300),    # prompt tiles with the split
])
def test_prefill_split_rows(sicu, oracle, wt, n_out, n_in, m):
    """Launches with few tiles split each row's super-blocks across CTAs and
    add the partial products afterwards: within the tolerance, and the same
    bits on every run (the partials are added in a fixed order)."""
    w, x, xq, want, got = _run(sicu, oracle, wt, n_out, n_in, m, seed=n_in + m)
    l1 = np.abs(_dequant_q8k(xq, n_in)) @ np.abs(_dequant_w(oracle, wt, w, n_in, n_out)).T
    _check_tol(got, want, l1, f"{Q.NAMES[wt]} prefill {n_out}x{n_in} m={m} (split)")
    y2 = empty_f32(m, n_out)
    sicu.gemm_prefill(wt, dev(w), n_in, n_out, dev(xq), m, y2)
    assert_bits_equal(host(y2), got, "second run")

"""Prefill from the re-tiled weight copy (sicu_prefill_pack,
sicu_gemm_prefill_packed) against the oracle's scalar per-row dots of the
reference (src/kernels.c:349-410 for Q4_K, 480-523 for Q6_K, 412-478 for
Q5_K, 289-347 for Q3_K, 249-287 for Q2_K).

The copy holds, per 128-row tile and super-block, the exact f16 operands the
tensor cores multiply, so two things are checked: the copy itself (decoded
here from its documented layout, it must give back the reference's
dequantized weights, src/kernels.c:603-801) and the products made from it,
held to the prefill tolerance

    |y - y_ref| <= PREFILL_TOL * L1,   L1 = sum_k |w_k| * |x_k|.
"""

from __future__ import annotations

import numpy as np
import pytest

from siphon_b200 import quant as Q
from siphon_b200 import synth
from tests.gpu_util import assert_bits_equal, dev, empty_f32, host
from tests.test_prefill_gpu import PREFILL_TOL, _check_tol, _dequant_q8k, _dequant_w

pytestmark = pytest.mark.gpu

ATILE = 128 * 64 * 2         # one K-step of a 128-row tile
MINT = 128 * 16 * 2          # one half of the Q4_K mins operand
KSTEPS = {Q.Q4_K: 4, Q.Q6_K: 8, Q.Q5_K: 4, Q.Q3_K: 4, Q.Q2_K: 4}
MINS = (Q.Q4_K, Q.Q5_K, Q.Q2_K)        # formats with a mins operand
K_TYPES = (Q.Q4_K, Q.Q5_K, Q.Q6_K, Q.Q3_K, Q.Q2_K)
COPY_ONLY = (Q.Q5_K, Q.Q3_K, Q.Q2_K)   # tensor-core kernels only from a prefill copy
SLOT = np.array([0, 2, 1, 3])
# byte offsets of d and dmin in a block, for the edge-row patches
D_OFF = {Q.Q4_K: (0, 2), Q.Q5_K: (0, 2), Q.Q2_K: (80, 82), Q.Q3_K: (108, None)}


def _zero_scales(wt, w, every_d=9, every_dmin=11):
    """Some blocks with d = 0 and (K formats with mins) some with dmin = 0."""
    w = w.copy()
    blocks = w.reshape(-1, Q.row_bytes(wt, 256))
    od, om = D_OFF[wt]
    blocks[::every_d, od:od + 2] = 0
    if om is not None:
        blocks[4::every_dmin, om:om + 2] = 0
    return w


def _pack(sicu, wt, w, n_in, n_out):
    import torch
    nbytes = sicu.prefill_pack_bytes(wt, n_in, n_out)
    dw = dev(w)
    dp = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    sicu.prefill_pack(wt, dw, n_in, n_out, dp, nbytes)
    return dw, dp, nbytes


def _unswizzle(tile: np.ndarray, row_bytes: int, mask_of_row) -> np.ndarray:
    """[rows, row_bytes] bytes of a swizzled K-major tile back in k order."""
    rows = tile.reshape(-1, row_bytes // 16, 16)
    out = np.empty_like(rows)
    for r in range(rows.shape[0]):
        for p in range(rows.shape[1]):
            out[r, p ^ mask_of_row(r)] = rows[r, p]
    return out.reshape(-1, row_bytes)


def _decode_pack(wt, pack: np.ndarray, n_in: int, n_out: int) -> np.ndarray:
    """The weights a packed copy stands for: [n_out, n_in] float64."""
    nsb, nrt = n_in // 256, (n_out + 127) // 128
    kst = KSTEPS[wt]
    chunk = kst * ATILE + (2 * MINT if wt in MINS else 0) + 512
    assert pack.size == nrt * nsb * chunk
    out = np.zeros((nrt * 128, n_in))
    for rt in range(nrt):
        for sb in range(nsb):
            c = pack[(rt * nsb + sb) * chunk:(rt * nsb + sb + 1) * chunk]
            f = c[kst * ATILE + (2 * MINT if wt in MINS else 0):].view(np.float32).astype(np.float64)
            # A tiles: 64 f16 per row, 16-byte unit j of row r at j ^ (r & 7)
            a = [_unswizzle(c[t * ATILE:(t + 1) * ATILE], 128, lambda r: r & 7).view(np.float16)
                 .astype(np.float64) for t in range(kst)]
            vals = np.zeros((128, 256))
            for t in range(kst):
                # slot s holds element 4 (s // 4) + (0, 2, 1, 3)[s % 4] of its 64
                e = 4 * (np.arange(64) // 4) + SLOT[np.arange(64) % 4]
                if wt != Q.Q6_K:    # one plane: sc q 2^-s
                    vals[:, 64 * t + e] = a[t]
                else:   # two planes per quarter: (q - 32) lo + 16 (q - 32) hi
                    vals[:, 64 * (t // 2) + e] += a[t] * (16.0 if t % 2 else 1.0)
            vals *= f[:, None]
            if wt in MINS:
                mins = [_unswizzle(c[kst * ATILE + h * MINT:kst * ATILE + (h + 1) * MINT], 32,
                                   lambda r: (r >> 2) & 1).view(np.float16).astype(np.float64) for h in range(2)]
                mterm = (mins[0] + mins[1]) * f[:, None]          # [128, 16]: per 16 elements
                vals += np.repeat(mterm, 16, axis=1)
            out[rt * 128:(rt + 1) * 128, 256 * sb:256 * (sb + 1)] = vals
    return out[:n_out]


@pytest.mark.parametrize("wt,n_out,n_in", [
    (Q.Q4_K, 200, 768),
    (Q.Q6_K, 130, 1280),    # 5 super-blocks: rows that are not 16-byte multiples
    (Q.Q5_K, 200, 768),
    (Q.Q3_K, 130, 1280),    # 110-byte blocks at even offsets
    (Q.Q2_K, 130, 1280),    # 84-byte blocks
])
def test_pack_layout_gives_back_the_weights(sicu, oracle, wt, n_out, n_in):
    """Decoded from its layout, the copy is the reference's dequantized
    weights: exactly d sc q for the main term (f16 sc q 2^-s times f = d 2^s),
    and the mins term (Q4_K, Q5_K, Q2_K) to the 22 bits of its hi + lo
    split."""
    w = synth.weights(wt, n_out, n_in, seed=5)
    if wt in D_OFF:   # a few blocks with d = 0 or dmin = 0
        w = _zero_scales(wt, w)
    _, dp, _ = _pack(sicu, wt, w, n_in, n_out)
    got = _decode_pack(wt, host(dp), n_in, n_out)
    want = _dequant_w(oracle, wt, w, n_in, n_out)
    scale = np.abs(want).max()
    err = np.abs(got - want)
    assert err.max() <= 2e-6 * scale, f"max err {err.max():.3g} of {scale:.3g}"
    if wt in (Q.Q6_K, Q.Q3_K):   # d sc q exactly, no mins (zero products may differ in sign)
        assert np.array_equal(got.astype(np.float32), want.astype(np.float32)), f"{Q.NAMES[wt]} copy"
    # the rows past n_out in the last tile are zero
    nrt, nsb = (n_out + 127) // 128, n_in // 256
    assert nrt * 128 > n_out


def _run_packed(sicu, oracle, wt, n_out, n_in, m, seed=0, patch=None, f32=False):
    w = synth.weights(wt, n_out, n_in, seed=seed)
    x = synth.activations(n_in, m, seed=seed + 1)
    if patch:
        w, x = patch(w, x)
    xq = oracle.quantize_pair(wt, x)
    dw, dp, _ = _pack(sicu, wt, w, n_in, n_out)
    y = empty_f32(m, n_out)
    if f32:
        sicu.gemm_prefill_packed_f32(wt, dw, dp, n_in, n_out, dev(x), m, y)
    else:
        sicu.gemm_prefill_packed(wt, dw, dp, n_in, n_out, dev(xq), m, y)
    return w, x, xq, dw, dp, host(y)


@pytest.mark.parametrize("wt", K_TYPES, ids=lambda t: Q.NAMES[t])
@pytest.mark.parametrize("n_out,n_in,m", [
    (128, 256, 128),     # one tile, one super-block, 128-token tile
    (200, 512, 77),      # ragged rows and tokens
    (256, 1024, 300),    # 256-token tiles, the second one partial
    (130, 1280, 140),    # 5 super-blocks (Q6_K rows not 16-byte multiples)
    (384, 4096, 64),     # long rows: the stage ring wraps many times
    (128, 2048, 513),    # three 256-token tiles
])
def test_packed_prefill_vs_reference(sicu, oracle, wt, n_out, n_in, m):
    w, x, xq, dw, dp, got = _run_packed(sicu, oracle, wt, n_out, n_in, m, seed=n_out + n_in + m)
    want = oracle.gemv_batch(wt, w, n_in, n_out, xq)
    l1 = np.abs(_dequant_q8k(xq, n_in)) @ np.abs(_dequant_w(oracle, wt, w, n_in, n_out)).T
    _check_tol(got, want, l1, f"{Q.NAMES[wt]} packed prefill {n_out}x{n_in} m={m}")
    assert np.isfinite(got).all()


def test_packed_prefill_exact_value(sicu, oracle):
    """Against the exact value of the product (float64 over the dequantized
    operands) at a larger size, through the f32 entry."""
    wt, n_out, n_in, m = Q.Q4_K, 1024, 4096, 512
    w = synth.weights(wt, n_out, n_in, seed=7)
    x = synth.activations(n_in, m, seed=8)
    xq = oracle.quantize_pair(wt, x)
    xd = _dequant_q8k(xq, n_in)
    wd = _dequant_w(oracle, wt, w, n_in, n_out)
    dw, dp, _ = _pack(sicu, wt, w, n_in, n_out)
    y = empty_f32(m, n_out)
    sicu.gemm_prefill_packed_f32(wt, dw, dp, n_in, n_out, dev(x), m, y)
    _check_tol(host(y), xd @ wd.T, np.abs(xd) @ np.abs(wd).T, "Q4_K packed prefill vs exact")


def test_packed_prefill_edge_rows(sicu, oracle):
    """Zero activation rows, weight blocks with d = 0 or dmin = 0, large
    activations."""
    wt, n_out, n_in, m = Q.Q4_K, 160, 768, 96

    def patch(w, x):
        w = w.copy()
        blocks = w.reshape(-1, 144)
        blocks[::5, 0:2] = 0
        blocks[1::7, 2:4] = 0
        x = x.copy()
        x[3] = 0.0
        x[10] *= 1e4
        return w, x

    w, x, xq, dw, dp, got = _run_packed(sicu, oracle, wt, n_out, n_in, m, seed=3, patch=patch)
    want = oracle.gemv_batch(wt, w, n_in, n_out, xq)
    l1 = np.abs(_dequant_q8k(xq, n_in)) @ np.abs(_dequant_w(oracle, wt, w, n_in, n_out)).T
    _check_tol(got, want, l1, "Q4_K packed prefill edge rows")
    assert (got[3] == 0).all()


@pytest.mark.parametrize("wt,n_out,n_in,m", [
    (Q.Q4_K, 640, 4096, 300),    # few tiles: each row's super-blocks split over CTAs
    (Q.Q6_K, 256, 5632, 200),
    (Q.Q5_K, 640, 4096, 300),
    (Q.Q3_K, 256, 5632, 200),
    (Q.Q2_K, 640, 4096, 130),
])
def test_packed_prefill_split_rows_repeatable(sicu, oracle, wt, n_out, n_in, m):
    w, x, xq, dw, dp, got = _run_packed(sicu, oracle, wt, n_out, n_in, m, seed=n_in + m)
    want = oracle.gemv_batch(wt, w, n_in, n_out, xq)
    l1 = np.abs(_dequant_q8k(xq, n_in)) @ np.abs(_dequant_w(oracle, wt, w, n_in, n_out)).T
    _check_tol(got, want, l1, f"{Q.NAMES[wt]} packed prefill {n_out}x{n_in} m={m} (split)")
    y2 = empty_f32(m, n_out)
    sicu.gemm_prefill_packed(wt, dw, dp, n_in, n_out, dev(xq), m, y2)
    assert_bits_equal(host(y2), got, "second run")


@pytest.mark.parametrize("m", [1, 8, 32])
def test_packed_small_blocks_use_raw_weights(sicu, oracle, m):
    """Blocks of <= 32 tokens read the raw blocks as before: the same bits as
    sicu_gemm_prefill."""
    wt, n_out, n_in = Q.Q4_K, 200, 1024
    w, x, xq, dw, dp, got = _run_packed(sicu, oracle, wt, n_out, n_in, m, seed=m)
    y = empty_f32(m, n_out)
    sicu.gemm_prefill(wt, dw, n_in, n_out, dev(xq), m, y)
    assert_bits_equal(got, host(y), f"m={m} with and without the copy")


def test_packed_null_copy_is_the_plain_product(sicu, oracle):
    wt, n_out, n_in, m = Q.Q6_K, 128, 512, 100
    w = synth.weights(wt, n_out, n_in, seed=9)
    x = synth.activations(n_in, m, seed=10)
    dw = dev(w)
    y1, y2 = empty_f32(m, n_out), empty_f32(m, n_out)
    sicu.gemm_prefill_f32(wt, dw, n_in, n_out, dev(x), m, y1)
    sicu.gemm_prefill_packed_f32(wt, dw, None, n_in, n_out, dev(x), m, y2)
    assert_bits_equal(host(y2), host(y1), "null copy")


def test_pack_errors(sicu):
    import torch
    from siphon_b200.lib import SicuError
    w = dev(synth.weights(Q.Q4_K, 128, 256, seed=1))
    n = sicu.prefill_pack_bytes(Q.Q4_K, 256, 128)
    p = torch.zeros(n, dtype=torch.uint8, device="cuda")
    with pytest.raises(SicuError):
        sicu.prefill_pack(Q.Q4_K, w, 256, 128, p, n - 16)          # too small
    with pytest.raises(SicuError):
        sicu.prefill_pack(Q.F32, w, 256, 128, p, n)                # no prefill copy
    with pytest.raises(SicuError):
        sicu.prefill_pack(Q.Q4_K, w, 200, 128, p, n)               # not whole super-blocks
    x = torch.zeros(256, dtype=torch.float32, device="cuda")
    y = empty_f32(64, 128)
    with pytest.raises(SicuError):
        sicu.gemm_prefill_packed_f32(Q.Q4_K, w, p[1:], 256, 128, x, 64, y)   # misaligned copy
    sicu.prefill_pack(Q.Q4_K, w, 256, 0, p, n)                     # no rows: nothing
    assert sicu.status() == 0


@pytest.mark.parametrize("wt,n_outs,n_in,m", [
    (Q.Q5_K, (640, 128), 1024, 300),
    (Q.Q3_K, (200, 130), 1280, 64),
    (Q.Q2_K, (256, 384, 128), 512, 77),
    (Q.Q2_K, (300, 100), 768, 20),           # at most 32 tokens, a copy-only format: the matvec per token
    (Q.Q4_K, (640, 128, 128), 1024, 300),    # Wq/Wk/Wv-like: one-tile matrices leave half a pair idle
    (Q.Q4_K, (1024, 1024), 4096, 512),       # W_gate/W_up-like
    (Q.Q6_K, (256, 384), 1280, 77),          # 5 super-blocks, 128-token tiles
    (Q.Q4_K, (200, 0, 130), 512, 64),        # a matrix without rows: the products one by one
    (Q.Q4_K, (300, 100), 768, 20),           # at most 32 tokens: the raw blocks
    (Q.Q6_K, (130, 260, 128, 64), 512, 6),   # a batch of decode steps: one batch launch
])
def test_packed_prefill_multi_vs_reference(sicu, oracle, wt, n_outs, n_in, m):
    """sicu_gemm_prefill_multi_f32: several matrices on one activation, each
    product within the prefill tolerance of the oracle's per-row dots, and
    the same bits on a second call."""
    x = synth.activations(n_in, m, seed=m + n_in)
    xq = oracle.quantize_pair(wt, x)
    ws, dws, dps, ys = [], [], [], []
    for i, n_out in enumerate(n_outs):
        w = synth.weights(wt, n_out, n_in, seed=10 * i + n_out + 1) if n_out else np.zeros(0, np.uint8)
        ws.append(w)
        if n_out:
            dw, dp, _ = _pack(sicu, wt, w, n_in, n_out)
        else:
            import torch
            dw = dp = torch.zeros(16, dtype=torch.uint8, device="cuda")
        dws.append(dw)
        dps.append(dp)
        ys.append(empty_f32(m, max(n_out, 1)))
    dx = dev(x)
    sicu.gemm_prefill_multi_f32(wt, dws, dps, list(n_outs), n_in, dx, m, ys)
    first = [host(y) for y in ys]
    sicu.gemm_prefill_multi_f32(wt, dws, dps, list(n_outs), n_in, dx, m, ys)
    xd = _dequant_q8k(xq, n_in)
    for i, n_out in enumerate(n_outs):
        if not n_out:
            continue
        got = host(ys[i])
        assert_bits_equal(got, first[i], f"matrix {i} second call")
        want = oracle.gemv_batch(wt, ws[i], n_in, n_out, xq)
        l1 = np.abs(xd) @ np.abs(_dequant_w(oracle, wt, ws[i], n_in, n_out)).T
        _check_tol(got, want, l1, f"{Q.NAMES[wt]} multi prefill matrix {i} {n_out}x{n_in} m={m}")
        assert np.isfinite(got).all()
    assert sicu.status() == 0


def test_packed_prefill_multi_without_copies(sicu, oracle):
    """No prefill copies: the products one by one from the raw blocks, the
    same bits as single sicu_gemm_prefill_f32 calls."""
    wt, n_outs, n_in, m = Q.Q4_K, (256, 128), 1024, 96
    x = dev(synth.activations(n_in, m, seed=2))
    ws = [dev(synth.weights(wt, n, n_in, seed=n)) for n in n_outs]
    ys = [empty_f32(m, n) for n in n_outs]
    sicu.gemm_prefill_multi_f32(wt, ws, None, list(n_outs), n_in, x, m, ys)
    for w, n, y in zip(ws, n_outs, ys):
        one = empty_f32(m, n)
        sicu.gemm_prefill_f32(wt, w, n_in, n, x, m, one)
        assert_bits_equal(host(y), host(one), f"{n} rows without copies")


def test_packed_prefill_many_pair_tiles(sicu, oracle):
    """More 256-row x 256-token tiles than two waves of CTA pairs hold (150
    on a 148-SM part), ragged tokens. Against the exact product, and the same
    bits on a second call."""
    wt, n_out, n_in, m = Q.Q4_K, 19200, 512, 300
    w = synth.weights(wt, n_out, n_in, seed=21)
    x = synth.activations(n_in, m, seed=22)
    xq = oracle.quantize_pair(wt, x)
    xd = _dequant_q8k(xq, n_in)
    wd = _dequant_w(oracle, wt, w, n_in, n_out)
    dw, dp, _ = _pack(sicu, wt, w, n_in, n_out)
    y = empty_f32(m, n_out)
    sicu.gemm_prefill_packed_f32(wt, dw, dp, n_in, n_out, dev(x), m, y)
    got = host(y)
    _check_tol(got, xd @ wd.T, np.abs(xd) @ np.abs(wd).T, "Q4_K packed prefill, 150 pair tiles")
    y2 = empty_f32(m, n_out)
    sicu.gemm_prefill_packed_f32(wt, dw, dp, n_in, n_out, dev(x), m, y2)
    assert_bits_equal(host(y2), got, "second run")


@pytest.mark.parametrize("wt", COPY_ONLY, ids=lambda t: Q.NAMES[t])
def test_packed_prefill_edge_rows_copy_only(sicu, oracle, wt):
    """Q5_K / Q3_K / Q2_K: blocks with d = 0 or dmin = 0, zero and large
    activation rows."""
    n_out, n_in, m = 260, 768, 96

    def patch(w, x):
        w = _zero_scales(wt, w, 5, 7)
        x = x.copy()
        x[3] = 0.0
        x[10] *= 1e4
        return w, x

    w, x, xq, dw, dp, got = _run_packed(sicu, oracle, wt, n_out, n_in, m, seed=4, patch=patch)
    want = oracle.gemv_batch(wt, w, n_in, n_out, xq)
    l1 = np.abs(_dequant_q8k(xq, n_in)) @ np.abs(_dequant_w(oracle, wt, w, n_in, n_out)).T
    _check_tol(got, want, l1, f"{Q.NAMES[wt]} packed prefill edge rows")
    assert (got[3] == 0).all()


@pytest.mark.parametrize("wt", COPY_ONLY, ids=lambda t: Q.NAMES[t])
@pytest.mark.parametrize("n_out,n_in,m", [
    (384, 1024, 100),    # CTA pairs, 128-token tiles
    (128, 512, 40),      # one row tile: the one-CTA kernel
    (130, 2048, 300),    # 256-token tiles, ragged rows
])
def test_copy_only_formats_without_a_copy(sicu, oracle, wt, n_out, n_in, m):
    """sicu_gemm_prefill(_f32) of a format whose tensor-core kernels read only
    the prefill copy: the call writes a copy into its workspace first. Within
    the prefill tolerance of the oracle, and the same bits as the call with
    the caller's own copy."""
    w = synth.weights(wt, n_out, n_in, seed=n_out + m)
    x = synth.activations(n_in, m, seed=n_in + m)
    xq = oracle.quantize_pair(wt, x)
    dw, dp, _ = _pack(sicu, wt, w, n_in, n_out)
    y = empty_f32(m, n_out)
    sicu.gemm_prefill(wt, dw, n_in, n_out, dev(xq), m, y)
    got = host(y)
    want = oracle.gemv_batch(wt, w, n_in, n_out, xq)
    l1 = np.abs(_dequant_q8k(xq, n_in)) @ np.abs(_dequant_w(oracle, wt, w, n_in, n_out)).T
    _check_tol(got, want, l1, f"{Q.NAMES[wt]} prefill without a copy {n_out}x{n_in} m={m}")
    y2 = empty_f32(m, n_out)
    sicu.gemm_prefill_packed(wt, dw, dp, n_in, n_out, dev(xq), m, y2)
    assert_bits_equal(host(y2), got, "with the caller's copy")
    y3 = empty_f32(m, n_out)
    sicu.gemm_prefill_f32(wt, dw, n_in, n_out, dev(x), m, y3)
    assert_bits_equal(host(y3), got, "f32 entry")
    assert sicu.status() == 0


def _f16_l1(x, w, n_in, n_out):
    """L1 = sum_k |x16_k| |w_k| of the F16 dot's products (x as the f16 the
    reference converts it to)."""
    xd = np.abs(x.astype(np.float16).astype(np.float64))
    wd = np.abs(w.view(np.float16).astype(np.float64).reshape(n_out, n_in))
    return xd @ wd.T


@pytest.mark.parametrize("n_out,n_in,m", [
    (128, 256, 64),      # one tile, one chunk
    (200, 1024, 77),     # ragged rows and tokens, CTA pairs
    (130, 4096, 300),    # long rows, 256-token tiles
])
def test_f16_prefill_vs_reference(sicu, oracle, n_out, n_in, m):
    """F16 weights on the tensor cores: the f16 weights re-tiled (no scale)
    against the activation converted to f16, 256-element chunks summed in
    tensor memory and added in the epilogue; within the prefill tolerance of
    the reference's F16 dot (src/kernels.c:189-195, exact products added into
    a double). With and without the caller's copy, f32 and f16 entries."""
    wt = Q.F16
    w = synth.weights(wt, n_out, n_in, seed=n_out + m)
    x = synth.activations(n_in, m, seed=n_in + m)
    xq = oracle.quantize_pair(wt, x)
    want = oracle.gemv_batch(wt, w, n_in, n_out, xq)
    l1 = _f16_l1(x, w, n_in, n_out)
    dw = dev(w)
    y = empty_f32(m, n_out)
    sicu.gemm_prefill_f32(wt, dw, n_in, n_out, dev(x), m, y)
    got = host(y)
    _check_tol(got, want, l1, f"F16 prefill {n_out}x{n_in} m={m}")
    dp = sicu.prefill_pack_bytes(wt, n_in, n_out)
    import torch
    pk = torch.zeros(dp, dtype=torch.uint8, device="cuda")
    sicu.prefill_pack(wt, dw, n_in, n_out, pk, dp)
    y2 = empty_f32(m, n_out)
    sicu.gemm_prefill_packed(wt, dw, pk, n_in, n_out, dev(xq), m, y2)
    assert_bits_equal(host(y2), got, "F16 prefill: f16 rows with the caller's copy")
    assert sicu.status() == 0


def test_f16_prefill_rows_not_whole_chunks_use_the_matvec(sicu, oracle):
    """F16 rows that are not whole 256-element chunks: the matvec per token,
    bit-identical with the reference's F16 dot."""
    wt, n_out, n_in, m = Q.F16, 96, 320, 40
    w = synth.weights(wt, n_out, n_in, seed=1)
    x = synth.activations(n_in, m, seed=2)
    y = empty_f32(m, n_out)
    sicu.gemm_prefill_f32(wt, dev(w), n_in, n_out, dev(x), m, y)
    assert_bits_equal(host(y), oracle.gemv_batch(wt, w, n_in, n_out, oracle.quantize_pair(wt, x)), "F16 K=320")

"""The activation steps between two products on the device: RMS norm (with
the residual add before it) and SwiGLU, on their own (sicu_rms_norm,
sicu_swiglu) and fused into the matvec (sicu_gemv_fused: prologues, and the
silu epilogue that splits SwiGLU across the gate product and W_down).

Everything is checked bit for bit against the oracle's restatement of the
reference's steps (src/engine.c:12-18, 162-179, 369, 379;
src/kernels.c:821-900), itself pinned to the reference by
tests/golden/steps.npz. That fixture also holds rows whose mean of squares
lies exactly halfway between two floats, where only the reference's
sequential double sum gives the right scale (the kernels' parallel sum must
notice and redo it in order).
"""

from __future__ import annotations

import numpy as np
import pytest

from siphon_b200 import quant as Q
from siphon_b200 import synth
from siphon_b200.lib import EPI_NONE, EPI_SILU, SicuError, mul_step, rms_norm_step, swiglu_step
from tests.gpu_util import assert_bits_equal, dev, empty_f32, host

pytestmark = pytest.mark.gpu

KQ = [Q.Q4_K, Q.Q5_K, Q.Q6_K, Q.Q3_K, Q.Q2_K, Q.Q4_0, Q.Q5_0, Q.Q8_0]
ALL = KQ + [Q.F16]
EPS = 1e-5


def _rows(golden_dir):
    g = np.load(golden_dir / "steps.npz")
    return g["rows256"], g["rows5120"], g["eps"]


def _gamma(n, seed):
    return (1.0 + 0.1 * np.random.default_rng(seed).standard_normal(n)).astype(np.float32)


def _want(oracle, wt, w, n_in, n_out, a):
    return oracle.gemv(wt, w, n_in, n_out, oracle.quantize_pair(wt, a[None, :])[0])


def test_rms_norm_rows_match_oracle(sicu, oracle, golden_dir):
    r256, r5120, epss = _rows(golden_dir)
    for rows in (r256, r5120):
        m, n = rows.shape
        w = _gamma(n, n)
        for eps in epss:
            eps = float(eps)
            y = empty_f32(m, n)
            sicu.rms_norm(dev(rows), dev(w), n, m, eps, y)
            want = np.stack([oracle.rms_norm(r, w, eps)[1] for r in rows])
            assert_bits_equal(host(y), want, f"rms norm n={n} eps={eps}")
            # the same rows arriving through the residual add (0 + r == r)
            zero = np.zeros_like(rows)
            y2, h = empty_f32(m, n), empty_f32(m, n)
            sicu.rms_norm(dev(zero), dev(w), n, m, eps, y2, dres=dev(rows), dsum=h)
            assert_bits_equal(host(y2), want, f"rms norm via residual n={n}")
            assert_bits_equal(host(h), rows, "residual sum")


def test_rms_norm_residual_add(sicu, oracle):
    rng = np.random.default_rng(5)
    m, n = 7, 4096
    x = (rng.standard_normal((m, n)) * 3).astype(np.float32)
    r = (rng.standard_normal((m, n)) * 0.7).astype(np.float32)
    w = _gamma(n, 6)
    y, h = empty_f32(m, n), empty_f32(m, n)
    sicu.rms_norm(dev(x), dev(w), n, m, EPS, y, dres=dev(r), dsum=h)
    hs, ys = zip(*[oracle.rms_norm(x[i], w, EPS, r[i]) for i in range(m)])
    assert_bits_equal(host(h), np.stack(hs), "h = x + r")
    assert_bits_equal(host(y), np.stack(ys), "norm of x + r")


def test_swiglu_matches_oracle(sicu, oracle, golden_dir):
    g = np.load(golden_dir / "steps.npz")
    ex = g["ex"]
    n = ex.size - ex.size % 8
    x = ex[:n]
    up = synth.activations(n, 1, seed=8)[0]
    y = empty_f32(n)
    sicu.swiglu(dev(x), dev(up), n, 1, y)
    assert_bits_equal(host(y), oracle.swiglu(x, up), "swiglu over the polynomial's range")
    rng = np.random.default_rng(9)
    m, n = 5, 13824
    gate = (rng.standard_normal((m, n)) * 4).astype(np.float32)
    up = rng.standard_normal((m, n)).astype(np.float32)
    y = empty_f32(m, n)
    sicu.swiglu(dev(gate), dev(up), n, m, y)
    assert_bits_equal(host(y), np.stack([oracle.swiglu(gate[i], up[i]) for i in range(m)]), "swiglu rows")


@pytest.mark.parametrize("wt", ALL, ids=lambda t: Q.NAMES[t])
def test_gemv_fused_rms_norm(sicu, oracle, golden_dir, wt):
    """RMS norm fused into the matvec: the halfway rows (n_in 256) and random
    rows with a residual (n_in 4096); sum_out holds x + residual."""
    r256, _, _ = _rows(golden_dir)
    n_out = 300
    w = synth.weights(wt, n_out, 256, seed=40 + wt)
    gam = _gamma(256, 41)
    for i, x in enumerate(r256):
        y = empty_f32(n_out)
        dw_, dx_, dg_ = dev(w), dev(x), dev(gam)      # held until the launch has run
        sicu.gemv_fused(wt, [dw_], [n_out], 256, dx_, rms_norm_step(dg_, EPS), [y])
        want = _want(oracle, wt, w, 256, n_out, oracle.rms_norm(x, gam, EPS)[1])
        assert_bits_equal(host(y), want, f"{Q.NAMES[wt]} fused norm, row {i}")
    n_in = 4096
    w = synth.weights(wt, n_out, n_in, seed=42 + wt)
    x = synth.activations(n_in, 1, seed=43)[0]
    res = synth.activations(n_in, 1, seed=44)[0]
    gam = _gamma(n_in, 45)
    dg, dres, h, y = dev(gam), dev(res), empty_f32(n_in), empty_f32(n_out)
    sicu.gemv_fused(wt, [dev(w)], [n_out], n_in, dev(x), rms_norm_step(dg, EPS, dres, h), [y])
    hw, a = oracle.rms_norm(x, gam, EPS, res)
    assert_bits_equal(host(h), hw, f"{Q.NAMES[wt]} sum_out")
    assert_bits_equal(host(y), _want(oracle, wt, w, n_in, n_out, a), f"{Q.NAMES[wt]} fused norm + residual")
    assert sicu.status() == 0


@pytest.mark.parametrize("wt", ALL, ids=lambda t: Q.NAMES[t])
def test_gemv_fused_swiglu(sicu, oracle, wt):
    n_in, n_out = 2048, 384
    w = synth.weights(wt, n_out, n_in, seed=50 + wt)
    rng = np.random.default_rng(51)
    gate = (rng.standard_normal(n_in) * 6).astype(np.float32)
    up = rng.standard_normal(n_in).astype(np.float32)
    y = empty_f32(n_out)
    dw_, dgate, dup = dev(w), dev(gate), dev(up)     # held until the launch has run
    sicu.gemv_fused(wt, [dw_], [n_out], n_in, dgate, swiglu_step(dup), [y])
    assert_bits_equal(host(y), _want(oracle, wt, w, n_in, n_out, oracle.swiglu(gate, up)), f"{Q.NAMES[wt]} swiglu")
    assert sicu.status() == 0


@pytest.mark.parametrize("wt", ALL, ids=lambda t: Q.NAMES[t])
def test_silu_epilogue_then_mul(sicu, oracle, wt):
    """SwiGLU split across two products: W_gate/W_up with the silu epilogue on
    the gate output, then W_down with the multiply step; the same bits as
    the reference's swiglu_row between the products."""
    d, ff = 512, 1536
    wg, wu = synth.weights(wt, ff, d, seed=90 + wt), synth.weights(wt, ff, d, seed=91 + wt)
    wd = synth.weights(wt, d, ff, seed=92 + wt)
    x = synth.activations(d, 1, seed=93)[0] * 4
    yg, yu, yd = empty_f32(ff), empty_f32(ff), empty_f32(d)
    sicu.gemv_fused(wt, [dev(wg), dev(wu)], [ff, ff], d, dev(x), None, [yg, yu], epi=[EPI_SILU, EPI_NONE])
    gate = _want(oracle, wt, wg, d, ff, x)
    up = _want(oracle, wt, wu, d, ff, x)
    assert_bits_equal(host(yg), oracle.silu_vec(gate), f"{Q.NAMES[wt]} silu epilogue")
    assert_bits_equal(host(yu), up, f"{Q.NAMES[wt]} plain output beside it")
    sicu.gemv_fused(wt, [dev(wd)], [d], ff, yg, mul_step(yu), [yd])
    assert_bits_equal(host(yd), _want(oracle, wt, wd, ff, d, oracle.swiglu(gate, up)), f"{Q.NAMES[wt]} down")
    assert sicu.status() == 0


@pytest.mark.parametrize("wt", [Q.Q4_K, Q.Q6_K, Q.Q5_K])
def test_gemv_fused_multi_large(sicu, oracle, wt):
    """Three products sharing one normed activation (the Wq/Wk/Wv shape of a
    5120-wide model, large enough for the flat kernel) with the residual
    add and the silu epilogue on the first, checked on a sample of rows."""
    n_in, outs = 5120, [5120, 1024, 1024]
    ws = [synth.weights(wt, n, n_in, seed=60 + j) for j, n in enumerate(outs)]
    x = synth.activations(n_in, 1, seed=61)[0]
    res = synth.activations(n_in, 1, seed=62)[0]
    gam = _gamma(n_in, 63)
    ys = [empty_f32(n) for n in outs]
    h = empty_f32(n_in)
    dws, dx_, dg_, dres_ = [dev(w) for w in ws], dev(x), dev(gam), dev(res)   # held until the launch has run
    sicu.gemv_fused(wt, dws, outs, n_in, dx_, rms_norm_step(dg_, EPS, dres_, h), ys,
                    epi=[EPI_SILU, EPI_NONE, EPI_NONE])
    hw, a = oracle.rms_norm(x, gam, EPS, res)
    assert_bits_equal(host(h), hw, "sum_out")
    xq = oracle.quantize_pair(wt, a[None, :])[0]
    rb = Q.row_bytes(wt, n_in)
    for j, (w, n) in enumerate(zip(ws, outs)):
        rows = np.unique(np.concatenate([np.arange(0, n, 97), [n - 1]]))
        sub = np.concatenate([w[r * rb:(r + 1) * rb] for r in rows])
        want = oracle.gemv(wt, sub, n_in, rows.size, xq)
        if j == 0:
            want = oracle.silu_vec(want)
        assert_bits_equal(host(ys[j])[rows], want, f"{Q.NAMES[wt]} matrix {j}")


@pytest.mark.parametrize("n_in", [27648, 13824])
def test_gemv_fused_mul_long_rows(sicu, oracle, n_in):
    """The W_down shapes of 32B-class models: the multiply step over rows of
    108 / 54 super-blocks (two pieces per thread)."""
    wt, n_out = Q.Q4_K, 640
    w = synth.weights(wt, n_out, n_in, seed=65)
    g = synth.activations(n_in, 1, seed=66)[0]
    u = synth.activations(n_in, 1, seed=67)[0]
    y = empty_f32(n_out)
    dw_, dg_, du_ = dev(w), dev(g), dev(u)           # held until the launch has run
    sicu.gemv_fused(wt, [dw_], [n_out], n_in, dg_, mul_step(du_), [y])
    assert_bits_equal(host(y), _want(oracle, wt, w, n_in, n_out, g * u), "mul step, long rows")


def test_fused_equals_separate_steps(sicu):
    """sicu_gemv_fused gives the bits of the step run on its own followed by
    sicu_gemv_f32."""
    wt, n_in, n_out = Q.Q4_K, 4096, 1000
    w = dev(synth.weights(wt, n_out, n_in, seed=70))
    x = dev(synth.activations(n_in, 1, seed=71)[0])
    res = dev(synth.activations(n_in, 1, seed=72)[0])
    gam = dev(_gamma(n_in, 73))
    a, y1, y2 = empty_f32(n_in), empty_f32(n_out), empty_f32(n_out)
    sicu.rms_norm(x, gam, n_in, 1, EPS, a, dres=res)
    sicu.gemv_f32(wt, w, n_in, n_out, a, y1)
    sicu.gemv_fused(wt, [w], [n_out], n_in, x, rms_norm_step(gam, EPS, res), [y2])
    assert_bits_equal(host(y2), host(y1), "norm: fused vs separate")
    up = dev(synth.activations(n_in, 1, seed=74)[0])
    sicu.swiglu(x, up, n_in, 1, a)
    sicu.gemv_f32(wt, w, n_in, n_out, a, y1)
    sicu.gemv_fused(wt, [w], [n_out], n_in, x, swiglu_step(up), [y2])
    assert_bits_equal(host(y2), host(y1), "swiglu: fused vs separate")


@pytest.mark.parametrize("wt", [Q.Q4_K, Q.Q6_K, Q.Q8_0])
def test_gemv_fused_swiglu_with_allreduce(sicu, oracle, wt):
    """The W_down form: SwiGLU fused into the row-split matvec with the
    all-reduce (a one-rank group), then with the silu epilogue on the sum."""
    n_in, d = 2048, 768
    w = synth.weights(wt, d, n_in, seed=80)
    gate = synth.activations(n_in, 1, seed=81)[0] * 3
    up = synth.activations(n_in, 1, seed=82)[0]
    g = sicu.ar_create(1, 0, d)
    g.open([g.local_handle])
    try:
        y = empty_f32(d)
        dw_, dgate, dup = dev(w), dev(gate), dev(up)     # held until the launches have run
        sicu.gemv_fused(wt, [dw_], [d], n_in, dgate, swiglu_step(dup), [y], group=g)
        want = _want(oracle, wt, w, n_in, d, oracle.swiglu(gate, up))
        assert_bits_equal(host(y), want, "swiglu + all-reduce")
        sicu.gemv_fused(wt, [dw_], [d], n_in, dgate, swiglu_step(dup), [y], group=g, epi=[EPI_SILU])
        assert_bits_equal(host(y), oracle.silu_vec(want), "swiglu + all-reduce + silu of the sum")
        assert sicu.status() == 0
    finally:
        g.destroy()


def test_step_argument_checks(sicu):
    n = 256
    x, y, gam = dev(np.ones(n, np.float32)), empty_f32(n), dev(np.ones(n, np.float32))
    w = dev(synth.weights(Q.Q4_K, 4, n, seed=1))
    with pytest.raises(SicuError):          # sum_out overlapping x
        sicu.gemv_fused(Q.Q4_K, [w], [4], n, x, rms_norm_step(gam, EPS, None, x), [y])
    with pytest.raises(SicuError):          # no norm weight
        sicu.gemv_fused(Q.Q4_K, [w], [4], n, x, rms_norm_step(None, EPS), [y])
    with pytest.raises(SicuError):          # SwiGLU row not a multiple of 8
        sicu.swiglu(x, x, 12, 1, y)
    with pytest.raises(SicuError):          # misaligned residual
        sicu.rms_norm(x, gam, n, 1, EPS, y, dres=x.data_ptr() + 4)


@pytest.mark.parametrize("wt", ALL, ids=lambda t: Q.NAMES[t])
def test_gemv_fused_bias_epilogue(sicu, oracle, wt):
    """Q/K/V-style launch with per-matrix biases (sicu_gemv_fused_ex): every
    output is the reference's product plus its bias, one f32 addition
    (src/engine.c:320-334); a NULL entry leaves that matrix unbiased; a silu
    epilogue applies after the bias. Covers whole-row, flattened-item and F16
    kernels (5120-wide rows take the flattened path for K formats)."""
    n_in = 5120 if wt in (Q.Q4_K, Q.Q6_K) else 1024
    outs = [256, 64, 64]
    ws = [synth.weights(wt, n, n_in, seed=40 + i) for i, n in enumerate(outs)]
    x = synth.activations(n_in, 1, seed=41)[0]
    g = _gamma(n_in, 42)
    rng = np.random.default_rng(43)
    bs = [(0.02 * rng.standard_normal(n)).astype(np.float32) for n in outs]
    _, a = oracle.rms_norm(x, g, EPS)
    ys = [empty_f32(n) for n in outs]
    # device buffers held until the (asynchronous) launch has run: the step
    # and the call keep only their addresses
    dws, dx, dg, db0, db2 = [dev(w) for w in ws], dev(x), dev(g), dev(bs[0]), dev(bs[2])
    sicu.gemv_fused(wt, dws, outs, n_in, dx, rms_norm_step(dg, EPS), ys, bias=[db0, None, db2],
                    epi=[EPI_NONE, EPI_NONE, EPI_SILU])
    for i, (w, n) in enumerate(zip(ws, outs)):
        want = _want(oracle, wt, w, n_in, n, a)
        if i != 1:
            want = (want + bs[i]).astype(np.float32)        # one f32 addition per element
        if i == 2:
            want = oracle.silu_vec(want)
        assert_bits_equal(host(ys[i]), want, f"{Q.NAMES[wt]} bias matrix {i}")


def test_add_bias_rows(sicu):
    """sicu_add_bias: m rows plus one bias row, one f32 addition per element
    (the reference's q[i] + bq[i], src/engine.c:319-333), for a prompt's
    Q/K/V rows; rows of odd widths, one row, and signed zeros."""
    import torch
    rng = np.random.default_rng(44)
    for n, m in ((1000, 7), (256, 1), (5120, 33)):
        y = (rng.standard_normal((m, n)) * 3).astype(np.float32)
        b = (0.02 * rng.standard_normal(n)).astype(np.float32)
        y[0, :4] = [0.0, -0.0, 0.0, -0.0]
        b[:4] = [-0.0, -0.0, 0.0, 0.0]
        dy = dev(y)
        sicu.add_bias(dy, dev(b), n, m)
        assert_bits_equal(host(dy), (y + b[None, :]).astype(np.float32), f"{m} rows of {n}")
    d = torch.zeros(8, device="cuda")
    with pytest.raises(SicuError):
        sicu.add_bias(d, d[4:], 4, 2)        # the bias inside the rows

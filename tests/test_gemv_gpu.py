"""Decode matvec parity: the CUDA kernels against the oracle's scalar
reference semantics, bit for bit, through the C ABI."""

from __future__ import annotations

import numpy as np
import pytest

from siphon_b200 import quant as Q
from siphon_b200 import synth
from tests.gpu_util import assert_bits_equal, assert_within_tol, dev, empty_f32, empty_u8, host

pytestmark = pytest.mark.gpu

K_TYPES = (Q.Q2_K, Q.Q3_K, Q.Q4_K, Q.Q5_K, Q.Q6_K)
C_TYPES = (Q.Q4_0, Q.Q5_0, Q.Q8_0)

# (n_out, n_in): tiny, ragged row counts, rows that are not 16-byte aligned
# (odd super-block counts), long rows that stream in chunks
K_SHAPES = [(1, 256), (5, 256), (37, 512), (64, 2048), (200, 768), (33, 1280), (129, 5632), (300, 12544)]
C_SHAPES = [(1, 32), (7, 96), (37, 160), (64, 2048), (33, 4128), (129, 5632), (100, 14336)]
F_SHAPES = [(1, 8), (7, 100), (64, 2048), (33, 4100)]


def _case(sicu, oracle, wt, n_out, n_in, seed=0, scale=1.0):
    w = synth.weights(wt, n_out, n_in, seed=seed)
    x = synth.activations(n_in, 1, seed=seed + 1) * np.float32(scale)
    xq = oracle.quantize_pair(wt, x)
    want = oracle.gemv(wt, w, n_in, n_out, xq[0])
    dw = dev(w)
    # pre-quantized activation
    y = empty_f32(n_out)
    sicu.gemv(wt, dw, n_in, n_out, dev(xq), y)
    got = host(y)
    assert_bits_equal(got, want, f"{Q.NAMES[wt]} {n_out}x{n_in} gemv")
    assert_within_tol(got, want, "gemv")
    # fused f32 activation
    y2 = empty_f32(n_out)
    sicu.gemv_f32(wt, dw, n_in, n_out, dev(x), y2)
    assert_bits_equal(host(y2), want, f"{Q.NAMES[wt]} {n_out}x{n_in} gemv_f32")


@pytest.mark.parametrize("shape", K_SHAPES, ids=str)
@pytest.mark.parametrize("wt", K_TYPES, ids=lambda t: Q.NAMES[t])
def test_k_formats(sicu, oracle, wt, shape):
    _case(sicu, oracle, wt, *shape)


@pytest.mark.parametrize("shape", C_SHAPES, ids=str)
@pytest.mark.parametrize("wt", C_TYPES, ids=lambda t: Q.NAMES[t])
def test_classic_formats(sicu, oracle, wt, shape):
    _case(sicu, oracle, wt, *shape)


@pytest.mark.parametrize("shape", F_SHAPES, ids=str)
def test_f16(sicu, oracle, shape):
    _case(sicu, oracle, Q.F16, *shape)


@pytest.mark.parametrize("wt", Q.WEIGHT_TYPES, ids=lambda t: Q.NAMES[t])
def test_activation_scales(sicu, oracle, wt):
    # F16 activations saturate past 65504 and go subnormal below 6e-5
    scales = (1e-6, 1e-3, 1e3, 1e4) if wt == Q.F16 else (1e-20, 1e-3, 1e3, 1e20)
    for s, scale in enumerate(scales):
        _case(sicu, oracle, wt, 24, 1024, seed=10 + s, scale=scale)


@pytest.mark.parametrize("wt", Q.WEIGHT_TYPES, ids=lambda t: Q.NAMES[t])
def test_zero_activation_blocks(sicu, oracle, wt):
    n_in, n_out = 1024, 40
    w = synth.weights(wt, n_out, n_in, seed=5)
    x = synth.activations(n_in, 1, seed=6)
    x[0, 256:512] = 0.0
    xq = oracle.quantize_pair(wt, x)
    want = oracle.gemv(wt, w, n_in, n_out, xq[0])
    y = empty_f32(n_out)
    sicu.gemv_f32(wt, dev(w), n_in, n_out, dev(x), y)
    assert_bits_equal(host(y), want, "zero block")


@pytest.mark.slow
@pytest.mark.parametrize("shape", [(4096, 4096), (14336, 4096), (4096, 14336), (5632, 2048)], ids=str)
@pytest.mark.parametrize("wt", Q.WEIGHT_TYPES, ids=lambda t: Q.NAMES[t])
def test_baseline_sizes(sicu, oracle, wt, shape):
    """The single-matvec shape 5632x2048 and the sweep shapes, bit-exact at full size."""
    n_out, n_in = shape
    w = synth.weights(wt, n_out, n_in, seed=wt)
    x = synth.activations(n_in, 1, seed=100 + wt)
    xq = oracle.quantize_pair(wt, x)
    want = oracle.gemv_batch(wt, w, n_in, n_out, xq)[0]
    y = empty_f32(n_out)
    sicu.gemv_f32(wt, dev(w), n_in, n_out, dev(x), y)
    assert_bits_equal(host(y), want, f"{Q.NAMES[wt]} {shape}")


def test_batched_rows(sicu, oracle):
    wt, n_in, n_out, m = Q.Q4_K, 2048, 96, 5
    w = synth.weights(wt, n_out, n_in, seed=8)
    x = synth.activations(n_in, m, seed=9)
    xq = oracle.quantize_pair(wt, x)
    want = oracle.gemv_batch(wt, w, n_in, n_out, xq)
    y = empty_f32(m, n_out)
    sicu.gemv(wt, dev(w), n_in, n_out, dev(xq), y, m=m)
    assert_bits_equal(host(y), want, "batched gemv")


def test_host_buffers(sicu, oracle):
    wt, n_in, n_out = Q.Q6_K, 2048, 300
    w = synth.weights(wt, n_out, n_in, seed=12)
    x = synth.activations(n_in, 1, seed=13)[0]
    want = oracle.gemv(wt, w, n_in, n_out, oracle.quantize_pair(wt, x)[0])
    hy = np.zeros(n_out, np.float32)
    sicu.gemv_host(wt, dev(w), n_in, n_out, x, hy)
    assert_bits_equal(hy, want, "gemv_host")


@pytest.mark.parametrize("wt,n_out,n_in", [(Q.Q6_K, 300, 2048), (Q.Q4_K, 5000, 5120), (Q.Q8_0, 77, 1024),
                                           (Q.F16, 64, 512)])
def test_host_buffers_page_locked(sicu, oracle, wt, n_out, n_in):
    """Page-locked host buffers take the path where the GPU reads x and
    writes y in host memory directly; pageable ones the copy-engine path.
    Both must give the reference's bits, several calls in a row."""
    import torch
    w = synth.weights(wt, n_out, n_in, seed=n_out)
    dw = dev(w)
    for call in range(3):
        x = synth.activations(n_in, 1, seed=100 + call)[0]
        want = oracle.gemv(wt, w, n_in, n_out, oracle.quantize_pair(wt, x)[0])
        hx = torch.from_numpy(x.copy()).pin_memory()
        hy = torch.full((n_out,), float("nan")).pin_memory()
        sicu.gemv_host(wt, dw, n_in, n_out, hx, hy)
        assert_bits_equal(hy.numpy(), want, f"{Q.NAMES[wt]} gemv_host, page-locked, call {call}")
        hy2 = np.full(n_out, np.nan, np.float32)
        sicu.gemv_host(wt, dw, n_in, n_out, x, hy2)
        assert_bits_equal(hy2, want, f"{Q.NAMES[wt]} gemv_host, pageable, call {call}")
    assert sicu.status() == 0


@pytest.mark.parametrize("wt", Q.WEIGHT_TYPES, ids=lambda t: Q.NAMES[t])
def test_row_to_f32(sicu, oracle, wt):
    n_in, n_out = 2048, 9
    w = synth.weights(wt, n_out, n_in, seed=14)
    rows = [8, 0, 3, 3]
    out = empty_f32(len(rows), n_in)
    sicu.row_to_f32(wt, dev(w), n_in, rows, out)
    rb = Q.row_bytes(wt, n_in)
    want = np.stack([oracle.dequant_row(wt, w[r * rb:(r + 1) * rb], n_in) for r in rows])
    assert_bits_equal(host(out), want, "row_to_f32")


def test_status_clean_after_runs(sicu):
    assert sicu.status() == 0


@pytest.mark.parametrize("wt", (Q.Q4_K, Q.Q6_K, Q.Q8_0), ids=lambda t: Q.NAMES[t])
def test_overlap_dependent_chain(sicu, oracle, wt):
    """With programmatic dependent launch on, a matvec whose activation is the
    previous matvec's output must still read it only after it is complete."""
    n = 2048
    ws = [synth.weights(wt, n, n, seed=40 + i) for i in range(4)]
    x = synth.activations(n, 1, seed=41)[0]
    want = x
    for w in ws:
        want = oracle.gemv(wt, w, n, n, oracle.quantize_pair(wt, want)[0])
    dws = [dev(w) for w in ws]
    bufs = [dev(x)] + [empty_f32(n) for _ in ws]
    sicu.set_overlap(True)
    try:
        for i, dw in enumerate(dws):
            sicu.gemv_f32(wt, dw, n, n, bufs[i], bufs[i + 1])
        got = host(bufs[-1])
    finally:
        sicu.set_overlap(False)
    assert_bits_equal(got, want, "overlapped chain")


@pytest.mark.parametrize("wt", Q.WEIGHT_TYPES, ids=lambda t: Q.NAMES[t])
def test_multi_matrix_launch(sicu, oracle, wt):
    """One launch over several matrices sharing an activation (the Q/K/V and
    gate/up pattern) equals separate matvecs, bit for bit; empty matrices and
    ragged row counts included."""
    n_in = 2048
    n_outs = [512, 128, 0, 77, 1024]
    ws = [synth.weights(wt, n, n_in, seed=60 + i) for i, n in enumerate(n_outs)]
    x = synth.activations(n_in, 1, seed=61)
    xq = oracle.quantize_pair(wt, x)[0]
    ys = [empty_f32(max(n, 1)) for n in n_outs]
    sicu.gemv_multi(wt, [dev(w) for w in ws], n_outs, n_in, dev(x), ys)
    for i, (w, n) in enumerate(zip(ws, n_outs)):
        if n:
            assert_bits_equal(host(ys[i])[:n], oracle.gemv(wt, w, n_in, n, xq), f"matrix {i}")


def test_multi_matrix_many_copies(sicu, oracle):
    wt, n_in, n_out, copies = Q.Q4_K, 4096, 1024, 40
    w = synth.weights(wt, n_out, n_in, seed=70)
    x = synth.activations(n_in, 1, seed=71)
    want = oracle.gemv(wt, w, n_in, n_out, oracle.quantize_pair(wt, x)[0])
    dw = dev(w)
    dws = [dw] + [dw.clone() for _ in range(copies - 1)]
    ys = [empty_f32(n_out) for _ in range(copies)]
    sicu.gemv_multi(wt, dws, [n_out] * copies, n_in, dev(x), ys)
    for i in range(copies):
        assert_bits_equal(host(ys[i]), want, f"copy {i}")

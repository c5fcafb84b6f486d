"""The flattened-item matvec (gemv_flat_kernel): rows whose super-block count
does not divide 32 are streamed as items of 32 consecutive super-blocks that
may span rows, and a row's float chains continue across items. The library
picks it by itself for launches with enough rows; `flat_rows` mirrors that
choice so each case here is known to take it. Outputs must be bit-identical
to the reference's scalar dots (the oracle)."""

from __future__ import annotations

import numpy as np
import pytest

from siphon_b200 import quant as Q
from siphon_b200 import synth
from tests.gpu_util import assert_bits_equal, dev, empty_f32, host

pytestmark = pytest.mark.gpu

CHAINS = {Q.Q4_K: 9, Q.Q5_K: 9, Q.Q6_K: 8, Q.Q3_K: 8, Q.Q2_K: 1}


def flat_rows(nu: int, n_outs: list[int], sms: int, chains: int) -> int:
    """Rows per task of the flattened kernel for this launch, 0 if the
    whole-row kernel is used (the library's launch choice, gemv.cu)."""
    if nu < 6:
        return 0
    if nu <= 32:
        rpt, nch = 32 // nu, 1
        rpt = min(rpt, 64 // chains) if chains > 1 else rpt
    else:
        nch = (nu + 31) // 32
        rpt = 1
    if rpt * nu / 32 >= 0.8 if nch == 1 else nu / (32 * nch) >= 0.8:
        return 0
    g = 2 * sms

    def busiest(rows, items):
        tasks = sum((n + rows - 1) // rows for n in n_outs)
        per_cta = (tasks + g - 1) // g
        return (per_cta + 7) // 8 * items

    best, pick = busiest(rpt, nch), 0
    for r in range(1, 9):
        v = busiest(r, (r * nu + 31) // 32)
        if v < best:
            best, pick = v, r
    return pick


@pytest.fixture(scope="module")
def sms():
    import torch
    return torch.cuda.get_device_properties(0).multi_processor_count


@pytest.mark.parametrize("wt", [Q.Q4_K, Q.Q5_K, Q.Q6_K, Q.Q3_K, Q.Q2_K])
@pytest.mark.parametrize("n_out,n_in", [
    (20000, 5120),     # 20 super-blocks per row (a 32B-class model's width)
    (30001, 3072),     # 12 per row, ragged last task
    (12000, 10240),    # 40 per row: items of 32 straddle rows
])
def test_flat_matches_reference(sicu, oracle, sms, wt, n_out, n_in):
    nu = n_in // 256
    assert flat_rows(nu, [n_out], sms, CHAINS[wt]) > 0, "shape does not take the flattened kernel"
    w = synth.weights(wt, n_out, n_in, seed=n_out + nu)
    x = synth.activations(n_in, 1, seed=nu)
    xq = oracle.quantize_pair(wt, x)[0]
    want = oracle.gemv(wt, w, n_in, n_out, xq)
    y = empty_f32(n_out)
    sicu.gemv_f32(wt, dev(w), n_in, n_out, dev(x[0]), y)
    assert_bits_equal(host(y), want, f"{Q.NAMES[wt]} {n_out}x{n_in} flattened")


def test_flat_multi_matrix_ragged(sicu, oracle, sms):
    """Several matrices in one launch, tasks ending mid-matrix."""
    wt, n_in = Q.Q4_K, 5120
    n_outs = [7001, 9000, 5003, 3]
    assert flat_rows(n_in // 256, n_outs, sms, 9) > 0
    x = synth.activations(n_in, 1, seed=5)
    xq = oracle.quantize_pair(wt, x)[0]
    ws = [synth.weights(wt, n, n_in, seed=100 + i) for i, n in enumerate(n_outs)]
    ys = [empty_f32(n) for n in n_outs]
    sicu.gemv_multi(wt, [dev(w) for w in ws], n_outs, n_in, dev(x[0]), ys)
    for i, (w, n) in enumerate(zip(ws, n_outs)):
        assert_bits_equal(host(ys[i]), oracle.gemv(wt, w, n_in, n, xq), f"matrix {i} ({n} rows)")


def test_flat_special_values(sicu, oracle, sms):
    """d = 0 blocks and a zero activation block pass through the straddled
    chains exactly."""
    wt, n_out, n_in = Q.Q4_K, 20000, 5120
    w = synth.weights(wt, n_out, n_in, seed=9).copy()
    blocks = w.reshape(-1, 144)
    blocks[::7, 0:2] = 0
    x = synth.activations(n_in, 1, seed=10)
    x[0, 256:512] = 0.0
    xq = oracle.quantize_pair(wt, x)[0]
    y = empty_f32(n_out)
    sicu.gemv_f32(wt, dev(w), n_in, n_out, dev(x[0]), y)
    assert_bits_equal(host(y), oracle.gemv(wt, w, n_in, n_out, xq), "flattened, special values")
    assert np.isfinite(host(y)).all()

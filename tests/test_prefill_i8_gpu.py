"""Prefill of the classic formats (Q4_0, Q5_0, Q8_0) on int8 tensor-core MMAs
against the oracle's scalar per-row dots of the reference
(src/kernels.c:197-247), bit for bit.

Each 32-element block's integer sum comes exactly out of one kind::i8 MMA
(the quants are int8 on both sides), and the epilogue adds the blocks' float
terms into each (row, token) sum in the reference's order, so unlike the
K-format prefill these products are held to equality, not to a tolerance.
"""

from __future__ import annotations

import numpy as np
import pytest

from siphon_b200 import quant as Q
from siphon_b200 import synth
from tests.gpu_util import assert_bits_equal, dev, empty_f32, host

pytestmark = pytest.mark.gpu

CLASSIC = (Q.Q4_0, Q.Q5_0, Q.Q8_0)


def _pack(sicu, wt, dw, n_in, n_out):
    import torch
    nb = sicu.prefill_pack_bytes(wt, n_in, n_out)
    dp = torch.zeros(nb, dtype=torch.uint8, device="cuda")
    sicu.prefill_pack(wt, dw, n_in, n_out, dp, nb)
    return dp


@pytest.mark.parametrize("wt", CLASSIC, ids=lambda t: Q.NAMES[t])
@pytest.mark.parametrize("n_out,n_in,m", [
    (128, 256, 64),      # one row tile, two K-steps
    (200, 512, 77),      # ragged rows and tokens
    (130, 4096, 300),    # three 128-token tiles, the last partial; long rows
    (256, 160, 40),      # five 32-blocks: a last K-step of one block
    (64, 1056, 129),     # 33 blocks; two token tiles, the second of one token
])
def test_i8_prefill_bit_exact(sicu, oracle, wt, n_out, n_in, m):
    w = synth.weights(wt, n_out, n_in, seed=n_out + n_in + m)
    x = synth.activations(n_in, m, seed=m)
    xq = oracle.quantize_pair(wt, x)
    want = oracle.gemv_batch(wt, w, n_in, n_out, xq)
    dw = dev(w)
    y = empty_f32(m, n_out)
    sicu.gemm_prefill(wt, dw, n_in, n_out, dev(xq), m, y)          # the copy made in the workspace
    assert_bits_equal(host(y), want, f"{Q.NAMES[wt]} {n_out}x{n_in} m={m}")
    dp = _pack(sicu, wt, dw, n_in, n_out)
    y2 = empty_f32(m, n_out)
    sicu.gemm_prefill_packed_f32(wt, dw, dp, n_in, n_out, dev(x), m, y2)   # caller's copy, f32 rows
    assert_bits_equal(host(y2), want, f"{Q.NAMES[wt]} {n_out}x{n_in} m={m} (copy, f32)")
    assert sicu.status() == 0


@pytest.mark.parametrize("wt", CLASSIC, ids=lambda t: Q.NAMES[t])
def test_i8_prefill_edge_rows(sicu, oracle, wt):
    """Zero activation rows, weight blocks with d = 0, activation rows at
    very different scales."""
    n_out, n_in, m = 160, 768, 96
    w = synth.weights(wt, n_out, n_in, seed=3).copy()
    blocks = w.reshape(-1, Q.row_bytes(wt, 32))
    blocks[::5, 0:2] = 0
    x = synth.activations(n_in, m, seed=4)
    x[3] = 0.0
    x[10] *= 1e4
    x[11] *= 1e-4
    xq = oracle.quantize_pair(wt, x)
    want = oracle.gemv_batch(wt, w, n_in, n_out, xq)
    y = empty_f32(m, n_out)
    sicu.gemm_prefill_f32(wt, dev(w), n_in, n_out, dev(x), m, y)
    got = host(y)
    assert_bits_equal(got, want, f"{Q.NAMES[wt]} edge rows")
    assert (got[3] == 0).all()


def test_i8_prefill_small_blocks_and_short_rows_use_the_matvec(sicu, oracle):
    """At most 32 tokens, or rows shorter than one 128-element K-step: the
    matvec per token, the same bits."""
    for wt, n_out, n_in, m in ((Q.Q8_0, 96, 512, 20), (Q.Q4_0, 96, 64, 50)):
        w = synth.weights(wt, n_out, n_in, seed=m)
        x = synth.activations(n_in, m, seed=m + 1)
        xq = oracle.quantize_pair(wt, x)
        y = empty_f32(m, n_out)
        sicu.gemm_prefill(wt, dev(w), n_in, n_out, dev(xq), m, y)
        assert_bits_equal(host(y), oracle.gemv_batch(wt, w, n_in, n_out, xq), f"{Q.NAMES[wt]} m={m} K={n_in}")


def test_i8_prefill_multi_products_one_by_one(sicu, oracle):
    """sicu_gemm_prefill_multi_f32 on a classic format: the products one by
    one from their copies, each bit-exact, and the same bits on a second call."""
    wt, n_outs, n_in, m = Q.Q8_0, (256, 128, 128), 1024, 300
    x = synth.activations(n_in, m, seed=9)
    xq = oracle.quantize_pair(wt, x)
    ws = [synth.weights(wt, n, n_in, seed=n + i) for i, n in enumerate(n_outs)]
    dws = [dev(w) for w in ws]
    dps = [_pack(sicu, wt, d, n_in, n) for d, n in zip(dws, n_outs)]
    ys = [empty_f32(m, n) for n in n_outs]
    dx = dev(x)
    sicu.gemm_prefill_multi_f32(wt, dws, dps, list(n_outs), n_in, dx, m, ys)
    first = [host(y) for y in ys]
    sicu.gemm_prefill_multi_f32(wt, dws, dps, list(n_outs), n_in, dx, m, ys)
    for i, n in enumerate(n_outs):
        assert_bits_equal(host(ys[i]), first[i], f"matrix {i} second call")
        assert_bits_equal(first[i], oracle.gemv_batch(wt, ws[i], n_in, n, xq), f"matrix {i}")
    assert sicu.status() == 0


def test_i8_pack_layout(sicu, oracle):
    """The classic copy decoded from its documented layout: int8 quants
    (128-byte swizzle, 16-byte unit j of row r at j ^ (r & 7)) times the row
    scales give back the reference's dequantized weights, exactly."""
    from tests.test_prefill_gpu import _dequant_w
    for wt in CLASSIC:
        n_out, n_in = 130, 160
        w = synth.weights(wt, n_out, n_in, seed=5)
        dp = host(_pack(sicu, wt, dev(w), n_in, n_out))
        nks, nrt = (n_in // 32 + 3) // 4, (n_out + 127) // 128
        chunk = 128 * 128 + 128 * 16
        got = np.zeros((nrt * 128, nks * 128))
        for rt in range(nrt):
            for ks in range(nks):
                c = dp[(rt * nks + ks) * chunk:(rt * nks + ks + 1) * chunk]
                q = c[:128 * 128].reshape(128, 8, 16)
                un = np.empty_like(q)
                for r in range(128):
                    for j in range(8):
                        un[r, j ^ (r & 7)] = q[r, j]
                qv = un.reshape(128, 128).view(np.int8).astype(np.float64)
                d = c[128 * 128:].view(np.float32).reshape(128, 4).astype(np.float64)
                got[rt * 128:(rt + 1) * 128, ks * 128:(ks + 1) * 128] = qv * np.repeat(d, 32, axis=1)
        want = _dequant_w(oracle, wt, w, n_in, n_out)
        assert np.array_equal(got[:n_out, :n_in].astype(np.float32), want.astype(np.float32)), Q.NAMES[wt]
        assert not got[n_out:].any() and not got[:, n_in:].any()

"""The reference's own kernel checks (tests/test_kernels.c) applied to the
oracle restatement: f16 spot values and round trips (:38-85), every dot
against an exact double evaluation within 2e-6 of the L1 norm (:177-260),
quantizer invariants (:264-321) and geometry (:403-417)."""

from __future__ import annotations

import numpy as np
import pytest

from siphon_b200 import quant as Q


class XorShift:
    """test_kernels.c:25-34"""

    def __init__(self, seed=0x9E3779B97F4A7C15):
        self.s = seed

    def next(self) -> int:
        s = self.s
        s ^= s >> 12
        s ^= (s << 25) & 0xFFFFFFFFFFFFFFFF
        s ^= s >> 27
        self.s = s
        return (s * 0x2545F4914F6CDD1D) & 0xFFFFFFFFFFFFFFFF

    def f(self) -> float:
        return float(np.float32((self.next() >> 40) / 524288.0 * 2.0 - 1.0))


def test_f16_spot_values(oracle):
    o = oracle
    assert o.f16_to_f32(0x0000) == 0.0 and np.signbit(o.f16_to_f32(0x8000))
    assert o.f16_to_f32(0x3C00) == 1.0
    assert 65500.0 < o.f16_to_f32(0x7BFF) < 65505.0
    assert o.f32_to_f16(1.0) == 0x3C00 and o.f32_to_f16(-1.0) == 0xBC00 and o.f32_to_f16(0.5) == 0x3800
    assert o.f32_to_f16(0.0) == 0 and (o.f32_to_f16(-0.0) & 0x8000)
    assert o.f32_to_f16(65504.0) == 0x7BFF and o.f32_to_f16(65520.0) == 0x7C00
    assert o.f32_to_f16(1e10) == 0x7C00 and o.f32_to_f16(1e-10) == 0 and o.f32_to_f16(6.0e-8) == 0x0001


def test_f16_roundtrip_all_patterns(oracle):
    for h in range(65536):
        f = oracle.f16_to_f32(h)
        if (h & 0x7C00) == 0x7C00:
            assert np.isinf(f) or np.isnan(f)
        else:
            assert oracle.f32_to_f16(f) == h


def _tame(wt: int, w: np.ndarray, rng: XorShift) -> None:
    """tame_scales_* (test_kernels.c:98-140): d in [0.01, 0.02), dmin in [0, 0.001)."""
    blck, bsz = Q.GEOMETRY[wt]
    blocks = w.reshape(-1, bsz)
    d_off = {Q.Q2_K: 80, Q.Q3_K: 108, Q.Q4_K: 0, Q.Q5_K: 0, Q.Q6_K: 208, Q.Q4_0: 0, Q.Q5_0: 0, Q.Q8_0: 0}[wt]
    m_off = {Q.Q2_K: 82, Q.Q4_K: 2, Q.Q5_K: 2}.get(wt)
    for b in blocks:
        d = np.float32(0.01 * (1.0 + (rng.next() % 100) / 100.0)).astype(np.float16)
        b[d_off:d_off + 2] = np.frombuffer(d.tobytes(), np.uint8)
        if m_off is not None:
            m = np.float32(0.001 * (rng.next() % 100) / 100.0).astype(np.float16)
            b[m_off:m_off + 2] = np.frombuffer(m.tobytes(), np.uint8)


@pytest.mark.parametrize("wt", [t for t in Q.WEIGHT_TYPES if t != Q.F16], ids=lambda t: Q.NAMES[t])
def test_dot_against_exact_double(oracle, wt):
    n = 1024
    rng = XorShift()
    pair = Q.pair_type(wt)
    worst = 0.0
    for _ in range(40):
        w = np.array([rng.next() & 0xFF for _ in range(Q.row_bytes(wt, n))], np.uint8)
        _tame(wt, w, rng)
        x = np.array([rng.f() for _ in range(n)], np.float32)
        xs = oracle.dequant_row(wt, w, n).astype(np.float64)
        xq = oracle.quantize_pair(wt, x)[0]
        if pair == Q.Q8_0:
            blk = xq.reshape(-1, 34)
            d = np.array([oracle.f16_to_f32(int(b[0]) | (int(b[1]) << 8)) for b in blk], np.float64)
            qa = blk[:, 2:].view(np.int8).astype(np.float64) * d[:, None]
        else:
            blk = xq.reshape(-1, 292)
            d = blk[:, :4].copy().view(np.float32).astype(np.float64)
            qa = blk[:, 4:260].view(np.int8).astype(np.float64) * d
        terms = xs * qa.reshape(-1)
        s = oracle.vec_dot(wt, n, w, xq)
        rel = abs(s - terms.sum()) / max(np.abs(terms).sum(), 1e-9)
        worst = max(worst, rel)
    assert worst <= 2e-6


def test_quantizer_invariants(oracle):
    rng = XorShift(12345)
    n = 1024
    for _ in range(20):
        x = np.array([rng.f() for _ in range(n)], np.float32)
        y8 = oracle.quant_q8_0(x).reshape(-1, 34)
        for b, blk in enumerate(y8):
            d = oracle.f16_to_f32(int(blk[0]) | (int(blk[1]) << 8))
            xb = x[32 * b:32 * b + 32]
            amax = float(np.abs(xb).max())
            assert abs(d - amax / 127.0) < 0.001 * (amax / 127.0 + 1e-6)
            q = blk[2:].view(np.int8).astype(np.float32)
            assert (np.abs(q * d - xb) <= d * 0.5 + np.abs(xb) * 5e-4 + 1e-6).all()
            assert q.min() >= -127 and q.max() <= 127
        yk = oracle.quant_q8_K(x).reshape(-1, 292)
        for b, blk in enumerate(yk):
            d = float(blk[:4].copy().view(np.float32)[0])
            xb = x[256 * b:256 * b + 256]
            i = int(np.argmax(np.abs(xb)))
            assert abs(d - xb[i] / -127.0) < abs(xb[i] / -127.0) * 1e-5 + 1e-9
            q = blk[4:260].view(np.int8).astype(np.int32)
            assert q.min() >= -127 and q.max() <= 127
            assert (np.abs(q * d - xb) <= abs(d) * 1.01).all()
            bs = blk[260:292].copy().view(np.int16)
            assert (bs == q.reshape(16, 16).sum(axis=1)).all()
    z = np.zeros(n, np.float32)
    assert (oracle.quant_q8_0(z).reshape(-1, 34)[:, :2] == 0).all()
    assert (oracle.quant_q8_K(z).reshape(-1, 292)[:, :4] == 0).all()


def test_geometry():
    assert Q.GEOMETRY[Q.Q4_K] == (256, 144) and Q.GEOMETRY[Q.Q6_K] == (256, 210)
    assert Q.GEOMETRY[Q.Q8_K] == (256, 292) and Q.GEOMETRY[Q.Q8_0] == (32, 34)
    assert Q.GEOMETRY[Q.Q5_0] == (32, 22) and 40 not in Q.GEOMETRY
    assert Q.NAMES[Q.Q4_K] == "Q4_K"

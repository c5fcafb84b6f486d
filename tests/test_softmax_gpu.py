"""sicu_softmax against the oracle's restatement of the reference's attention
softmax (itself pinned to the reference build in tests/test_softmax.py), bit
for bit: row lengths with and without a tail (the n % 8 elements that go
through libm's expf), masked and equal entries, many rows at once, in place."""

from __future__ import annotations

import numpy as np
import pytest

from tests.gpu_util import assert_bits_equal, dev, empty_f32, host
from tests.test_softmax import _rows

pytestmark = pytest.mark.gpu


def test_rows_match_oracle(sicu, oracle):
    for i, x in enumerate(_rows(1)):
        y = empty_f32(x.size)
        sicu.softmax(dev(x), y, x.size)
        assert_bits_equal(host(y), oracle.softmax(x), f"row {i} (n={x.size})")


def test_many_rows_and_in_place(sicu, oracle):
    rng = np.random.default_rng(7)
    for n, m, s in ((15, 20000, 30.0), (257, 300, 5.0), (2048, 16, 8.0)):
        x = (rng.standard_normal((m, n)) * s).astype(np.float32)
        y = empty_f32(m, n)
        sicu.softmax(dev(x), y, n, m)
        want = np.stack([oracle.softmax(r) for r in x])
        assert_bits_equal(host(y), want, f"n={n} m={m}")
        xd = dev(x)
        sicu.softmax(xd, xd, n, m)
        assert_bits_equal(host(xd), want, f"in place n={n} m={m}")


def test_tail_hard_case(sicu, oracle):
    """A tail element whose exp argument is the one input where the FMA
    build of glibc's expf rounds differently from its plain build."""
    hard = np.array([0xC27C65D9], np.uint32).view(np.float32)[0]
    x = np.zeros(9, np.float32)
    x[8] = hard                          # tail element; the maximum is 0
    y = empty_f32(9)
    sicu.softmax(dev(x), y, 9)
    assert_bits_equal(host(y), oracle.softmax(x), "hard tail case")

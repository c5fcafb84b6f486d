"""The attention softmax (src/engine.c:124-130, src/kernels.c:855-890): the
oracle's restatement against the reference build, the restated libm expf
the device uses for the n % 8 tail against the host's expf, and the table
it reads against its definition."""

from __future__ import annotations

import re
import struct
from decimal import Decimal, getcontext
from pathlib import Path

import numpy as np
import pytest

SRC = Path(__file__).resolve().parents[1] / "siphon_b200" / "csrc" / "softmax.cu"


def _rows(seed=0):
    rng = np.random.default_rng(seed)
    rows = []
    for n in list(range(1, 40)) + [127, 128, 129, 511, 1000, 2047, 2048]:
        for s in (0.05, 3.0, 40.0):
            rows.append((rng.standard_normal(n) * s).astype(np.float32))
    x = rng.standard_normal(37).astype(np.float32)
    x[[3, 20]] = -np.inf                       # masked positions: exp -> 0
    rows.append(x)
    rows.append(np.full(19, 2.5, np.float32))  # all equal
    return rows


def test_oracle_softmax_matches_reference(oracle, reference):
    for i, x in enumerate(_rows()):
        a, b = oracle.softmax(x), reference.softmax(x)
        assert (a.view(np.uint32) == b.view(np.uint32)).all(), f"row {i} (n={x.size})"


def test_exp2_table_is_its_definition():
    tab = [int(v.rstrip("ul"), 16) for v in re.findall(r"0x[0-9a-f]+ull", re.search(
        r"kExp2Tab\[32\] = \{(.*?)\};", SRC.read_text(), re.S).group(1))]
    assert len(tab) == 32
    getcontext().prec = 60
    ln2 = Decimal(2).ln()
    for i, t in enumerate(tab):
        d = float((Decimal(i) / 32 * ln2).exp())          # correctly rounded
        bits = struct.unpack("<Q", struct.pack("<d", d))[0]
        assert t == (bits - (i << 47)) & (2 ** 64 - 1), i


def test_restated_expf_matches_host_libm(oracle):
    """The algorithm the device uses for the softmax tail, on a stride of the
    negative floats down to the underflow bound (every one of them agrees in
    a full sweep) and of the positives up to overflow."""
    lib = oracle.lib
    assert lib.orc_expf_restated_mismatches(0x80000000, 0xC2CFF1B4, 97) == 0
    assert lib.orc_expf_restated_mismatches(0x00000000, 0x42B17217, 101) == 0
    assert lib.orc_expf_restated_mismatches(0xC27C65D0, 0xC27C65E0, 1) == 0   # a hard case of the FMA build

"""The oracle restatement reproduces fixtures produced by the reference itself
(tests/golden/gen_golden.py ran the reference built from its own sources)."""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

from siphon_b200 import quant as Q


def test_quantizers_match_golden(oracle, golden_dir):
    g = np.load(golden_dir / "quant.npz")
    for i, row in enumerate(g["x"]):
        assert (oracle.quant_q8_K(row) == g["q8_K"][i]).all(), f"q8_K row {i}"
        assert (oracle.quant_q8_0(row) == g["q8_0"][i]).all(), f"q8_0 row {i}"


@pytest.mark.parametrize("wt", Q.WEIGHT_TYPES, ids=lambda t: Q.NAMES[t])
def test_dots_match_golden(oracle, golden_dir, wt):
    g = np.load(golden_dir / f"dot_{Q.NAMES[wt]}.npz")
    n_in, n_out = int(g["n_in"]), int(g["n_out"])
    for i, x in enumerate(g["x"]):
        xq = oracle.quantize_pair(wt, x)[0]
        assert (xq == g["xq"][i]).all()
        y = oracle.gemv(wt, g["w"], n_in, n_out, xq)
        assert (y.view(np.uint32) == g["y_scalar"][i].view(np.uint32)).all()


def test_dequant_matches_golden(oracle, golden_dir):
    g = np.load(golden_dir / "dequant.npz")
    for wt in Q.WEIGHT_TYPES:
        w, y = g[f"w_{wt}"], g[f"y_{wt}"]
        rb = Q.row_bytes(wt, 512)
        for r in range(2):
            got = oracle.dequant_row(wt, w[r * rb:(r + 1) * rb], 512)
            assert (got.view(np.uint32) == y[r].view(np.uint32)).all(), Q.NAMES[wt]


def test_f16_conversions_match_golden(oracle, golden_dir):
    g = np.load(golden_dir / "f16.npz")
    got = np.array([oracle.f32_to_f16(float(v)) for v in g["f32"]], np.uint16)
    assert (got == g["f16"]).all()
    table = np.array([oracle.f16_to_f32(i) for i in range(65536)], np.float32)
    assert hashlib.sha256(table.tobytes()).hexdigest() == str(g["table_sha256"])


def test_activation_steps_match_golden(oracle, golden_dir):
    g = np.load(golden_dir / "steps.npz")
    ex = g["ex"]
    assert (np.array([oracle.expf(float(v)) for v in ex], np.float32).view(np.uint32) == g["expf"].view(np.uint32)).all()
    assert (np.array([oracle.silu(float(v)) for v in ex], np.float32).view(np.uint32) == g["silu"].view(np.uint32)).all()
    for rows, scales in ((g["rows256"], g["scale256"]), (g["rows5120"], g["scale5120"])):
        for i, r in enumerate(rows):
            got = np.array([oracle.rms_scale(r, float(e)) for e in g["eps"]], np.float32)
            assert (got.view(np.uint32) == scales[i].view(np.uint32)).all(), f"row {i}"


def test_halfway_rows_depend_on_summation_order(golden_dir):
    """The fixture's last two rows hold the same values, yet the reference's
    scales differ: a kernel must follow the reference's sequential sum there,
    not any exact or reordered sum."""
    g = np.load(golden_dir / "steps.npz")
    rows, sc = g["rows256"], g["scale256"]
    a, c = rows[-2], rows[-1]
    assert sorted(a.tolist()) == sorted(c.tolist())
    assert (sc[-2] != sc[-1]).all()

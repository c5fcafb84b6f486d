"""Synthetic GGUF models: the weight quantizers are faithful and the files
load and run in the reference's own engine (CPU backend, no GPU)."""

from __future__ import annotations

import numpy as np
import pytest

from siphon_b200 import quant as Q
from siphon_b200 import synth_model, wquant


@pytest.mark.parametrize("wt", (Q.Q4_K, Q.Q6_K, Q.Q8_0), ids=lambda t: Q.NAMES[t])
def test_weight_quantizers_roundtrip(oracle, wt):
    rng = np.random.default_rng(0)
    x = (rng.standard_normal((4, 1024)) * 0.02).astype(np.float32)
    b = wquant.quantize(wt, x)
    assert b.size == 4 * Q.row_bytes(wt, 1024)
    rb = Q.row_bytes(wt, 1024)
    y = np.stack([oracle.dequant_row(wt, b[i * rb:(i + 1) * rb], 1024) for i in range(4)])
    assert np.isfinite(y).all()
    rel = np.linalg.norm(y - x) / np.linalg.norm(x)
    assert rel < {Q.Q4_K: 0.12, Q.Q6_K: 0.03, Q.Q8_0: 0.01}[wt]


@pytest.fixture(scope="module")
def small_model(tmp_path_factory):
    return synth_model.write_llama(tmp_path_factory.mktemp("m") / "small.gguf", synth_model.SMALL, seed=3)


def test_small_model_runs_in_reference_engine(small_model):
    from oracle.oracle import E2E_SO, RefEngine
    if not E2E_SO.exists():
        pytest.skip("reference engine harness not built")
    e = RefEngine(small_model, use_cuda=False, n_ctx=64, scalar=True)
    try:
        assert e.n_vocab == synth_model.SMALL.n_vocab
        for tok in (1, 17, 900):
            logits = e.forward(tok)
            assert np.isfinite(logits).all() and logits.std() > 0
    finally:
        e.close()

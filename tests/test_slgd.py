"""SLGD v1 logit dumps and the golden protocol (siphon_b200/slgd.py), checked
against the reference's own `run --golden` (src/cmd_run.c:132-248), built
unmodified from its sources into oracle/_ref/siphon."""

from __future__ import annotations

import os
import re
import struct
import subprocess

import numpy as np
import pytest

from siphon_b200 import slgd, synth_model

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CLI = os.path.join(ROOT, "oracle", "_ref", "siphon")


def test_file_layout_round_trip(tmp_path):
    toks = [5, 1, 9]
    lg = np.arange(12, dtype=np.float32).reshape(3, 4) - 3.5
    p = slgd.write(tmp_path / "a.slgd", toks, lg, n_prompt=2)
    raw = p.read_bytes()
    assert raw[:20] == b"SLGD" + struct.pack("<IIII", 1, 3, 2, 4)
    assert raw[20:32] == np.array(toks, "<i4").tobytes()
    assert raw[32:] == lg.astype("<f4").tobytes()
    g = slgd.read(p)
    assert g.n_prompt == 2 and g.n_total == 3 and g.n_vocab == 4
    assert (g.tokens == toks).all() and (g.logits == lg).all()
    p.write_bytes(raw[:-4])
    with pytest.raises(ValueError, match="truncated logits"):
        slgd.read(p)
    p.write_bytes(b"XLGD" + raw[4:])
    with pytest.raises(ValueError, match="not an SLGD"):
        slgd.read(p)


def test_verify_statistics_and_acceptance():
    rng = np.random.default_rng(0)
    lg = rng.standard_normal((30, 50)).astype(np.float32)
    lg[:, 7] += 6.0                       # a clear winner everywhere: gap > 1
    g = slgd.Golden(10, np.arange(30, dtype=np.int32), lg)
    v = slgd.verify(lambda t: lg[t], g)
    assert v.passed and v.prefill_max == 0 and v.flips == 0 and v.threshold == 1.0
    bump = lg.copy()
    bump[3, 2] += 0.5                     # prompt position: counted in the prefill max
    bump[12, 7] -= 20.0                   # generated position inside the window: a real flip
    v = slgd.verify(lambda t: bump[t], g)
    assert v.prefill_max == pytest.approx(0.5, rel=1e-6)
    assert v.decode_max == pytest.approx(20.0, rel=1e-6)
    assert v.flips == 1 and v.real_flips == 1 and not v.passed
    short = slgd.Golden(8, g.tokens[:16], lg[:16])
    assert slgd.verify(lambda t: lg[t], short).threshold == 0.6


def _cli(golden, model, scalar=True):
    env = dict(os.environ, SI_SCALAR="1" if scalar else "0")
    r = subprocess.run([CLI, "run", "--golden", str(golden), "--ctx", "256", "-t", "2", str(model)],
                       capture_output=True, text=True, env=env, timeout=300)
    return r.returncode, r.stdout


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    return synth_model.write_llama(tmp_path_factory.mktemp("m") / "small.gguf", synth_model.SMALL, seed=7)


def test_reference_cli_accepts_our_dump(tmp_path, model):
    """A golden recorded through the reference engine (CPU backend) and
    written by slgd.write passes the reference's own verification with zero
    difference, and slgd.verify reports the same."""
    if not os.path.exists(CLI):
        pytest.skip("reference CLI oracle/_ref/siphon not built")
    from oracle.oracle import RefEngine
    prompt = np.random.default_rng(3).integers(0, synth_model.SMALL.n_vocab, 8).tolist()
    eng = RefEngine(model, use_cuda=False, n_ctx=256, scalar=True)
    try:
        g = slgd.record(eng.forward, prompt, 8)
    finally:
        eng.close()
    path = slgd.write(tmp_path / "cpu.slgd", g.tokens, g.logits, g.n_prompt)
    rc, out = _cli(path, model)
    assert rc == 0, out
    assert "result: PASS" in out and re.search(r"prefill logits: max abs diff 0\.0000", out), out
    eng = RefEngine(model, use_cuda=False, n_ctx=256, scalar=True)
    try:
        v = slgd.verify(eng.forward, slgd.read(path))
    finally:
        eng.close()
    assert v.passed and v.prefill_max == 0.0 and v.decode_max == 0.0 and v.flips == 0

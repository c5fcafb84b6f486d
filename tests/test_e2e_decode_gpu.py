"""End-to-end greedy decode through the reference's own engine
(si_engine_forward): every layer's matvec on the CUDA backend adapter versus
the reference CPU backend, on a synthetic llama model (N(0,0.02) weights,
Q4_K_M-style mix). A 32-token seeded prompt, then 128 greedy tokens: the
logits of every step must be bit-identical, hence so are the tokens."""

from __future__ import annotations

import numpy as np
import pytest

from siphon_b200 import synth_model
from tests.gpu_util import assert_bits_equal

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    return synth_model.write_llama(tmp_path_factory.mktemp("m") / "small.gguf", synth_model.SMALL, seed=7)


def test_greedy_decode_128_tokens_token_identical(sicu, model):
    from oracle.oracle import RefEngine
    rng = np.random.default_rng(11)
    prompt = rng.integers(0, synth_model.SMALL.n_vocab, 32).tolist()
    cpu = RefEngine(model, use_cuda=False, n_ctx=256, scalar=True)
    gpu = RefEngine(model, use_cuda=True, n_ctx=256, scalar=True)
    assert cpu.kern_impl == "scalar"
    try:
        tokens_cpu, tokens_gpu = [], []
        tok_c = tok_g = None
        for step in range(32 + 128):
            feed_c = prompt[step] if step < 32 else tok_c
            feed_g = prompt[step] if step < 32 else tok_g
            lc, lg = cpu.forward(feed_c), gpu.forward(feed_g)
            assert_bits_equal(lg, lc, f"logits at step {step}")
            tok_c, tok_g = int(np.argmax(lc)), int(np.argmax(lg))   # greedy: first maximum
            if step >= 32:
                tokens_cpu.append(tok_c)
                tokens_gpu.append(tok_g)
        assert tokens_gpu == tokens_cpu
        assert len(set(tokens_cpu)) > 1
    finally:
        cpu.close()
        gpu.close()


def test_cuda_backend_dump_passes_reference_golden_check(sicu, model, tmp_path):
    """The reference's golden protocol (src/cmd_run.c:132-248) on a dump made
    through the CUDA backend: the reference CLI (CPU backend, scalar kernels)
    teacher-forces its tokens and finds every logit identical."""
    import os
    import subprocess
    from oracle.oracle import RefEngine
    from siphon_b200 import slgd
    cli = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref", "siphon")
    if not os.path.exists(cli):
        pytest.skip("reference CLI oracle/_ref/siphon not built")
    prompt = np.random.default_rng(5).integers(0, synth_model.SMALL.n_vocab, 16).tolist()
    gpu = RefEngine(model, use_cuda=True, n_ctx=256, scalar=True)
    try:
        g = slgd.record(gpu.forward, prompt, 32)
    finally:
        gpu.close()
    path = slgd.write(tmp_path / "gpu.slgd", g.tokens, g.logits, g.n_prompt)
    r = subprocess.run([cli, "run", "--golden", str(path), "--ctx", "256", "-t", "2", str(model)],
                       capture_output=True, text=True, env=dict(os.environ, SI_SCALAR="1"), timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "result: PASS" in r.stdout
    assert "prefill logits: max abs diff 0.0000" in r.stdout
    assert "decode  logits: max abs diff 0.0000" in r.stdout
    assert "argmax flips: 0 total" in r.stdout

"""End-to-end greedy decode against the reference's own engine
(si_engine_forward, src/engine.c:288-398) run on the CPU with its scalar
kernels (the parity target), on synthetic llama models (N(0,0.02) weights,
Q4_K_M-style mix, seeded norm weights):

* the reference engine with the CUDA backend adapter: every layer's products,
  the embedding lookup (src/engine.c:302) and the output head (:393) on the
  GPU, the rest of the engine on the host;
* the device-resident decode loop (siphon_b200.model_path.MatrixPath with the
  model file's tensors): every step of the forward pass and the greedy choice
  on the GPU, the chosen token fed back on the device.

A 32-token seeded prompt, then 128 greedy tokens: the logits of every step
must be bit-identical to the reference engine's, hence so are the tokens
(greedy = the first maximum, src/sampler.c:6-12). Run on the TinyLlama-1.1B
shape (22 layers, d_model 2048, 32000-row Q6_K head) and on a small model.
"""

from __future__ import annotations

import numpy as np
import pytest

from siphon_b200 import synth_model
from tests.gpu_util import assert_bits_equal

pytestmark = pytest.mark.gpu

N_PROMPT, N_GEN = 32, 128
N_CTX = 256


def _reference_run(path, sh, seed):
    """Prompt tokens, the reference CPU engine's logits of every step, and the
    greedy token after every step."""
    from oracle.oracle import RefEngine
    prompt = np.random.default_rng(seed).integers(0, sh.n_vocab, N_PROMPT).tolist()
    cpu = RefEngine(path, use_cuda=False, n_ctx=N_CTX, scalar=True)
    assert cpu.kern_impl == "scalar"
    logits, greedy = [], []
    try:
        tok = None
        for step in range(N_PROMPT + N_GEN):
            lc = cpu.forward(prompt[step] if step < N_PROMPT else tok)
            tok = int(np.argmax(lc))           # first maximum, like si_sample_greedy
            logits.append(lc)
            greedy.append(tok)
    finally:
        cpu.close()
    assert len(set(greedy[N_PROMPT:])) > 1
    return {"prompt": prompt, "logits": logits, "greedy": greedy}


@pytest.fixture(scope="module")
def small(tmp_path_factory):
    path = synth_model.write_llama(tmp_path_factory.mktemp("m") / "small.gguf", synth_model.SMALL, seed=7)
    return path, synth_model.SMALL, _reference_run(path, synth_model.SMALL, 11)


@pytest.fixture(scope="module")
def small_qwen(tmp_path_factory):
    """A small Qwen2-architecture model: Q/K/V biases, half-split RoPE."""
    path = synth_model.write_llama(tmp_path_factory.mktemp("m") / "qwen.gguf", synth_model.SMALL_QWEN, seed=9)
    return path, synth_model.SMALL_QWEN, _reference_run(path, synth_model.SMALL_QWEN, 17)


@pytest.fixture(scope="module")
def tinyllama(tmp_path_factory):
    sh = synth_model.TINYLLAMA
    path = synth_model.write_llama(tmp_path_factory.mktemp("m") / "tinyllama.gguf", sh, seed=7)
    return path, sh, _reference_run(path, sh, 13)


def _reference_engine_on_cuda(model):
    from oracle.oracle import RefEngine
    path, sh, ref = model
    gpu = RefEngine(path, use_cuda=True, n_ctx=N_CTX, scalar=True)
    try:
        tok = None
        for step in range(N_PROMPT + N_GEN):
            lg = gpu.forward(ref["prompt"][step] if step < N_PROMPT else tok)
            assert_bits_equal(lg, ref["logits"][step], f"logits at step {step}")
            tok = int(np.argmax(lg))
            assert tok == ref["greedy"][step]
    finally:
        gpu.close()


def _device_resident_loop(sicu, model):
    import torch
    from siphon_b200 import model_path as mp
    path, sh, ref = model
    m = mp.MatrixPath(sicu, sh, torch.device("cuda", 0), embed=True, n_ctx=N_CTX, gguf_path=path)
    stream = torch.cuda.Stream()
    try:
        for step in range(N_PROMPT + N_GEN):
            if step >= N_PROMPT:         # the token the previous step chose, on the device
                assert int(m.token.cpu()[0]) == ref["greedy"][step - 1]
            m.pos = step
            with torch.cuda.stream(stream):
                if step < N_PROMPT:
                    m.token.fill_(ref["prompt"][step])
                m.decode_step(stream)
            torch.cuda.synchronize()
            assert_bits_equal(m.y["head"][0].cpu().numpy(), ref["logits"][step], f"logits at step {step}")
        assert int(m.token.cpu()[0]) == ref["greedy"][-1]
        assert sicu.status() == 0
    finally:
        m.close()


def test_reference_engine_cuda_backend_small(sicu, small):
    _reference_engine_on_cuda(small)


def test_device_resident_loop_small(sicu, small):
    _device_resident_loop(sicu, small)


def test_reference_engine_cuda_backend_qwen2(sicu, small_qwen):
    _reference_engine_on_cuda(small_qwen)


def test_device_resident_loop_qwen2(sicu, small_qwen):
    """Qwen2 architecture: the Q/K/V bias adds ride in the QKV product's
    epilogue, RoPE in the half-split form."""
    _device_resident_loop(sicu, small_qwen)


def test_reference_engine_cuda_backend_tinyllama(sicu, tinyllama):
    """configs[2] shape: the reference engine's whole 32 + 128-token greedy
    run with every matrix product, the embedding and the head on the GPU."""
    _reference_engine_on_cuda(tinyllama)


def test_device_resident_loop_tinyllama(sicu, tinyllama):
    """configs[2] shape: the decode loop the benchmark times (every step on
    the device, tokens chosen and fed back there), 32 + 128 steps."""
    _device_resident_loop(sicu, tinyllama)


def test_cuda_backend_dump_passes_reference_golden_check(sicu, small, tmp_path):
    """The reference's golden protocol (src/cmd_run.c:132-248) on a dump made
    through the CUDA backend: the reference CLI (CPU backend, scalar kernels)
    teacher-forces its tokens and finds every logit identical."""
    import os
    import subprocess
    from oracle.oracle import RefEngine
    from siphon_b200 import slgd
    path, sh, _ = small
    cli = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref", "siphon")
    if not os.path.exists(cli):
        pytest.skip("reference CLI oracle/_ref/siphon not built")
    prompt = np.random.default_rng(5).integers(0, sh.n_vocab, 16).tolist()
    gpu = RefEngine(path, use_cuda=True, n_ctx=N_CTX, scalar=True)
    try:
        g = slgd.record(gpu.forward, prompt, 32)
    finally:
        gpu.close()
    dump = slgd.write(tmp_path / "gpu.slgd", g.tokens, g.logits, g.n_prompt)
    r = subprocess.run([cli, "run", "--golden", str(dump), "--ctx", str(N_CTX), "-t", "2", str(path)],
                       capture_output=True, text=True, env=dict(os.environ, SI_SCALAR="1"), timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "result: PASS" in r.stdout
    assert "prefill logits: max abs diff 0.0000" in r.stdout
    assert "decode  logits: max abs diff 0.0000" in r.stdout
    assert "argmax flips: 0 total" in r.stdout

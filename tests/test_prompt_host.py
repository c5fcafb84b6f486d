"""The host side of MatrixPath.prompt_step on the CPU, with a recording
stand-in for the CUDA library: the order of the library calls per layer
(the reference's per-token order of steps, src/engine.c:290-398, with m rows
at each step), the residual streams used in turn (a norm never writes the
sum over its own input), the chunk's positions and RoPE table rows, the
Qwen2 bias adds, and the argument errors. The numerics are the GPU tests'."""

from __future__ import annotations

import inspect

import pytest

from siphon_b200 import lib
from siphon_b200 import model_path as mp
from siphon_b200 import synth_model as sm


class _Recorder:
    """Every SiphonCuda method: the arguments bound against the real
    signature, recorded, nothing run."""

    def __init__(self):
        self.calls = []

    def __getattr__(self, name):
        sig = inspect.signature(getattr(lib.SiphonCuda, name))

        def call(*a, **k):
            sig.bind(None, *a, **k)
            self.calls.append((name, a, k))
            return 4096 if name == "prefill_pack_bytes" else None
        return call


class _Stream:
    cuda_stream = None


def _path(tmp_path, sh, max_tokens):
    import torch
    path = sm.write_llama(tmp_path / "m.gguf", sh, seed=3)
    rec = _Recorder()
    m = mp.MatrixPath(rec, sh, torch.device("cpu"), embed=True, n_ctx=64, gguf_path=path, max_tokens=max_tokens)
    rec.calls.clear()
    return m, rec


def test_prompt_step_call_order_and_buffers(tmp_path):
    sh = sm.SMALL
    m, rec = _path(tmp_path, sh, 12)
    m.pos = 20
    n = m.prompt_step(_Stream(), 12)
    names = [c[0] for c in rec.calls]
    assert n == len(rec.calls)
    assert names[0] == "row_to_f32_dev" and rec.calls[0][1][5] == 12        # m embedding rows
    assert names[-1] == "argmax" and names[-3] == "rms_norm"
    per_layer = []
    for nm in names[1:-3]:
        if nm.startswith("gemm_prefill"):
            nm = "product"
        if not per_layer or not (nm == "product" and per_layer[-1] == "product"):
            per_layer.append(nm)
    assert per_layer == ["rms_norm", "product", "attention_prompt", "product", "rms_norm", "product", "swiglu",
                         "product"] * sh.n_layer
    norms = [c for c in rec.calls if c[0] == "rms_norm"]
    assert norms[0][2].get("dres") is None                                # layer 0 norms the embedding rows
    for _, a, k in norms[1:]:
        assert k["dsum"] is not None and k["dsum"].data_ptr() != a[0].data_ptr()
        assert k["dres"] is not None
    att = [c for c in rec.calls if c[0] == "attention_prompt"]
    hd = sh.head_dim
    for _, a, k in att:
        assert a[12:14] == (20, 12)                                       # pos0, m
        assert a[5].data_ptr() == m.rope_cos[20].data_ptr() and a[6].data_ptr() == m.rope_sin[20].data_ptr()
        assert a[7:11] == (sh.n_head, sh.n_head_kv, hd, hd)
        assert k["neox"] == sh.neox
    _, a, _ = rec.calls[-2]                                               # the head over the output norm's rows
    assert a[2:4] == (sh.n_embd, sh.n_vocab) and a[4].data_ptr() == m.xn.data_ptr() and a[5] == 12
    assert rec.calls[-1][1][0].data_ptr() == m.y["head"][11].data_ptr()     # the last token's logits


def test_prompt_step_qwen2_bias_adds(tmp_path):
    sh = sm.SMALL_QWEN
    m, rec = _path(tmp_path, sh, 8)
    m.prompt_step(_Stream(), 8)
    names = [c[0] for c in rec.calls]
    adds = [c for c in rec.calls if c[0] == "add_bias"]
    assert len(adds) == 3 * sh.n_layer
    kv = sh.n_head_kv * sh.head_dim
    assert [(a[2], a[3]) for _, a, _ in adds[:3]] == [(sh.n_embd, 8), (kv, 8), (kv, 8)]
    first_att = names.index("attention_prompt")
    assert names[first_att - 3:first_att] == ["add_bias"] * 3                # after Q/K/V, before RoPE
    assert all(k["neox"] for nm, _, k in rec.calls if nm == "attention_prompt")


def test_prompt_step_argument_errors(tmp_path):
    sh = sm.SMALL
    m, _ = _path(tmp_path, sh, 8)
    with pytest.raises(ValueError):
        m.prompt_step(_Stream(), 9)                                       # more than the buffers
    m.pos = 60
    with pytest.raises(ValueError):
        m.prompt_step(_Stream(), 8)                                       # past the context
    m.pos = 0
    with pytest.raises(ValueError):
        m.prompt_step(_Stream(), 0)

"""A decode step of a small llama-shaped model through the device path with
the activation steps fused into the products (MatrixPath(steps=True)):
every layer's residual adds, both RMS norms and SwiGLU run inside the
matvecs that read their results. The oracle replays the same step on the CPU
in the reference's order (src/engine.c:313-389 without attention and RoPE:
Wo reads the same fixed activation on both sides) and the logits, the last
layer's products and the residual stream must agree bit for bit.
"""

from __future__ import annotations

import pytest

from siphon_b200 import model_path as mp
from siphon_b200 import synth_model as sm
from tests.gpu_util import assert_bits_equal, host

pytestmark = pytest.mark.gpu


def _gemv(oracle, wt, w, n_out, a):
    return oracle.gemv(wt, w, a.size, n_out, oracle.quantize_pair(wt, a[None, :])[0])


@pytest.mark.parametrize("shape", [sm.SMALL, sm.LlamaShape(2, 1024, 2816, 16, 4, 2048, 10000.0, 1e-6, 1024)],
                         ids=["small", "wide"])
def test_decode_step_with_steps_matches_oracle(sicu, oracle, shape):
    import torch
    dev = torch.device("cuda", 0)
    m = mp.MatrixPath(sicu, shape, dev, seed=3, steps=True)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        m.decode_step(stream)
    torch.cuda.synchronize()
    assert sicu.status() == 0

    eps, d = shape.rms_eps, shape.n_embd
    cur, res = host(m.x_model[0]), None
    x_attn = host(m.x_attn[0])
    for il, lay in enumerate(m.layers):
        W = {k: (t, host(w)) for k, (t, w) in lay.items()}
        h, a = oracle.rms_norm(cur, host(m.attn_norm[il]), eps, res)
        q = _gemv(oracle, *W["q"], m.shapes["q"][0], a)
        k = _gemv(oracle, *W["k"], m.shapes["k"][0], a)
        v = _gemv(oracle, *W["v"], m.shapes["v"][0], a)
        o = _gemv(oracle, *W["o"], d, x_attn)
        h2, a2 = oracle.rms_norm(h, host(m.ffn_norm[il]), eps, o)
        gate = _gemv(oracle, *W["gate"], m.shapes["gate"][0], a2)
        up = _gemv(oracle, *W["up"], m.shapes["up"][0], a2)
        down = _gemv(oracle, *W["down"], d, oracle.swiglu(gate, up))
        cur, res = h2, down
    _, a = oracle.rms_norm(cur, host(m.out_norm), eps, res)
    logits = _gemv(oracle, m.head[0], host(m.head[1]), m.shapes["head"][0], a)

    silu_gate = oracle.silu_vec(gate)            # the gate product writes silu(gate)
    for name, want in (("q", q), ("k", k), ("v", v), ("o", o), ("gate", silu_gate), ("up", up), ("down", down)):
        assert_bits_equal(host(m.y[name][0]), want, f"last layer {name}")
    assert_bits_equal(host(m.resid[1]), cur, "residual stream")
    assert_bits_equal(host(m.y["head"][0]), logits, "logits")
    m.close()

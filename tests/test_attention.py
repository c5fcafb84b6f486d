"""The oracle's restatement of the reference's attention step (rope_apply,
attn_head on the scalar f16 dot, src/engine.c:42-147) checked against the
reference build's own pieces: its si_dot_f16 for every score and value dot,
its si_softmax with its row-max loop, its f32 -> f16 conversion."""

from __future__ import annotations

import numpy as np

from siphon_b200 import quant as Q


def random_cache(rng, n_head_kv, hd, n_ctx, scale=1.0):
    k = (rng.standard_normal((n_head_kv, n_ctx, hd)) * scale).astype(np.float16).view(np.uint16)
    v = (rng.standard_normal((n_head_kv, hd, n_ctx)) * scale).astype(np.float16).view(np.uint16)
    return k, v


def test_attention_matches_reference_pieces(oracle, reference):
    rng = np.random.default_rng(4)
    n_head, n_head_kv, hd, n_ctx = 4, 2, 64, 96
    k, v = random_cache(rng, n_head_kv, hd, n_ctx)
    q = (rng.standard_normal(n_head * hd) * 2).astype(np.float32)
    ks = np.float32(1.0 / np.sqrt(hd))
    for pos in (0, 7, 40, 95):
        got = oracle.attention(q, k, v, n_head, n_head_kv, hd, n_ctx, pos, float(ks))
        want = np.zeros_like(got)
        for h in range(n_head):
            hk = h // (n_head // n_head_kv)
            q16 = reference.convert_f16(q[h * hd:(h + 1) * hd])
            sc = np.array([reference.vec_dot(Q.F16, hd, np.ascontiguousarray(k[hk, j]).view(np.uint8), q16)
                           for j in range(pos + 1)], np.float32) * ks
            pr16 = reference.convert_f16(reference.softmax(sc))
            for c in range(hd):
                want[h * hd + c] = reference.vec_dot(Q.F16, pos + 1,
                                                     np.ascontiguousarray(v[hk, c, :pos + 1]).view(np.uint8), pr16)
        assert (got.view(np.uint32) == want.view(np.uint32)).all(), pos


def test_rope_forms():
    """Both rotation forms on a hand-checked pair (the oracle's rope_apply)."""
    from oracle.oracle import Oracle
    o = Oracle()
    x = np.array([1.0, 2.0, 3.0, 4.0], np.float32)
    c, s = np.array([0.5, 0.25], np.float32), np.array([0.75, -1.0], np.float32)
    inter = o.rope(x, 1, 4, 4, c, s, neox=False)
    assert inter.tolist() == [1 * 0.5 - 2 * 0.75, 1 * 0.75 + 2 * 0.5, 3 * 0.25 + 4 * 1.0, 3 * -1.0 + 4 * 0.25]
    neox = o.rope(x, 1, 4, 4, c, s, neox=True)
    assert neox.tolist() == [1 * 0.5 - 3 * 0.75, 2 * 0.25 + 4 * 1.0, 1 * 0.75 + 3 * 0.5, 2 * -1.0 + 4 * 0.25]

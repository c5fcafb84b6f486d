"""Host-side helpers: geometry mirror, byte model, seeded synthetic inputs."""

from __future__ import annotations

import numpy as np

from siphon_b200 import quant as Q
from siphon_b200 import synth


def test_geometry_matches_oracle(oracle):
    import ctypes as C
    for t, (blck, size) in Q.GEOMETRY.items():
        b, s = C.c_uint32(), C.c_uint32()
        assert oracle.lib.orc_geometry(t, C.byref(b), C.byref(s)) == 1
        assert (b.value, s.value) == (blck, size)


def test_matvec_byte_model_configs0():
    # Q4_K 5632x2048 batch 1: weights + Q8_K activation + f32 out + f32 in
    assert Q.matvec_bytes(Q.Q4_K, 5632, 2048) == 6_521_120


def test_synthetic_weights_are_seeded_and_scaled():
    a = synth.weights(Q.Q4_K, 8, 512, seed=3)
    b = synth.weights(Q.Q4_K, 8, 512, seed=3)
    assert (a == b).all() and a.size == 8 * Q.row_bytes(Q.Q4_K, 512)
    d = a.reshape(-1, 144)[:, 0:2].copy().view(np.float16).astype(np.float32)
    assert (d >= 1e-4 * 0.999).all() and (d <= 1e-2 * 1.001).all()
    f = synth.weights(Q.F16, 4, 64, seed=1).view(np.float16)
    assert np.isfinite(f).all() and np.abs(f).max() <= 1.0


def test_rope_tables_match_engine_restatement(oracle):
    """The device decode loop's RoPE tables are the reference engine's
    (src/engine.c:26-40, 196) bit for bit, for both benchmark bases."""
    from siphon_b200 import model_path as mp
    from siphon_b200 import synth_model as sm
    for sh in (sm.TINYLLAMA, sm.QWEN25_32B, sm.SMALL):
        cos, sin = mp.rope_tables(sh, 300)
        want_c, want_s = oracle.rope_table(sh.rope_base, sh.head_dim, 300)
        assert (cos.view(np.uint32) == want_c.view(np.uint32)).all()
        assert (sin.view(np.uint32) == want_s.view(np.uint32)).all()


def test_gguf_reader_round_trip(tmp_path):
    """The GGUF writer's file reads back through the reader: key-values,
    tensor dims, types and bytes."""
    from siphon_b200 import gguf
    from siphon_b200 import synth_model as sm
    sh = sm.SMALL_QWEN
    path = sm.write_llama(tmp_path / "q.gguf", sh, seed=2)
    r = gguf.Reader(path)
    assert r.kv["general.architecture"] == "qwen2" and r.kv["qwen2.block_count"] == sh.n_layer
    names = [n for n, *_ in sm.matrices(sh)] + [n for n, _ in sm.vectors(sh)]
    assert sorted(r.tensors) == sorted(names)
    for name, wt, n_out, n_in in sm.matrices(sh):
        t = r.tensors[name]
        assert t.type == wt and t.dims == (n_in, n_out) and t.offset % 32 == 0
        assert r.data(name).size == n_out * Q.row_bytes(wt, n_in)
    b = r.data("blk.1.attn_k.bias").view(np.float32)
    assert b.size == sh.n_head_kv * sh.head_dim and 0 < np.abs(b).max() < 0.2
    assert r.data("blk.0.ffn_norm.weight").view(np.float32).std() > 0.01

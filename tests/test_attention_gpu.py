"""RoPE, the f16 KV-cache store and the per-head attention on the device
(sicu_rope, sicu_kv_store, sicu_attention) against the oracle's restatement
of the reference's attention step (src/engine.c:42-147, 336-366; scalar f16
dots), bit for bit."""

from __future__ import annotations

import numpy as np
import pytest

from tests.gpu_util import assert_bits_equal, dev, empty_f32, host
from tests.test_attention import random_cache

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("neox", [False, True])
def test_rope(sicu, oracle, neox):
    import torch
    rng = np.random.default_rng(1)
    for n_heads, hd, n_rot in ((32, 64, 64), (8, 128, 128), (4, 128, 64)):
        x = (rng.standard_normal(n_heads * hd) * 3).astype(np.float32)
        theta = rng.uniform(-50, 50, n_rot // 2)
        c, s = np.cos(theta).astype(np.float32), np.sin(theta).astype(np.float32)
        d = dev(x)
        sicu.rope(d, n_heads, hd, n_rot, dev(c), dev(s), neox=neox)
        assert_bits_equal(host(d), oracle.rope(x, n_heads, hd, n_rot, c, s, neox=neox), f"rope {n_heads}x{hd}/{n_rot}")
    del torch


def test_kv_store_layout(sicu, oracle):
    import torch
    rng = np.random.default_rng(2)
    nkv, hd, n_ctx = 3, 64, 40
    kc = torch.zeros(nkv * n_ctx * hd, dtype=torch.int16, device="cuda")
    vc = torch.zeros(nkv * hd * n_ctx, dtype=torch.int16, device="cuda")
    want_k = np.zeros((nkv, n_ctx, hd), np.uint16)
    want_v = np.zeros((nkv, hd, n_ctx), np.uint16)
    for pos in (0, 5, 39):
        k = (rng.standard_normal(nkv * hd) * 4).astype(np.float32)
        v = (rng.standard_normal(nkv * hd) * 4).astype(np.float32)
        sicu.kv_store(dev(k), dev(v), kc, vc, nkv, hd, n_ctx, pos)
        want_k[:, pos, :] = oracle.convert_f16(k).view(np.uint16).reshape(nkv, hd)
        want_v[:, :, pos] = oracle.convert_f16(v).view(np.uint16).reshape(nkv, hd)
    assert (host(kc).view(np.uint16) == want_k.reshape(-1)).all()
    assert (host(vc).view(np.uint16) == want_v.reshape(-1)).all()


@pytest.mark.parametrize("n_head,n_head_kv,hd,n_ctx", [(8, 2, 64, 512), (32, 8, 128, 2048), (4, 4, 64, 64)])
def test_attention(sicu, oracle, n_head, n_head_kv, hd, n_ctx):
    import torch
    rng = np.random.default_rng(n_ctx + hd)
    k, v = random_cache(rng, n_head_kv, hd, n_ctx)
    kd = torch.from_numpy(k.view(np.int16).reshape(-1).copy()).cuda()
    vd = torch.from_numpy(v.view(np.int16).reshape(-1).copy()).cuda()
    ks = float(np.float32(1.0 / np.sqrt(hd)))
    for pos in sorted({0, 1, 7, 8, 63, n_ctx // 2 + 3, n_ctx - 1}):
        if pos >= n_ctx:
            continue
        q = (rng.standard_normal(n_head * hd) * 2).astype(np.float32)
        out = empty_f32(n_head * hd)
        sicu.attention(dev(q), kd, vd, n_head, n_head_kv, hd, n_ctx, pos, ks, out)
        assert_bits_equal(host(out), oracle.attention(q, k, v, n_head, n_head_kv, hd, n_ctx, pos, ks),
                          f"attention pos {pos}")


@pytest.mark.parametrize("neox", [False, True])
def test_attention_step_equals_separate_launches(sicu, oracle, neox):
    """sicu_attention_step (RoPE, cache store and attention in one launch)
    against the three separate entry points: the same caches and outputs."""
    import torch
    rng = np.random.default_rng(11)
    n_head, nkv, hd, n_ctx = 8, 2, 128, 64
    k0, v0 = random_cache(rng, nkv, hd, n_ctx)
    theta = rng.uniform(-20, 20, hd // 2)
    c, s = dev(np.cos(theta).astype(np.float32)), dev(np.sin(theta).astype(np.float32))
    ks = float(np.float32(1.0 / np.sqrt(hd)))
    for pos in (0, 9, 63):
        q = (rng.standard_normal(n_head * hd) * 2).astype(np.float32)
        k = (rng.standard_normal(nkv * hd) * 2).astype(np.float32)
        v = (rng.standard_normal(nkv * hd) * 2).astype(np.float32)
        kc1 = torch.from_numpy(k0.view(np.int16).reshape(-1).copy()).cuda()
        vc1 = torch.from_numpy(v0.view(np.int16).reshape(-1).copy()).cuda()
        kc2, vc2 = kc1.clone(), vc1.clone()
        o1, o2 = empty_f32(n_head * hd), empty_f32(n_head * hd)
        qd, kd, vd = dev(q), dev(k), dev(v)
        sicu.attention_step(qd, kd, vd, kc1, vc1, c, s, n_head, nkv, hd, hd, n_ctx, pos, ks, o1, neox=neox)
        q2, k2 = dev(q), dev(k)
        sicu.rope(q2, n_head, hd, hd, c, s, neox=neox)
        sicu.rope(k2, nkv, hd, hd, c, s, neox=neox)
        sicu.kv_store(k2, vd, kc2, vc2, nkv, hd, n_ctx, pos)
        sicu.attention(q2, kc2, vc2, n_head, nkv, hd, n_ctx, pos, ks, o2)
        assert_bits_equal(host(o1), host(o2), f"pos {pos} output")
        assert (host(kc1) == host(kc2)).all() and (host(vc1) == host(vc2)).all(), f"pos {pos} caches"
        assert_bits_equal(host(qd), q, "q left unrotated")


@pytest.mark.parametrize("case", ["parallel", "values_fallback", "scores_fallback", "both_fallback"])
def test_attention_exactness_bound_and_fallback(sicu, oracle, case):
    """The value dots are summed in parallel when no addition can round
    (max|a| * sum|b| below 2^(53 + the smallest last-bit weights)) and
    sequentially otherwise, the scores always sequentially; every form gives
    the reference's bits. Large V values
    (|v| ~ 100 against subnormal probabilities) and a subnormal query
    component with large K values push the bound over."""
    import torch
    rng = np.random.default_rng(31)
    n_head, nkv, hd, n_ctx, pos = 4, 2, 64, 256, 200
    k, v = random_cache(rng, nkv, hd, n_ctx)
    q = (rng.standard_normal(n_head * hd) * 2).astype(np.float32)
    if case in ("values_fallback", "both_fallback"):
        v = (v.view(np.float16).astype(np.float32) * 150).astype(np.float16).view(np.uint16)
    if case in ("scores_fallback", "both_fallback"):
        k = (k.view(np.float16).astype(np.float32) * 200).astype(np.float16).view(np.uint16)
        q[::hd] = 3e-7                                   # a subnormal f16 component in every head
        q = q * np.float32(0.02)                          # keep the scores' softmax spread
    kd = torch.from_numpy(k.view(np.int16).reshape(-1).copy()).cuda()
    vd = torch.from_numpy(v.view(np.int16).reshape(-1).copy()).cuda()
    ks = float(np.float32(1.0 / np.sqrt(hd)))
    out = empty_f32(n_head * hd)
    sicu.attention(dev(q), kd, vd, n_head, nkv, hd, n_ctx, pos, ks, out)
    assert_bits_equal(host(out), oracle.attention(q, k, v, n_head, nkv, hd, n_ctx, pos, ks), case)


@pytest.mark.parametrize("n_head,nkv,hd,n_ctx,neox,n_rot,pos0,m", [
    (8, 2, 128, 96, False, 128, 0, 37),     # 4 heads per KV head
    (8, 2, 128, 96, True, 128, 20, 44),
    (8, 2, 128, 96, False, 64, 5, 1),       # partial rotation, one token
    (32, 4, 64, 160, False, 64, 3, 70),     # TinyLlama's groups of 8
    (10, 2, 128, 100, True, 128, 7, 40),    # groups of 5; V rows not 16-byte aligned
    (4, 4, 64, 64, False, 64, 0, 33),       # no grouping
    (16, 2, 96, 80, False, 96, 1, 30),      # head 96: 4 heads per value task
    (16, 1, 64, 64, False, 64, 2, 20),      # 16 per KV head: the per-head kernel
])
def test_attention_prompt_equals_token_steps(sicu, oracle, n_head, nkv, hd, n_ctx, neox, n_rot, pos0, m):
    """sicu_attention_prompt (m consecutive positions in one call) against m
    sicu_attention_step calls, the engine's token-serial order: the same
    outputs and caches, bit for bit; the last token's heads also against the
    oracle's attention over the final caches. Up to 8 query heads per KV head
    run in the grouped kernel (fma chains over widened f16 values), more in
    the per-head one."""
    import torch
    rng = np.random.default_rng(pos0 * 100 + m)
    k0, v0 = random_cache(rng, nkv, hd, n_ctx)
    theta = rng.uniform(-20, 20, (m, n_rot // 2))
    c = np.cos(theta).astype(np.float32)
    s = np.sin(theta).astype(np.float32)
    ks = float(np.float32(1.0 / np.sqrt(hd)))
    q = (rng.standard_normal((m, n_head * hd)) * 2).astype(np.float32)
    k = (rng.standard_normal((m, nkv * hd)) * 2).astype(np.float32)
    v = (rng.standard_normal((m, nkv * hd)) * 2).astype(np.float32)
    kc1 = torch.from_numpy(k0.view(np.int16).reshape(-1).copy()).cuda()
    vc1 = torch.from_numpy(v0.view(np.int16).reshape(-1).copy()).cuda()
    kc2, vc2 = kc1.clone(), vc1.clone()
    out1 = empty_f32(m, n_head * hd)
    qd, kd, vd = dev(q), dev(k), dev(v)
    sicu.attention_prompt(qd, kd, vd, kc1, vc1, dev(c), dev(s), n_head, nkv, hd, n_rot, n_ctx, pos0, m, ks, out1,
                          neox=neox)
    out2 = np.zeros((m, n_head * hd), np.float32)
    for t in range(m):
        o = empty_f32(n_head * hd)
        sicu.attention_step(dev(q[t]), dev(k[t]), dev(v[t]), kc2, vc2, dev(c[t]), dev(s[t]), n_head, nkv, hd, n_rot,
                            n_ctx, pos0 + t, ks, o, neox=neox)
        out2[t] = host(o)
    assert_bits_equal(host(out1), out2, f"prompt pos0={pos0} m={m} outputs")
    assert (host(kc1) == host(kc2)).all() and (host(vc1) == host(vc2)).all(), "caches"
    assert_bits_equal(host(qd), q, "q left unrotated")
    # the last token's attention, with its q rotated on the host by the oracle
    qr = oracle.rope(q[m - 1], n_head, hd, n_rot, c[m - 1], s[m - 1], neox=neox)
    kf = host(kc1).view(np.uint16).reshape(nkv, n_ctx, hd)
    vf = host(vc1).view(np.uint16).reshape(nkv, hd, n_ctx)
    want = oracle.attention(qr, kf, vf, n_head, nkv, hd, n_ctx, pos0 + m - 1, ks)
    assert_bits_equal(host(out1)[m - 1], want, "last token vs oracle")

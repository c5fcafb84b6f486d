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
from siphon_b200 import quant as Q
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


def _free_port() -> int:
    import socket
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _tp_rank(rank, world, port, q, attention=False):
    """One rank of the tensor-parallel step flow: a decode step with the
    all-reduces fused into Wo / W_down and the steps fused into the products,
    then every rank replays the whole step on the CPU from every rank's shards
    (rank-order f32 sums for the row-split products) and checks its residual
    stream, W_down sum and head shard bit for bit. With attention, two
    consecutive positions run through RoPE, each rank's f16 caches and its
    own heads' attention, and the replay does the same per rank."""
    import datetime
    import os

    import numpy as np
    import torch
    import torch.distributed as dist

    from oracle.oracle import Oracle
    from siphon_b200 import lib

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    m = None
    try:
        s = lib.load()
        s.init(rank)
        orc = Oracle()
        shape = sm.LlamaShape(2, 1024, 2048, 16, 4, 2048, 10000.0, 1e-5, 1024)
        dev = torch.device("cuda", rank)
        n_ctx = 8
        m = mp.MatrixPath(s, shape, dev, world, rank, None, seed=9, fused=True, steps=True, attention=attention,
                          n_ctx=n_ctx)
        st = torch.cuda.Stream(device=dev)
        mine = {"layers": [{k: (t, host(w)) for k, (t, w) in lay.items()} for lay in m.layers],
                "head": (m.head[0], host(m.head[1])), "x_attn": host(m.x_attn[0])}
        shards = [None] * world
        dist.all_gather_object(shards, mine)
        eps, d, hd = shape.rms_eps, shape.n_embd, shape.head_dim
        x0 = host(m.x_model[0])

        def gemv(wt, w, n_out, a):
            return orc.gemv(wt, w, a.size, n_out, orc.quantize_pair(wt, a[None, :])[0])

        def rows(wt, w):
            return w.size // Q.row_bytes(wt, d)

        def rank_sum(parts):
            total = parts[0].copy()
            for p in parts[1:]:
                total = (total + p).astype(np.float32)
            return total

        if attention:
            cos, sin = host(m.rope_cos), host(m.rope_sin)
            caches = []
            for sh in shards:
                nkv = rows(*sh["layers"][0]["k"]) // hd
                caches.append([(np.zeros((nkv, n_ctx, hd), np.uint16), np.zeros((nkv, hd, n_ctx), np.uint16))
                               for _ in range(shape.n_layer)])
        for pos in range(2 if attention else 1):
            m.pos = pos
            with torch.cuda.stream(st):
                m.decode_step(st)
            torch.cuda.synchronize()
            assert s.status() == 0
            cur, res = x0, None
            for il in range(shape.n_layer):
                h, a = orc.rms_norm(cur, host(m.attn_norm[il]), eps, res)
                if attention:
                    xa = []
                    for r, sh in enumerate(shards):
                        lw = sh["layers"][il]
                        nq, nk = rows(*lw["q"]), rows(*lw["k"])
                        nh, nkv = nq // hd, nk // hd
                        qv = orc.rope(gemv(*lw["q"], nq, a), nh, hd, hd, cos[pos], sin[pos])
                        kv = orc.rope(gemv(*lw["k"], nk, a), nkv, hd, hd, cos[pos], sin[pos])
                        vv = gemv(*lw["v"], nk, a)
                        kc, vc = caches[r][il]
                        kc[:, pos, :] = orc.convert_f16(kv).view(np.uint16).reshape(nkv, hd)
                        vc[:, :, pos] = orc.convert_f16(vv).view(np.uint16).reshape(nkv, hd)
                        xa.append(orc.attention(qv, kc, vc, nh, nkv, hd, n_ctx, pos, m.kq_scale))
                else:
                    xa = [sh["x_attn"] for sh in shards]
                o = rank_sum([gemv(*sh["layers"][il]["o"], d, xa[r]) for r, sh in enumerate(shards)])
                h2, a2 = orc.rms_norm(h, host(m.ffn_norm[il]), eps, o)
                parts = []
                for sh in shards:
                    lw = sh["layers"][il]
                    (tg, wg), (tu, wu), (td, wd) = lw["gate"], lw["up"], lw["down"]
                    nff = rows(tg, wg)
                    gate, up = gemv(tg, wg, nff, a2), gemv(tu, wu, nff, a2)
                    parts.append(gemv(td, wd, d, orc.swiglu(gate, up)))
                down = rank_sum(parts)
                cur, res = h2, down
            _, a = orc.rms_norm(cur, host(m.out_norm), eps, res)
            th, wh = shards[rank]["head"]
            logits = gemv(th, wh, rows(th, wh), a)
            if attention:
                assert_bits_equal(host(m.x_attn_buf), xa[rank], f"rank {rank} pos {pos}: attention output")
            assert_bits_equal(host(m.resid[1]), cur, f"rank {rank} pos {pos}: residual stream")
            assert_bits_equal(host(m.y["down"][0]), down, f"rank {rank} pos {pos}: W_down sum")
            assert_bits_equal(host(m.y["head"][0]), logits, f"rank {rank} pos {pos}: head shard")
        torch.cuda.synchronize()
        dist.barrier()
        if rank == 0:
            q.put(("ok", None))
    except BaseException as e:
        q.put(("fail", f"rank {rank}: {type(e).__name__}: {e}"))
        raise
    finally:
        try:
            if m is not None:
                m.close()
        finally:
            dist.destroy_process_group()


@pytest.mark.parametrize("attention", [False, True], ids=["fixed_x_attn", "attention"])
def test_tensor_parallel_step_flow_matches_oracle(attention):
    import torch
    ngpu = torch.cuda.device_count()
    if ngpu < 2:
        pytest.skip("needs two or more GPUs")
    world = 2 if ngpu < 4 else 4
    import torch.multiprocessing as tmp
    ctx = tmp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_rank, args=(r, world, port, q, attention)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    for p in procs:
        if p.is_alive():
            p.kill()
    msgs = []
    while not q.empty():
        msgs.append(q.get())
    assert all(p.exitcode == 0 for p in procs), msgs
    assert ("ok", None) in msgs, msgs


@pytest.mark.parametrize("shape", [sm.SMALL, sm.LlamaShape(2, 1024, 2816, 16, 4, 2048, 10000.0, 1e-6, 1024)],
                         ids=["small", "wide"])
def test_decode_steps_with_attention_match_oracle(sicu, oracle, shape):
    """Three consecutive positions through the device step with attention:
    RoPE on q and k, the f16 caches, each head's attention over the positions
    so far feeding Wo. The oracle replays every step in the reference's order
    (its caches filled the same way) and the logits and the last layer's
    attention output must agree bit for bit at every position."""
    import numpy as np
    import torch
    dev = torch.device("cuda", 0)
    n_ctx = 16
    m = mp.MatrixPath(sicu, shape, dev, seed=5, attention=True, n_ctx=n_ctx)
    stream = torch.cuda.Stream()
    eps, d, hd = shape.rms_eps, shape.n_embd, shape.head_dim
    nh, nkv = m.shapes["q"][0] // hd, m.shapes["k"][0] // hd
    W = [{k: (t, host(w)) for k, (t, w) in lay.items()} for lay in m.layers]
    cos, sin = host(m.rope_cos), host(m.rope_sin)
    kc = [np.zeros((nkv, n_ctx, hd), np.uint16) for _ in m.layers]
    vc = [np.zeros((nkv, hd, n_ctx), np.uint16) for _ in m.layers]
    x0 = host(m.x_model[0])
    for pos in range(3):
        m.pos = pos
        with torch.cuda.stream(stream):
            m.decode_step(stream)
        torch.cuda.synchronize()
        assert sicu.status() == 0
        # the device flow starts every step from the same embedding row
        cur, res = x0, None
        for il, lw in enumerate(W):
            h, a = oracle.rms_norm(cur, host(m.attn_norm[il]), eps, res)
            q = _gemv(oracle, *lw["q"], nh * hd, a)
            k = _gemv(oracle, *lw["k"], nkv * hd, a)
            v = _gemv(oracle, *lw["v"], nkv * hd, a)
            q = oracle.rope(q, nh, hd, hd, cos[pos], sin[pos])
            k = oracle.rope(k, nkv, hd, hd, cos[pos], sin[pos])
            kc[il][:, pos, :] = oracle.convert_f16(k).view(np.uint16).reshape(nkv, hd)
            vc[il][:, :, pos] = oracle.convert_f16(v).view(np.uint16).reshape(nkv, hd)
            att = oracle.attention(q, kc[il], vc[il], nh, nkv, hd, n_ctx, pos, m.kq_scale)
            o = _gemv(oracle, *lw["o"], d, att)
            h2, a2 = oracle.rms_norm(h, host(m.ffn_norm[il]), eps, o)
            gate = _gemv(oracle, *lw["gate"], m.shapes["gate"][0], a2)
            up = _gemv(oracle, *lw["up"], m.shapes["up"][0], a2)
            down = _gemv(oracle, *lw["down"], d, oracle.swiglu(gate, up))
            cur, res = h2, down
        _, a = oracle.rms_norm(cur, host(m.out_norm), eps, res)
        logits = _gemv(oracle, m.head[0], host(m.head[1]), m.shapes["head"][0], a)
        assert_bits_equal(host(m.x_attn_buf), att, f"pos {pos}: last layer's attention output")
        assert_bits_equal(host(m.y["head"][0]), logits, f"pos {pos}: logits")
    m.close()


def test_device_resident_greedy_decode(sicu, oracle):
    """Four greedy tokens with the whole loop on the device: the embedding
    row of the token the previous step chose (sicu_row_to_f32_dev), every
    layer's steps and attention, the head, and the greedy choice
    (sicu_argmax) written back for the next step. The oracle replays each step
    from the same token and must choose the same token with bit-identical
    logits."""
    import numpy as np
    import torch
    shape = sm.SMALL
    dev = torch.device("cuda", 0)
    n_ctx = 16
    m = mp.MatrixPath(sicu, shape, dev, seed=6, embed=True, n_ctx=n_ctx)
    stream = torch.cuda.Stream()
    eps, d, hd = shape.rms_eps, shape.n_embd, shape.head_dim
    nh, nkv = m.shapes["q"][0] // hd, m.shapes["k"][0] // hd
    W = [{k: (t, host(w)) for k, (t, w) in lay.items()} for lay in m.layers]
    emb = host(m.embd)
    rb = Q.row_bytes(Q.Q4_K, d)
    cos, sin = host(m.rope_cos), host(m.rope_sin)
    kc = [np.zeros((nkv, n_ctx, hd), np.uint16) for _ in m.layers]
    vc = [np.zeros((nkv, hd, n_ctx), np.uint16) for _ in m.layers]
    m.token.fill_(123)
    tok = 123
    for pos in range(4):
        m.pos = pos
        with torch.cuda.stream(stream):
            m.decode_step(stream)
        torch.cuda.synchronize()
        assert sicu.status() == 0
        cur, res = oracle.dequant_row(Q.Q4_K, emb[tok * rb:(tok + 1) * rb], d), None
        for il, lw in enumerate(W):
            h, a = oracle.rms_norm(cur, host(m.attn_norm[il]), eps, res)
            q = oracle.rope(_gemv(oracle, *lw["q"], nh * hd, a), nh, hd, hd, cos[pos], sin[pos])
            k = oracle.rope(_gemv(oracle, *lw["k"], nkv * hd, a), nkv, hd, hd, cos[pos], sin[pos])
            v = _gemv(oracle, *lw["v"], nkv * hd, a)
            kc[il][:, pos, :] = oracle.convert_f16(k).view(np.uint16).reshape(nkv, hd)
            vc[il][:, :, pos] = oracle.convert_f16(v).view(np.uint16).reshape(nkv, hd)
            att = oracle.attention(q, kc[il], vc[il], nh, nkv, hd, n_ctx, pos, m.kq_scale)
            o = _gemv(oracle, *lw["o"], d, att)
            h2, a2 = oracle.rms_norm(h, host(m.ffn_norm[il]), eps, o)
            gate = _gemv(oracle, *lw["gate"], m.shapes["gate"][0], a2)
            up = _gemv(oracle, *lw["up"], m.shapes["up"][0], a2)
            cur, res = h2, _gemv(oracle, *lw["down"], d, oracle.swiglu(gate, up))
        _, a = oracle.rms_norm(cur, host(m.out_norm), eps, res)
        logits = _gemv(oracle, m.head[0], host(m.head[1]), m.shapes["head"][0], a)
        assert_bits_equal(host(m.y["head"][0]), logits, f"pos {pos}: logits")
        tok = int(np.argmax(logits))
        assert int(host(m.token)[0]) == tok, f"pos {pos}: greedy token"
    m.close()


def test_argmax_and_device_rows(sicu, oracle):
    import numpy as np
    import torch
    from siphon_b200.lib import STATUS_BAD_ROW
    from tests.gpu_util import dev as todev
    x = np.random.default_rng(3).standard_normal((5, 1000)).astype(np.float32)
    x[1, [10, 500]] = 9.0                       # tie: the first one
    x[2, 0] = np.nan                            # NaN first: 0
    x[3, [7, 8]] = np.nan
    x[4, :] = -np.inf
    out = torch.zeros(5, dtype=torch.int64, device="cuda")
    sicu.argmax(todev(x), 1000, 5, out)
    assert host(out).tolist() == [int(np.argmax(x[0])), 10, 0, int(np.nanargmax(x[3])), 0]
    w = todev(oracle_rows := np.random.default_rng(4).integers(0, 256, Q.row_bytes(Q.Q6_K, 512) * 6, dtype=np.uint8))
    ids = torch.tensor([5, 0, 6], dtype=torch.int64, device="cuda")
    y = torch.empty(3, 512, device="cuda")
    sicu.row_to_f32_dev(Q.Q6_K, w, 512, 6, ids, 3, y)
    rb = Q.row_bytes(Q.Q6_K, 512)
    got = host(y)
    for i, r in enumerate((5, 0)):
        assert (got[i].view(np.uint32) == oracle.dequant_row(Q.Q6_K, oracle_rows[r * rb:(r + 1) * rb], 512).view(np.uint32)).all()
    assert np.isnan(got[2]).all()               # id 6 of 6 rows: out of range
    assert sicu.status() & STATUS_BAD_ROW

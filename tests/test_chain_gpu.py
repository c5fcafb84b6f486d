"""Chains of dependent matvecs in one launch (sicu_chain_*).

Every stage must produce exactly what the separate matvec calls produce, bit
for bit, including stages whose activation is an earlier stage's output (the
grid barrier between stages) and row-split stages with the fused all-reduce.
Expected values come from the oracle, following the same dependencies.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from siphon_b200 import quant as Q
from siphon_b200 import synth
from tests.gpu_util import assert_bits_equal, dev, empty_f32, host

pytestmark = pytest.mark.gpu


def _layer_chain(sicu, oracle, d, ff, nq, nkv, n_layers, seed, group=None):
    """A llama-style chain: per layer QKV (reads the previous FFN output),
    Wo (fixed attention input, row-split when a group is given), gate/up
    (read Wo's output), W_down (reads gate's output); then a Q6_K head.
    Returns (stages, device tensors, host expectation function)."""
    rng = np.random.default_rng(seed)
    mats, stages, expect = [], [], []
    x0 = synth.activations(d, 1, seed=seed)[0]
    xa = synth.activations(nq, 1, seed=seed + 1)[0]
    dx0, dxa = dev(x0), dev(xa)
    keep = [dx0, dxa]
    prev = ("dev", dx0, dx0)
    for il in range(n_layers):
        tv = Q.Q6_K if il % 2 == 0 else Q.Q4_K
        ws = {}
        for name, t, n_out, n_in in (("q", Q.Q4_K, nq, d), ("k", Q.Q4_K, nkv, d), ("v", tv, nkv, d),
                                     ("o", Q.Q4_K, d, nq), ("gate", Q.Q4_K, ff, d), ("up", Q.Q4_K, ff, d),
                                     ("down", tv, d, ff)):
            w = synth.weights(t, n_out, n_in, seed=int(rng.integers(1 << 30)))
            ys = empty_f32(n_out)
            ws[name] = (t, w, dev(w), n_out, n_in, ys)
            keep += [ws[name][2], ys]
        # QKV: one stage per weight type
        groups = [["q", "k", "v"]] if tv == Q.Q4_K else [["q", "k"], ["v"]]
        for g in groups:
            t = ws[g[0]][0]
            stages.append({"wtype": t, "w": [ws[n][2] for n in g], "n_out": [ws[n][3] for n in g],
                           "y": [ws[n][5] for n in g], "n_in": d, "x": prev[2]})
            expect.append((g, ws, prev))
        stages.append({"wtype": Q.Q4_K, "w": [ws["o"][2]], "n_out": [d], "y": [ws["o"][5]], "n_in": nq, "x": dxa,
                       "all_reduce": group is not None})
        expect.append((["o"], ws, ("host", xa, dxa)))
        o_out = ("dev", ws["o"][5], ws["o"][5])
        stages.append({"wtype": Q.Q4_K, "w": [ws["gate"][2], ws["up"][2]], "n_out": [ff, ff],
                       "y": [ws["gate"][5], ws["up"][5]], "n_in": d, "x": ws["o"][5]})
        expect.append((["gate", "up"], ws, o_out))
        g_out = ("dev", ws["gate"][5], ws["gate"][5])
        stages.append({"wtype": tv, "w": [ws["down"][2]], "n_out": [d], "y": [ws["down"][5]], "n_in": ff,
                       "x": ws["gate"][5], "all_reduce": group is not None})
        expect.append((["down"], ws, g_out))
        prev = ("dev", ws["down"][5], ws["down"][5])
    wh = synth.weights(Q.Q6_K, 700, d, seed=seed + 99)
    yh = empty_f32(700)
    dwh = dev(wh)
    keep += [dwh, yh]
    stages.append({"wtype": Q.Q6_K, "w": [dwh], "n_out": [700], "y": [yh], "n_in": d, "x": prev[2]})
    expect.append((["head"], {"head": (Q.Q6_K, wh, dwh, 700, d, yh)}, prev))

    def check(what):
        """Stage by stage: the oracle's matvec of the activation the stage
        read (host copy of the device buffer it names) must equal its outputs."""
        for si, (names, ws, src) in enumerate(expect):
            x = src[1] if src[0] == "host" else host(src[1])
            for n in names:
                t, w, _, n_out, n_in, ys = ws[n]
                want = oracle.gemv(t, w, n_in, n_out, oracle.quantize_pair(t, x[None, :])[0])
                assert_bits_equal(host(ys), want, f"{what}: stage {si} ({n})")

    return stages, keep, check


def test_chain_matches_reference_stage_by_stage(sicu, oracle):
    stages, keep, check = _layer_chain(sicu, oracle, d=1024, ff=2816, nq=1024, nkv=256, n_layers=3, seed=11)
    ch = sicu.chain_create(stages)
    try:
        ch.run()
        check("first run")
        ch.run()                                   # the barrier counter restarts every run
        check("second run")
        assert sicu.status() == 0
    finally:
        ch.destroy()


def test_chain_long_rows_and_ragged_matrices(sicu, oracle):
    """Rows in chunks (36 super-blocks), several matrices of ragged sizes,
    a stage reading its predecessor's output."""
    d1, d2 = 9216, 2304
    w1 = [synth.weights(Q.Q4_K, n, d1, seed=20 + i) for i, n in enumerate((2304, 300, 7))]
    w2 = synth.weights(Q.Q6_K, 1001, d2, seed=30)
    x = synth.activations(d1, 1, seed=31)[0]
    y1 = [empty_f32(n) for n in (2304, 300, 7)]
    y2 = empty_f32(1001)
    dw1, dw2, dx = [dev(w) for w in w1], dev(w2), dev(x)
    stages = [{"wtype": Q.Q4_K, "w": dw1, "n_out": [2304, 300, 7], "y": y1, "n_in": d1, "x": dx},
              {"wtype": Q.Q6_K, "w": [dw2], "n_out": [1001], "y": [y2], "n_in": d2, "x": y1[0]}]
    ch = sicu.chain_create(stages)
    try:
        ch.run()
        xq = oracle.quantize_pair(Q.Q4_K, x[None, :])[0]
        for i, n in enumerate((2304, 300, 7)):
            assert_bits_equal(host(y1[i]), oracle.gemv(Q.Q4_K, w1[i], d1, n, xq), f"stage 0 matrix {i}")
        x2 = host(y1[0])
        want = oracle.gemv(Q.Q6_K, w2, d2, 1001, oracle.quantize_pair(Q.Q6_K, x2[None, :])[0])
        assert_bits_equal(host(y2), want, "stage 1")
        assert sicu.status() == 0
    finally:
        ch.destroy()


def test_chain_replays_in_a_cuda_graph(sicu, oracle):
    import torch
    stages, keep, check = _layer_chain(sicu, oracle, d=768, ff=2048, nq=768, nkv=256, n_layers=2, seed=12)
    ch = sicu.chain_create(stages)
    try:
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            ch.run(stream=s.cuda_stream)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            ch.run(stream=s.cuda_stream)
            ch.run(stream=s.cuda_stream)
        x0 = keep[0]                               # the first stage's activation
        for rep in range(2):
            x0.copy_(torch.from_numpy(synth.activations(768, 1, seed=40 + rep)[0]))
            g.replay()
            torch.cuda.synchronize()
            check(f"graph replay {rep}")
        del g
        assert sicu.status() == 0
    finally:
        ch.destroy()


def test_chain_all_reduce_one_rank(sicu, oracle):
    """Row-split stages with a one-rank group equal the plain products, and
    the group's delivery count stays consistent with sicu_gemv_ar calls."""
    d = 1024
    g = sicu.ar_create(1, 0, d)
    g.open([g.local_handle])
    try:
        stages, keep, check = _layer_chain(sicu, oracle, d=d, ff=2048, nq=1024, nkv=256, n_layers=2, seed=13,
                                           group=g)
        ch = sicu.chain_create(stages, group=g)
        try:
            ch.run()
            check("chain with all-reduce stages")
            w = synth.weights(Q.Q4_K, d, 512, seed=50)
            x = synth.activations(512, 1, seed=51)[0]
            y = empty_f32(d)
            sicu.gemv_ar(Q.Q4_K, dev(w), 512, d, dev(x), y, g)
            want = oracle.gemv(Q.Q4_K, w, 512, d, oracle.quantize_pair(Q.Q4_K, x[None, :])[0])
            assert_bits_equal(host(y), want, "gemv_ar after the chain")
            ch.run()
            check("chain again")
            assert sicu.status() == 0
        finally:
            ch.destroy()
    finally:
        g.destroy()


def test_chain_argument_errors(sicu):
    from siphon_b200.lib import SicuError
    x = empty_f32(256)
    w = dev(synth.weights(Q.Q4_K, 8, 256, seed=1))
    y = empty_f32(8)
    with pytest.raises(SicuError):      # Q8_0 stages are not supported
        sicu.chain_create([{"wtype": Q.Q8_0, "w": [w], "n_out": [8], "y": [y], "n_in": 256, "x": x}])
    with pytest.raises(SicuError):      # an all-reduce stage needs a group
        sicu.chain_create([{"wtype": Q.Q4_K, "w": [w], "n_out": [8], "y": [y], "n_in": 256, "x": x,
                            "all_reduce": True}])
    with pytest.raises(SicuError):      # row length not whole super-blocks
        sicu.chain_create([{"wtype": Q.Q4_K, "w": [w], "n_out": [8], "y": [y], "n_in": 200, "x": x}])
    assert sicu.status() == 0


# ---- several GPUs ---------------------------------------------------------------------

def _free_port() -> int:
    with socket.socket() as so:
        so.bind(("127.0.0.1", 0))
        return so.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, q) -> None:
    """Each rank runs a two-stage chain: its W_down column shard as a row-split
    stage (summed over the group inside the launch), then a column-split
    product reading that sum; three runs, each checked bit for bit."""
    import datetime

    import torch
    import torch.distributed as dist

    from oracle.oracle import Oracle
    from siphon_b200 import lib

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    g = ch = None
    try:
        s = lib.load()
        s.init(rank)
        orc = Oracle()
        d, k, n2 = 1280, 768, 640
        g = s.ar_create(world, rank, d)
        handles = [None] * world
        dist.all_gather_object(handles, g.local_handle)
        g.open(handles)
        g.set_timeout(500_000_000)
        wt = Q.Q4_K if rank % 2 == 0 else Q.Q6_K
        w1 = synth.weights(wt, d, k, seed=200 + rank)
        w2 = synth.weights(Q.Q4_K, n2, d, seed=300 + rank)
        xbuf = torch.zeros(k, dtype=torch.float32, device="cuda")
        y1, y2 = empty_f32(d), empty_f32(n2)
        dw1, dw2 = dev(w1), dev(w2)
        ch = s.chain_create([{"wtype": wt, "w": [dw1], "n_out": [d], "y": [y1], "n_in": k, "x": xbuf,
                              "all_reduce": True},
                             {"wtype": Q.Q4_K, "w": [dw2], "n_out": [n2], "y": [y2], "n_in": d, "x": y1}], group=g)
        for cycle in range(3):
            x = synth.activations(k, 1, seed=500 * cycle + rank)[0]
            xbuf.copy_(torch.from_numpy(x))
            ch.run()
            part = orc.gemv(wt, w1, k, d, orc.quantize_pair(wt, x[None, :])[0])
            parts = [None] * world
            dist.all_gather_object(parts, part)
            total = parts[0].copy()
            for p in parts[1:]:
                total = (total + p).astype(np.float32)
            assert_bits_equal(host(y1), total, f"rank {rank} cycle {cycle}: row-split stage")
            want2 = orc.gemv(Q.Q4_K, w2, d, n2, orc.quantize_pair(Q.Q4_K, total[None, :])[0])
            assert_bits_equal(host(y2), want2, f"rank {rank} cycle {cycle}: next stage")
        assert s.status() == 0
        if rank == 0:
            q.put(("ok", None))
    except BaseException as e:
        q.put(("fail", f"rank {rank}: {type(e).__name__}: {e}"))
        raise
    finally:
        try:
            torch.cuda.synchronize()
            dist.barrier()
            if ch is not None:
                ch.destroy()
            if g is not None:
                g.destroy()
            dist.barrier()
        finally:
            dist.destroy_process_group()


def test_chain_multi_gpu_all_reduce():
    import torch
    ngpu = torch.cuda.device_count()
    if ngpu < 2:
        pytest.skip("needs two or more GPUs")
    world = min(ngpu, 8)
    import torch.multiprocessing as tmp
    ctx = tmp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    msgs = []
    while not q.empty():
        msgs.append(q.get())
    assert all(p.exitcode == 0 for p in procs), msgs
    assert ("ok", None) in msgs, msgs

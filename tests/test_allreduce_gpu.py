"""Fused tensor-parallel all-reduce (sicu_ar_* and sicu_gemv_ar).

The consumed activation is the sum of the ranks' partial vectors added in
rank order in f32, so every result is checked bit for bit: a consumer matvec
against the oracle's matvec of that exact sum, a delivering matvec against
the plain matvec.

One-GPU tests use one-rank groups (the consumer's flag was raised by an
earlier kernel of the same stream, so no kernel waits on a running one).
The multi-rank tests run one process per GPU and are skipped with fewer than
two GPUs; their failure case is a flag that nothing raises (one rank skips a
delivery), which the consumer's bounded wait turns into a status bit.
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

KQ = [Q.Q4_K, Q.Q5_K, Q.Q6_K, Q.Q3_K, Q.Q2_K, Q.Q4_0, Q.Q5_0, Q.Q8_0]


def _group(sicu, length, n=1, rank=0):
    g = sicu.ar_create(n, rank, length)
    g.open([g.local_handle])
    return g


def _plain(sicu, wt, w, n_in, n_out, x):
    y = empty_f32(n_out)
    sicu.gemv_f32(wt, w, n_in, n_out, x, y)
    return host(y)


def test_deliver_then_reduce_is_the_vector(sicu):
    from siphon_b200.lib import SicuError
    g = _group(sicu, 1024)
    try:
        for seed in range(3):                       # both parities, then the first again
            v = synth.activations(1024, 1, seed=seed)[0]
            out = empty_f32(1024)
            g.deliver(dev(v))
            g.reduce(out)
            assert_bits_equal(host(out), v, f"reduce of one rank, delivery {seed}")
        assert sicu.status() == 0
        with pytest.raises(SicuError):
            g.deliver(dev(np.zeros(1024, np.float32))[1:])      # misaligned source
    finally:
        g.destroy()


@pytest.mark.parametrize("wt", KQ)
def test_fused_deliver_and_consume_match_plain_matvecs(sicu, oracle, wt):
    """o-projection style: a delivering matvec (its output must equal the plain
    matvec's) followed by gate/up style consumers of that output."""
    n_in, d = 512, 768
    w_o = synth.weights(wt, d, n_in, seed=31)
    w_g = synth.weights(wt, 300, d, seed=32)
    w_u = synth.weights(wt, 200, d, seed=33)
    x = synth.activations(n_in, 1, seed=34)[0]
    g = _group(sicu, d)
    try:
        dwo, dwg, dwu, dx = dev(w_o), dev(w_g), dev(w_u), dev(x)
        y_o = empty_f32(d)
        sicu.gemv_ar(wt, [dwo], [d], n_in, dx, [y_o], deliver=g)
        yo = host(y_o)
        assert_bits_equal(yo, _plain(sicu, wt, dwo, n_in, d, dx), "delivering matvec")
        y_g, y_u = empty_f32(300), empty_f32(200)
        sicu.gemv_ar(wt, [dwg, dwu], [300, 200], d, None, [y_g, y_u], consume=g)
        xq = oracle.quantize_pair(wt, yo[None, :])[0]
        assert_bits_equal(host(y_g), oracle.gemv(wt, w_g, d, 300, xq), "consumer (gate)")
        assert_bits_equal(host(y_u), oracle.gemv(wt, w_u, d, 200, xq), "consumer (up)")
        assert sicu.status() == 0
    finally:
        g.destroy()


def test_order_violations_break_the_group(sicu):
    from siphon_b200 import lib
    wt, d = Q.Q4_K, 256
    w = dev(synth.weights(wt, d, d, seed=41))
    x = dev(synth.activations(d, 1, seed=42)[0])
    y = empty_f32(d)
    # a consumption before any delivery
    g = _group(sicu, d)
    try:
        sicu.gemv_ar(wt, [w], [d], d, None, [y], consume=g)
        assert sicu.status() & lib.STATUS_AR_ORDER
        # broken from now on: a delivery returns at once with the timeout bit
        sicu.gemv_ar(wt, [w], [d], d, x, [y], deliver=g)
        assert sicu.status() & lib.STATUS_AR_TIMEOUT
    finally:
        g.destroy()
    # two deliveries without a consumption between them
    g = _group(sicu, d)
    try:
        sicu.gemv_ar(wt, [w], [d], d, x, [y], deliver=g)
        assert sicu.status() == 0
        sicu.gemv_ar(wt, [w], [d], d, x, [y], deliver=g)
        assert sicu.status() & lib.STATUS_AR_ORDER
    finally:
        g.destroy()


def test_group_steps_replay_in_a_cuda_graph(sicu, oracle):
    """The counters live on the device: a captured deliver/consume pair
    replays with fresh inputs and stays in step."""
    import torch
    wt, n_in, d, n_out = Q.Q6_K, 1024, 512, 384
    w_o, w_g = synth.weights(wt, d, n_in, seed=51), synth.weights(wt, n_out, d, seed=52)
    dwo, dwg = dev(w_o), dev(w_g)
    xbuf = torch.zeros(n_in, dtype=torch.float32, device="cuda")
    y_o, y_g = empty_f32(d), empty_f32(n_out)
    g = _group(sicu, d)
    try:
        s = torch.cuda.Stream()
        xbuf.copy_(torch.from_numpy(synth.activations(n_in, 1, seed=50)[0]))
        with torch.cuda.stream(s):
            # one eager pair first (also sets the launch attributes)
            sicu.gemv_ar(wt, [dwo], [d], n_in, xbuf, [y_o], deliver=g, stream=s.cuda_stream)
            sicu.gemv_ar(wt, [dwg], [n_out], d, None, [y_g], consume=g, stream=s.cuda_stream)
        s.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            sicu.gemv_ar(wt, [dwo], [d], n_in, xbuf, [y_o], deliver=g, stream=s.cuda_stream)
            sicu.gemv_ar(wt, [dwg], [n_out], d, None, [y_g], consume=g, stream=s.cuda_stream)
        for rep in range(4):
            x = synth.activations(n_in, 1, seed=60 + rep)[0]
            xbuf.copy_(torch.from_numpy(x))
            graph.replay()
            torch.cuda.synchronize()
            yo = host(y_o)
            want_o = oracle.gemv(wt, w_o, n_in, d, oracle.quantize_pair(wt, x[None, :])[0])
            assert_bits_equal(yo, want_o, f"replay {rep}: delivering matvec")
            want_g = oracle.gemv(wt, w_g, d, n_out, oracle.quantize_pair(wt, yo[None, :])[0])
            assert_bits_equal(host(y_g), want_g, f"replay {rep}: consumer")
        del graph
        assert sicu.status() == 0
    finally:
        g.destroy()


# ---- several GPUs: one process per GPU ---------------------------------------------------

def _free_port() -> int:
    with socket.socket() as so:
        so.bind(("127.0.0.1", 0))
        return so.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, q) -> None:
    """One rank: row-split product -> fused all-reduce -> consumer, several
    cycles, each checked bit for bit; then the failure case."""
    import datetime

    import torch
    import torch.distributed as dist

    from oracle.oracle import Oracle
    from siphon_b200 import lib

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    g = None
    try:
        s = lib.load()
        s.init(rank)
        orc = Oracle()
        d, n_ff = 1280, 256 * 3 * world          # model width (5 super-blocks); FFN rows
        g = s.ar_create(world, rank, d)
        handles = [None] * world
        dist.all_gather_object(handles, g.local_handle)
        g.open(handles)
        g.set_timeout(200_000_000)               # 0.2 s
        wt = Q.Q4_K
        # this rank's column shard of W_down (ff slice of 3 super-blocks) and W_gate rows
        w_dn = synth.weights(wt, d, 768, seed=100 + rank)
        w_g = synth.weights(Q.Q6_K, 320, d, seed=200 + rank)
        dw_dn, dw_g = dev(w_dn), dev(w_g)
        y_dn, y_g = empty_f32(d), empty_f32(320)
        out = empty_f32(d)
        for cycle in range(5):
            x = synth.activations(768, 1, seed=1000 * cycle + rank)[0]
            s.gemv_ar(wt, [dw_dn], [d], 768, dev(x), [y_dn], deliver=g)
            s.gemv_ar(Q.Q6_K, [dw_g], [320], d, None, [y_g], consume=g)
            part = host(y_dn)
            want_part = orc.gemv(wt, w_dn, 768, d, orc.quantize_pair(wt, x[None, :])[0])
            assert_bits_equal(part, want_part, f"rank {rank} cycle {cycle}: partial")
            parts = [None] * world
            dist.all_gather_object(parts, part)
            total = parts[0].copy()
            for p in parts[1:]:
                total = (total + p).astype(np.float32)          # rank order, f32
            want_g = orc.gemv(Q.Q6_K, w_g, d, 320, orc.quantize_pair(Q.Q6_K, total[None, :])[0])
            assert_bits_equal(host(y_g), want_g, f"rank {rank} cycle {cycle}: consumer")
            # a standalone consumption of the same delivery gives the sum itself
            g.reduce(out)
            assert_bits_equal(host(out), total, f"rank {rank} cycle {cycle}: reduce")
        assert s.status() == 0
        torch.cuda.synchronize()
        dist.barrier()
        # failure: the last rank skips a delivery; everyone else's consumer
        # gives up after the timeout and reports it
        x = dev(synth.activations(768, 1, seed=7)[0])
        if rank != world - 1:
            s.gemv_ar(wt, [dw_dn], [d], 768, x, [y_dn], deliver=g)
            s.gemv_ar(Q.Q6_K, [dw_g], [320], d, None, [y_g], consume=g)
            st = s.status()
            assert st & lib.STATUS_AR_TIMEOUT, st
        torch.cuda.synchronize()
        dist.barrier()
        if rank == 0:
            q.put(("ok", None))
    except BaseException as e:                     # report, then leave at the barrier below
        q.put(("fail", f"rank {rank}: {type(e).__name__}: {e}"))
        raise
    finally:
        try:
            torch.cuda.synchronize()
            dist.barrier()
            if g is not None:
                g.destroy()
            dist.barrier()
        finally:
            dist.destroy_process_group()


def test_multi_gpu_row_split_allreduce():
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

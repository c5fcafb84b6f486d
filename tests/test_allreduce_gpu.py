"""All-reduce fused into the row-split matvec (sicu_gemv_ar) and the
standalone all-reduce (sicu_ar_allreduce).

The sum over ranks is added in rank order in f32, so every result is checked
bit for bit: sicu_gemv_ar's output against the rank-order sum of the ranks'
partial products, each of which must equal the oracle's matvec of that
rank's shard.

One-GPU tests use one-rank groups (a CTA's wait is for the part it sent
itself). The multi-rank tests run one process per GPU and are skipped with
fewer than two GPUs; their failure case is a part that nobody sends (one
rank skips an operation), which the bounded wait turns into a status bit.
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


def test_allreduce_one_rank_is_identity(sicu):
    from siphon_b200.lib import SicuError
    g = _group(sicu, 1024)
    try:
        for seed in range(3):                       # both buffers, then the first again
            v = synth.activations(1024, 1, seed=seed)[0]
            out = empty_f32(1024)
            g.allreduce(dev(v), out)
            assert_bits_equal(host(out), v, f"one-rank all-reduce {seed}")
        x = dev(synth.activations(1024, 1, seed=9)[0])
        want = host(x).copy()
        g.allreduce(x, x)                           # in place
        assert_bits_equal(host(x), want, "in place")
        assert sicu.status() == 0
        with pytest.raises(SicuError):
            g.allreduce(None, x)
    finally:
        g.destroy()


@pytest.mark.parametrize("wt", KQ)
def test_gemv_ar_one_rank_matches_plain(sicu, oracle, wt):
    n_in, d = 512, 768
    w = synth.weights(wt, d, n_in, seed=31)
    x = synth.activations(n_in, 1, seed=34)[0]
    g = _group(sicu, d)
    try:
        y = empty_f32(d)
        sicu.gemv_ar(wt, dev(w), n_in, d, dev(x), y, g)
        want = oracle.gemv(wt, w, n_in, d, oracle.quantize_pair(wt, x[None, :])[0])
        assert_bits_equal(host(y), want, f"{Q.NAMES[wt]} gemv_ar, one rank")
        assert sicu.status() == 0
    finally:
        g.destroy()


@pytest.mark.parametrize("n_out,n_in", [
    (768, 256),      # 32 rows per task
    (1280, 2304),    # 3 rows per task, the last task partial
    (512, 14336),    # rows in two chunks
])
def test_gemv_ar_row_layouts(sicu, oracle, n_out, n_in):
    """Every row's sum lands where its task put it, for every task shape."""
    wt = Q.Q4_K
    w = synth.weights(wt, n_out, n_in, seed=n_in)
    x = synth.activations(n_in, 1, seed=n_out)[0]
    g = _group(sicu, n_out)
    try:
        y = empty_f32(n_out)
        for _ in range(3):
            sicu.gemv_ar(wt, dev(w), n_in, n_out, dev(x), y, g)
        want = oracle.gemv(wt, w, n_in, n_out, oracle.quantize_pair(wt, x[None, :])[0])
        assert_bits_equal(host(y), want, f"gemv_ar {n_out}x{n_in}")
        assert sicu.status() == 0
    finally:
        g.destroy()


def test_gemv_ar_replays_in_a_cuda_graph(sicu, oracle):
    """The delivery counter lives on the device: a captured row-split product
    followed by a matvec reading its output replays with fresh inputs."""
    import torch
    wt, n_in, d, n_out = Q.Q6_K, 1024, 512, 384
    w_o, w_g = synth.weights(wt, d, n_in, seed=51), synth.weights(wt, n_out, d, seed=52)
    dwo, dwg = dev(w_o), dev(w_g)
    xbuf = torch.zeros(n_in, dtype=torch.float32, device="cuda")
    y_o, y_g = empty_f32(d), empty_f32(n_out)
    g = _group(sicu, d)
    try:
        s = torch.cuda.Stream()

        def step():
            sicu.gemv_ar(wt, dwo, n_in, d, xbuf, y_o, g, stream=s.cuda_stream)
            sicu.gemv_f32(wt, dwg, d, n_out, y_o, y_g, stream=s.cuda_stream)

        with torch.cuda.stream(s):
            step()                                  # eager first: sets the launch attributes
        s.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            step()
            step()
        for rep in range(3):
            x = synth.activations(n_in, 1, seed=60 + rep)[0]
            xbuf.copy_(torch.from_numpy(x))
            graph.replay()
            torch.cuda.synchronize()
            yo = host(y_o)
            want_o = oracle.gemv(wt, w_o, n_in, d, oracle.quantize_pair(wt, x[None, :])[0])
            assert_bits_equal(yo, want_o, f"replay {rep}: row-split product")
            want_g = oracle.gemv(wt, w_g, d, n_out, oracle.quantize_pair(wt, yo[None, :])[0])
            assert_bits_equal(host(y_g), want_g, f"replay {rep}: next product")
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
    """One rank: row-split product with the fused all-reduce, several cycles,
    each checked bit for bit against the rank-order sum; the standalone
    all-reduce; then the failure case."""
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
        d, k = 1280, 768                         # model width; this rank's W_down columns
        g = s.ar_create(world, rank, d)
        handles = [None] * world
        dist.all_gather_object(handles, g.local_handle)
        g.open(handles)
        g.set_timeout(200_000_000)               # 0.2 s
        wt = Q.Q4_K if rank % 2 == 0 else Q.Q6_K  # shards of different types are fine
        w = synth.weights(wt, d, k, seed=100 + rank)
        dw = dev(w)
        y = empty_f32(d)

        def gathered_sum(part):
            parts = [None] * world
            dist.all_gather_object(parts, part)
            total = parts[0].copy()
            for p in parts[1:]:
                total = (total + p).astype(np.float32)          # rank order, f32
            return total

        for cycle in range(5):
            x = synth.activations(k, 1, seed=1000 * cycle + rank)[0]
            s.gemv_ar(wt, dw, k, d, dev(x), y, g)
            part = orc.gemv(wt, w, k, d, orc.quantize_pair(wt, x[None, :])[0])
            assert_bits_equal(host(y), gathered_sum(part), f"rank {rank} cycle {cycle}: gemv_ar")
            v = synth.activations(d, 1, seed=77 + cycle + 10 * rank)[0]
            out = empty_f32(d)
            g.allreduce(dev(v), out)
            assert_bits_equal(host(out), gathered_sum(v), f"rank {rank} cycle {cycle}: allreduce")
        assert s.status() == 0
        torch.cuda.synchronize()
        dist.barrier()
        # failure: the last rank skips an operation; everyone else's wait for
        # its part gives up after the timeout and reports it
        if rank != world - 1:
            s.gemv_ar(wt, dw, k, d, dev(synth.activations(k, 1, seed=7)[0]), y, g)
            st = s.status()
            assert st & lib.STATUS_AR_TIMEOUT, st
            # the group is broken now: the next operation returns at once
            s.gemv_ar(wt, dw, k, d, dev(synth.activations(k, 1, seed=8)[0]), y, g)
            assert s.status() & lib.STATUS_AR_TIMEOUT
        torch.cuda.synchronize()
        dist.barrier()
        if rank == 0:
            q.put(("ok", None))
    except BaseException as e:                     # report, then leave through the barriers below
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

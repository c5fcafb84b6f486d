"""Tensor-parallel layout of the matrix path (CPU: partition logic, and a
two-rank gloo emulation of the row-split product + all-reduce against the
oracle)."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from siphon_b200 import model_path as mp
from siphon_b200 import quant as Q
from siphon_b200 import synth
from siphon_b200 import synth_model as sm


@pytest.mark.parametrize("shape", [sm.TINYLLAMA, sm.LLAMA3_8B, sm.QWEN25_32B, sm.SMALL])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_partition_covers_everything_once(shape, world):
    if world > shape.n_head // (256 // np.gcd(256, shape.head_dim)):
        pytest.skip("more ranks than head units")
    heads, ff, vocab = [], [], []
    for r in range(world):
        s = mp.tp_partition(shape, world, r)
        heads += list(s.heads)
        ff += list(s.ff)
        vocab += list(s.vocab)
        # Wo / W_down column shards are whole super-blocks
        assert (len(s.heads) * shape.head_dim) % 256 == 0
        assert len(s.ff) % 256 == 0 and s.ff.start % 256 == 0
        # every query head's kv head is present
        group = shape.n_head // shape.n_head_kv
        assert {h // group for h in s.heads} == set(s.kv_heads)
    assert heads == list(range(shape.n_head))
    assert ff == list(range(shape.n_ff))
    assert vocab == list(range(shape.n_vocab))


def test_partition_qwen32b_8way_is_uneven_as_required():
    shards = [mp.tp_partition(sm.QWEN25_32B, 8, r) for r in range(8)]
    # 20 super-blocks of Wo's input: 3,3,3,3,2,2,2,2; 108 of W_down's: 14 x 4, 13 x 4
    assert [len(s.heads) * 128 // 256 for s in shards] == [3, 3, 3, 3, 2, 2, 2, 2]
    assert [len(s.ff) // 256 for s in shards] == [14, 14, 14, 14, 13, 13, 13, 13]


def test_step_bytes_match_model_sizes():
    # weight bytes per decode token (whole model, one GPU)
    assert abs(mp.step_weight_bytes(sm.TINYLLAMA) - 0.633e9) < 0.001e9
    assert abs(mp.step_weight_bytes(sm.LLAMA3_8B) - 4.616e9) < 0.001e9
    assert abs(mp.step_weight_bytes(sm.QWEN25_32B) - 19.40e9) < 0.01e9
    # shards add up to the whole (replicated kv heads aside)
    tot = sum(mp.step_weight_bytes(sm.QWEN25_32B, 4, r) for r in range(4))
    assert tot >= mp.step_weight_bytes(sm.QWEN25_32B)


def _free_port() -> int:
    with socket.socket() as so:
        so.bind(("127.0.0.1", 0))
        return so.getsockname()[1]


def _rank_main(rank, world, port, q):
    import torch.distributed as dist
    import torch

    from oracle.oracle import Oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        orc = Oracle()
        wt, n_out, n_in = Q.Q4_K, 48, 1280            # 5 super-blocks: shards 3 + 2
        w = synth.weights(wt, n_out, n_in, seed=5)
        x = synth.activations(n_in, 1, seed=6)
        sbs = mp._split(n_in // 256, world, rank)
        k0, k1 = sbs.start * 256, sbs.stop * 256
        rb = Q.row_bytes(wt, n_in)
        wsh = w.reshape(n_out, rb)[:, sbs.start * 144:sbs.stop * 144].copy().reshape(-1)
        xq = orc.quantize_pair(wt, x[:, k0:k1])
        part = orc.gemv(wt, wsh, k1 - k0, n_out, xq[0])
        t = torch.from_numpy(part.copy())
        dist.all_reduce(t)
        if rank == 0:
            full = orc.gemv(wt, w, n_in, n_out, orc.quantize_pair(wt, x)[0])
            wd = np.stack([orc.dequant_row(wt, w[i * rb:(i + 1) * rb], n_in) for i in range(n_out)]).astype(np.float64)
            xq_full = orc.quantize_pair(wt, x)[0].reshape(-1, 292)
            d = xq_full[:, 0:4].copy().view(np.float32)[:, 0].astype(np.float64)
            xd = (xq_full[:, 4:260].view(np.int8).astype(np.float64) * d[:, None]).reshape(-1)
            l1 = np.abs(wd) @ np.abs(xd)
            q.put((t.numpy(), full, l1))
    finally:
        dist.destroy_process_group()


def test_row_split_allreduce_matches_unsharded():
    import torch.multiprocessing as tmp
    ctx = tmp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got, full, l1 = q.get()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    # the split changes the float summation order only: within 1e-5 of L1
    assert (np.abs(got.astype(np.float64) - full) <= 1e-5 * l1).all()
    # quantizing a 256-aligned slice gives the same blocks as the whole row
    # (blocks are independent), so the integer work is identical

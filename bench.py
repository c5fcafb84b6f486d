#!/usr/bin/env python
"""Q4_K decode-matvec HBM throughput on B200, with the model-level decode and
prefill rates of the quantized matrix path beside it.

Headline workload (the Q4_K leg of the per-format matvec sweep): batch-1
matvecs y = W x with W a random Q4_K matrix of shape (rows x K) 4096x4096,
14336x4096 and 4096x14336, x ~ N(0,1) f32 quantized to Q8_K. One step streams
every weight copy of every shape once: each shape rotates through distinct
device copies totalling >= 4x the L2 size, so no step reads weights from L2.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python bench.py --case NAME      # one small profiling workload (below)

Under torchrun each rank runs the same sweep on its own GPU (independent
replicas, weak scaling; there is no data-path collective in a matvec sweep).
Rank 0 prints one JSON line. value = algorithmic bytes of all ranks' steps /
max-over-ranks device time. e2e = the same metric through sicu_gemv_host, the
call shape of the reference's backend gemv slot: pinned host x in, host y out,
per matvec. --impl reference times the reference's own CPU matvec
(si_backend_cpu()->gemv, AVX2, all host threads) on host copies of the sweep.

Beside the headline: `per_format` (every weight format at every sweep shape
and the 5632x2048 single-matvec shape, batched and one launch per matvec),
`model_path` (decode / prefill tok/s of llama-shaped models: TinyLlama-1.1B,
Llama-3-8B, Qwen2.5-32B tensor parallel over the run's GPUs), the reference
engine's own CPU rates on the same model shapes (si_engine_forward, token
serial, all host threads), and last `tp_curve`, the Qwen2.5-32B rates at this
GPU count against one GPU measured in the same run.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from siphon_b200 import quant as Q  # noqa: E402
from siphon_b200 import synth  # noqa: E402

METRIC = "Q4_K matvec HBM GB/s (% of peak)"
UNIT = "GB/s"
SHAPES = [(4096, 4096), (14336, 4096), (4096, 14336)]   # rows x K
WTYPE = Q.Q4_K
PEAKS = ROOT / "MEASURED_PEAKS.json"
FALLBACK_HBM = 6650.0
# DRAM traffic of the dominant kernel from an ncu capture (--set full) of one
# batched launch of 17 Q4_K 14336x4096 copies: it read and wrote 1.005x its
# algorithmic bytes; traffic grows with the matrices a launch streams, so a
# bench launch's traffic is that ratio times its bytes
NCU_TRAFFIC = {"ratio_to_algorithmic": 1.005,
               "source": "ncu --set full of one batched launch of 17 x Q4_K 14336x4096 (gemv_kernel<12>)"}


def peak_hbm() -> tuple[float, str]:
    try:
        return float(json.loads(PEAKS.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM, "fallback"


def workload_config(copies: dict | None, extra: dict | None = None) -> dict:
    cfg = {
        "workload": "configs[1] Q4_K matvec sweep: 4096x4096, 14336x4096, 4096x14336 (rows x K), batch 1, "
                    "f32 activation quantized to Q8_K inside the matvec kernel",
        "weights": "seeded random Q4_K blocks (f16 d,dmin U[1e-4,1e-2]; other bits uniform); x ~ N(0,1)",
        "l2": "inputs larger than L2: each shape rotates through distinct weight copies totalling >= 4x L2",
        "parallelism": "replicas",
        "launch": "one CUDA graph of K steps; per step and shape one sicu_gemv_multi launch over the shape's "
                  "weight copies (shared activation); programmatic dependent launch between launches",
    }
    if copies:
        cfg["copies_per_shape"] = copies
    if extra:
        cfg.update(extra)
    return cfg


# ---- clocks during the timed region -------------------------------------------------
class ClockSampler:
    """Polls NVML for SM clock and throttle reasons on a background thread."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, device: int):
        self.samples: list[int] = []
        self.reasons: int = 0
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None
        self._stop = threading.Event()

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                self.reasons |= self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:
                pass
            time.sleep(0.0002)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self) -> dict:
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "samples": len(self.samples),
                "reasons": [n for bit, n in self.REASONS.items() if self.reasons & bit]}


# ---- distributed plumbing ----------------------------------------------------------------
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def max_over_ranks(v: float, world: int, device) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ---- the reference's CPU matvec ------------------------------------------------------------
def cpu_sweep_setup(copies: dict):
    """Host copies of the sweep for the reference's CPU gemv."""
    mats = []
    for (n_out, n_in) in SHAPES:
        w = synth.weights(WTYPE, n_out, n_in, seed=n_out + n_in)
        x = synth.activations(n_in, 1, seed=7)[0]
        c = copies[f"{n_out}x{n_in}"]
        mats.append((n_out, n_in, [w] + [w.copy() for _ in range(c - 1)], x, np.zeros(n_out, np.float32)))
    return mats


def cpu_run_pass(gemv, mats) -> int:
    done = 0
    for n_out, n_in, ws, x, y in mats:
        for w in ws:
            gemv(gemv.tensor(WTYPE, w, n_in, n_out), x, y)
            done += Q.matvec_bytes(WTYPE, n_out, n_in)
    return done


def cpu_gemv_handle():
    from oracle.oracle import RefCpuGemv, Reference, have_reference
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    if have_reference():
        return RefCpuGemv(Reference(), threads), "reference", threads
    return None, "port", 1


def cpu_baseline(copies: dict, budget_s: float = 12.0) -> dict:
    """The reference's AVX2 matvec on the host cores over a bounded sample of
    the sweep (whole passes until ~budget_s)."""
    gemv, kind, threads = cpu_gemv_handle()
    if gemv is None:
        return port_baseline(budget_s)
    mats = cpu_sweep_setup(copies)
    cpu_run_pass(gemv, mats)   # warm
    t0 = time.perf_counter()
    nbytes = 0
    passes = 0
    while True:
        nbytes += cpu_run_pass(gemv, mats)
        passes += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    gemv.close()
    return {"value": round(nbytes / dt / 1e9, 3), "unit": UNIT, "cores": threads, "kind": kind,
            "sample": f"{passes} pass(es) over the sweep ({sum(copies.values())} matvecs each), "
                      f"si_backend_cpu()->gemv ({'AVX2' if kind == 'reference' else 'scalar'}), {threads} threads, "
                      f"{dt:.1f} s", "cpu": cpu_model()}


def port_baseline(budget_s: float) -> dict:
    from oracle.oracle import Oracle
    o = Oracle()
    n_out, n_in = SHAPES[0]
    w = synth.weights(WTYPE, n_out, n_in, seed=1)
    x = synth.activations(n_in, 1, seed=7)
    t0 = time.perf_counter()
    nbytes = reps = 0
    while time.perf_counter() - t0 < budget_s:
        o.gemv(WTYPE, w, n_in, n_out, o.quantize_pair(WTYPE, x)[0])
        nbytes += Q.matvec_bytes(WTYPE, n_out, n_in)
        reps += 1
    dt = time.perf_counter() - t0
    return {"value": round(nbytes / dt / 1e9, 3), "unit": UNIT, "cores": 1, "kind": "port",
            "sample": f"{reps} x 4096x4096 matvec, oracle restatement, 1 thread", "cpu": cpu_model()}


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def copies_for(l2_bytes: int) -> dict:
    out = {}
    for n_out, n_in in SHAPES:
        wb = n_out * Q.row_bytes(WTYPE, n_in)
        out[f"{n_out}x{n_in}"] = max(2, math.ceil(4 * l2_bytes / wb))
    return out


def run_reference(args, world, rank) -> None:
    if rank != 0:
        return
    gemv, kind, threads = cpu_gemv_handle()
    copies = copies_for(126 * 2 ** 20)
    if gemv is None:
        bl = port_baseline(5.0)
        line = {"impl": "reference", "metric": METRIC, "value": bl["value"], "unit": UNIT, "n_gpus": args.gpus,
                "steps": 0, "warmup": 0, "higher_is_better": True, "note": "oracle port: reference build absent",
                "cpu_baseline": bl, "e2e": {"value": bl["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                                            "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return
    mats = cpu_sweep_setup(copies)
    for _ in range(args.warmup):
        cpu_run_pass(gemv, mats)
    t0 = time.perf_counter()
    nbytes = 0
    for _ in range(args.steps):
        nbytes += cpu_run_pass(gemv, mats)
    dt = time.perf_counter() - t0
    gemv.close()
    value = nbytes / dt / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3 / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": workload_config(copies),
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": kind,
                         "sample": f"{args.steps} timed passes over the sweep, si_backend_cpu()->gemv (AVX2), "
                                   f"{threads} threads", "cpu": cpu_model()},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


# ---- our arm ----------------------------------------------------------------------------------
# ---- model-level matrix path (configs[2..4]) -----------------------------------------
DECODE_PER_GRAPH = 8      # decode tokens per captured graph


def _time_graph(torch, g, stream, reps, world, dev) -> float:
    """ms of `reps` replays of graph g on `stream` (max over ranks)."""
    with torch.cuda.stream(stream):
        for _ in range(3):
            g.replay()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(e0.elapsed_time(e1), world, dev)


def _heads_align(shape, world) -> bool:
    """Every rank's query heads cover whole KV groups (the device attention
    step maps local heads to local KV heads by that)."""
    from siphon_b200 import model_path as mp
    group = shape.n_head // shape.n_head_kv
    for r in range(world):
        sh = mp.tp_partition(shape, world, r)
        if not (len(sh.heads) == len(sh.kv_heads) * group or len(sh.kv_heads) == 1):
            return False
    return True


def model_decode(torch, s, shape, dev, stream, world, rank, group, reps, fused=False, steps=False,
                 attention_ctx=0) -> dict:
    """Decode tok/s of the matrix path of `shape` (batch 1), tensor parallel
    over the world: every weight matrix of one token per step, with (steps)
    the residual adds, RMS norms and SwiGLU between them fused into the
    products (sicu_gemv_fused). fused: the all-reduces ride in the matvecs
    too, else NCCL all-reduces."""
    from siphon_b200 import model_path as mp
    if attention_ctx:
        # the whole step but the embedding lookup, at the last position of an
        # attention_ctx-long context
        m = mp.MatrixPath(s, shape, dev, world, rank, group, seed=4, fused=fused, attention=True, n_ctx=attention_ctx)
        m.pos = attention_ctx - 1
    else:
        m = mp.MatrixPath(s, shape, dev, world, rank, group, seed=4, fused=fused, steps=steps)
    with torch.cuda.stream(stream):
        for _ in range(2):
            launches = m.decode_step(stream)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for _ in range(DECODE_PER_GRAPH):
            m.decode_step(stream)
    ms = _time_graph(torch, g, stream, reps, world, dev)
    del g
    tok = reps * DECODE_PER_GRAPH
    us = ms * 1e3 / tok
    gbps = m.weight_bytes / (us * 1e-6) / 1e9
    peak, peak_kind = peak_hbm()
    out = {"tok_s": round(tok / (ms * 1e-3), 1), "us_per_token": round(us, 2),
           "weight_bytes_per_token_per_gpu": m.weight_bytes, "GBps_per_gpu": round(gbps, 1),
           "hbm_frac": round(gbps / peak, 4), "peak_kind": peak_kind,
           "kernel_launches_per_token": launches, "allreduces_per_token": 2 * shape.n_layer if world > 1 else 0}
    if world > 1:
        out["allreduce"] = "fused into the matvecs (NVLink peer stores, sicu_gemv_ar)" if fused else "NCCL"
    assert s.status() == 0, "a matvec or all-reduce wait gave up"
    m.close()
    del m
    torch.cuda.empty_cache()
    return out


_TC_PEAKS: dict = {}


def tensor_peaks(s, dev) -> dict:
    """Dense tensor-core rates of this GPU from the library's own probe
    (sicu_tc_peak: every SM issuing M = 128, N = 256 MMAs from shared memory,
    about 30 ms per kind): kind::f16 (what the prefill kernels run) and
    kind::i8, the int8 denominator of the prefill roofline. Measured once per
    process."""
    if not _TC_PEAKS:
        import torch
        from siphon_b200.lib import TC_F16, TC_I8
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        out = {}
        for name, kind in (("f16_TFLOPs", TC_F16), ("i8_TOPs", TC_I8)):
            s.tc_peak(kind, 200, sms)                       # warm-up
            ms, tf = s.tc_peak(kind, 7000, sms)
            out[name] = round(tf, 1)
            out[name.split("_")[0] + "_ms"] = round(ms, 2)
        out["source"] = ("sicu_tc_peak: one CTA per SM, back-to-back tcgen05.mma M=128 N=256 from shared memory, "
                         "7000 rounds of 64 MMAs")
        _TC_PEAKS.update(out)
    return dict(_TC_PEAKS)


def model_prefill(torch, s, shape, dev, stream, world, rank, group, m_tok, reps) -> dict:
    """Prefill tok/s of the matrix path of `shape` for an m_tok-token prompt,
    from the prefill copies of the weights (sicu_prefill_pack, made at load
    beside the raw blocks)."""
    from siphon_b200 import model_path as mp
    m = mp.MatrixPath(s, shape, dev, world, rank, group, seed=5, max_tokens=m_tok, packed=True)
    with torch.cuda.stream(stream):
        m.prefill(stream, m_tok)          # sizes the workspace outside capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        m.prefill(stream, m_tok)
    ms = _time_graph(torch, g, stream, reps, world, dev)
    del g
    sec = ms * 1e-3 / reps
    params = sum(n_out * n_in for n_out, n_in in
                 [m.shapes[k] for k in ("q", "k", "v", "o", "gate", "up", "down")]) * shape.n_layer \
        + m.shapes["head"][0] * m.shapes["head"][1]
    tflops = 2.0 * m_tok * params / sec / 1e12
    try:
        f16_peak = float(json.loads(PEAKS.read_text())["bf16_tflops"])
        kind = "measured"
    except Exception:
        f16_peak, kind = 1590.0, "fallback"
    tc = tensor_peaks(s, dev)
    out = {"tok_s": round(m_tok / sec, 1), "ms_per_prompt": round(sec * 1e3, 3), "prompt_tokens": m_tok,
           "TFLOPs": round(tflops, 1), "f16_tensor_frac": round(tflops / f16_peak, 4), "peak_kind": kind,
           "f16_probe_frac": round(tflops / tc["f16_TFLOPs"], 4), "int8_tensor_frac": round(tflops / tc["i8_TOPs"], 4),
           "tensor_peaks_measured": tc,
           "pack_bytes_per_gpu": int(sum(t.numel() for t in m.pack.values())),
           "note": "tensor-core kernels (kind::f16 MMAs on exact f16 (scale x quant) operands) reading the "
                   "prefill copies of the Q4_K and Q6_K weights; f16_tensor_frac against the measured cuBLAS bf16 "
                   "peak, f16_probe_frac / int8_tensor_frac against this GPU's kind::f16 / kind::i8 MMA rates "
                   "measured by sicu_tc_peak"}
    del m
    torch.cuda.empty_cache()
    return out


def model_prompt(torch, s, shape, dev, stream, m_tok, reps) -> dict:
    """A whole prompt's forward pass in one pass (MatrixPath.prompt_step, one
    GPU): m_tok token ids in device memory -> the embedding rows, every
    layer's norms, products (from the prefill copies), RoPE, KV-cache stores
    and each token's attention over its prefix, SwiGLU, the head's logits of
    every token and the greedy choice after the last. Graph-timed."""
    from siphon_b200 import model_path as mp
    m = mp.MatrixPath(s, shape, dev, seed=6, embed=True, n_ctx=m_tok, max_tokens=m_tok, packed=True)
    gen = torch.Generator(device=dev)
    gen.manual_seed(3)
    m.tokens.copy_(torch.randint(0, shape.n_vocab, (m_tok,), device=dev, generator=gen))
    with torch.cuda.stream(stream):
        launches = m.prompt_step(stream, m_tok)     # sizes the workspace outside capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        m.prompt_step(stream, m_tok)
    ms = _time_graph(torch, g, stream, reps, 1, dev)
    del g
    sec = ms * 1e-3 / reps
    assert s.status() == 0, "a kernel of the prompt pass reported a device-side status"
    out = {"tok_s": round(m_tok / sec, 1), "ms_per_prompt": round(sec * 1e3, 3), "prompt_tokens": m_tok,
           "library_calls_per_prompt": launches,
           "pack_bytes": int(sum(t.numel() for t in m.pack.values()))}
    m.close()
    del m
    torch.cuda.empty_cache()
    return out


def model_batch_decode(torch, s, shape, dev, stream, world, rank, group, batch, reps) -> dict:
    """Decode tok/s of the matrix path for `batch` sequences per step (one
    token each): every weight product once per step for all of them, through
    sicu_gemv_batch (the batch decode kernel: weights decoded in registers,
    mma.sync tiles of 16 rows x 8 tokens)."""
    from siphon_b200 import model_path as mp
    m = mp.MatrixPath(s, shape, dev, world, rank, group, seed=6, max_tokens=batch)
    with torch.cuda.stream(stream):
        launches = m.batch_step(stream, batch)     # sizes the workspace outside capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for _ in range(DECODE_PER_GRAPH):
            m.batch_step(stream, batch)
    ms = _time_graph(torch, g, stream, reps, world, dev)
    del g
    steps = reps * DECODE_PER_GRAPH
    us = ms * 1e3 / steps
    gbps = m.weight_bytes / (us * 1e-6) / 1e9
    peak, peak_kind = peak_hbm()
    out = {"batch": batch, "tok_s": round(batch * steps / (ms * 1e-3), 1), "us_per_step": round(us, 2),
           "weight_bytes_per_step_per_gpu": m.weight_bytes, "GBps_per_gpu": round(gbps, 1),
           "hbm_frac": round(gbps / peak, 4), "peak_kind": peak_kind, "library_calls_per_step": launches,
           "allreduces_per_step": 2 * shape.n_layer if world > 1 else 0}
    assert s.status() == 0, "a batch matvec wait gave up"
    del m
    torch.cuda.empty_cache()
    return out


def _host_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


def _scratch_dir(need_bytes: int) -> str:
    """A directory for temporary model files: RAM-backed /dev/shm when it has
    room, else the system temporary directory."""
    import shutil
    import tempfile
    for d in ("/dev/shm", tempfile.gettempdir()):
        try:
            if shutil.disk_usage(d).free > need_bytes * 1.2:
                return d
        except OSError:
            pass
    return tempfile.gettempdir()


def engine_cpu_baseline(dev) -> dict | None:
    """The reference engine's own CPU rates on the model shapes the GPU lines
    run: si_engine_forward token-serial (src/engine.c:288-398; the reference's
    prompt loop is token-serial too, src/cmd_run.c:273-321), its default
    dispatch (AVX2 dots), a pthread pool of all host threads. Each model is a
    synthetic GGUF of the full shape with random blocks (generated on the GPU,
    written to RAM-backed storage), timed on a bounded sample:

    * TinyLlama-1.1B shape: a 32-token prompt, then 128 greedy tokens (whole);
    * Llama-3-8B shape: the first 64 tokens of a 512-token prompt;
    * Qwen2.5-32B shape: the first 16 tokens of a 512-token prompt, then 16
      greedy tokens. Batch-8 decode on the CPU is eight sequences run one
      after the other, so its rate is the batch-1 rate."""
    import zlib

    from oracle.oracle import E2E_SO, RefEngine
    from siphon_b200 import model_path as mp
    from siphon_b200 import synth_model as sm
    if not E2E_SO.exists():
        return None
    threads = _host_threads()

    def gpu_blocks(wt, n_out, n_in, key):
        seed = zlib.crc32(repr(key).encode())
        return mp.device_weights(wt, n_out, n_in, seed, dev).cpu().numpy()

    def run(sh, name, n_prompt, n_gen, prompt_len):
        nbytes = sum(n_out * Q.row_bytes(wt, n_in) for _, wt, n_out, n_in in sm.matrices(sh))
        path = Path(_scratch_dir(nbytes)) / f"siphon_bench_{name}_{os.getpid()}.gguf"
        t0 = time.perf_counter()
        sm.write_llama(path, sh, seed=1, blocks=gpu_blocks)
        t_write = time.perf_counter() - t0
        try:
            e = RefEngine(path, use_cuda=False, n_ctx=max(512, n_prompt + n_gen), threads=threads, scalar=False)
            try:
                prompt = np.random.default_rng(2).integers(0, sh.n_vocab, n_prompt).tolist()
                e.forward(prompt[0])                       # pages the mapped file in
                t0 = time.perf_counter()
                for tok in prompt[1:]:
                    logits = e.forward(tok)
                t1 = time.perf_counter()
                tok = int(np.argmax(logits))
                for _ in range(n_gen):
                    tok = int(np.argmax(e.forward(tok)))
                t2 = time.perf_counter()
            finally:
                e.close()
        finally:
            path.unlink(missing_ok=True)
        out = {"prompt_tok_s": round((n_prompt - 1) / (t1 - t0), 3)}
        if n_gen:
            out["decode_tok_s"] = round(n_gen / (t2 - t1), 3)
        out["sample"] = (f"prompt tokens 2..{n_prompt} of a {prompt_len}-token prompt"
                         + (f", then {n_gen} greedy tokens" if n_gen else "")
                         + f" (model file of random blocks written in {t_write:.1f} s)")
        return out

    res = {"engine": "si_engine_forward token-serial, AVX2 dispatch", "cores": threads, "kind": "reference",
           "cpu": cpu_model(),
           "decode_tinyllama": run(sm.TINYLLAMA, "tinyllama", 32, 128, 32),
           "prefill_llama3_8b": run(sm.LLAMA3_8B, "llama3_8b", 64, 0, 512),
           "qwen32b": run(sm.QWEN25_32B, "qwen32b", 16, 16, 512)}
    res["qwen32b"]["note"] = ("prompt rate over the first tokens of a 512-token prompt; batch-8 decode on the CPU "
                              "runs the 8 sequences one after the other (the batch-1 rate)")
    torch_empty_cache()
    return res


def torch_empty_cache() -> None:
    try:
        import torch
        torch.cuda.empty_cache()
    except Exception:
        pass


def bench_weights(wt: int, n_out: int, n_in: int, seed: int, dev):
    """Device weight blocks of the sweep's distribution: random blocks with
    f16 scales U[1e-4, 1e-2] for the quantized formats, f16(U[-1, 1)) for F16."""
    import torch

    from siphon_b200 import model_path as mp
    if wt == Q.F16:
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        v = torch.rand(n_out * n_in, device=dev, generator=g) * 2 - 1
        return v.half().view(torch.uint8)
    return mp.device_weights(wt, n_out, n_in, seed, dev)


PER_FORMAT_SHAPES = [(4096, 4096), (14336, 4096), (4096, 14336), (5632, 2048)]


def per_format(torch, s, dev, stream, l2: int) -> dict:
    """Every weight format at every sweep shape and at the single-matvec shape
    5632x2048: GB/s (algorithmic bytes / device time) batched (one
    sicu_gemv_multi launch over copies totalling >= 4x L2) and one launch per
    matvec, each as a fraction of the measured HBM copy bandwidth."""
    peak, peak_kind = peak_hbm()
    out = {"peak_GBps": peak, "peak_kind": peak_kind,
           "l2": "per shape, distinct weight copies totalling >= 4x L2, capped at 64 copies (>= 1.8x L2 for "
                 "the smallest matrices)"}
    h = stream.cuda_stream
    for wt in Q.WEIGHT_TYPES:
        row = {}
        for n_out, n_in in PER_FORMAT_SHAPES:
            wb = n_out * Q.row_bytes(wt, n_in)
            c = min(64, max(2, math.ceil(4 * l2 / wb)))    # a launch takes up to 64 matrices
            ws = [bench_weights(wt, n_out, n_in, 11 + i, dev) for i in range(c)]
            x = torch.from_numpy(synth.activations(n_in, 1, seed=7)[0]).to(dev)
            ys = [torch.empty(n_out, device=dev) for _ in range(c)]

            def batched():
                s.gemv_multi(wt, ws, [n_out] * c, n_in, x, ys, stream=h)

            def single():
                for w, y in zip(ws, ys):
                    s.gemv_f32(wt, w, n_in, n_out, x, y, stream=h)

            b = Q.matvec_bytes(wt, n_out, n_in)
            res = {}
            for name, fn, reps in (("batched", batched, 6), ("single", single, 2)):
                with torch.cuda.stream(stream):
                    fn()
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    for _ in range(reps):
                        fn()
                ms = _time_graph(torch, g, stream, 2, 1, dev) / 2
                del g
                us = ms * 1e3 / (reps * c)
                gbps = b / (us * 1e-6) / 1e9
                res[f"{name}_GBps"] = round(gbps, 1)
                res[f"{name}_frac"] = round(gbps / peak, 4)
            row[f"{n_out}x{n_in}"] = res
            del ws, ys
        out[Q.NAMES[wt]] = row
    torch.cuda.empty_cache()
    assert s.status() == 0, "a matvec wait gave up"
    return out


PREFILL_FORMAT_SHAPES = [(14336, 4096), (4096, 4096)]


def prefill_per_format(torch, s, dev, stream, m_tok: int = 512) -> dict:
    """Every quantized format's tensor-core prompt product from its prefill
    copy (sicu_gemm_prefill_packed_f32, f32 prompt rows quantized inside the
    launch): TFLOP/s = 2 m rows K / device time, against the measured f16
    dense peak (the K formats run kind::f16 MMAs on exact f16 scale x quant)
    and the measured int8 rate (the classic formats run kind::i8 MMAs)."""
    try:
        f16_peak = float(json.loads(PEAKS.read_text())["bf16_tflops"])
        kind = "measured"
    except Exception:
        f16_peak, kind = 1590.0, "fallback"
    tc = tensor_peaks(s, dev)
    out = {"prompt_tokens": m_tok, "f16_peak_TFLOPs": f16_peak, "peak_kind": kind,
           "i8_peak_TOPs_measured": tc["i8_TOPs"]}
    h = stream.cuda_stream
    x = torch.from_numpy(synth.activations(max(k for _, k in PREFILL_FORMAT_SHAPES), m_tok, seed=3)).to(dev)
    for wt in (Q.Q4_K, Q.Q5_K, Q.Q6_K, Q.Q3_K, Q.Q2_K, Q.Q4_0, Q.Q5_0, Q.Q8_0, Q.F16):
        row = {}
        for n_out, n_in in PREFILL_FORMAT_SHAPES:
            w = bench_weights(wt, n_out, n_in, 31, dev)
            nb = s.prefill_pack_bytes(wt, n_in, n_out)
            pk = torch.empty(nb, dtype=torch.uint8, device=dev)
            s.prefill_pack(wt, w, n_in, n_out, pk, nb, stream=h)
            xi = x[:, :n_in].contiguous()
            y = torch.empty(m_tok, n_out, device=dev)

            def run():
                s.gemm_prefill_packed_f32(wt, w, pk, n_in, n_out, xi, m_tok, y, stream=h)

            with torch.cuda.stream(stream):
                run()                      # sizes the workspace outside capture
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for _ in range(4):
                    run()
            ms = _time_graph(torch, g, stream, 3, 1, dev) / 12
            del g
            tf = 2.0 * m_tok * n_out * n_in / (ms * 1e-3) / 1e12
            row[f"{n_out}x{n_in}"] = {"us": round(ms * 1e3, 1), "TFLOPs": round(tf, 1),
                                      "f16_frac": round(tf / f16_peak, 4), "int8_frac": round(tf / tc["i8_TOPs"], 4)}
            del w, pk, y
        out[Q.NAMES[wt]] = row
    torch.cuda.empty_cache()
    assert s.status() == 0, "a prefill wait gave up"
    return out


TP_ROWS = ("decode_b1", "decode_b1_steps", "decode_b1_full", "decode_b1_nccl", "decode_b8", "prefill512")


def tp_rows(torch, s, shape, dev, stream, world, rank, reps) -> dict:
    """The configs[4] measurements at this world size: batch-1 decode (matrix
    path with the all-reduces fused into the matvecs; with the activation
    steps; the whole step with attention; with NCCL all-reduces), batch-8
    decode and the 512-token prefill."""
    rows = {}
    rows["decode_b1"] = model_decode(torch, s, shape, dev, stream, world, rank, None, reps, fused=world > 1)
    rows["decode_b1_steps"] = model_decode(torch, s, shape, dev, stream, world, rank, None, reps,
                                           fused=world > 1, steps=True)
    if _heads_align(shape, world):
        rows["decode_b1_full"] = model_decode(torch, s, shape, dev, stream, world, rank, None, reps,
                                              fused=world > 1, attention_ctx=512)
    if world > 1:
        rows["decode_b1_nccl"] = model_decode(torch, s, shape, dev, stream, world, rank, None, reps)
    rows["decode_b8"] = model_batch_decode(torch, s, shape, dev, stream, world, rank, None, 8, reps)
    rows["prefill512"] = model_prefill(torch, s, shape, dev, stream, world, rank, None, 512, max(2, reps // 2))
    return rows


def tp_curve(world: int, rows: dict, one: dict) -> dict:
    """Compact Qwen2.5-32B summary (printed last in the line): tok/s at this
    GPU count, at one GPU in the same run, and the efficiency
    (tok/s at N) / (N x tok/s at 1)."""
    cur = {k: rows[k]["tok_s"] for k in TP_ROWS if k in rows}
    base = {k: one[k]["tok_s"] for k in TP_ROWS if k in one}
    eff = {}
    for k, v in cur.items():
        b = base.get("decode_b1" if k == "decode_b1_nccl" else k)
        if b:
            eff[k] = round(v / (world * b), 3)
    return {"shape": "Qwen2.5-32B", "n_gpus": world, "tok_s": cur, "tok_s_1gpu": base, "efficiency": eff,
            "allreduce": "fused into the matvecs over NVLink peer stores (decode_b1*), NCCL (decode_b1_nccl, "
                         "decode_b8, prefill512)" if world > 1 else "none (one GPU)"}


def model_metrics(torch, s, dev, stream, world, rank, quick: bool) -> tuple[dict, dict]:
    from siphon_b200 import synth_model as sm
    out = {}
    reps = 3 if quick else 10
    sh = sm.QWEN25_32B
    tp_desc = (f"configs[4] Qwen2.5-32B shape, tensor parallel x{world} (column-split QKV/gate/up/head, row-split "
               "o/down, an all-reduce after o and after down per layer)" if world > 1
               else "configs[4] Qwen2.5-32B shape, one GPU")
    rows = tp_rows(torch, s, sh, dev, stream, world, rank, reps)
    # at N > 1 the same measurements on this rank's GPU alone, for the
    # efficiency (every rank runs them at the same time; no collective)
    one = tp_rows(torch, s, sh, dev, stream, 1, 0, reps) if world > 1 else rows
    out["tp"] = {"config": tp_desc, "rows": rows,
                 "notes": {"decode_b1": "matrix path, batch 1 (every weight product of a token)",
                           "decode_b1_steps": "plus the residual adds, RMS norms and SwiGLU fused into the products",
                           "decode_b1_full": "plus RoPE, the f16 KV cache and attention, the token at position 511",
                           "decode_b1_nccl": "decode_b1 with NCCL all-reduces between the matvecs",
                           "decode_b8": "8 sequences per step, every weight product once per step for all 8",
                           "prefill512": "a 512-token prompt's products"}}
    if world == 1:
        out["decode"] = {"config": "configs[2] TinyLlama-1.1B shape, batch 1, matrix path",
                         **model_decode(torch, s, sm.TINYLLAMA, dev, stream, 1, 0, None, reps * 4)}
        out["decode_steps"] = {"config": "as decode, with the residual adds, RMS norms and SwiGLU between the "
                                         "products fused into them (sicu_gemv_fused)",
                               **model_decode(torch, s, sm.TINYLLAMA, dev, stream, 1, 0, None, reps * 4, steps=True)}
        out["decode_full"] = {"config": "as decode_steps, plus RoPE, the f16 KV-cache store and attention over a "
                                        "512-position context (the token at position 511): every step of the "
                                        "reference's forward pass but the embedding lookup",
                              **model_decode(torch, s, sm.TINYLLAMA, dev, stream, 1, 0, None, reps * 4,
                                             attention_ctx=512)}
        out["prompt_full"] = {"config": "configs[2] TinyLlama-1.1B shape, a 512-token prompt's whole forward pass "
                                        "in one pass: embedding, norms, products, RoPE, KV cache, each token's "
                                        "attention over its prefix, SwiGLU, the logits of every token, the greedy "
                                        "choice (MatrixPath.prompt_step); the reference engine runs a prompt "
                                        "token by token (engine_cpu decode_tinyllama prompt_tok_s)",
                              **model_prompt(torch, s, sm.TINYLLAMA, dev, stream, 512, max(2, reps // 2))}
        out["prefill"] = {"config": "configs[3] Llama-3-8B shape, 512-token prompt, matrix path",
                          **model_prefill(torch, s, sm.LLAMA3_8B, dev, stream, 1, 0, None, 512, max(2, reps // 2))}
        out["prefill_per_format"] = prefill_per_format(torch, s, dev, stream)
    out["scope"] = ("every weight-matrix product of the forward pass (per layer Wq, Wk, Wv, Wo, W_gate, W_up, "
                    "W_down; then the output head) with synthetic Q4_K_M-style weights; the *_steps lines also run "
                    "the residual adds, RMS norms and SwiGLU between them, fused into the products (Wo reading a "
                    "fixed activation); *_full lines also run RoPE, the KV cache and attention: the whole step but "
                    "the embedding lookup")
    return out, tp_curve(world, rows, one)


def run_ours(args, world, rank, local) -> None:
    import torch

    from siphon_b200 import lib

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    s = lib.load()
    s.init(local)
    # programmatic dependent launch: each matvec starts streaming its (immutable)
    # weights while the previous one drains
    s.set_overlap(True)
    props = torch.cuda.get_device_properties(dev)
    l2 = int(getattr(props, "L2_cache_size", 126 * 2 ** 20))
    copies = copies_for(l2)

    stream = torch.cuda.Stream(device=dev)
    mats = []
    for (n_out, n_in) in SHAPES:
        w = torch.from_numpy(synth.weights(WTYPE, n_out, n_in, seed=n_out + n_in)).to(dev)
        c = copies[f"{n_out}x{n_in}"]
        ws = [w] + [w.clone() for _ in range(c - 1)]
        x = torch.from_numpy(synth.activations(n_in, 1, seed=7)[0]).to(dev)
        ys = [torch.empty(n_out, dtype=torch.float32, device=dev) for _ in range(c)]
        mats.append((n_out, n_in, ws, x, ys))
    torch.cuda.synchronize()
    step_bytes = sum(len(ws) * Q.matvec_bytes(WTYPE, n_out, n_in) for n_out, n_in, ws, _, _ in mats)
    launches_per_step = sum(len(ws) for _, _, ws, _, _ in mats)

    def step(st, evs=None, single=False):
        # one launch per shape: the shape's weight copies share the activation
        # (sicu_gemv_multi); single=True launches one matvec per copy instead
        h = st.cuda_stream
        for si, (n_out, n_in, ws, x, ys) in enumerate(mats):
            if evs is not None:
                evs[si][0].record(st)
            if single:
                for w, y in zip(ws, ys):
                    s.gemv_f32(WTYPE, w, n_in, n_out, x, y, stream=h)
            else:
                s.gemv_multi(WTYPE, ws, [n_out] * len(ws), n_in, x, ys, stream=h)
            if evs is not None:
                evs[si][1].record(st)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step(stream)
            step(stream, single=True)
    torch.cuda.synchronize()
    for n_out, n_in, ws, x, ys in mats:
        assert torch.isfinite(ys[-1]).all(), "non-finite matvec output"

    # the K timed steps as one CUDA graph, with timing events around each
    # shape's group of launches
    evs = [[[torch.cuda.Event(enable_timing=True, external=True) for _ in range(2)] for _ in SHAPES]
           for _ in range(args.steps)]
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for k in range(args.steps):
            step(stream, evs[k])
    with torch.cuda.stream(stream):
        g.replay()                   # graph upload + K more warm-up steps
    torch.cuda.synchronize()

    barrier(world)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk, torch.cuda.stream(stream):
        e0.record(stream)
        g.replay()                   # replays on the current stream: `stream`
        e1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ms = e0.elapsed_time(e1)
    ms_max = max_over_ranks(ms, world, dev)
    value = world * args.steps * step_bytes / (ms_max * 1e-3) / 1e9

    # dominant kernel: gemv_kernel<Q4_K>, one launch per shape per step
    per_shape_ms = [0.0] * len(SHAPES)
    for k in range(args.steps):
        for si in range(len(SHAPES)):
            per_shape_ms[si] += evs[k][si][0].elapsed_time(evs[k][si][1])
    kern_bytes = args.steps * step_bytes
    achieved = kern_bytes / (sum(per_shape_ms) * 1e-3) / 1e9
    peak, peak_kind = peak_hbm()
    # per launch (one launch = all copies of one shape), averaged over the shapes
    per_launch = step_bytes / len(SHAPES)
    traffic = round(NCU_TRAFFIC["ratio_to_algorithmic"] * per_launch) if NCU_TRAFFIC else None

    # the same sweep with one launch per matvec (informational)
    sevs = [[[torch.cuda.Event(enable_timing=True, external=True) for _ in range(2)] for _ in SHAPES]
            for _ in range(2)]
    g1 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g1, stream=stream):
        for k in range(2):
            step(stream, sevs[k], single=True)
    with torch.cuda.stream(stream):
        g1.replay()
        g1.replay()
    torch.cuda.synchronize()
    shape_detail = {}
    for si, (n_out, n_in, ws, _, _) in enumerate(mats):
        b = Q.matvec_bytes(WTYPE, n_out, n_in)
        us = per_shape_ms[si] * 1e3 / (args.steps * len(ws))
        us1 = sum(sevs[k][si][0].elapsed_time(sevs[k][si][1]) for k in range(2)) * 1e3 / (2 * len(ws))
        shape_detail[f"{n_out}x{n_in}"] = {
            "batched_us_per_matrix": round(us, 3), "batched_GBps": round(b / (us * 1e-6) / 1e9, 1),
            "single_launch_us": round(us1, 3), "single_launch_GBps": round(b / (us1 * 1e-6) / 1e9, 1),
            "bytes_per_matrix": b}
    del g1

    # e2e through the host-buffer entry point (reference backend call shape)
    hx = [torch.from_numpy(synth.activations(n_in, 1, seed=7)[0]).pin_memory() for _, n_in, _, _, _ in mats]
    hy = [[torch.empty(n_out, dtype=torch.float32).pin_memory() for _ in ws] for n_out, _, ws, _, _ in mats]

    # the C entry point with its arguments bound ahead (as a C caller holds
    # them), so the loop times the call rather than the Python binding
    fn_host = s.lib.sicu_gemv_host
    calls = [(WTYPE, w.data_ptr(), n_in, n_out, hx[si].data_ptr(), hy[si][ci].data_ptr(), stream.cuda_stream)
             for si, (n_out, n_in, ws, _, _) in enumerate(mats) for ci, w in enumerate(ws)]

    def e2e_step():
        for a in calls:
            rc = fn_host(*a)
            if rc:
                s.check(rc)

    for _ in range(max(1, min(args.warmup, 3))):
        e2e_step()
    e2e_steps = max(3, min(args.steps, 20))
    barrier(world)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    e2e_s = max_over_ranks(time.perf_counter() - t0, world, dev)
    e2e_value = world * e2e_steps * step_bytes / e2e_s / 1e9
    h2d = sum(len(ws) * 4 * n_in for _, n_in, ws, _, _ in mats)
    d2h = sum(len(ws) * 4 * n_out for n_out, _, ws, _, _ in mats)

    del g
    fmt = None
    if world == 1 and not args.no_model:
        fmt = per_format(torch, s, dev, stream, l2)
    model = curve = None
    if not args.no_model:
        model, curve = model_metrics(torch, s, dev, stream, world, rank, quick=args.steps < 10)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(copies)
        if model is not None:
            mc = engine_cpu_baseline(dev)
            if mc is not None:
                model["cpu_baseline"] = mc

    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": workload_config(copies, {"parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                                           "per_shape": shape_detail}),
        "roofline": {"bound": "hbm", "kernel": "gemv_kernel<Q4_K> (one launch = all copies of a shape)", "achieved": round(achieved, 1),
                     "peak": peak, "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "traffic": traffic, "algorithmic_bytes_per_launch": round(per_launch),
                     "traffic_source": NCU_TRAFFIC.get("source")},
        "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "path": "sicu_gemv_host per matvec (page-locked host x and y, read and written by the GPU "
                        "directly; stream sync per call)"},
        "gpu_launches": args.steps * len(SHAPES),
        "clocks": clk.summary(),
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if fmt is not None:
        line["per_format"] = fmt
    if model is not None:
        line["model_path"] = model
    if curve is not None:
        line["tp_curve"] = curve            # last: kept by a reader of the line's tail
    print(json.dumps(line))


# ---- single profiling workloads (run under ncu on one GPU) -----------------------------------
CASES = {
    "flat": "gemv_flat_kernel<Q4_K>: one sicu_gemv_multi launch over 4 copies of Q4_K 27648x5120, 4 times",
    "ar": "gemv_kernel<Q4_K, AR> (one-rank group) and the plain gemv_kernel<Q4_K> alternating, Q4_K 5120x13824",
    "prefill": "prefill_kernel<Q4_K>: 4096x4096, 512 tokens, twice",
    "prefill_packed": "prefill_packed_kernel<Q4_K, 256>: 14336x4096 from its prefill copy, 512 tokens, twice",
    "steps": "Q4_K Wq/Wk/Wv of the 32B shape (5120 -> 5120+1024+1024): plain and with the residual add + "
             "RMS norm fused, alternating, 4 each",
    "decode_full": "three eager decode steps of the TinyLlama-1.1B shape with the steps and attention, "
                   "the token at position 511 of a 512-position context",
    "batch8": "the batch-8 decode matvec: Q4_K and Q6_K 5120x27648, 8 tokens, 4 times each",
    "prefill_i8": "prefill_i8_kernel<Q8_0>: 4096x4096 from its int8 prefill copy, 512 f32 tokens, twice",
    "prompt_full": "two eager whole-prompt passes (MatrixPath.prompt_step) of the TinyLlama-1.1B shape, "
                   "512 tokens",
}


def run_case(case: str, reps: int = 4) -> int:
    """Run one small workload on GPU 0 for an ncu capture; exits non-zero if
    the library reports a device-side status bit."""
    import torch

    from siphon_b200 import lib
    from siphon_b200 import model_path as mp
    from siphon_b200 import synth_model as sm
    if case not in CASES:
        raise SystemExit(f"unknown case {case!r}: " + ", ".join(CASES))
    torch.cuda.set_device(0)
    s = lib.load()
    s.init(0)
    s.set_overlap(True)
    dev = torch.device("cuda", 0)
    if case == "flat":
        wt, n_out, n_in, c = Q.Q4_K, 27648, 5120, 4
        ws = [mp.device_weights(wt, n_out, n_in, 1 + i, dev) for i in range(c)]
        x = torch.from_numpy(synth.activations(n_in, 1, seed=2)[0]).to(dev)
        ys = [torch.empty(n_out, device=dev) for _ in range(c)]
        for _ in range(reps):
            s.gemv_multi(wt, ws, [n_out] * c, n_in, x, ys)
    elif case == "ar":
        wt, n_out, n_in = Q.Q4_K, 5120, 13824
        g = s.ar_create(1, 0, n_out)
        g.open([g.local_handle])
        w = mp.device_weights(wt, n_out, n_in, 1, dev)
        x = torch.from_numpy(synth.activations(n_in, 1, seed=2)[0]).to(dev)
        y = torch.empty(n_out, device=dev)
        for _ in range(reps):
            s.gemv_ar(wt, w, n_in, n_out, x, y, g)
            s.gemv_f32(wt, w, n_in, n_out, x, y)
        torch.cuda.synchronize()
        g.destroy()
    elif case == "prefill_i8":
        wt, n, m = Q.Q8_0, 4096, 512
        w = bench_weights(wt, n, n, 1, dev)
        nb = s.prefill_pack_bytes(wt, n, n)
        pk = torch.empty(nb, dtype=torch.uint8, device=dev)
        s.prefill_pack(wt, w, n, n, pk, nb)
        x = torch.randn(m, n, device=dev)
        y = torch.empty(m, n, device=dev)
        for _ in range(2):
            s.gemm_prefill_packed_f32(wt, w, pk, n, n, x, m, y)
    elif case == "prefill":
        wt, n, m = Q.Q4_K, 4096, 512
        w = mp.device_weights(wt, n, n, 1, dev)
        x = torch.randn(m, n, device=dev)
        y = torch.empty(m, n, device=dev)
        for _ in range(2):
            s.gemm_prefill_f32(wt, w, n, n, x, m, y)
    elif case == "prefill_packed":
        wt, n_out, n_in, m = Q.Q4_K, 14336, 4096, 512
        w = mp.device_weights(wt, n_out, n_in, 1, dev)
        nb = s.prefill_pack_bytes(wt, n_in, n_out)
        p = torch.empty(nb, dtype=torch.uint8, device=dev)
        s.prefill_pack(wt, w, n_in, n_out, p, nb)
        x = torch.randn(m, n_in, device=dev)
        y = torch.empty(m, n_out, device=dev)
        for _ in range(2):
            s.gemm_prefill_packed_f32(wt, w, p, n_in, n_out, x, m, y)
    elif case == "steps":
        wt, n_in, outs = Q.Q4_K, 5120, [5120, 1024, 1024]
        ws = [mp.device_weights(wt, n, n_in, 1 + i, dev) for i, n in enumerate(outs)]
        x = torch.randn(n_in, device=dev)
        r = torch.randn(n_in, device=dev)
        gam = 1.0 + 0.1 * torch.randn(n_in, device=dev)
        h = torch.empty(n_in, device=dev)
        ys = [torch.empty(n, device=dev) for n in outs]
        for _ in range(reps):
            s.gemv_multi(wt, ws, outs, n_in, x, ys)
            s.gemv_fused(wt, ws, outs, n_in, x, lib.rms_norm_step(gam, 1e-6, r, h), ys)
    elif case == "decode_full":
        m = mp.MatrixPath(s, sm.TINYLLAMA, dev, seed=4, attention=True, n_ctx=512)
        m.pos = 511
        st = torch.cuda.Stream(device=dev)
        with torch.cuda.stream(st):
            for _ in range(3):
                m.decode_step(st)
        torch.cuda.synchronize()
        m.close()
    elif case == "prompt_full":
        m = mp.MatrixPath(s, sm.TINYLLAMA, dev, seed=6, embed=True, n_ctx=512, max_tokens=512, packed=True)
        st = torch.cuda.Stream(device=dev)
        with torch.cuda.stream(st):
            for _ in range(2):
                m.prompt_step(st, 512)
        torch.cuda.synchronize()
        m.close()
    elif case == "batch8":
        n_out, n_in, m = 5120, 27648, 8
        x = torch.randn(m, n_in, device=dev)
        y = torch.empty(m, n_out, device=dev)
        for wt in (Q.Q4_K, Q.Q6_K):
            w = mp.device_weights(wt, n_out, n_in, 1, dev)
            for _ in range(reps):
                s.gemm_prefill_f32(wt, w, n_in, n_out, x, m, y)
    torch.cuda.synchronize()
    st = s.status()
    print(case, "status", st)
    return 1 if st else 0


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", choices=sorted(CASES), help="run one profiling workload and exit")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-model", action="store_true", help="skip the model-level matrix-path measurements")
    args = ap.parse_args()
    if args.case:
        sys.exit(run_case(args.case))
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    world, rank, local = dist_setup()
    if args.impl == "reference":
        run_reference(args, world, rank)
    else:
        run_ours(args, world, rank, local)


if __name__ == "__main__":
    main()

"""The C-ABI library loads on a CPU-only machine, exports every entry point
include/siphon_cuda.h declares, and rejects bad arguments on the host with
the reference's error codes before touching CUDA."""

from __future__ import annotations

import ctypes as C
import re

import numpy as np
import pytest

from siphon_b200 import lib as L
from siphon_b200 import quant as Q

HEADER = L.LIB_PATH.parents[1] / "include" / "siphon_cuda.h"


def declared() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"SICU_API\s+int\s+(sicu_\w+)\s*\(", text)


@pytest.fixture(scope="module")
def so():
    return L.SiphonCuda()


def test_every_declared_symbol_is_exported(so):
    names = declared()
    assert len(names) >= 20
    for n in names:
        assert hasattr(so.lib, n), n
    assert set(names) == set(L.SIGNATURES), "binding and header disagree"


def test_geometry_and_pairing_without_gpu(so):
    for t, (blck, size) in Q.GEOMETRY.items():
        assert so.geometry(t) == (blck, size)
    for t in Q.WEIGHT_TYPES:
        assert so.pair_type(t) == Q.pair_type(t)
    with pytest.raises(L.SicuError) as e:
        so.pair_type(3)   # Q4_1: recognised by ggml, not on this path
    assert e.value.code == L.SICU_ENOTSUP


def _call_gemv(so, wt=Q.Q4_K, w=16, n_in=256, n_out=4, x=32, y=64, m=1):
    return so.lib.sicu_gemv(wt, w, n_in, n_out, x, y, m, None)


def test_matvec_argument_checks_run_on_host(so):
    assert _call_gemv(so, wt=3) == L.SICU_ENOTSUP          # unsupported type
    assert _call_gemv(so, n_in=300) == L.SICU_EINVAL        # not a whole super-block
    assert _call_gemv(so, n_in=0) == L.SICU_EINVAL
    assert _call_gemv(so, m=0) == L.SICU_EINVAL
    assert _call_gemv(so, w=None) == L.SICU_EINVAL          # null
    assert _call_gemv(so, w=24) == L.SICU_EINVAL            # weight not 16-byte aligned
    assert _call_gemv(so, y=66) == L.SICU_EINVAL            # output misaligned
    assert "aligned" in so.last_error()
    # well-formed, but no device initialised: refused without a CUDA call
    assert _call_gemv(so) == L.SICU_EINVAL
    assert "sicu_init" in so.last_error()


def test_quantizer_argument_checks_run_on_host(so):
    assert so.lib.sicu_quantize_q8_K(16, 32, 300, 1, None) == L.SICU_EINVAL
    assert so.lib.sicu_quantize_q8_0(16, 32, 40, 1, None) == L.SICU_EINVAL
    assert so.lib.sicu_quantize_q8_K(20, 32, 256, 1, None) == L.SICU_EINVAL   # f32 input misaligned
    assert so.lib.sicu_quantize_pair(3, 16, 32, 256, 1, None) == L.SICU_ENOTSUP
    assert so.lib.sicu_quantize_q8_K(16, 32, 256, 1, None) == L.SICU_EINVAL   # not initialised


def test_last_error_is_per_thread(so):
    import threading
    _call_gemv(so, wt=3)
    msgs = {}

    def other():
        msgs["t"] = so.last_error()

    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert "unsupported" in so.last_error()
    assert msgs["t"] == ""


def test_allreduce_group_checks_run_on_host(so):
    h = C.c_void_p()
    buf = C.create_string_buffer(L.AR_HANDLE_BYTES)
    assert so.lib.sicu_ar_create(0, 0, 256, C.byref(h), buf) == L.SICU_EINVAL      # no ranks
    assert so.lib.sicu_ar_create(9, 0, 256, C.byref(h), buf) == L.SICU_EINVAL      # more than 8
    assert so.lib.sicu_ar_create(2, 2, 256, C.byref(h), buf) == L.SICU_EINVAL      # rank out of range
    assert so.lib.sicu_ar_create(2, 0, 300, C.byref(h), buf) == L.SICU_EINVAL      # not whole super-blocks
    assert so.lib.sicu_ar_create(2, 0, 256, None, buf) == L.SICU_EINVAL
    # well-formed, but no device initialised: refused without a CUDA call
    assert so.lib.sicu_ar_create(2, 0, 256, C.byref(h), buf) == L.SICU_EINVAL
    assert "sicu_init" in so.last_error()
    assert h.value is None
    assert so.lib.sicu_ar_open(None, buf) == L.SICU_EINVAL
    assert so.lib.sicu_ar_allreduce(None, 16, 16, None) == L.SICU_EINVAL
    assert so.lib.sicu_ar_set_timeout(None, 1000) == L.SICU_EINVAL
    assert so.lib.sicu_ar_destroy(None) == L.SICU_OK
    # the fused matvec: F16 has no fused form; shapes are checked first
    assert so.lib.sicu_gemv_ar(Q.F16, 4096, 256, 256, 16, 8192, None, None) == L.SICU_ENOTSUP
    assert so.lib.sicu_gemv_ar(Q.Q4_K, 4096, 300, 256, 16, 8192, None, None) == L.SICU_EINVAL
    assert so.lib.sicu_gemv_ar(Q.Q4_K, 4096, 256, 256, 16, 8192, None, None) == L.SICU_EINVAL   # no group


def test_activation_step_checks_run_on_host(so):
    """sicu_gemv_fused / sicu_rms_norm / sicu_swiglu reject malformed steps
    before any CUDA call (fake, aligned device addresses; no device)."""
    one = (C.c_void_p * 1)(0x10000)
    outs = (C.c_void_p * 1)(0x20000)
    rows = (C.c_int64 * 1)(64)

    def fused(step, n_in=256):
        return so.lib.sicu_gemv_fused(Q.Q4_K, 1, one, rows, n_in, 0x30000, C.byref(step) if step else None,
                                      None, outs, None, None)

    assert fused(L.Prologue(7, 0.0, None, None, None, None)) == L.SICU_EINVAL            # unknown kind
    assert fused(L.Prologue(L.PRO_RMS_NORM, 1e-5, None, None, None, None)) == L.SICU_EINVAL  # no weight
    assert fused(L.Prologue(L.PRO_RMS_NORM, 1e-5, 0x40004, None, None, None)) == L.SICU_EINVAL  # misaligned
    assert fused(L.Prologue(L.PRO_RMS_NORM, -1.0, 0x40000, None, None, None)) == L.SICU_EINVAL  # eps < 0
    assert fused(L.Prologue(L.PRO_RMS_NORM, 1e-5, 0x40000, None, 0x30000, None)) == L.SICU_EINVAL  # sum_out == x
    assert fused(L.Prologue(L.PRO_RMS_NORM, 1e-5, 0x40000, None, 0x20000, None)) == L.SICU_EINVAL  # sum_out == y
    assert fused(L.Prologue(L.PRO_SWIGLU, 0.0, None, None, None, None)) == L.SICU_EINVAL       # no up vector
    assert fused(L.Prologue(L.PRO_MUL, 0.0, None, None, None, None)) == L.SICU_EINVAL          # no up vector
    bad_epi = (C.c_int32 * 1)(5)
    assert so.lib.sicu_gemv_fused(Q.Q4_K, 1, one, rows, 256, 0x30000, None, bad_epi, outs, None, None) == L.SICU_EINVAL
    assert "epilogue" in so.last_error()
    # well-formed: refused only for want of an initialised device
    assert fused(L.Prologue(L.PRO_RMS_NORM, 1e-5, 0x40000, 0x50000, 0x60000, None)) == L.SICU_EINVAL
    assert "sicu_init" in so.last_error()
    assert fused(L.Prologue(L.PRO_SWIGLU, 0.0, None, None, None, 0x50000)) == L.SICU_EINVAL
    assert "sicu_init" in so.last_error()
    assert fused(None) == L.SICU_EINVAL and "sicu_init" in so.last_error()
    assert so.lib.sicu_swiglu(0x10000, 0x20000, 12, 1, 0x30000, None) == L.SICU_EINVAL      # 12 % 8
    assert "multiple of 8" in so.last_error()
    assert so.lib.sicu_rms_norm(0x10000, None, None, None, 256, 1, 1e-5, 0x30000, None) == L.SICU_EINVAL
    assert so.lib.sicu_rms_norm(0x10000, None, 0x10000, 0x20000, 256, 1, 1e-5, 0x30000, None) == L.SICU_EINVAL
    assert "overlaps" in so.last_error()


def test_softmax_checks_run_on_host(so):
    assert so.lib.sicu_softmax(0x10000, 0x20000, 0, 1, None) == L.SICU_EINVAL       # empty row
    assert so.lib.sicu_softmax(None, 0x20000, 16, 1, None) == L.SICU_EINVAL
    assert so.lib.sicu_softmax(0x10000, 0x10004, 16, 1, None) == L.SICU_EINVAL     # partial overlap
    assert "overlap" in so.last_error()
    assert so.lib.sicu_softmax(0x10000, 0x10000, 16, 1, None) == L.SICU_EINVAL     # in place: needs a device
    assert "sicu_init" in so.last_error()


def test_prefill_copy_size_and_checks_run_on_host(so):
    """The size of a prefill weight copy needs no GPU: per 128-row tile and
    super-block 4 x 16 KiB of f16 operands + 8 KiB of mins + 512 B of row
    scales (Q4_K), 8 x 16 KiB + 512 B (Q6_K)."""
    assert so.prefill_pack_bytes(Q.Q4_K, 4096, 4096) == 32 * 16 * (4 * 16384 + 8192 + 512)
    assert so.prefill_pack_bytes(Q.Q6_K, 1280, 130) == 2 * 5 * (8 * 16384 + 512)
    assert so.prefill_pack_bytes(Q.Q4_K, 256, 0) == 0
    # one f16 plane per K-step; Q5_K and Q2_K with the mins operand
    assert so.prefill_pack_bytes(Q.Q5_K, 4096, 4096) == 32 * 16 * (4 * 16384 + 8192 + 512)
    assert so.prefill_pack_bytes(Q.Q2_K, 1024, 300) == 3 * 4 * (4 * 16384 + 8192 + 512)
    assert so.prefill_pack_bytes(Q.Q3_K, 1280, 130) == 2 * 5 * (4 * 16384 + 512)
    n = C.c_size_t(7)
    assert so.lib.sicu_prefill_pack_bytes(Q.F32, 256, 128, C.byref(n)) == L.SICU_ENOTSUP and n.value == 0
    assert so.prefill_pack_bytes(Q.F16, 512, 130) == 2 * 2 * (4 * 16384 + 512)   # the f16 weights re-tiled
    # classic formats: per 128-row tile and K-step of four 32-blocks, 16 KiB of
    # int8 quants + 2 KiB of row scales; at least one 128-element K-step
    assert so.prefill_pack_bytes(Q.Q8_0, 4096, 4096) == 32 * 32 * (16384 + 2048)
    assert so.prefill_pack_bytes(Q.Q4_0, 160, 130) == 2 * 2 * (16384 + 2048)
    assert so.lib.sicu_prefill_pack_bytes(Q.Q5_0, 96, 128, C.byref(n)) == L.SICU_EINVAL
    assert so.lib.sicu_prefill_pack_bytes(Q.Q4_K, 300, 128, C.byref(n)) == L.SICU_EINVAL
    need = so.prefill_pack_bytes(Q.Q4_K, 256, 128)
    assert so.lib.sicu_prefill_pack(Q.Q4_K, 16, 256, 128, 32, need - 1, None) == L.SICU_EINVAL
    assert so.lib.sicu_prefill_pack(Q.Q4_K, 24, 256, 128, 32, need, None) == L.SICU_EINVAL   # misaligned
    assert so.lib.sicu_prefill_pack(Q.Q4_K, 16, 256, 128, 32, need, None) == L.SICU_EINVAL   # not initialised
    assert "sicu_init" in so.last_error()
    # a copy given for a type without one
    assert so.lib.sicu_gemm_prefill_packed_f32(Q.F32, 16, 32, 256, 128, 64, 64, 128, None) != L.SICU_OK


def test_prefill_multi_checks_run_on_host(so):
    """The grouped prefill entry checks its arrays and every matrix before any
    CUDA call: 1..4 matrices, null arrays, a copy for a type without one, a
    misaligned copy."""
    P = C.c_void_p
    w = (P * 2)(16, 16)
    ok_packs = (P * 2)(32, 48)
    bad_packs = (P * 2)(32, 40)
    n_out = (C.c_int64 * 2)(128, 128)
    y = (P * 2)(64, 64)
    f = so.lib.sicu_gemm_prefill_multi_f32
    assert f(Q.Q4_K, 0, w, ok_packs, n_out, 256, 128, 64, y, None) == L.SICU_EINVAL
    assert f(Q.Q4_K, 5, w, ok_packs, n_out, 256, 128, 64, y, None) == L.SICU_EINVAL
    assert f(Q.Q4_K, 2, None, ok_packs, n_out, 256, 128, 64, y, None) == L.SICU_EINVAL
    assert f(Q.Q4_K, 2, w, ok_packs, None, 256, 128, 64, y, None) == L.SICU_EINVAL
    assert f(Q.Q4_K, 2, w, bad_packs, n_out, 256, 128, 64, y, None) == L.SICU_EINVAL     # misaligned copy
    assert "aligned" in so.last_error()
    assert f(Q.F32, 2, w, ok_packs, n_out, 256, 128, 64, y, None) != L.SICU_OK          # no copies for F32
    assert f(Q.Q4_K, 2, w, ok_packs, n_out, 300, 128, 64, y, None) == L.SICU_EINVAL      # not whole super-blocks
    assert f(Q.Q4_K, 2, w, ok_packs, n_out, 256, 128, 64, y, None) == L.SICU_EINVAL      # not initialised
    assert "sicu_init" in so.last_error()


def test_attention_prompt_checks_run_on_host(so):
    """sicu_attention_prompt rejects bad shapes and positions before any
    device work: a prompt past the cache, GQA that does not divide, an odd
    or too large n_rot, null or misaligned buffers."""
    f = so.lib.sicu_attention_prompt
    p = 0x10000

    def call(n_head=8, nkv=2, hd=64, n_rot=64, n_ctx=64, pos0=0, m=4, ptr=p, cache=p):
        return f(ptr, ptr, ptr, cache, cache, ptr, ptr, n_head, nkv, hd, n_rot, 0, n_ctx, pos0, m, 0.125, ptr, None)
    assert call(pos0=60, m=5) == L.SICU_EINVAL               # past the cache
    assert call(nkv=3) == L.SICU_EINVAL                      # heads not a multiple of KV heads
    assert call(n_rot=63) == L.SICU_EINVAL
    assert call(n_rot=128) == L.SICU_EINVAL                  # more than the head
    assert call(hd=2048, n_rot=64) == L.SICU_EINVAL          # head larger than 1024
    assert call(m=-1) == L.SICU_EINVAL
    assert call(ptr=None) == L.SICU_EINVAL
    assert call(cache=p + 1) == L.SICU_EINVAL                # caches not 2-byte aligned
    assert call(n_ctx=40000, pos0=29000, m=1001) == L.SICU_EINVAL   # more than 30000 positions


def test_add_bias_checks_run_on_host(so):
    f = so.lib.sicu_add_bias
    p = 0x10000
    assert f(p, p + 0x8000, 0, 4, None) == L.SICU_EINVAL          # no columns
    assert f(p, p + 0x8000, 16, -1, None) == L.SICU_EINVAL
    assert f(None, p, 16, 4, None) == L.SICU_EINVAL
    assert f(p + 2, p + 0x8000, 16, 4, None) == L.SICU_EINVAL     # rows misaligned
    assert f(p, p + 64, 16, 4, None) == L.SICU_EINVAL             # bias inside the rows


def test_model_path_packs_what_the_library_accepts(so):
    """model_path.packable (which matrices get a prefill copy at load) agrees
    with sicu_prefill_pack_bytes for every type and a spread of row lengths."""
    from siphon_b200 import model_path as mp
    for wt in Q.WEIGHT_TYPES + (Q.F32,):
        blk = Q.GEOMETRY[wt][0]
        for n_in in (32, 64, 96, 128, 160, 256, 512, 640, 4096, 5120):
            if n_in % blk:
                continue                      # not a whole row of blocks: no model matrix
            n = C.c_size_t(0)
            ok = so.lib.sicu_prefill_pack_bytes(wt, n_in, 256, C.byref(n)) == 0
            assert ok == mp.packable(wt, n_in), (Q.NAMES[wt], n_in, ok)

"""ctypes binding of libsiphon_cuda.so (the C ABI in include/siphon_cuda.h).

This is the Python mirror of the reference's backend interface for the
quantized matrix path: ``gemv`` / ``gemv_f32`` / ``gemv_host`` stand where
``si_backend.gemv`` (include/siphon/tensor.h:43-55) stands, ``quantize_*``
where ``si_quant_row_q8_K`` / ``si_quant_row_q8_0`` stand, ``row_to_f32``
where ``si_backend.row_to_f32`` stands. Errors raise :class:`SicuError`
carrying the reference-style negative code and the library's message.

There is no fallback: if the shared library is missing the import of any
compute entry point raises.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

from . import quant as Q

LIB_PATH = Path(__file__).resolve().parent / "libsiphon_cuda.so"

SICU_OK, SICU_ENOMEM, SICU_EIO, SICU_EFORMAT, SICU_ENOTSUP, SICU_EINVAL = 0, -1, -2, -3, -4, -5

# every entry point of include/siphon_cuda.h with its ctypes signature
_i64, _u32, _vp, _fp = C.c_int64, C.c_uint32, C.c_void_p, C.c_void_p
SIGNATURES = {
    "sicu_init": [C.c_int],
    "sicu_shutdown": [],
    "sicu_last_error": [C.c_char_p, C.c_size_t],
    "sicu_status": [C.POINTER(C.c_int)],
    "sicu_tc_peak": [C.c_int, C.c_int, C.c_int, C.POINTER(C.c_float), C.POINTER(C.c_double)],
    "sicu_set_overlap": [C.c_int],
    "sicu_malloc": [C.POINTER(C.c_void_p), C.c_size_t],
    "sicu_free": [_vp],
    "sicu_upload": [_vp, C.c_size_t, C.POINTER(C.c_void_p)],
    "sicu_memcpy_h2d": [_vp, _vp, C.c_size_t, _vp],
    "sicu_memcpy_d2h": [_vp, _vp, C.c_size_t, _vp],
    "sicu_stream_sync": [_vp],
    "sicu_quant_geometry": [_u32, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32)],
    "sicu_vec_dot_pair": [_u32, C.POINTER(C.c_uint32)],
    "sicu_quantize_q8_K": [_fp, _vp, _i64, _i64, _vp],
    "sicu_quantize_q8_0": [_fp, _vp, _i64, _i64, _vp],
    "sicu_convert_f16": [_fp, _vp, _i64, _i64, _vp],
    "sicu_quantize_pair": [_u32, _fp, _vp, _i64, _i64, _vp],
    "sicu_gemv": [_u32, _vp, _i64, _i64, _vp, _fp, _i64, _vp],
    "sicu_gemv_f32": [_u32, _vp, _i64, _i64, _fp, _fp, _i64, _vp],
    "sicu_gemv_multi": [_u32, C.c_int, C.POINTER(C.c_void_p), C.POINTER(C.c_int64), _i64, _fp,
                        C.POINTER(C.c_void_p), _vp],
    "sicu_gemv_batch": [_u32, C.c_int, C.POINTER(C.c_void_p), C.POINTER(C.c_int64), _i64, _fp, _i64,
                        C.POINTER(C.c_void_p), _vp],
    "sicu_gemv_host": [_u32, _vp, _i64, _i64, _fp, _fp, _vp],
    "sicu_gemv_host_noalloc": [_u32, _vp, _i64, _i64, _fp, _fp, _vp],
    "sicu_row_to_f32": [_u32, _vp, _i64, C.POINTER(C.c_int64), _i64, _fp, _vp],
    "sicu_gemm_prefill": [_u32, _vp, _i64, _i64, _vp, _i64, _fp, _vp],
    "sicu_gemm_prefill_f32": [_u32, _vp, _i64, _i64, _fp, _i64, _fp, _vp],
    "sicu_prefill_pack_bytes": [_u32, _i64, _i64, C.POINTER(C.c_size_t)],
    "sicu_prefill_pack": [_u32, _vp, _i64, _i64, _vp, C.c_size_t, _vp],
    "sicu_gemm_prefill_packed": [_u32, _vp, _vp, _i64, _i64, _vp, _i64, _fp, _vp],
    "sicu_gemm_prefill_packed_f32": [_u32, _vp, _vp, _i64, _i64, _fp, _i64, _fp, _vp],
    "sicu_gemm_prefill_multi_f32": [_u32, C.c_int, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
                                    C.POINTER(C.c_int64), _i64, _fp, _i64, C.POINTER(C.c_void_p), _vp],
    "sicu_ar_create": [C.c_int, C.c_int, _i64, C.POINTER(C.c_void_p), _vp],
    "sicu_ar_open": [_vp, _vp],
    "sicu_ar_set_timeout": [_vp, C.c_uint64],
    "sicu_ar_destroy": [_vp],
    "sicu_ar_allreduce": [_vp, _fp, _fp, _vp],
    "sicu_gemv_ar": [_u32, _vp, _i64, _i64, _fp, _fp, _vp, _vp],
    "sicu_gemv_fused": [_u32, C.c_int, C.POINTER(C.c_void_p), C.POINTER(C.c_int64), _i64, _fp, _vp, _vp,
                        C.POINTER(C.c_void_p), _vp, _vp],
    "sicu_gemv_fused_ex": [_u32, C.c_int, C.POINTER(C.c_void_p), C.POINTER(C.c_int64), _i64, _fp, _vp, _vp,
                           C.POINTER(C.c_void_p), C.POINTER(C.c_void_p), _vp, _vp],
    "sicu_rms_norm": [_fp, _fp, _fp, _fp, _i64, _i64, C.c_float, _fp, _vp],
    "sicu_swiglu": [_fp, _fp, _i64, _i64, _fp, _vp],
    "sicu_add_bias": [_fp, _fp, _i64, _i64, _vp],
    "sicu_softmax": [_fp, _fp, _i64, _i64, _vp],
    "sicu_rope": [_fp, _i64, _i64, _i64, _fp, _fp, C.c_int, _vp],
    "sicu_kv_store": [_fp, _fp, _vp, _vp, _i64, _i64, _i64, _i64, _vp],
    "sicu_attention": [_fp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, C.c_float, _fp, _vp],
    "sicu_row_to_f32_dev": [_u32, _vp, _i64, _i64, _vp, _i64, _fp, _vp],
    "sicu_argmax": [_fp, _i64, _i64, _vp, _vp],
    "sicu_attention_step": [_fp, _fp, _fp, _vp, _vp, _fp, _fp, _i64, _i64, _i64, _i64, C.c_int, _i64, _i64,
                            C.c_float, _fp, _vp],
    "sicu_attention_prompt": [_fp, _fp, _fp, _vp, _vp, _fp, _fp, _i64, _i64, _i64, _i64, C.c_int, _i64, _i64,
                              _i64, C.c_float, _fp, _vp],
}

PRO_NONE, PRO_RMS_NORM, PRO_SWIGLU, PRO_MUL = 0, 1, 2, 3
EPI_NONE, EPI_SILU = 0, 1


class Prologue(C.Structure):
    """sicu_prologue: the activation step sicu_gemv_fused applies before
    quantizing (RMS norm with an optional residual add, SwiGLU, or the
    multiply that completes a SwiGLU whose silu ran as the gate's epilogue)."""
    _fields_ = [("kind", C.c_int32), ("eps", C.c_float), ("weight", C.c_void_p), ("residual", C.c_void_p),
                ("sum_out", C.c_void_p), ("up", C.c_void_p)]

TC_F16, TC_I8 = 0, 1       # sicu_tc_peak kinds
AR_HANDLE_BYTES = 64
STATUS_WAIT_TIMEOUT, STATUS_AR_TIMEOUT, STATUS_BAD_ROW = 1, 2, 4


def rms_norm_step(weight, eps: float, residual=None, sum_out=None) -> Prologue:
    """a = (x + residual) * rms_scale * weight; sum_out receives x + residual."""
    return Prologue(PRO_RMS_NORM, eps, _ptr(weight), _ptr(residual), _ptr(sum_out), None)


def swiglu_step(up) -> Prologue:
    """a = silu(x) * up."""
    return Prologue(PRO_SWIGLU, 0.0, None, None, None, _ptr(up))


def mul_step(up) -> Prologue:
    """a = x * up (x already through silu: the gate product's EPI_SILU)."""
    return Prologue(PRO_MUL, 0.0, None, None, None, _ptr(up))


class SicuError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"libsiphon_cuda error {code}: {msg}")
        self.code = code


def _ptr(x) -> int | None:
    """Device/host address of a torch tensor, numpy array or int."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if hasattr(x, "ctypes"):
        return x.ctypes.data
    raise TypeError(f"cannot take the address of {type(x)}")


class SiphonCuda:
    def __init__(self, path: Path = LIB_PATH):
        if not Path(path).exists():
            raise FileNotFoundError(f"{path} is not built; run `python -m siphon_b200.build`")
        self.lib = C.CDLL(str(path))
        for name, args in SIGNATURES.items():
            f = getattr(self.lib, name)
            f.argtypes = args
            f.restype = C.c_int

    # -- errors ---------------------------------------------------------------
    def last_error(self) -> str:
        buf = C.create_string_buffer(512)
        self.lib.sicu_last_error(buf, 512)
        return buf.value.decode(errors="replace")

    def check(self, rc: int) -> None:
        if rc != SICU_OK:
            raise SicuError(rc, self.last_error())

    # -- lifecycle --------------------------------------------------------------
    def init(self, device: int = 0) -> None:
        self.check(self.lib.sicu_init(device))

    def shutdown(self) -> None:
        self.check(self.lib.sicu_shutdown())

    def set_overlap(self, on: bool) -> None:
        self.check(self.lib.sicu_set_overlap(1 if on else 0))

    def tc_peak(self, kind: int, rounds: int, sms: int) -> tuple[float, float]:
        """(ms, TFLOP/s) of the tensor-core throughput probe (kind TC_F16 or TC_I8)."""
        ms, tf = C.c_float(), C.c_double()
        self.check(self.lib.sicu_tc_peak(kind, rounds, sms, C.byref(ms), C.byref(tf)))
        return ms.value, tf.value

    def status(self) -> int:
        flags = C.c_int(0)
        self.check(self.lib.sicu_status(C.byref(flags)))
        return flags.value

    # -- geometry -----------------------------------------------------------------
    def geometry(self, t: int) -> tuple[int, int]:
        b, s = C.c_uint32(), C.c_uint32()
        self.check(self.lib.sicu_quant_geometry(t, C.byref(b), C.byref(s)))
        return b.value, s.value

    def pair_type(self, wtype: int) -> int:
        p = C.c_uint32()
        self.check(self.lib.sicu_vec_dot_pair(wtype, C.byref(p)))
        return p.value

    # -- compute ----------------------------------------------------------------------
    def quantize_q8_K(self, dx, dy, n: int, m: int = 1, stream=None) -> None:
        self.check(self.lib.sicu_quantize_q8_K(_ptr(dx), _ptr(dy), n, m, _ptr(stream)))

    def quantize_q8_0(self, dx, dy, n: int, m: int = 1, stream=None) -> None:
        self.check(self.lib.sicu_quantize_q8_0(_ptr(dx), _ptr(dy), n, m, _ptr(stream)))

    def convert_f16(self, dx, dy, n: int, m: int = 1, stream=None) -> None:
        self.check(self.lib.sicu_convert_f16(_ptr(dx), _ptr(dy), n, m, _ptr(stream)))

    def quantize_pair(self, wtype: int, dx, dxq, n: int, m: int = 1, stream=None) -> None:
        self.check(self.lib.sicu_quantize_pair(wtype, _ptr(dx), _ptr(dxq), n, m, _ptr(stream)))

    def gemv(self, wtype: int, dw, n_in: int, n_out: int, dxq, dy, m: int = 1, stream=None) -> None:
        self.check(self.lib.sicu_gemv(wtype, _ptr(dw), n_in, n_out, _ptr(dxq), _ptr(dy), m, _ptr(stream)))

    def gemv_f32(self, wtype: int, dw, n_in: int, n_out: int, dx, dy, m: int = 1, stream=None) -> None:
        self.check(self.lib.sicu_gemv_f32(wtype, _ptr(dw), n_in, n_out, _ptr(dx), _ptr(dy), m, _ptr(stream)))

    def gemv_multi(self, wtype: int, dws, n_outs, n_in: int, dx, dys, stream=None) -> None:
        n = len(dws)
        w_arr = (C.c_void_p * n)(*[_ptr(w) for w in dws])
        y_arr = (C.c_void_p * n)(*[_ptr(y) for y in dys])
        o_arr = (C.c_int64 * n)(*n_outs)
        self.check(self.lib.sicu_gemv_multi(wtype, n, w_arr, o_arr, n_in, _ptr(dx), y_arr, _ptr(stream)))

    def gemv_batch(self, wtype: int, dws, n_outs, n_in: int, dx, m: int, dys, stream=None) -> None:
        """dys[i][t] = W_i x_t for the m <= 8 f32 rows of dx (each dys[i] is [m][n_outs[i]])."""
        n = len(dws)
        w_arr = (C.c_void_p * n)(*[_ptr(w) for w in dws])
        y_arr = (C.c_void_p * n)(*[_ptr(y) for y in dys])
        o_arr = (C.c_int64 * n)(*n_outs)
        self.check(self.lib.sicu_gemv_batch(wtype, n, w_arr, o_arr, n_in, _ptr(dx), m, y_arr, _ptr(stream)))

    def gemv_host(self, wtype: int, dw, n_in: int, n_out: int, hx, hy, stream=None) -> None:
        self.check(self.lib.sicu_gemv_host(wtype, _ptr(dw), n_in, n_out, _ptr(hx), _ptr(hy), _ptr(stream)))

    def gemv_host_noalloc(self, wtype: int, dw, n_in: int, n_out: int, hx, hy, stream=None) -> None:
        self.check(self.lib.sicu_gemv_host_noalloc(wtype, _ptr(dw), n_in, n_out, _ptr(hx), _ptr(hy), _ptr(stream)))

    def gemm_prefill(self, wtype: int, dw, n_in: int, n_out: int, dxq, m: int, dy, stream=None) -> None:
        self.check(self.lib.sicu_gemm_prefill(wtype, _ptr(dw), n_in, n_out, _ptr(dxq), m, _ptr(dy), _ptr(stream)))

    def gemm_prefill_f32(self, wtype: int, dw, n_in: int, n_out: int, dx, m: int, dy, stream=None) -> None:
        self.check(self.lib.sicu_gemm_prefill_f32(wtype, _ptr(dw), n_in, n_out, _ptr(dx), m, _ptr(dy), _ptr(stream)))

    # -- prefill copies of the weights -------------------------------------------------
    def prefill_pack_bytes(self, wtype: int, n_in: int, n_out: int) -> int:
        n = C.c_size_t(0)
        self.check(self.lib.sicu_prefill_pack_bytes(wtype, n_in, n_out, C.byref(n)))
        return n.value

    def prefill_pack(self, wtype: int, dw, n_in: int, n_out: int, dpack, pack_bytes: int, stream=None) -> None:
        self.check(self.lib.sicu_prefill_pack(wtype, _ptr(dw), n_in, n_out, _ptr(dpack), pack_bytes, _ptr(stream)))

    def gemm_prefill_packed(self, wtype: int, dw, dpack, n_in: int, n_out: int, dxq, m: int, dy, stream=None) -> None:
        self.check(self.lib.sicu_gemm_prefill_packed(wtype, _ptr(dw), _ptr(dpack), n_in, n_out, _ptr(dxq), m,
                                                     _ptr(dy), _ptr(stream)))

    def gemm_prefill_packed_f32(self, wtype: int, dw, dpack, n_in: int, n_out: int, dx, m: int, dy,
                                stream=None) -> None:
        self.check(self.lib.sicu_gemm_prefill_packed_f32(wtype, _ptr(dw), _ptr(dpack), n_in, n_out, _ptr(dx), m,
                                                         _ptr(dy), _ptr(stream)))

    def gemm_prefill_multi_f32(self, wtype: int, dws, dpacks, n_outs, n_in: int, dx, m: int, dys,
                               stream=None) -> None:
        """sicu_gemm_prefill_multi_f32: the products of several matrices that
        read one m-token activation, from their prefill copies (dpacks may be
        None, or hold None entries)."""
        n = len(dws)
        w_arr = (C.c_void_p * n)(*[_ptr(w) for w in dws])
        p_arr = (C.c_void_p * n)(*[_ptr(p) for p in dpacks]) if dpacks is not None else None
        o_arr = (C.c_int64 * n)(*n_outs)
        y_arr = (C.c_void_p * n)(*[_ptr(y) for y in dys])
        self.check(self.lib.sicu_gemm_prefill_multi_f32(wtype, n, w_arr, p_arr, o_arr, n_in, _ptr(dx), m, y_arr,
                                                        _ptr(stream)))

    # -- fused all-reduce groups ---------------------------------------------------
    def ar_create(self, n_ranks: int, rank: int, length: int) -> "ArGroup":
        return ArGroup(self, n_ranks, rank, length)

    def gemv_ar(self, wtype: int, dw, n_in: int, n_out: int, dx, dy, group: "ArGroup", stream=None) -> None:
        """sicu_gemv_ar: this rank's column shard times x, summed over the group."""
        self.check(self.lib.sicu_gemv_ar(wtype, _ptr(dw), n_in, n_out, _ptr(dx), _ptr(dy), group.handle,
                                         _ptr(stream)))

    # -- activation steps ------------------------------------------------------------
    def gemv_fused(self, wtype: int, dws, n_outs, n_in: int, dx, step: Prologue | None, dys,
                   group: "ArGroup | None" = None, stream=None, epi=None, bias=None) -> None:
        """sicu_gemv_fused: dys[i] = epi[i](W_i (step applied to dx) [+ bias[i]]),
        optionally all-reduced over group (one matrix)."""
        n = len(dws)
        w_arr = (C.c_void_p * n)(*[_ptr(w) for w in dws])
        y_arr = (C.c_void_p * n)(*[_ptr(y) for y in dys])
        o_arr = (C.c_int64 * n)(*n_outs)
        e_arr = (C.c_int32 * n)(*epi) if epi is not None else None
        pro = C.byref(step) if step is not None else None
        grp = group.handle if group is not None else None
        if bias is None:
            self.check(self.lib.sicu_gemv_fused(wtype, n, w_arr, o_arr, n_in, _ptr(dx), pro, e_arr, y_arr, grp,
                                                _ptr(stream)))
        else:
            b_arr = (C.c_void_p * n)(*[_ptr(b) for b in bias])
            self.check(self.lib.sicu_gemv_fused_ex(wtype, n, w_arr, o_arr, n_in, _ptr(dx), pro, e_arr, b_arr, y_arr,
                                                   grp, _ptr(stream)))

    def rms_norm(self, dx, dw, n: int, m: int, eps: float, dy, dres=None, dsum=None, stream=None) -> None:
        self.check(self.lib.sicu_rms_norm(_ptr(dx), _ptr(dres), _ptr(dsum), _ptr(dw), n, m, eps, _ptr(dy),
                                          _ptr(stream)))

    def swiglu(self, dx, dup, n: int, m: int, dy, stream=None) -> None:
        self.check(self.lib.sicu_swiglu(_ptr(dx), _ptr(dup), n, m, _ptr(dy), _ptr(stream)))

    def add_bias(self, dy, db, n: int, m: int, stream=None) -> None:
        """sicu_add_bias: dy_r += db for m rows of n floats."""
        self.check(self.lib.sicu_add_bias(_ptr(dy), _ptr(db), n, m, _ptr(stream)))

    def softmax(self, dx, dy, n: int, m: int = 1, stream=None) -> None:
        """sicu_softmax: the reference's attention softmax over m rows."""
        self.check(self.lib.sicu_softmax(_ptr(dx), _ptr(dy), n, m, _ptr(stream)))

    def rope(self, dx, n_heads: int, head_dim: int, n_rot: int, dcos, dsin, neox: bool = False, stream=None) -> None:
        self.check(self.lib.sicu_rope(_ptr(dx), n_heads, head_dim, n_rot, _ptr(dcos), _ptr(dsin), 1 if neox else 0,
                                      _ptr(stream)))

    def kv_store(self, dk, dv, dk_cache, dv_cache, n_head_kv: int, head_dim: int, n_ctx: int, pos: int,
                 stream=None) -> None:
        self.check(self.lib.sicu_kv_store(_ptr(dk), _ptr(dv), _ptr(dk_cache), _ptr(dv_cache), n_head_kv, head_dim,
                                          n_ctx, pos, _ptr(stream)))

    def attention(self, dq, dk_cache, dv_cache, n_head: int, n_head_kv: int, head_dim: int, n_ctx: int, pos: int,
                  kq_scale: float, dout, stream=None) -> None:
        self.check(self.lib.sicu_attention(_ptr(dq), _ptr(dk_cache), _ptr(dv_cache), n_head, n_head_kv, head_dim,
                                           n_ctx, pos, kq_scale, _ptr(dout), _ptr(stream)))

    def attention_step(self, dq, dk, dv, dk_cache, dv_cache, dcos, dsin, n_head: int, n_head_kv: int, head_dim: int,
                       n_rot: int, n_ctx: int, pos: int, kq_scale: float, dout, neox: bool = False,
                       stream=None) -> None:
        self.check(self.lib.sicu_attention_step(_ptr(dq), _ptr(dk), _ptr(dv), _ptr(dk_cache), _ptr(dv_cache),
                                                _ptr(dcos), _ptr(dsin), n_head, n_head_kv, head_dim, n_rot,
                                                1 if neox else 0, n_ctx, pos, kq_scale, _ptr(dout), _ptr(stream)))

    def attention_prompt(self, dq, dk, dv, dk_cache, dv_cache, dcos, dsin, n_head: int, n_head_kv: int,
                         head_dim: int, n_rot: int, n_ctx: int, pos0: int, m: int, kq_scale: float, dout,
                         neox: bool = False, stream=None) -> None:
        """attention_step for the m consecutive positions pos0 .. pos0 + m - 1 (a prompt)."""
        self.check(self.lib.sicu_attention_prompt(_ptr(dq), _ptr(dk), _ptr(dv), _ptr(dk_cache), _ptr(dv_cache),
                                                  _ptr(dcos), _ptr(dsin), n_head, n_head_kv, head_dim, n_rot,
                                                  1 if neox else 0, n_ctx, pos0, m, kq_scale, _ptr(dout),
                                                  _ptr(stream)))

    def row_to_f32_dev(self, wtype: int, dw, n_in: int, n_rows: int, drows, nrows: int, dout, stream=None) -> None:
        self.check(self.lib.sicu_row_to_f32_dev(wtype, _ptr(dw), n_in, n_rows, _ptr(drows), nrows, _ptr(dout),
                                                _ptr(stream)))

    def argmax(self, dx, n: int, m: int, dout, stream=None) -> None:
        self.check(self.lib.sicu_argmax(_ptr(dx), n, m, _ptr(dout), _ptr(stream)))

    def row_to_f32(self, wtype: int, dw, n_in: int, rows, dout, stream=None) -> None:
        arr = (C.c_int64 * len(rows))(*rows)
        self.check(self.lib.sicu_row_to_f32(wtype, _ptr(dw), n_in, arr, len(rows), _ptr(dout), _ptr(stream)))

    # -- memory ---------------------------------------------------------------------
    def upload(self, host) -> int:
        p = C.c_void_p()
        self.check(self.lib.sicu_upload(_ptr(host), host.nbytes, C.byref(p)))
        return p.value

    def free(self, dev: int) -> None:
        self.check(self.lib.sicu_free(dev))


class ArGroup:
    """One rank's member of an all-reduce group (sicu_ar_*): create, exchange
    `local_handle` with the other ranks, `open` with all of them in rank
    order, then pass it to gemv_ar / allreduce."""

    def __init__(self, sicu: SiphonCuda, n_ranks: int, rank: int, length: int):
        self.s, self.n, self.rank, self.len = sicu, n_ranks, rank, length
        h = C.c_void_p()
        buf = C.create_string_buffer(AR_HANDLE_BYTES)
        sicu.check(sicu.lib.sicu_ar_create(n_ranks, rank, length, C.byref(h), buf))
        self.handle = h.value
        self.local_handle = buf.raw

    def open(self, handles: list[bytes]) -> None:
        if len(handles) != self.n or any(len(x) != AR_HANDLE_BYTES for x in handles):
            raise ValueError("one 64-byte handle per rank expected")
        blob = C.create_string_buffer(b"".join(handles), AR_HANDLE_BYTES * self.n)
        self.s.check(self.s.lib.sicu_ar_open(self.handle, blob))

    def set_timeout(self, ns: int) -> None:
        self.s.check(self.s.lib.sicu_ar_set_timeout(self.handle, ns))

    def allreduce(self, dsrc, ddst, stream=None) -> None:
        self.s.check(self.s.lib.sicu_ar_allreduce(self.handle, _ptr(dsrc), _ptr(ddst), _ptr(stream)))

    def destroy(self) -> None:
        if self.handle:
            self.s.check(self.s.lib.sicu_ar_destroy(self.handle))
            self.handle = None


_LIB: SiphonCuda | None = None


def load() -> SiphonCuda:
    """The process-wide binding (raises if the library is not built)."""
    global _LIB
    if _LIB is None:
        _LIB = SiphonCuda()
    return _LIB


def pair_row_bytes(wtype: int, n: int) -> int:
    return Q.row_bytes(Q.pair_type(wtype), n)

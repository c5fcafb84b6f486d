"""Python binding of the CPU checkers in oracle/ (TEST INFRASTRUCTURE ONLY).

Two libraries, both built by oracle/Makefile:

* ``Oracle``  -- libsiphon_oracle.so, our C restatement of the reference's
  quantized matrix path (siphon_oracle.c). Always present once built.
* ``Reference`` -- _ref/libsiphon_ref.so, the reference compiled unmodified
  from its own sources. Present wherever it was built (this container, and
  the GPU box because built files travel with the tree).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import
this module. The CUDA product never does.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "libsiphon_oracle.so"
REF_SO = HERE / "_ref" / "libsiphon_ref.so"

_fp = np.ctypeslib.ndpointer
_u8 = _fp(dtype=np.uint8, flags="C_CONTIGUOUS")
_f32 = _fp(dtype=np.float32, flags="C_CONTIGUOUS")
_u16 = _fp(dtype=np.uint16, flags="C_CONTIGUOUS")

# ggml ids and block geometry (include/siphon/quant.h:92-119)
F32, F16, Q4_0, Q5_0, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, Q8_K = 0, 1, 2, 6, 8, 10, 11, 12, 13, 14, 15
GEOM = {F32: (1, 4), F16: (1, 2), Q4_0: (32, 18), Q5_0: (32, 22), Q8_0: (32, 34), Q2_K: (256, 84),
        Q3_K: (256, 110), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210), Q8_K: (256, 292)}
PAIR = {F32: F32, F16: F16, Q4_0: Q8_0, Q5_0: Q8_0, Q8_0: Q8_0,
        Q2_K: Q8_K, Q3_K: Q8_K, Q4_K: Q8_K, Q5_K: Q8_K, Q6_K: Q8_K}
DOT_NAME = {F16: "f16", Q4_0: "q4_0", Q5_0: "q5_0", Q8_0: "q8_0", Q2_K: "q2_K", Q3_K: "q3_K",
            Q4_K: "q4_K", Q5_K: "q5_K", Q6_K: "q6_K"}
REF_DOT_NAME = {F16: "f16", Q4_0: "q4_0_q8_0", Q5_0: "q5_0_q8_0", Q8_0: "q8_0_q8_0", Q2_K: "q2_K_q8_K",
                Q3_K: "q3_K_q8_K", Q4_K: "q4_K_q8_K", Q5_K: "q5_K_q8_K", Q6_K: "q6_K_q8_K"}


def row_bytes(t: int, n: int) -> int:
    blck, size = GEOM[t]
    assert n % blck == 0
    return n // blck * size


def _as_f32(x) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32)


class Oracle:
    """Our C restatement (siphon_oracle.c)."""

    def __init__(self, path: Path = ORACLE_SO):
        if not path.exists():
            raise FileNotFoundError(f"{path} not built (run make -C oracle)")
        L = self.lib = C.CDLL(str(path))
        L.orc_f16_to_f32.argtypes = [C.c_uint16]
        L.orc_f16_to_f32.restype = C.c_float
        L.orc_f32_to_f16.argtypes = [C.c_float]
        L.orc_f32_to_f16.restype = C.c_uint16
        for name in ("orc_quant_q8_K", "orc_quant_q8_0", "orc_quant_q8_0_scalar"):
            getattr(L, name).argtypes = [_f32, _u8, C.c_int]
            getattr(L, name).restype = None
        L.orc_convert_f16.argtypes = [_f32, _u16, C.c_int]
        L.orc_quantize_pair.argtypes = [C.c_uint32, _f32, C.c_void_p, C.c_int]
        L.orc_quantize_pair.restype = C.c_int
        L.orc_vec_dot.argtypes = [C.c_uint32, C.c_int, C.c_void_p, C.c_void_p, C.POINTER(C.c_float)]
        L.orc_vec_dot.restype = C.c_int
        L.orc_gemv_rows.argtypes = [C.c_uint32, C.c_void_p, C.c_int64, C.c_int, C.c_int64, C.c_int64,
                                    C.c_void_p, _f32]
        L.orc_gemv_rows.restype = C.c_int
        L.orc_dequant_row.argtypes = [C.c_uint32, C.c_void_p, _f32, C.c_int]
        L.orc_dequant_row.restype = C.c_int
        L.orc_geometry.argtypes = [C.c_uint32, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32)]
        L.orc_geometry.restype = C.c_int
        L.orc_pair_type.argtypes = [C.c_uint32, C.POINTER(C.c_uint32)]
        L.orc_pair_type.restype = C.c_int
        for name in ("orc_expf", "orc_silu"):
            getattr(L, name).argtypes = [C.c_float]
            getattr(L, name).restype = C.c_float
        L.orc_rms_scale.argtypes = [_f32, C.c_int, C.c_float]
        L.orc_rms_scale.restype = C.c_float
        L.orc_rms_norm.argtypes = [_f32, C.c_void_p, _f32, _f32, C.c_int, C.c_float, _f32]
        L.orc_rms_norm.restype = None
        L.orc_swiglu.argtypes = [_f32, _f32, C.c_int, _f32]
        L.orc_swiglu.restype = None
        L.orc_softmax.argtypes = [_f32, _f32, C.c_int]
        L.orc_softmax.restype = None
        L.orc_expf_restated_mismatches.argtypes = [C.c_uint32, C.c_uint32, C.c_uint32]
        L.orc_expf_restated_mismatches.restype = C.c_long
        L.orc_rope_table.argtypes = [C.c_float, C.c_int, C.c_int, _f32, _f32]
        L.orc_rope_table.restype = None
        L.orc_rope.argtypes = [_f32, C.c_int, C.c_int, C.c_int, _f32, _f32, C.c_int]
        L.orc_rope.restype = None
        L.orc_attention.argtypes = [_f32, _u16, _u16, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, _f32]
        L.orc_attention.restype = None

    # -- conversions / quantizers ------------------------------------------
    def f16_to_f32(self, h: int) -> float:
        return self.lib.orc_f16_to_f32(h)

    def f32_to_f16(self, f: float) -> int:
        return self.lib.orc_f32_to_f16(f)

    def quant_q8_K(self, x) -> np.ndarray:
        x = _as_f32(x).reshape(-1)
        y = np.zeros(row_bytes(Q8_K, x.size), np.uint8)
        self.lib.orc_quant_q8_K(x, y, x.size)
        return y

    def quant_q8_0(self, x, scalar: bool = False) -> np.ndarray:
        x = _as_f32(x).reshape(-1)
        y = np.zeros(row_bytes(Q8_0, x.size), np.uint8)
        (self.lib.orc_quant_q8_0_scalar if scalar else self.lib.orc_quant_q8_0)(x, y, x.size)
        return y

    def convert_f16(self, x) -> np.ndarray:
        x = _as_f32(x).reshape(-1)
        y = np.zeros(x.size, np.uint16)
        self.lib.orc_convert_f16(x, y, x.size)
        return y.view(np.uint8)

    def quantize_pair(self, wtype: int, x) -> np.ndarray:
        """[m, n] f32 -> [m, pair_row_bytes] uint8, each row quantized alone."""
        x = _as_f32(x)
        x2 = x.reshape(-1, x.shape[-1])
        n = x2.shape[1]
        out = np.zeros((x2.shape[0], row_bytes(PAIR[wtype], n)), np.uint8)
        for i in range(x2.shape[0]):
            row = np.ascontiguousarray(x2[i])
            rc = self.lib.orc_quantize_pair(wtype, row, out[i].ctypes.data, n)
            assert rc == 0
        return out

    # -- activation steps between products -----------------------------------
    def expf(self, x: float) -> float:
        return self.lib.orc_expf(x)

    def silu(self, x: float) -> float:
        return self.lib.orc_silu(x)

    def rms_scale(self, x, eps: float) -> float:
        x = _as_f32(x).reshape(-1)
        return self.lib.orc_rms_scale(x, x.size, eps)

    def rms_norm(self, x, w, eps: float, res=None):
        """(h, y): h = x (+ res), y = h * rms_scale(h) * w, one row."""
        x, w = _as_f32(x).reshape(-1), _as_f32(w).reshape(-1)
        h = np.zeros_like(x)
        y = np.zeros_like(x)
        r = None if res is None else _as_f32(res).reshape(-1)
        self.lib.orc_rms_norm(x, None if r is None else r.ctypes.data, h, w, x.size, eps, y)
        return h, y

    def swiglu(self, x, g) -> np.ndarray:
        """swiglu_row: silu(x) * g, the n % 8 tail through libm's expf."""
        x, g = _as_f32(x).reshape(-1), _as_f32(g).reshape(-1)
        y = np.zeros_like(x)
        self.lib.orc_swiglu(x, g, x.size, y)
        return y

    def softmax(self, x) -> np.ndarray:
        """The attention softmax of one row (row max, then si_softmax)."""
        x = _as_f32(x).reshape(-1)
        y = np.zeros_like(x)
        self.lib.orc_softmax(x, y, x.size)
        return y

    def rope_table(self, base: float, n_rot: int, n_pos: int) -> tuple[np.ndarray, np.ndarray]:
        cs = np.zeros((n_pos, n_rot // 2), np.float32)
        sn = np.zeros((n_pos, n_rot // 2), np.float32)
        self.lib.orc_rope_table(base, n_rot, n_pos, cs, sn)
        return cs, sn

    def rope(self, x, n_heads: int, hd: int, n_rot: int, cs, sn, neox: bool = False) -> np.ndarray:
        y = _as_f32(x).reshape(-1).copy()
        self.lib.orc_rope(y, n_heads, hd, n_rot, _as_f32(cs), _as_f32(sn), 1 if neox else 0)
        return y

    def attention(self, q, k_cache, v_cache, n_head: int, n_head_kv: int, hd: int, n_ctx: int, pos: int,
                  ks: float) -> np.ndarray:
        """attn_head for every query head; caches as uint16 f16 bits."""
        out = np.zeros(n_head * hd, np.float32)
        self.lib.orc_attention(_as_f32(q).reshape(-1), np.ascontiguousarray(k_cache, np.uint16).reshape(-1),
                               np.ascontiguousarray(v_cache, np.uint16).reshape(-1), n_head, n_head_kv, hd, n_ctx,
                               pos, ks, out)
        return out

    def silu_vec(self, x) -> np.ndarray:
        """si_silu element by element (no tail rule)."""
        return np.array([self.lib.orc_silu(float(v)) for v in np.asarray(x, np.float32).reshape(-1)], np.float32)

    # -- products -------------------------------------------------------------
    def vec_dot(self, wtype: int, n: int, x: np.ndarray, y: np.ndarray) -> float:
        s = C.c_float()
        rc = self.lib.orc_vec_dot(wtype, n, x.ctypes.data, y.ctypes.data, C.byref(s))
        assert rc == 0
        return s.value

    def gemv(self, wtype: int, w: np.ndarray, n_in: int, n_out: int, xq: np.ndarray) -> np.ndarray:
        """y[n_out] = W xq with xq already in the pair format (one activation row)."""
        y = np.zeros(n_out, np.float32)
        w = np.ascontiguousarray(w)
        xq = np.ascontiguousarray(xq)
        rc = self.lib.orc_gemv_rows(wtype, w.ctypes.data, row_bytes(wtype, n_in), n_in, 0, n_out,
                                    xq.ctypes.data, y)
        assert rc == 0
        return y

    def gemv_batch(self, wtype: int, w: np.ndarray, n_in: int, n_out: int, xq: np.ndarray,
                   threads: int = 0) -> np.ndarray:
        """[m, n_out] results for m pair-format activation rows; rows of W are
        split over threads (ctypes releases the GIL)."""
        xq = np.ascontiguousarray(xq).reshape(-1, row_bytes(PAIR[wtype], n_in))
        m = xq.shape[0]
        y = np.zeros((m, n_out), np.float32)
        w = np.ascontiguousarray(w)
        threads = threads or min(os.cpu_count() or 1, 16)
        rb = row_bytes(wtype, n_in)
        jobs = []
        for i in range(m):
            step = (n_out + threads - 1) // threads
            for r0 in range(0, n_out, step):
                jobs.append((i, r0, min(n_out, r0 + step)))

        def run(job):
            i, r0, r1 = job
            yi = y[i]
            rc = self.lib.orc_gemv_rows(wtype, w.ctypes.data, rb, n_in, r0, r1, xq[i].ctypes.data, yi)
            assert rc == 0

        if threads == 1 or len(jobs) == 1:
            for j in jobs:
                run(j)
        else:
            from concurrent.futures import ThreadPoolExecutor
            with ThreadPoolExecutor(threads) as ex:
                list(ex.map(run, jobs))
        return y

    def dequant_row(self, t: int, x: np.ndarray, n: int) -> np.ndarray:
        y = np.zeros(n, np.float32)
        rc = self.lib.orc_dequant_row(t, np.ascontiguousarray(x).ctypes.data, y, n)
        assert rc == 0
        return y


# ---- the reference itself ---------------------------------------------------------

class SiTensor(C.Structure):
    """si_tensor, include/siphon/tensor.h:33-41"""
    _fields_ = [("type", C.c_uint32), ("ne", C.c_uint64 * 4), ("n_elems", C.c_uint64),
                ("n_bytes", C.c_uint64), ("data", C.c_void_p), ("loc", C.c_int), ("be", C.c_void_p)]


GEMV_FN = C.CFUNCTYPE(None, C.c_void_p, C.POINTER(SiTensor), C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p)
ROW_FN = C.CFUNCTYPE(None, C.c_void_p, C.POINTER(SiTensor), C.c_uint64, C.c_void_p)


class SiBackend(C.Structure):
    """si_backend, include/siphon/tensor.h:43-55"""
    _fields_ = [("name", C.c_char_p), ("loc", C.c_int), ("gemv", GEMV_FN), ("row_to_f32", ROW_FN)]


class Reference:
    """The reference compiled from its own sources (oracle/_ref)."""

    def __init__(self, path: Path = REF_SO):
        if not path.exists():
            raise FileNotFoundError(f"{path} not built (run make -C oracle ref)")
        L = self.lib = C.CDLL(str(path))
        L.si_kern_init.restype = None
        L.si_kern_init()
        L.si_kern_impl_name.restype = C.c_char_p
        L.si_f16_to_f32.argtypes = [C.c_uint16]
        L.si_f16_to_f32.restype = C.c_float
        L.si_f32_to_f16.argtypes = [C.c_float]
        L.si_f32_to_f16.restype = C.c_uint16
        for name in ("si_quant_row_q8_K", "si_quant_row_q8_0", "si_avx2_quant_row_q8_0"):
            getattr(L, name).argtypes = [_f32, _u8, C.c_int]
            getattr(L, name).restype = None
        for t, nm in REF_DOT_NAME.items():
            for pre in ("si_dot_", "si_avx2_dot_"):
                f = getattr(L, pre + nm)
                f.argtypes = [C.c_int, C.POINTER(C.c_float), C.c_void_p, C.c_void_p]
                f.restype = None
        L.si_dequant_row.argtypes = [C.c_uint32, C.c_void_p, _f32, C.c_int]
        L.si_dequant_row.restype = C.c_bool
        L.si_backend_cpu.restype = C.POINTER(SiBackend)
        L.si_tp_create.argtypes = [C.c_int]
        L.si_tp_create.restype = C.c_void_p
        L.si_tp_free.argtypes = [C.c_void_p]
        L.si_tp_free.restype = None
        for name in ("si_expf", "si_silu"):
            getattr(L, name).argtypes = [C.c_float]
            getattr(L, name).restype = C.c_float
        L.si_rms_scale.argtypes = [_f32, C.c_int, C.c_float]
        L.si_rms_scale.restype = C.c_float
        L.si_softmax.argtypes = [_f32, _f32, C.c_int, C.c_float]
        L.si_softmax.restype = None

    @property
    def impl(self) -> str:
        return self.lib.si_kern_impl_name().decode()

    def quant_q8_K(self, x) -> np.ndarray:
        x = _as_f32(x).reshape(-1)
        y = np.zeros(row_bytes(Q8_K, x.size), np.uint8)
        self.lib.si_quant_row_q8_K(x, y, x.size)
        return y

    def quant_q8_0(self, x, form: str = "avx2") -> np.ndarray:
        x = _as_f32(x).reshape(-1)
        y = np.zeros(row_bytes(Q8_0, x.size), np.uint8)
        fn = {"avx2": self.lib.si_avx2_quant_row_q8_0, "dispatch": self.lib.si_quant_row_q8_0}[form]
        fn(x, y, x.size)
        return y

    def convert_f16(self, x) -> np.ndarray:
        x = _as_f32(x).reshape(-1)
        return np.array([self.lib.si_f32_to_f16(float(v)) for v in x], np.uint16).view(np.uint8)

    def vec_dot(self, wtype: int, n: int, x: np.ndarray, y: np.ndarray, avx2: bool = False) -> float:
        s = C.c_float()
        fn = getattr(self.lib, ("si_avx2_dot_" if avx2 else "si_dot_") + REF_DOT_NAME[wtype])
        fn(n, C.byref(s), x.ctypes.data, y.ctypes.data)
        return s.value

    def gemv_scalar(self, wtype: int, w: np.ndarray, n_in: int, n_out: int, xq: np.ndarray) -> np.ndarray:
        rb = row_bytes(wtype, n_in)
        y = np.zeros(n_out, np.float32)
        for r in range(n_out):
            y[r] = self.vec_dot(wtype, n_in, w[r * rb:(r + 1) * rb], xq)
        return y

    def expf(self, x: float) -> float:
        return self.lib.si_expf(x)

    def silu(self, x: float) -> float:
        return self.lib.si_silu(x)

    def rms_scale(self, x, eps: float) -> float:
        x = _as_f32(x).reshape(-1)
        return self.lib.si_rms_scale(x, x.size, eps)

    def softmax(self, x) -> np.ndarray:
        """The reference's attention softmax: its row-max loop
        (src/engine.c:124-128) written here, then its si_softmax."""
        x = _as_f32(x).reshape(-1)
        mx = -np.inf
        for v in x:
            if v > mx:
                mx = v
        y = np.zeros_like(x)
        self.lib.si_softmax(y, x, x.size, np.float32(mx))
        return y

    def dequant_row(self, t: int, x: np.ndarray, n: int) -> np.ndarray:
        y = np.zeros(n, np.float32)
        ok = self.lib.si_dequant_row(t, np.ascontiguousarray(x).ctypes.data, y, n)
        assert ok
        return y


class RefCpuGemv:
    """The reference's own matvec, si_backend_cpu()->gemv (src/backend.c:85-120):
    quantize once, then AVX2 dots over a pthread pool of ``threads`` lanes."""

    def __init__(self, ref: Reference, threads: int):
        self.ref = ref
        self.threads = threads
        self.tp = ref.lib.si_tp_create(threads)
        self.be = ref.lib.si_backend_cpu()

    def tensor(self, wtype: int, w: np.ndarray, n_in: int, n_out: int) -> SiTensor:
        t = SiTensor()
        t.type = wtype
        t.ne[0], t.ne[1], t.ne[2], t.ne[3] = n_in, n_out, 1, 1
        t.n_elems = n_in * n_out
        t.n_bytes = w.nbytes
        t.data = w.ctypes.data
        t.loc = 1
        t.be = C.cast(self.be, C.c_void_p)
        return t

    def __call__(self, t: SiTensor, x: np.ndarray, y: np.ndarray) -> None:
        self.be.contents.gemv(C.cast(self.be, C.c_void_p), C.byref(t), x.ctypes.data, y.ctypes.data,
                              int(t.ne[1]), self.tp)

    def close(self) -> None:
        if self.tp:
            self.ref.lib.si_tp_free(self.tp)
            self.tp = None


def have_reference() -> bool:
    return REF_SO.exists()


# ---- the reference engine, with the CPU or the CUDA backend ---------------------------

E2E_SO = HERE / "_ref" / "libsiphon_e2e.so"


class RefEngine:
    """The reference's forward pass (si_engine_forward) on a GGUF file, every
    matrix product on the reference CPU backend or on the CUDA backend adapter
    (siphon_b200/csrc/backend_cuda.c): with use_cuda, every layer's gemv, the
    embedding lookup (src/engine.c:302) and the output head (:393) run on the
    GPU. scalar=True runs the reference's scalar kernels for all host work
    (the parity target); the first engine of a process fixes the mode."""

    _lib = None

    def __init__(self, path, use_cuda: bool = False, device: int = 0, n_ctx: int = 512, threads: int = 0,
                 scalar: bool = True):
        if RefEngine._lib is None:
            if not E2E_SO.exists():
                raise FileNotFoundError(f"{E2E_SO} not built (make -C oracle e2e)")
            L = C.CDLL(str(E2E_SO))
            L.e2e_error.restype = C.c_char_p
            L.e2e_open.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_void_p)]
            L.e2e_kern_impl.restype = C.c_char_p
            L.e2e_open.restype = C.c_int
            L.e2e_forward.argtypes = [C.c_void_p, C.c_uint32]
            L.e2e_forward.restype = C.POINTER(C.c_float)
            L.e2e_n_vocab.argtypes = [C.c_void_p]
            L.e2e_n_vocab.restype = C.c_uint32
            L.e2e_close.argtypes = [C.c_void_p]
            L.e2e_close.restype = None
            RefEngine._lib = L
        self.L = RefEngine._lib
        threads = threads or min(os.cpu_count() or 1, 16)
        h = C.c_void_p()
        rc = self.L.e2e_open(str(path).encode(), 1 if use_cuda else 0, device, n_ctx, threads,
                             1 if scalar else 0, C.byref(h))
        if rc != 0:
            raise RuntimeError(f"e2e_open failed ({rc}): {self.L.e2e_error().decode()}")
        self.h = h
        self.n_vocab = self.L.e2e_n_vocab(h)
        self.kern_impl = self.L.e2e_kern_impl().decode()

    def forward(self, token: int) -> np.ndarray:
        p = self.L.e2e_forward(self.h, token)
        if not p:
            raise RuntimeError(f"forward failed: {self.L.e2e_error().decode()}")
        return np.ctypeslib.as_array(p, shape=(self.n_vocab,)).copy()

    def close(self) -> None:
        if self.h:
            self.L.e2e_close(self.h)
            self.h = None

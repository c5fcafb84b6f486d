"""Generate tests/golden/*.npz by running the REFERENCE ITSELF.

The reference is compiled from its own sources into oracle/_ref/ (see
oracle/Makefile); this script calls its exported functions on seeded inputs
and stores inputs and outputs as compact fixtures. The fixtures pin the
oracle restatement (tests/test_oracle_golden.py) on machines where the
reference tree is absent (the GPU box).

    python tests/golden/gen_golden.py

Contents:
  quant.npz   f32 rows (random at several scales plus edge cases: zero
              blocks, tied maxima, negative max, subnormal and huge values)
              with their Q8_K bytes (si_quant_row_q8_K) and their Q8_0 bytes
              in the AVX2 form x86 hosts dispatch to (si_avx2_quant_row_q8_0).
  dot_<T>.npz per weight type: weight bytes, f32 activation, its pair-format
              bytes, scalar-path outputs (si_dot_*) and AVX2-path outputs.
  dequant.npz per type: two rows of bytes and si_dequant_row outputs.
  f16.npz     f32 -> f16 of edge values and random bit patterns, and a
              digest of the f16 -> f32 table over all 65536 halves.
  steps.npz   the activation steps between products: si_expf and si_silu
              of edge values and random floats over the polynomial's whole
              range, and si_rms_scale of rows of 256 and 5120 floats at two
              epsilons, among them rows whose mean of squares lies exactly
              halfway between two floats (the last two rows of rows256: the
              same values in two orders, whose sequential double sums round
              the mean to different floats).
"""

from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle.oracle import PAIR, Reference, row_bytes  # noqa: E402
from siphon_b200 import quant as Q  # noqa: E402
from siphon_b200 import synth  # noqa: E402

OUT = Path(__file__).resolve().parent


def quant_inputs() -> np.ndarray:
    rng = np.random.default_rng(1234)
    n = 512
    rows = [rng.standard_normal(n) * s for s in (1.0, 1e-3, 37.0, 1e4)]
    rows.append(np.zeros(n))                                   # all-zero blocks
    tie = rng.standard_normal(n); tie[[3, 70, 200]] = 5.0; tie[300] = -5.0; tie[301] = 5.0
    rows.append(tie)                                           # equal-magnitude maxima
    neg = rng.standard_normal(n); neg[17] = -9.0
    rows.append(neg)                                           # negative max
    half = rng.standard_normal(n); half[:256] = 0.0
    rows.append(half)                                          # zero block then normal
    tiny = rng.standard_normal(n) * 1e-30                      # subnormal products
    rows.append(tiny)
    huge = rng.standard_normal(n) * 1e30
    rows.append(huge)
    ints = np.round(rng.standard_normal(n) * 50)               # exact .5 roundings after scaling
    rows.append(ints)
    spiky = np.zeros(n); spiky[::37] = rng.standard_normal(len(spiky[::37]))
    rows.append(spiky)
    return np.stack(rows).astype(np.float32)


def halfway_rows() -> np.ndarray:
    """Rows of 256 floats whose f32 mean of squares is decided by the
    reference's summation order. x0 = 16.279024 (0x41823b71) squares to t0
    with t0 + 247 exactly halfway between two multiples of the f32 spacing
    of the mean times 256 (the lower one even), so rounding the mean is a tie
    that goes down. Eight elements of 2^-23 (squares 2^-46) follow x0 in the
    second row: each is below half a double ulp of the running sum and is
    lost, the tie stands and the mean rounds down. In the third row they come
    first, add up to 2^-43 and survive, the sum is above halfway and the mean
    rounds up. The first row has zeros in their place (an exact tie)."""
    x0 = np.array([0x41823B71], np.uint32).view(np.float32)[0]
    tiny = np.float32(2.0 ** -23)
    a = np.ones(256, np.float32); a[0] = x0; a[1:9] = tiny
    c = np.ones(256, np.float32); c[0:8] = tiny; c[8] = x0
    z = np.ones(256, np.float32); z[0] = x0; z[1:9] = 0.0
    return np.stack([z, a, c])


def steps_inputs():
    rng = np.random.default_rng(4321)
    edge = np.array([0.0, -0.0, 1.0, -1.0, 88.0, 88.7, 89.0, -87.0, -88.0, -103.0, -104.0, 126.0 * 0.6931472,
                     -126.0 * 0.6931472, 130.0, -130.0, 150.0, -150.0, 192.0 * 0.6931472, 200.0, -200.0, 1e-30,
                     -1e-30, 1e-45, 3e38, -3e38, np.inf, -np.inf], np.float32)
    ex = np.concatenate([edge, rng.standard_normal(4000) * 8, rng.uniform(-220, 220, 4000),
                         rng.standard_normal(1000) * 1e-3]).astype(np.float32)
    r256 = [rng.standard_normal(256) * s for s in (1.0, 1e-3, 40.0)]
    r256.append(np.zeros(256))
    r256.append(rng.standard_normal(256) * 1e20)                # squares overflow to inf: scale 0
    spread = rng.standard_normal(256) * np.exp2(rng.uniform(-40, 20, 256))
    r256.append(spread)                                         # squares over 120 binades
    r256 = np.concatenate([np.stack(r256).astype(np.float32), halfway_rows()])
    r5120 = np.stack([rng.standard_normal(5120) * s for s in (1.0, 0.05, 3.0)]).astype(np.float32)
    return ex, r256, r5120


def main() -> None:
    ref = Reference()
    print("reference kernels:", ref.impl)

    x = quant_inputs()
    q8k = np.stack([ref.quant_q8_K(r) for r in x])
    q80 = np.stack([ref.quant_q8_0(r, "avx2") for r in x])
    np.savez_compressed(OUT / "quant.npz", x=x, q8_K=q8k, q8_0=q80)

    shapes = {t: (12, 1024) for t in Q.WEIGHT_TYPES}
    for wt in Q.WEIGHT_TYPES:
        n_out, n_in = shapes[wt]
        w = synth.weights(wt, n_out, n_in, seed=100 + wt)
        xs = synth.activations(n_in, 3, seed=200 + wt)
        xq, ys, ya = [], [], []
        for r in xs:
            if PAIR[wt] == Q.Q8_K:
                q = ref.quant_q8_K(r)
            elif PAIR[wt] == Q.Q8_0:
                q = ref.quant_q8_0(r, "avx2")
            else:
                q = ref.convert_f16(r)
            rb = row_bytes(wt, n_in)
            xq.append(q)
            ys.append([ref.vec_dot(wt, n_in, w[i * rb:(i + 1) * rb], q) for i in range(n_out)])
            ya.append([ref.vec_dot(wt, n_in, w[i * rb:(i + 1) * rb], q, avx2=True) for i in range(n_out)])
        np.savez_compressed(OUT / f"dot_{Q.NAMES[wt]}.npz", w=w, x=xs, xq=np.stack(xq),
                            y_scalar=np.array(ys, np.float32), y_avx2=np.array(ya, np.float32),
                            n_in=n_in, n_out=n_out, wtype=wt)

    deq = {}
    for wt in Q.WEIGHT_TYPES:
        n_in = 512
        w = synth.weights(wt, 2, n_in, seed=300 + wt)
        rb = row_bytes(wt, n_in)
        deq[f"w_{wt}"] = w
        deq[f"y_{wt}"] = np.stack([ref.dequant_row(wt, w[i * rb:(i + 1) * rb], n_in) for i in range(2)])
    np.savez_compressed(OUT / "dequant.npz", **deq)

    rng = np.random.default_rng(99)
    edge = np.array([0.0, -0.0, 1.0, -1.0, 0.5, 65504.0, 65519.99, 65520.0, 1e10, -1e10, 1e-10,
                     6.0e-8, 5.96e-8, 2.98e-8, 2.99e-8, 6.1e-5, 6.09e-5, np.inf, -np.inf], np.float32)
    nans = np.array([0x7fc00000, 0xffc00000, 0x7f800001, 0x7fa00000, 0xff800123], np.uint32).view(np.float32)
    bits = rng.integers(0, 2 ** 32, 20000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    f = np.concatenate([edge, nans, bits]).astype(np.float32)
    h = np.array([ref.lib.si_f32_to_f16(float(v)) for v in f], np.uint16)
    table = np.array([ref.lib.si_f16_to_f32(i) for i in range(65536)], np.float32)
    digest = hashlib.sha256(table.tobytes()).hexdigest()
    np.savez_compressed(OUT / "f16.npz", f32=f, f16=h, table_sha256=np.array(digest))

    ex, r256, r5120 = steps_inputs()
    eps = np.array([1e-5, 1e-6], np.float32)
    np.savez_compressed(OUT / "steps.npz", ex=ex,
                        expf=np.array([ref.expf(float(v)) for v in ex], np.float32),
                        silu=np.array([ref.silu(float(v)) for v in ex], np.float32),
                        eps=eps, rows256=r256, rows5120=r5120,
                        scale256=np.array([[ref.rms_scale(r, float(e)) for e in eps] for r in r256], np.float32),
                        scale5120=np.array([[ref.rms_scale(r, float(e)) for e in eps] for r in r5120], np.float32))
    print("wrote", sorted(p.name for p in OUT.glob("*.npz")))


if __name__ == "__main__":
    main()

"""Block geometry of the GGUF weight formats on the quantized matrix path.

Host-side mirror of the reference's ``include/siphon/quant.h`` (type ids at
:103-119, block sizes at :92-100) and of ``si_quant_geometry`` /
``si_quant_vec_dot_pair`` (``src/kernels.c:904-919, 946-960``). The numbers
are the on-disk GGUF layout, which is what the CUDA library consumes byte for
byte, so they cannot differ from the reference's.
"""

from __future__ import annotations

F32, F16, Q4_0, Q5_0, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, Q8_K = 0, 1, 2, 6, 8, 10, 11, 12, 13, 14, 15

NAMES = {F32: "F32", F16: "F16", Q4_0: "Q4_0", Q5_0: "Q5_0", Q8_0: "Q8_0", Q2_K: "Q2_K",
         Q3_K: "Q3_K", Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K", Q8_K: "Q8_K"}
BY_NAME = {v: k for k, v in NAMES.items()}

# (elements per block, bytes per block)
GEOMETRY = {
    F32: (1, 4), F16: (1, 2),
    Q4_0: (32, 18), Q5_0: (32, 22), Q8_0: (32, 34),
    Q2_K: (256, 84), Q3_K: (256, 110), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210),
    Q8_K: (256, 292),
}

# weight formats of the quantized matrix path (the north-star list)
WEIGHT_TYPES = (F16, Q4_0, Q5_0, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K)


def pair_type(wtype: int) -> int:
    """Activation format the dot product of ``wtype`` consumes."""
    if wtype in (F32, F16):
        return wtype
    if wtype in (Q4_0, Q5_0, Q8_0):
        return Q8_0
    if wtype in (Q2_K, Q3_K, Q4_K, Q5_K, Q6_K):
        return Q8_K
    raise ValueError(f"no dot product for type {wtype}")


def row_bytes(t: int, n: int) -> int:
    blck, size = GEOMETRY[t]
    if n % blck:
        raise ValueError(f"{NAMES[t]} row of {n} elements is not a whole number of {blck}-blocks")
    return n // blck * size


def bytes_per_elem(t: int) -> float:
    blck, size = GEOMETRY[t]
    return size / blck


def matvec_bytes(wtype: int, n_out: int, n_in: int, m: int = 1) -> int:
    """Algorithmic HBM bytes of one y = W x: the weight blocks once, the
    pair-format activation and the f32 output per batch row, the f32 input
    per batch row (the quantizer reads it)."""
    return (n_out * row_bytes(wtype, n_in) + m * row_bytes(pair_type(wtype), n_in)
            + 4 * m * n_out + 4 * m * n_in)

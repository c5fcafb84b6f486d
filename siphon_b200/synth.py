"""Seeded synthetic inputs for the quantized matrix path.

The reference publishes no dataset for this path; its benchmark configs
describe random blocks. Weight blocks here follow that description: every
f16 super-block / block scale (``d``, ``dmin``) is drawn uniform in
[1e-4, 1e-2] and every other bit (quants, packed 6-bit scales and mins, high
bits, int8 sub-scales) is uniform over its full range. F16 weight rows hold
f16(U[-1, 1)) values (an all-bit-patterns draw would include inf/NaN).
Activations are f32 ~ N(0, 1).
"""

from __future__ import annotations

import numpy as np

from . import quant as Q

# byte offsets of the f16 scale fields inside one block (quant.h:32-89)
_F16_FIELDS = {
    Q.Q4_0: (0,), Q.Q5_0: (0,), Q.Q8_0: (0,),
    Q.Q2_K: (80, 82), Q.Q3_K: (108,), Q.Q4_K: (0, 2), Q.Q5_K: (0, 2), Q.Q6_K: (208,),
}


def weights(wtype: int, n_out: int, n_in: int, seed: int = 0,
            scale_lo: float = 1e-4, scale_hi: float = 1e-2) -> np.ndarray:
    """Raw GGUF block bytes of an [n_out, n_in] weight matrix (uint8, row-major)."""
    rng = np.random.default_rng(seed)
    rb = Q.row_bytes(wtype, n_in)
    if wtype == Q.F16:
        vals = rng.uniform(-1.0, 1.0, size=n_out * n_in).astype(np.float32).astype(np.float16)
        return vals.view(np.uint8).copy()
    if wtype == Q.F32:
        return rng.uniform(-1.0, 1.0, size=n_out * n_in).astype(np.float32).view(np.uint8).copy()
    raw = rng.integers(0, 256, size=n_out * rb, dtype=np.uint8)
    _, bsz = Q.GEOMETRY[wtype]
    blocks = raw.reshape(-1, bsz)
    for off in _F16_FIELDS[wtype]:
        d = rng.uniform(scale_lo, scale_hi, size=blocks.shape[0]).astype(np.float16)
        blocks[:, off:off + 2] = d.view(np.uint8).reshape(-1, 2)
    return raw


def activations(n: int, m: int = 1, seed: int = 1) -> np.ndarray:
    """f32 activations ~ N(0, 1), shape [m, n]."""
    rng = np.random.default_rng(seed)
    return rng.standard_normal(size=(m, n)).astype(np.float32)

"""f32 -> GGUF block quantizers for synthetic model weights.

The reference only quantizes activations (Q8_K / Q8_0); its models come
quantized from elsewhere. Synthetic models here need weight blocks, so these
are simple deterministic quantizers (min/max per sub-block, 6-bit scales per
super-block): any well-formed block is a valid input to both the reference
and the CUDA kernels, which then have to agree bit for bit.
"""

from __future__ import annotations

import numpy as np

from . import quant as Q


def _f16(a: np.ndarray) -> np.ndarray:
    return a.astype(np.float16)


def q4_k(x: np.ndarray) -> np.ndarray:
    """[..., K] f32 with K % 256 == 0 -> raw Q4_K bytes (144 per 256)."""
    xs = np.ascontiguousarray(x, np.float32).reshape(-1, 8, 32)
    nb = xs.shape[0]
    mn = np.minimum(xs.min(axis=2), 0.0)
    mx = xs.max(axis=2)
    s = (mx - mn) / 15.0
    m = -mn
    d16 = _f16(s.max(axis=1) / 63.0)
    dm16 = _f16(m.max(axis=1) / 63.0)
    d, dm = d16.astype(np.float32)[:, None], dm16.astype(np.float32)[:, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.clip(np.where(d > 0, np.rint(s / d), 0), 0, 63).astype(np.uint8)
        mm = np.clip(np.where(dm > 0, np.rint(m / dm), 0), 0, 63).astype(np.uint8)
        scale = (d * sc)[:, :, None]
        off = (dm * mm)[:, :, None]
        q = np.clip(np.where(scale > 0, np.rint((xs + off) / scale), 0), 0, 15).astype(np.uint8)
    out = np.zeros((nb, 144), np.uint8)
    out[:, 0:2] = d16.view(np.uint8).reshape(nb, 2)
    out[:, 2:4] = dm16.view(np.uint8).reshape(nb, 2)
    # 6-bit scales/mins: bytes 0-3 sc[0..3] (+ top bits of sc[4..7]), 4-7 mins
    # likewise, 8-11 low nibbles of sc[4..7] and mins[4..7]
    out[:, 4:8] = sc[:, :4] | ((sc[:, 4:] >> 4) << 6)
    out[:, 8:12] = mm[:, :4] | ((mm[:, 4:] >> 4) << 6)
    out[:, 12:16] = (sc[:, 4:] & 15) | ((mm[:, 4:] & 15) << 4)
    # chunk c of 32 bytes: low nibbles = sub-block 2c, high nibbles = 2c+1
    qq = q.reshape(nb, 4, 2, 32)
    out[:, 16:].reshape(nb, 4, 32)[:] = qq[:, :, 0, :] | (qq[:, :, 1, :] << 4)
    return out.reshape(-1)


def q6_k(x: np.ndarray) -> np.ndarray:
    """[..., K] f32 with K % 256 == 0 -> raw Q6_K bytes (210 per 256)."""
    xs = np.ascontiguousarray(x, np.float32).reshape(-1, 16, 16)
    nb = xs.shape[0]
    s = np.abs(xs).max(axis=2) / 31.0
    d16 = _f16(s.max(axis=1) / 127.0)
    d = d16.astype(np.float32)[:, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.clip(np.where(d > 0, np.rint(s / d), 0), -128, 127).astype(np.int8)
        eff = (d * sc)[:, :, None]
        q = np.clip(np.where(eff != 0, np.rint(xs / eff), 0), -32, 31).astype(np.int32) + 32
    u = q.reshape(nb, 2, 4, 32).astype(np.uint8)        # [block, half h, group g, lane l]
    out = np.zeros((nb, 210), np.uint8)
    ql = out[:, 0:128].reshape(nb, 2, 2, 32)            # [block, h, g & 1, l]
    ql[:] = (u[:, :, 0:2, :] & 15) | ((u[:, :, 2:4, :] & 15) << 4)
    qh = out[:, 128:192].reshape(nb, 2, 32)
    qh[:] = (u[:, :, 0] >> 4) | ((u[:, :, 1] >> 4) << 2) | ((u[:, :, 2] >> 4) << 4) | ((u[:, :, 3] >> 4) << 6)
    out[:, 192:208] = sc.view(np.uint8)
    out[:, 208:210] = d16.view(np.uint8).reshape(nb, 2)
    return out.reshape(-1)


def q8_0(x: np.ndarray) -> np.ndarray:
    xs = np.ascontiguousarray(x, np.float32).reshape(-1, 32)
    d16 = _f16(np.abs(xs).max(axis=1) / 127.0)
    d = d16.astype(np.float32)[:, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.clip(np.where(d > 0, np.rint(xs / d), 0), -127, 127).astype(np.int8)
    out = np.zeros((xs.shape[0], 34), np.uint8)
    out[:, 0:2] = d16.view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.reshape(-1)


def quantize(wtype: int, x: np.ndarray) -> np.ndarray:
    if wtype == Q.Q4_K:
        return q4_k(x)
    if wtype == Q.Q6_K:
        return q6_k(x)
    if wtype == Q.Q8_0:
        return q8_0(x)
    if wtype == Q.F16:
        return np.ascontiguousarray(x, np.float32).astype(np.float16).view(np.uint8).reshape(-1)
    if wtype == Q.F32:
        return np.ascontiguousarray(x, np.float32).view(np.uint8).reshape(-1)
    raise ValueError(f"no weight quantizer for {Q.NAMES.get(wtype, wtype)}")

"""Small helpers for the GPU tests (device buffers via torch)."""

from __future__ import annotations

import numpy as np


def dev(a: np.ndarray):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def empty_u8(n: int):
    import torch
    return torch.zeros(n, dtype=torch.uint8, device="cuda")


def empty_f32(*shape):
    import torch
    return torch.full(shape, float("nan"), dtype=torch.float32, device="cuda")


def host(t) -> np.ndarray:
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


def assert_bits_equal(got: np.ndarray, want: np.ndarray, what: str) -> None:
    """Bit-identical outputs (NaN == NaN); on failure report the worst
    relative error against the north-star tolerance of 1e-5."""
    g = np.asarray(got, np.float32).reshape(-1)
    w = np.asarray(want, np.float32).reshape(-1)
    same = (g.view(np.uint32) == w.view(np.uint32)) | (np.isnan(g) & np.isnan(w))
    if not same.all():
        bad = np.flatnonzero(~same)
        rel = np.abs(g[bad] - w[bad]) / np.maximum(np.abs(w[bad]), 1e-30)
        raise AssertionError(f"{what}: {bad.size}/{g.size} outputs differ; first {bad[:5].tolist()}, "
                             f"got {g[bad[:3]].tolist()} want {w[bad[:3]].tolist()}, max rel {rel.max():.3g}")


REL_TOL = 1e-5   # north-star bound per output element; the kernels are bit-exact (stricter)


def assert_within_tol(got: np.ndarray, want: np.ndarray, what: str) -> None:
    g32 = np.asarray(got, np.float32).reshape(-1)
    w32 = np.asarray(want, np.float32).reshape(-1)
    same = (g32.view(np.uint32) == w32.view(np.uint32)) | (np.isnan(g32) & np.isnan(w32))
    g, w = g32[~same].astype(np.float64), w32[~same].astype(np.float64)
    rel = np.abs(g - w) / np.maximum(np.abs(w), 1e-30)
    assert not rel.size or (rel <= REL_TOL).all(), f"{what}: max rel {rel.max():.3g} > {REL_TOL}"

"""SLGD v1 logit dumps, the reference's golden-file format, and its
verification protocol.

The reference writes and reads these files in its `run` command
(src/cmd_run.c:21-81): a 20-byte header ("SLGD", version 1, n_total,
n_prompt, n_vocab as little-endian u32), n_total int32 tokens, then
n_total x n_vocab f32 logits, one row per position. `run --golden FILE`
teacher-forces the file's tokens through the engine one position at a time
and compares every logits row with the recorded one (src/cmd_run.c:132-248).

This module writes such files from any engine that maps a token to its
logits (the reference engine on the CUDA backend included), reads them, and
restates the comparison and its acceptance rule, so a run of this library
can be checked against a golden made by the reference and vice versa.
"""

from __future__ import annotations

import struct
from dataclasses import dataclass
from pathlib import Path
from typing import Callable, Sequence

import numpy as np

MAGIC = b"SLGD"
VERSION = 1
_HEADER = struct.Struct("<4sIIII")


@dataclass
class Golden:
    n_prompt: int
    tokens: np.ndarray        # int32 [n_total]
    logits: np.ndarray        # float32 [n_total, n_vocab]

    @property
    def n_total(self) -> int:
        return int(self.tokens.size)

    @property
    def n_vocab(self) -> int:
        return int(self.logits.shape[1])


def write(path: str | Path, tokens: Sequence[int], logits: np.ndarray, n_prompt: int) -> Path:
    """slgd_write (src/cmd_run.c:61-81): header, tokens, logits rows."""
    toks = np.asarray(tokens, dtype="<i4")
    lg = np.ascontiguousarray(logits, dtype="<f4")
    if lg.ndim != 2 or lg.shape[0] != toks.size:
        raise ValueError(f"logits {lg.shape} do not match {toks.size} tokens")
    if not 0 <= n_prompt <= toks.size:
        raise ValueError("n_prompt out of range")
    path = Path(path)
    with open(path, "wb") as f:
        f.write(_HEADER.pack(MAGIC, VERSION, toks.size, n_prompt, lg.shape[1]))
        f.write(toks.tobytes())
        f.write(lg.tobytes())
    return path


def read(path: str | Path) -> Golden:
    """slgd_read (src/cmd_run.c:32-59), with the same checks: magic and
    version, then complete token and logits sections."""
    data = Path(path).read_bytes()
    if len(data) < _HEADER.size:
        raise ValueError(f"{path}: not an SLGD v1 file")
    magic, version, n_total, n_prompt, n_vocab = _HEADER.unpack_from(data)
    if magic != MAGIC or version != VERSION:
        raise ValueError(f"{path}: not an SLGD v1 file")
    off = _HEADER.size
    if len(data) < off + 4 * n_total:
        raise ValueError(f"{path}: truncated token section")
    toks = np.frombuffer(data, "<i4", n_total, off).copy()
    off += 4 * n_total
    if len(data) < off + 4 * n_total * n_vocab:
        raise ValueError(f"{path}: truncated logits section")
    lg = np.frombuffer(data, "<f4", n_total * n_vocab, off).reshape(n_total, n_vocab).copy()
    return Golden(int(n_prompt), toks, lg)


def record(forward: Callable[[int], np.ndarray], prompt: Sequence[int], n_gen: int) -> Golden:
    """Run a prompt then n_gen greedy tokens through `forward` (token ->
    logits) and keep every position's logits, as the reference's dump mode
    does: the token stream holds the prompt followed by the generated
    tokens, and row t holds the logits after feeding token t."""
    toks, rows = [], []
    tok = None
    for step in range(len(prompt) + n_gen):
        t = int(prompt[step]) if step < len(prompt) else tok
        lg = np.asarray(forward(t), np.float32)
        toks.append(t)
        rows.append(lg.copy())
        tok = int(np.argmax(lg))          # greedy: the first maximum
    return Golden(len(prompt), np.array(toks, np.int32), np.stack(rows))


@dataclass
class Verdict:
    prefill_max: float
    prefill_mean: float
    decode_max: float
    decode_mean: float
    flips: int
    real_flips: int
    threshold: float
    passed: bool


# acceptance constants of cmd_run_golden (src/cmd_run.c:166-167, 227-241)
REAL_FLIP_WINDOW = 24
REAL_FLIP_GAP = 1.0


def verify(forward: Callable[[int], np.ndarray], golden: Golden) -> Verdict:
    """cmd_run_golden (src/cmd_run.c:149-248): teacher-force the golden's
    tokens, compare every logits row (max and mean absolute difference,
    prompt and generated positions apart), count argmax flips and the real
    ones (reference top-2 gap above 1.0 within the first 24 positions), and
    pass when the prompt's max difference is within 0.6 (prompts of at most
    8 tokens) or 1.0 and no flip is real."""
    pre, gen = [], []
    flips = real = 0
    for step in range(golden.n_total):
        lg = np.asarray(forward(int(golden.tokens[step])), np.float32)
        ref = golden.logits[step]
        d = np.abs(lg.astype(np.float64) - ref.astype(np.float64))
        (pre if step < golden.n_prompt else gen).append(d)
        ours = int(np.argmax(lg))
        ref_arg = int(np.argmax(ref))
        if ours != ref_arg:
            flips += 1
            top2 = np.sort(ref.astype(np.float64))[-2:]
            gap = top2[1] - top2[0]
            if gap > REAL_FLIP_GAP and step < REAL_FLIP_WINDOW:
                real += 1

    def stats(ds):
        if not ds:
            return 0.0, 0.0
        a = np.concatenate(ds)
        return float(a.max()), float(a.mean())

    pmax, pmean = stats(pre)
    gmax, gmean = stats(gen)
    thr = 0.6 if golden.n_prompt <= 8 else 1.0
    return Verdict(pmax, pmean, gmax, gmean, flips, real, thr, pmax <= thr and real == 0)

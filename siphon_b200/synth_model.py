"""Synthetic llama-architecture GGUF models of the benchmark shapes.

Weights are random-init N(0, 0.02), quantized "Q4_K_M-style": Q6_K for the
output head and for attn_v / ffn_down on every other layer, Q4_K for the other
matrices and the token embedding. Norm weights are F32, 1 + 0.1 N(0, 1).
Qwen2-architecture models (``arch="qwen2"``) also carry F32 Q/K/V biases
(0.02 N(0, 1)), which the reference adds after the Q, K and V products
(src/engine.c:320-334), and rotate with the half-split (NEOX) RoPE form
(src/engine.c:61-71). The file uses the GGUF keys and tensor names the
reference's loader reads (src/model.c:26-172).

``blocks="random"`` writes uniformly random block bytes instead (every f16
scale U[1e-4, 1e-2], every other bit uniform), for models whose values do not
matter (timing runs): far faster to make for the 8B and 32B shapes. A
function ``blocks(wtype, n_out, n_in, key) -> uint8 array`` supplies the
blocks of each matrix itself (e.g. generated on a GPU).
"""

from __future__ import annotations

import zlib
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from . import gguf
from . import quant as Q
from . import synth
from .wquant import quantize


@dataclass(frozen=True)
class LlamaShape:
    n_layer: int
    n_embd: int
    n_ff: int
    n_head: int
    n_head_kv: int
    n_vocab: int
    rope_base: float = 10000.0
    rms_eps: float = 1e-5
    n_ctx: int = 2048
    arch: str = "llama"

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_head

    @property
    def qkv_bias(self) -> bool:
        return self.arch == "qwen2"

    @property
    def neox(self) -> bool:
        """Half-split RoPE pairs (the reference's form for qwen2)."""
        return self.arch == "qwen2"

    def with_layers(self, n_layer: int) -> "LlamaShape":
        return LlamaShape(n_layer, self.n_embd, self.n_ff, self.n_head, self.n_head_kv, self.n_vocab,
                          self.rope_base, self.rms_eps, self.n_ctx, self.arch)


# TinyLlama-1.1B shape (decode benchmark)
TINYLLAMA = LlamaShape(22, 2048, 5632, 32, 4, 32000, 10000.0, 1e-5, 2048)
# Llama-3-8B shape (prefill benchmark)
LLAMA3_8B = LlamaShape(32, 4096, 14336, 32, 8, 128256, 500000.0, 1e-5, 2048)
# Qwen2.5-32B shape (tensor-parallel benchmark): qwen2 architecture, QKV bias
QWEN25_32B = LlamaShape(64, 5120, 27648, 40, 8, 152064, 1000000.0, 1e-6, 2048, "qwen2")
# small models of the same families for parity tests
SMALL = LlamaShape(3, 512, 1536, 8, 2, 1024, 10000.0, 1e-5, 1024)
SMALL_QWEN = LlamaShape(2, 512, 1024, 8, 2, 1024, 1000000.0, 1e-6, 1024, "qwen2")


def layer_types(il: int) -> dict:
    """Q4_K_M-style mix: Q6_K for attn_v and ffn_down on even layers."""
    mix = Q.Q6_K if il % 2 == 0 else Q.Q4_K
    return {"q": Q.Q4_K, "k": Q.Q4_K, "v": mix, "o": Q.Q4_K, "gate": Q.Q4_K, "up": Q.Q4_K, "down": mix}


GGUF_NAMES = {"q": "attn_q", "k": "attn_k", "v": "attn_v", "o": "attn_output", "gate": "ffn_gate",
              "up": "ffn_up", "down": "ffn_down"}


def matrices(sh: LlamaShape, wtype: int | None = None) -> list[tuple[str, int, int, int]]:
    """(tensor name, ggml type, n_out, n_in) of every weight matrix: the
    Q4_K_M-style mix, or every matrix (embedding and head included) of one
    type `wtype`."""
    kv = sh.n_head_kv * sh.head_dim
    out = [("token_embd.weight", wtype or Q.Q4_K, sh.n_vocab, sh.n_embd),
           ("output.weight", wtype or Q.Q6_K, sh.n_vocab, sh.n_embd)]
    shapes = {"q": (sh.n_embd, sh.n_embd), "k": (kv, sh.n_embd), "v": (kv, sh.n_embd), "o": (sh.n_embd, sh.n_embd),
              "gate": (sh.n_ff, sh.n_embd), "up": (sh.n_ff, sh.n_embd), "down": (sh.n_embd, sh.n_ff)}
    for il in range(sh.n_layer):
        t = layer_types(il)
        for k in ("q", "k", "v", "o", "gate", "up", "down"):
            out.append((f"blk.{il}.{GGUF_NAMES[k]}.weight", wtype or t[k], *shapes[k]))
    return out


def vectors(sh: LlamaShape) -> list[tuple[str, int]]:
    """(tensor name, length) of every F32 vector: norms, then biases."""
    out = [("output_norm.weight", sh.n_embd)]
    kv = sh.n_head_kv * sh.head_dim
    for il in range(sh.n_layer):
        out += [(f"blk.{il}.attn_norm.weight", sh.n_embd), (f"blk.{il}.ffn_norm.weight", sh.n_embd)]
        if sh.qkv_bias:
            out += [(f"blk.{il}.attn_q.bias", sh.n_embd), (f"blk.{il}.attn_k.bias", kv),
                    (f"blk.{il}.attn_v.bias", kv)]
    return out


def _quantized(wt: int, n_out: int, n_in: int, rng_seed) -> np.ndarray:
    """N(0, 0.02) rows quantized in slabs of about 4M elements (keeps the
    temporaries small)."""
    rng = np.random.default_rng(rng_seed)
    out = np.empty(n_out * Q.row_bytes(wt, n_in), np.uint8)
    rows = max(1, (1 << 22) // n_in)
    rb = Q.row_bytes(wt, n_in)
    for r0 in range(0, n_out, rows):
        r1 = min(n_out, r0 + rows)
        w = rng.standard_normal((r1 - r0, n_in), dtype=np.float32) * np.float32(0.02)
        out[r0 * rb:r1 * rb] = quantize(wt, w)
    return out


def _vector(name: str, n: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng([seed, zlib.crc32(name.encode())])
    z = rng.standard_normal(n, dtype=np.float32)
    v = z * np.float32(0.02) if name.endswith(".bias") else np.float32(1.0) + np.float32(0.1) * z
    return v.astype(np.float32)


def write_llama(path: str | Path, sh: LlamaShape, seed: int = 0, blocks="quantized", wtype: int | None = None) -> Path:
    a = sh.arch
    kvs = [
        ("general.architecture", gguf.STRING, a),
        ("general.alignment", gguf.U32, 32),
        (f"{a}.block_count", gguf.U32, sh.n_layer),
        (f"{a}.context_length", gguf.U32, sh.n_ctx),
        (f"{a}.embedding_length", gguf.U32, sh.n_embd),
        (f"{a}.feed_forward_length", gguf.U32, sh.n_ff),
        (f"{a}.attention.head_count", gguf.U32, sh.n_head),
        (f"{a}.attention.head_count_kv", gguf.U32, sh.n_head_kv),
        (f"{a}.attention.layer_norm_rms_epsilon", gguf.F32, sh.rms_eps),
        (f"{a}.rope.freq_base", gguf.F32, sh.rope_base),
    ]
    tensors = []
    for name, wt, n_out, n_in in matrices(sh, wtype):
        key = [seed, zlib.crc32(name.encode())]
        if callable(blocks):
            fn = (lambda wt=wt, n_out=n_out, n_in=n_in, key=key: blocks(wt, n_out, n_in, key))
        elif blocks == "random":
            fn = (lambda wt=wt, n_out=n_out, n_in=n_in, key=key:
                  synth.weights(wt, n_out, n_in, seed=key))
        elif blocks == "quantized":
            fn = (lambda wt=wt, n_out=n_out, n_in=n_in, key=key: _quantized(wt, n_out, n_in, key))
        else:
            raise ValueError(f"blocks={blocks!r}")
        tensors.append((name, (n_in, n_out), wt, fn))
    for name, n in vectors(sh):
        tensors.append((name, (n,), Q.F32, (lambda name=name, n=n: _vector(name, n, seed).view(np.uint8))))
    return gguf.write(path, kvs, tensors)

"""Synthetic llama-architecture GGUF models (BASELINE.json configs[2..4]).

Weights are random-init N(0, 0.02), quantized "Q4_K_M-style": Q6_K for the
output head and for attn_v / ffn_down on every other layer, Q4_K for the other
matrices and the token embedding, F32 (ones) for the norms. The file uses the
GGUF keys and tensor names the reference's loader reads (src/model.c:51-172).
"""

from __future__ import annotations

import zlib
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from . import gguf
from . import quant as Q
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

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_head


# TinyLlama-1.1B shape
TINYLLAMA = LlamaShape(22, 2048, 5632, 32, 4, 32000, 10000.0, 1e-5, 2048)
# Llama-3-8B shape
LLAMA3_8B = LlamaShape(32, 4096, 14336, 32, 8, 128256, 500000.0, 1e-5, 2048)
# Qwen2.5-32B shape (its QKV bias adds are vector
# work outside the matrix path)
QWEN25_32B = LlamaShape(64, 5120, 27648, 40, 8, 152064, 1000000.0, 1e-6, 2048)
# a small model of the same family for parity tests
SMALL = LlamaShape(3, 512, 1536, 8, 2, 1024, 10000.0, 1e-5, 1024)


def matrices(sh: LlamaShape) -> list[tuple[str, int, int, int]]:
    """(tensor name, ggml type, n_out, n_in) of every weight matrix."""
    kv = sh.n_head_kv * sh.head_dim
    out = [("token_embd.weight", Q.Q4_K, sh.n_vocab, sh.n_embd),
           ("output.weight", Q.Q6_K, sh.n_vocab, sh.n_embd)]
    for il in range(sh.n_layer):
        mix = Q.Q6_K if il % 2 == 0 else Q.Q4_K
        out += [(f"blk.{il}.attn_q.weight", Q.Q4_K, sh.n_embd, sh.n_embd),
                (f"blk.{il}.attn_k.weight", Q.Q4_K, kv, sh.n_embd),
                (f"blk.{il}.attn_v.weight", mix, kv, sh.n_embd),
                (f"blk.{il}.attn_output.weight", Q.Q4_K, sh.n_embd, sh.n_embd),
                (f"blk.{il}.ffn_gate.weight", Q.Q4_K, sh.n_ff, sh.n_embd),
                (f"blk.{il}.ffn_up.weight", Q.Q4_K, sh.n_ff, sh.n_embd),
                (f"blk.{il}.ffn_down.weight", mix, sh.n_embd, sh.n_ff)]
    return out


def write_llama(path: str | Path, sh: LlamaShape, seed: int = 0) -> Path:
    kvs = [
        ("general.architecture", gguf.STRING, "llama"),
        ("general.alignment", gguf.U32, 32),
        ("llama.block_count", gguf.U32, sh.n_layer),
        ("llama.context_length", gguf.U32, sh.n_ctx),
        ("llama.embedding_length", gguf.U32, sh.n_embd),
        ("llama.feed_forward_length", gguf.U32, sh.n_ff),
        ("llama.attention.head_count", gguf.U32, sh.n_head),
        ("llama.attention.head_count_kv", gguf.U32, sh.n_head_kv),
        ("llama.attention.layer_norm_rms_epsilon", gguf.F32, sh.rms_eps),
        ("llama.rope.freq_base", gguf.F32, sh.rope_base),
    ]
    tensors = []
    for name, wt, n_out, n_in in matrices(sh):
        rng = np.random.default_rng([seed, zlib.crc32(name.encode())])
        w = (rng.standard_normal((n_out, n_in), dtype=np.float32) * np.float32(0.02))
        tensors.append((name, (n_in, n_out), wt, quantize(wt, w)))
    ones = np.ones(sh.n_embd, np.float32)
    tensors.append(("output_norm.weight", (sh.n_embd,), Q.F32, ones.view(np.uint8)))
    for il in range(sh.n_layer):
        tensors.append((f"blk.{il}.attn_norm.weight", (sh.n_embd,), Q.F32, ones.view(np.uint8)))
        tensors.append((f"blk.{il}.ffn_norm.weight", (sh.n_embd,), Q.F32, ones.view(np.uint8)))
    return gguf.write(path, kvs, tensors)

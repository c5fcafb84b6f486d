"""The quantized matrix path of a llama-architecture forward pass, on device.

The reference's forward pass (src/engine.c:290-400) calls its backend gemv
once per weight matrix and token: Wq, Wk, Wv (engine.c:317-319), Wo
(engine.c:368), W_gate and W_up (engine.c:375-376), W_down (engine.c:378) per
layer, then the output head (engine.c:393). This module runs exactly that
sequence of products through libsiphon_cuda for the model shapes of the
benchmark configs (synthetic Q4_K_M-style weights generated on the device):

* ``decode_step``: one token (batch 1), sicu_gemv_multi for products that
  share an activation and type (Wq/Wk[/Wv], W_gate/W_up), sicu_gemv_f32 for
  the rest;
* ``prefill``: m tokens at once through sicu_gemm_prefill_f32;
* ``prompt_step`` (``embed=True``, ``max_tokens`` > 1, one GPU): a prompt's
  whole forward pass, m tokens at once: the embedding rows, the RMS norms
  with their residual adds (sicu_rms_norm), the products (sicu_gemm_prefill_*),
  RoPE, the KV-cache stores and each token's attention over its prefix
  (sicu_attention_prompt), SwiGLU (sicu_swiglu), the head's logits for every
  token and the greedy choice after the last; the caches are left as the
  token-serial engine leaves them (src/cmd_run.c:275-276), so decode_step
  carries on at position pos + m.

With ``steps=True`` the decode step also runs the activation steps between
the products the way the reference's forward pass does (engine.c:313-315,
367-379, 387-389), each fused into the product that reads its result
(sicu_gemv_fused): the residual add and RMS norm before Wq/Wk/Wv, before
W_gate/W_up and before the output head, SwiGLU split into a silu epilogue on
W_gate's output and a multiply in W_down's prologue, and for Qwen2-shaped
models the Q/K/V bias adds as the QKV products' epilogue (engine.c:320-334). The
residual stream starts from a fixed embedding row, and Wo reads a fixed
activation in place of the attention output. ``attention=True`` adds RoPE,
the f16 KV-cache store and the heads' attention (sicu_attention_step, one
launch per layer), and ``embed=True`` the embedding lookup from a token id in
device memory and the greedy choice after the head: every step of the
reference's forward pass on the device. Without ``steps`` each product reads
a fixed activation buffer of its input length, so a step is the matrix work
of one token (or one prompt) and nothing else.

Tensor parallelism (``world > 1``) follows the layout the 32B-class configs
name: Wq/Wk/Wv, W_gate/W_up and the output head are split by output rows
(attention heads, FFN rows, vocabulary), Wo and W_down by input columns, and
the partial Wo and W_down outputs are summed with one all-reduce each per
layer (attention block and FFN block). Column shards are whole 256-element
super-blocks (Q8_K quantizes whole blocks), so shards can be uneven.

Two forms of that all-reduce:

* ``fused=True`` (decode): sicu_gemv_ar runs Wo and W_down as row-split
  products with the all-reduce inside the kernel (NVLink peer stores of the
  partial rows, a bounded wait for the other ranks' parts, the sum in rank
  order). The next products read the sum: W_gate/W_up read Wo's, the next
  layer's Wq/Wk/Wv (or the head) read W_down's, where a full forward pass
  would put the residual add and norm between them.
* otherwise: ``torch.distributed.all_reduce`` (NCCL) on each partial output,
  and every product reads a fixed activation.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

from . import quant as Q
from .synth_model import GGUF_NAMES, LlamaShape, layer_types

# byte offsets of the f16 scale fields inside one block (include/siphon/quant.h)
F16_FIELDS = {
    Q.Q4_0: (0,), Q.Q5_0: (0,), Q.Q8_0: (0,),
    Q.Q2_K: (80, 82), Q.Q3_K: (108,), Q.Q4_K: (0, 2), Q.Q5_K: (0, 2), Q.Q6_K: (208,),
}


def _split(n_units: int, world: int, rank: int) -> range:
    """Units [start, stop) of rank in a balanced split (first ranks get the extra)."""
    base, extra = divmod(n_units, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


@dataclass(frozen=True)
class Shard:
    heads: range          # query heads
    kv_heads: tuple       # key/value heads those query heads read (replicated where shared)
    ff: range             # FFN rows (elements)
    vocab: range          # output-head rows


def tp_partition(sh: LlamaShape, world: int, rank: int) -> Shard:
    hd = sh.head_dim
    heads_per_unit = 256 // math.gcd(256, hd)        # Wo's column shard must be whole super-blocks
    if sh.n_head % heads_per_unit or sh.n_ff % 256:
        raise ValueError("shape cannot be split on 256-element boundaries")
    hu = _split(sh.n_head // heads_per_unit, world, rank)
    heads = range(hu.start * heads_per_unit, hu.stop * heads_per_unit)
    group = sh.n_head // sh.n_head_kv
    kv = tuple(sorted({h // group for h in heads}))
    fu = _split(sh.n_ff // 256, world, rank)
    vu = _split(sh.n_vocab, world, rank)
    return Shard(heads, kv, range(fu.start * 256, fu.stop * 256), vu)


def rope_tables(sh: LlamaShape, n_ctx: int):
    """cos / sin tables [n_ctx][n_rot / 2] of every position, computed as the
    reference engine computes them on the host (src/engine.c:26-40, 196):
    theta_scale = powf(base, -2 / n_rot); per position theta starts at the
    position and is multiplied by theta_scale (f32) after each pair; cosf /
    sinf from the C library (the same libm the reference build calls)."""
    import ctypes
    import ctypes.util

    import numpy as np
    libm = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
    for fn in ("powf", "cosf", "sinf"):
        getattr(libm, fn).restype = ctypes.c_float
    libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]
    libm.cosf.argtypes = libm.sinf.argtypes = [ctypes.c_float]
    n_rot = sh.head_dim
    theta_scale = np.float32(libm.powf(np.float32(sh.rope_base), np.float32(-2.0) / np.float32(n_rot)))
    cos = np.zeros((n_ctx, n_rot // 2), np.float32)
    sin = np.zeros((n_ctx, n_rot // 2), np.float32)
    for p in range(n_ctx):
        th = np.float32(p)
        for j in range(n_rot // 2):
            cos[p, j], sin[p, j] = libm.cosf(th), libm.sinf(th)
            th = np.float32(th * theta_scale)
    return cos, sin


def packable(wtype: int, n_in: int) -> bool:
    """Whether sicu_prefill_pack makes a prefill copy of a matrix of this
    type and row length: the K formats; the classic formats with rows of at
    least one 128-element K-step; F16 rows of whole 256-element chunks."""
    if wtype in (Q.Q2_K, Q.Q3_K, Q.Q4_K, Q.Q5_K, Q.Q6_K):
        return True
    if wtype in (Q.Q4_0, Q.Q5_0, Q.Q8_0):
        return n_in >= 128
    return wtype == Q.F16 and n_in % 256 == 0


def shard_shapes(sh: LlamaShape, shard: Shard) -> dict:
    """(n_out, n_in) of every matrix one rank holds."""
    hd = sh.head_dim
    nq, nkv, nff = len(shard.heads) * hd, len(shard.kv_heads) * hd, len(shard.ff)
    return {"q": (nq, sh.n_embd), "k": (nkv, sh.n_embd), "v": (nkv, sh.n_embd), "o": (sh.n_embd, nq),
            "gate": (nff, sh.n_embd), "up": (nff, sh.n_embd), "down": (sh.n_embd, nff),
            "head": (len(shard.vocab), sh.n_embd)}


def step_weight_bytes(sh: LlamaShape, world: int = 1, rank: int = 0) -> int:
    """Weight bytes one rank streams per decode token."""
    shp = shard_shapes(sh, tp_partition(sh, world, rank))
    total = Q.row_bytes(Q.Q6_K, sh.n_embd) * shp["head"][0]
    for il in range(sh.n_layer):
        t = layer_types(il)
        for name in ("q", "k", "v", "o", "gate", "up", "down"):
            n_out, n_in = shp[name]
            total += n_out * Q.row_bytes(t[name], n_in)
    return total


def device_weights(wtype: int, n_out: int, n_in: int, seed: int, device):
    """Synthetic GGUF blocks generated on the device (same distribution as
    synth.weights: f16 scales U[1e-4, 1e-2], every other bit uniform)."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    rb = Q.row_bytes(wtype, n_in)
    raw = torch.randint(0, 256, (n_out * rb,), dtype=torch.uint8, device=device, generator=g)
    bsz = Q.GEOMETRY[wtype][1]
    blocks = raw.view(-1, bsz)
    for off in F16_FIELDS[wtype]:
        d = torch.empty(blocks.shape[0], dtype=torch.float32, device=device).uniform_(1e-4, 1e-2, generator=g)
        blocks[:, off:off + 2] = d.half().view(torch.uint8).view(-1, 2)
    return raw


class MatrixPath:
    """One rank's shard of the model's weight matrices and the launch
    sequence of a decode step / a prefill over them.

    Weights are synthetic blocks generated on the device, or, with
    ``gguf_path`` (one GPU), a model file's tensors uploaded unchanged: the
    matrices, the embedding, the norm weights and any Q/K/V biases."""

    def __init__(self, sicu, sh: LlamaShape, device, world: int = 1, rank: int = 0, group=None, seed: int = 0,
                 max_tokens: int = 1, fused: bool = False, steps: bool = False, attention: bool = False,
                 n_ctx: int = 256, embed: bool = False, gguf_path=None, packed: bool = False):
        import numpy as np
        import torch
        self.s, self.sh, self.dev, self.world, self.group = sicu, sh, device, world, group
        self.ar = None
        self.steps = steps or attention or embed
        self.attention = attention or embed
        self.embed = embed
        self.pos = 0
        self.shard = tp_partition(sh, world, rank)
        self.shapes = shard_shapes(sh, self.shard)
        reader = None
        if gguf_path is not None:
            from . import gguf
            if world != 1:
                raise ValueError("a model file is loaded on one GPU")
            reader = gguf.Reader(gguf_path)

        def from_file(name, n_out=None, n_in=None):
            info = reader.tensors[name]
            if n_out is not None and info.dims[:2] != (n_in, n_out):
                raise ValueError(f"{name}: dims {info.dims} in the file, ({n_in}, {n_out}) expected")
            return info.type, torch.from_numpy(np.array(reader.data(name))).to(device)

        self.layers = []
        for il in range(sh.n_layer):
            t = layer_types(il)
            lay = {}
            for j, name in enumerate(("q", "k", "v", "o", "gate", "up", "down")):
                n_out, n_in = self.shapes[name]
                if reader is not None:
                    lay[name] = from_file(f"blk.{il}.{GGUF_NAMES[name]}.weight", n_out, n_in)
                else:
                    lay[name] = (t[name], device_weights(t[name], n_out, n_in,
                                                         seed * 7919 + il * 16 + j + 1000 * rank, device))
            self.layers.append(lay)
        n_out, n_in = self.shapes["head"]
        if reader is not None:
            self.head = from_file("output.weight", n_out, n_in)
        else:
            self.head = (Q.Q6_K, device_weights(Q.Q6_K, n_out, n_in, seed * 7919 + 999 + 1000 * rank, device))
        # prefill copies (sicu_prefill_pack) of the matrices, made once here
        # beside the raw blocks
        self.pack = {}
        if packed:
            mats = [((il, name), lay[name]) for il, lay in enumerate(self.layers) for name in lay]
            mats.append((("head",), self.head))
            for key, (t, w) in mats:
                n_out, n_in = self.shapes[key[-1]]
                if not packable(t, n_in):
                    continue
                nb = sicu.prefill_pack_bytes(t, n_in, n_out)
                buf = torch.empty(nb, dtype=torch.uint8, device=device)
                sicu.prefill_pack(t, w, n_in, n_out, buf, nb)
                self.pack[key] = buf
            torch.cuda.synchronize(device)
        m = max_tokens
        gen = torch.Generator(device=device)
        gen.manual_seed(seed + 17)

        def act(n):
            return torch.randn(m, n, device=device, generator=gen)

        nq, nff = self.shapes["q"][0], self.shapes["gate"][0]
        # fixed inputs per input length; outputs per product
        self.x_model, self.x_attn, self.x_ff = act(sh.n_embd), act(nq), act(nff)
        self.y = {name: torch.empty(m, self.shapes[name][0], device=device) for name in self.shapes}
        self.weight_bytes = step_weight_bytes(sh, world, rank)

        def vec(name):
            return torch.from_numpy(np.array(reader.data(name)).view(np.float32)).to(device)

        if self.steps:
            # norm weights (near 1 when synthetic; replicated on every rank),
            # two residual stream buffers used in turn
            def norm_w():
                return 1.0 + 0.1 * torch.randn(sh.n_embd, device=device, generator=gen)
            if reader is not None:
                self.attn_norm = [vec(f"blk.{il}.attn_norm.weight") for il in range(sh.n_layer)]
                self.ffn_norm = [vec(f"blk.{il}.ffn_norm.weight") for il in range(sh.n_layer)]
                self.out_norm = vec("output_norm.weight")
            else:
                self.attn_norm = [norm_w() for _ in range(sh.n_layer)]
                self.ffn_norm = [norm_w() for _ in range(sh.n_layer)]
                self.out_norm = norm_w()
            self.resid = [torch.empty(sh.n_embd, device=device) for _ in range(2)]
            # Qwen2-architecture Q/K/V biases, added after those products
            # (synthetic: 0.02 N(0, 1), this rank's heads)
            self.bias = None
            if sh.qkv_bias:
                def bias_vec(il, name, n):
                    if reader is not None:
                        return vec(f"blk.{il}.attn_{name}.bias")
                    return 0.02 * torch.randn(n, device=device, generator=gen)
                nq_, nkv_ = self.shapes["q"][0], self.shapes["k"][0]
                self.bias = [{"q": bias_vec(il, "q", nq_), "k": bias_vec(il, "k", nkv_), "v": bias_vec(il, "v", nkv_)}
                             for il in range(sh.n_layer)]
        if self.attention:
            # f16 caches per layer in the engine's layout (K [kv][n_ctx][hd],
            # V [kv][hd][n_ctx]), zero; the RoPE tables of every position as
            # the engine computes them
            hd, nkv = sh.head_dim, len(self.shard.kv_heads)
            per_kv = sh.n_head // sh.n_head_kv
            if not (len(self.shard.heads) == nkv * per_kv or nkv == 1):
                raise ValueError("a rank's query heads must cover whole KV groups")
            self.n_ctx = n_ctx
            self.kc = [torch.zeros(nkv * n_ctx * hd, dtype=torch.int16, device=device) for _ in range(sh.n_layer)]
            self.vc = [torch.zeros(nkv * hd * n_ctx, dtype=torch.int16, device=device) for _ in range(sh.n_layer)]
            cos, sin = rope_tables(sh, n_ctx)
            self.rope_cos = torch.from_numpy(cos).to(device)
            self.rope_sin = torch.from_numpy(sin).to(device)
            self.kq_scale = float(np.float32(1.0) / np.sqrt(np.float32(hd)))
            self.x_attn_buf = torch.empty(len(self.shard.heads) * hd, device=device)
        if embed:
            # a device-resident token loop: the step starts from the embedding
            # row of self.token (on the device) and ends by writing the greedy
            # choice of its logits back into it (one GPU: the head is whole)
            if world != 1:
                raise ValueError("the device token loop needs the whole output head on one GPU")
            if reader is not None:
                self.embd_type, self.embd = from_file("token_embd.weight", sh.n_vocab, sh.n_embd)
            else:
                self.embd_type = Q.Q4_K
                self.embd = device_weights(Q.Q4_K, sh.n_vocab, sh.n_embd, seed * 7919 + 555, device)
            self.token = torch.zeros(1, dtype=torch.int64, device=device)
            self.x_embed = torch.empty(sh.n_embd, device=device)
            if m > 1:
                # a prompt of up to m tokens (prompt_step): its token ids, two
                # residual streams used in turn, the normed rows, the attention
                # output and the SwiGLU rows
                self.tokens = torch.zeros(m, dtype=torch.int64, device=device)
                self.xp = [torch.empty(m, sh.n_embd, device=device) for _ in range(2)]
                self.xn = torch.empty(m, sh.n_embd, device=device)
                self.att = torch.empty(m, nq, device=device)
                self.ffp = torch.empty(m, nff, device=device)
        if fused and world > 1:
            import torch.distributed as dist
            self.ar = sicu.ar_create(world, rank, sh.n_embd)
            handles = [None] * world
            dist.all_gather_object(handles, self.ar.local_handle, group=self.group)
            self.ar.open(handles)

    def close(self) -> None:
        """Release the fused group (every rank calls this at the same point:
        streams are drained and the ranks meet before and after)."""
        if self.ar is not None:
            import torch
            import torch.distributed as dist
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
            self.ar.destroy()
            self.ar = None
            dist.barrier(group=self.group)

    def _allreduce(self, t) -> None:
        if self.world > 1:
            import torch.distributed as dist
            dist.all_reduce(t, group=self.group)

    def decode_step(self, stream) -> int:
        """Launch one token's products on `stream`; returns the number of
        library kernel launches."""
        if self.steps:
            return self._decode_step_steps(stream)
        if self.ar is not None:
            return self._decode_step_fused(stream)
        s, h, y = self.s, stream.cuda_stream, self.y
        x, xa, xf = self.x_model[0], self.x_attn[0], self.x_ff[0]
        n = 0
        for lay in self.layers:
            (tq, wq), (tk, wk), (tv, wv) = lay["q"], lay["k"], lay["v"]
            (nq, _), (nkv, _) = self.shapes["q"], self.shapes["k"]
            if tv == tq:
                s.gemv_multi(tq, [wq, wk, wv], [nq, nkv, nkv], self.sh.n_embd, x, [y["q"], y["k"], y["v"]], stream=h)
                n += 1
            else:
                s.gemv_multi(tq, [wq, wk], [nq, nkv], self.sh.n_embd, x, [y["q"], y["k"]], stream=h)
                s.gemv_f32(tv, wv, self.sh.n_embd, nkv, x, y["v"], stream=h)
                n += 2
            to, wo = lay["o"]
            s.gemv_f32(to, wo, nq, self.sh.n_embd, xa, y["o"], stream=h)
            self._allreduce(y["o"])
            (tg, wg), (_, wu) = lay["gate"], lay["up"]
            nff = self.shapes["gate"][0]
            s.gemv_multi(tg, [wg, wu], [nff, nff], self.sh.n_embd, x, [y["gate"], y["up"]], stream=h)
            td, wd = lay["down"]
            s.gemv_f32(td, wd, nff, self.sh.n_embd, xf, y["down"], stream=h)
            self._allreduce(y["down"])
            n += 3
        th, wh = self.head
        s.gemv_f32(th, wh, self.sh.n_embd, self.shapes["head"][0], x, y["head"], stream=h)
        return n + 1

    def _decode_step_fused(self, stream) -> int:
        """decode_step with the all-reduces fused into Wo and W_down: 4 or 5
        launches per layer and no collective launches."""
        s, h, y, ar, d = self.s, stream.cuda_stream, self.y, self.ar, self.sh.n_embd
        (nq, _), (nkv, _) = self.shapes["q"], self.shapes["k"]
        nff = self.shapes["gate"][0]
        x = self.x_model[0]                  # layer 0 reads the embedding row
        n = 0
        for lay in self.layers:
            (tq, wq), (tk, wk), (tv, wv) = lay["q"], lay["k"], lay["v"]
            if tv == tq:
                s.gemv_multi(tq, [wq, wk, wv], [nq, nkv, nkv], d, x, [y["q"], y["k"], y["v"]], stream=h)
                n += 1
            else:
                s.gemv_multi(tq, [wq, wk], [nq, nkv], d, x, [y["q"], y["k"]], stream=h)
                s.gemv_f32(tv, wv, d, nkv, x, y["v"], stream=h)
                n += 2
            to, wo = lay["o"]
            s.gemv_ar(to, wo, nq, d, self.x_attn[0], y["o"][0], ar, stream=h)
            (tg, wg), (_, wu) = lay["gate"], lay["up"]
            s.gemv_multi(tg, [wg, wu], [nff, nff], d, y["o"][0], [y["gate"], y["up"]], stream=h)
            td, wd = lay["down"]
            s.gemv_ar(td, wd, nff, d, self.x_ff[0], y["down"][0], ar, stream=h)
            x = y["down"][0]
            n += 3
        th, wh = self.head
        s.gemv_f32(th, wh, d, self.shapes["head"][0], x, y["head"], stream=h)
        return n + 1

    def _decode_step_steps(self, stream) -> int:
        """One token with the activation steps fused into the products:
        per layer h += (previous W_down output); Wq/Wk/Wv of norm(h); h += Wo
        output; W_gate/W_up of norm(h), the gate output written through silu;
        W_down of silu(gate) * up; after the last layer the head of
        norm(h + W_down output). The residual sums are written by the
        products that norm them (sum_out). Row-split products all-reduce in
        the kernel (fused groups) or through NCCL. y["gate"] ends up holding
        silu(gate)."""
        from .lib import EPI_NONE, EPI_SILU, mul_step, rms_norm_step
        s, h, y, d, eps = self.s, stream.cuda_stream, self.y, self.sh.n_embd, self.sh.rms_eps
        (nq, _), (nkv, _) = self.shapes["q"], self.shapes["k"]
        nff = self.shapes["gate"][0]
        cur, res = self.x_model[0], None      # residual stream so far, and the output still to be added
        nxt = 0
        n = 0
        if self.embed:
            s.row_to_f32_dev(self.embd_type, self.embd, d, self.sh.n_vocab, self.token, 1, self.x_embed, stream=h)
            cur = self.x_embed
            n += 1
        for il, lay in enumerate(self.layers):
            (tq, wq), (tk, wk), (tv, wv) = lay["q"], lay["k"], lay["v"]
            out = self.resid[nxt]
            step = rms_norm_step(self.attn_norm[il], eps, res, out)
            b = self.bias[il] if self.bias is not None else None
            if tv == tq:
                s.gemv_fused(tq, [wq, wk, wv], [nq, nkv, nkv], d, cur, step, [y["q"], y["k"], y["v"]], stream=h,
                             bias=[b["q"], b["k"], b["v"]] if b else None)
                n += 1
            else:
                s.gemv_fused(tq, [wq, wk], [nq, nkv], d, cur, step, [y["q"], y["k"]], stream=h,
                             bias=[b["q"], b["k"]] if b else None)
                s.gemv_fused(tv, [wv], [nkv], d, out, rms_norm_step(self.attn_norm[il], eps), [y["v"]], stream=h,
                             bias=[b["v"]] if b else None)
                n += 2
            cur, nxt = out, 1 - nxt
            xa = self.x_attn[0]
            if self.attention:
                # RoPE on q and k, this position's K / V into the caches, the
                # heads' attention over positions 0..pos (src/engine.c:336-366)
                hd, p = self.sh.head_dim, self.pos
                nh, nkvl = nq // hd, nkv // hd
                s.attention_step(y["q"], y["k"], y["v"], self.kc[il], self.vc[il], self.rope_cos[p],
                                 self.rope_sin[p], nh, nkvl, hd, hd, self.n_ctx, p, self.kq_scale, self.x_attn_buf,
                                 neox=self.sh.neox, stream=h)
                xa = self.x_attn_buf
                n += 1
            to, wo = lay["o"]
            s.gemv_fused(to, [wo], [d], nq, xa, None, [y["o"]], group=self.ar, stream=h)
            if self.ar is None:
                self._allreduce(y["o"])
            (tg, wg), (_, wu) = lay["gate"], lay["up"]
            out = self.resid[nxt]
            # SwiGLU split in two: silu in the gate product's epilogue (once
            # per element), the product with up in W_down's prologue
            s.gemv_fused(tg, [wg, wu], [nff, nff], d, cur, rms_norm_step(self.ffn_norm[il], eps, y["o"][0], out),
                         [y["gate"], y["up"]], stream=h, epi=[EPI_SILU, EPI_NONE])
            cur, nxt = out, 1 - nxt
            td, wd = lay["down"]
            s.gemv_fused(td, [wd], [d], nff, y["gate"][0], mul_step(y["up"][0]), [y["down"]], group=self.ar,
                         stream=h)
            if self.ar is None:
                self._allreduce(y["down"])
            res = y["down"][0]
            n += 3
        th, wh = self.head
        s.gemv_fused(th, [wh], [self.shapes["head"][0]], d, cur, rms_norm_step(self.out_norm, eps, res),
                     [y["head"]], stream=h)
        if self.embed:
            s.argmax(y["head"], self.shapes["head"][0], 1, self.token, stream=h)
            n += 1
        return n + 1

    def batch_step(self, stream, m: int) -> int:
        """One decode step of m <= 8 sequences (one token each): every weight
        product once for all m activation rows (sicu_gemv_batch; products that
        share an activation and type in one launch), row-split partials
        all-reduced through NCCL. Returns the number of library calls."""
        s, h, y = self.s, stream.cuda_stream, self.y
        d = self.sh.n_embd
        nq, nkv, nff = self.shapes["q"][0], self.shapes["k"][0], self.shapes["gate"][0]
        n = 0
        for lay in self.layers:
            (tq, wq), (tk, wk), (tv, wv) = lay["q"], lay["k"], lay["v"]
            if tv == tq:
                s.gemv_batch(tq, [wq, wk, wv], [nq, nkv, nkv], d, self.x_model, m, [y["q"], y["k"], y["v"]], stream=h)
                n += 1
            else:
                s.gemv_batch(tq, [wq, wk], [nq, nkv], d, self.x_model, m, [y["q"], y["k"]], stream=h)
                s.gemv_batch(tv, [wv], [nkv], d, self.x_model, m, [y["v"]], stream=h)
                n += 2
            to, wo = lay["o"]
            s.gemv_batch(to, [wo], [d], nq, self.x_attn, m, [y["o"]], stream=h)
            self._allreduce(y["o"][:m])
            (tg, wg), (_, wu) = lay["gate"], lay["up"]
            s.gemv_batch(tg, [wg, wu], [nff, nff], d, self.x_model, m, [y["gate"], y["up"]], stream=h)
            td, wd = lay["down"]
            s.gemv_batch(td, [wd], [d], nff, self.x_ff, m, [y["down"]], stream=h)
            self._allreduce(y["down"][:m])
            n += 3
        th, wh = self.head
        s.gemv_batch(th, [wh], [self.shapes["head"][0]], d, self.x_model, m, [y["head"]], stream=h)
        return n + 1

    def _prompt_products(self, il: int, group, n_in: int, xin, m: int, h) -> int:
        """The m-row products of layer il's matrices `group` (one activation
        xin): those with one weight type and prefill copies as one grouped
        launch (Wq/Wk[/Wv], W_gate/W_up), the rest one by one. Returns the
        number of library calls."""
        s, y, lay = self.s, self.y, self.layers[il]
        runs = []
        for name in group:
            t = lay[name][0]
            pk = self.pack.get((il, name))
            if runs and runs[-1][0] == t and pk is not None and runs[-1][1][-1][1] is not None:
                runs[-1][1].append((name, pk))
            else:
                runs.append((t, [(name, pk)]))
        for t, members in runs:
            if len(members) > 1:
                names = [nm for nm, _ in members]
                s.gemm_prefill_multi_f32(t, [lay[nm][1] for nm in names], [pk for _, pk in members],
                                         [self.shapes[nm][0] for nm in names], n_in, xin, m,
                                         [y[nm] for nm in names], stream=h)
                continue
            name, pk = members[0]
            w = lay[name][1]
            if pk is not None:
                s.gemm_prefill_packed_f32(t, w, pk, n_in, self.shapes[name][0], xin, m, y[name], stream=h)
            else:
                s.gemm_prefill_f32(t, w, n_in, self.shapes[name][0], xin, m, y[name], stream=h)
        return len(runs)

    def _prompt_head(self, x, m: int, h) -> None:
        s, d = self.s, self.sh.n_embd
        th, wh = self.head
        pk = self.pack.get(("head",))
        if pk is not None:
            s.gemm_prefill_packed_f32(th, wh, pk, d, self.shapes["head"][0], x, m, self.y["head"], stream=h)
        else:
            s.gemm_prefill_f32(th, wh, d, self.shapes["head"][0], x, m, self.y["head"], stream=h)

    def prefill(self, stream, m: int) -> None:
        """Launch the products of an m-token prompt on `stream` (or, with m
        up to the batch size, one decode step of a batch of m sequences:
        the same products, every weight matrix streamed once for all m)."""
        h, y = stream.cuda_stream, self.y
        d = self.sh.n_embd
        nq, nff = self.shapes["q"][0], self.shapes["gate"][0]
        for il in range(len(self.layers)):
            for group, n_in, xin in ((("q", "k", "v"), d, self.x_model), (("o",), nq, self.x_attn),
                                     (("gate", "up"), d, self.x_model), (("down",), nff, self.x_ff)):
                self._prompt_products(il, group, n_in, xin, m, h)
                if group[0] in ("o", "down"):
                    self._allreduce(y[group[0]][:m])
        self._prompt_head(self.x_model, m, h)

    def prompt_step(self, stream, m: int) -> int:
        """The forward pass of the m prompt tokens in self.tokens[:m] at
        positions self.pos .. self.pos + m - 1, all tokens at once, in the
        reference's per-token order of steps (src/engine.c:290-398):
        embedding rows; per layer h += (previous W_down output) and its RMS
        norm, Wq/Wk/Wv (and the Q/K/V bias adds of Qwen2 models), RoPE +
        cache stores + each token's attention over
        positions 0 .. its own, Wo, h += Wo output and its RMS norm,
        W_gate/W_up, SwiGLU, W_down; the output norm and the head's logits of
        every token (y["head"][:m]); the greedy choice after the last token
        into self.token. Every step but the products repeats the reference's
        arithmetic per row; the products are the prefill kernels' (bit-exact
        for the classic formats and the matvec sizes, within 1e-5 of each
        output's L1 norm for the K formats and F16 on tensor cores). Returns
        the number of library calls."""
        if not (self.embed and hasattr(self, "tokens")):
            raise ValueError("prompt_step needs MatrixPath(embed=True, max_tokens > 1)")
        if not 0 < m <= self.tokens.numel() or self.pos + m > self.n_ctx:
            raise ValueError(f"prompt of {m} tokens at position {self.pos}: past the buffers or the context")
        s, h, y, d, eps = self.s, stream.cuda_stream, self.y, self.sh.n_embd, self.sh.rms_eps
        nq, nkv, nff = self.shapes["q"][0], self.shapes["k"][0], self.shapes["gate"][0]
        hd, p = self.sh.head_dim, self.pos
        xp, xn = self.xp, self.xn
        s.row_to_f32_dev(self.embd_type, self.embd, d, self.sh.n_vocab, self.tokens, m, xp[0], stream=h)
        cur, nxt, res, n = 0, 1, None, 1
        for il in range(len(self.layers)):
            if res is None:
                s.rms_norm(xp[cur], self.attn_norm[il], d, m, eps, xn, stream=h)
            else:
                s.rms_norm(xp[cur], self.attn_norm[il], d, m, eps, xn, dres=res, dsum=xp[nxt], stream=h)
                cur, nxt = nxt, cur
            n += 1 + self._prompt_products(il, ("q", "k", "v"), d, xn, m, h)
            if self.bias is not None:
                # Qwen2: the Q/K/V bias adds over the m rows (src/engine.c:319-333)
                b = self.bias[il]
                for name, width in (("q", nq), ("k", nkv), ("v", nkv)):
                    s.add_bias(y[name], b[name], width, m, stream=h)
                n += 3
            s.attention_prompt(y["q"], y["k"], y["v"], self.kc[il], self.vc[il], self.rope_cos[p:],
                               self.rope_sin[p:], nq // hd, nkv // hd, hd, hd, self.n_ctx, p, m, self.kq_scale,
                               self.att, neox=self.sh.neox, stream=h)
            n += 1 + self._prompt_products(il, ("o",), nq, self.att, m, h)
            s.rms_norm(xp[cur], self.ffn_norm[il], d, m, eps, xn, dres=y["o"], dsum=xp[nxt], stream=h)
            cur, nxt = nxt, cur
            n += 1 + self._prompt_products(il, ("gate", "up"), d, xn, m, h)
            s.swiglu(y["gate"], y["up"], nff, m, self.ffp, stream=h)
            n += 1 + self._prompt_products(il, ("down",), nff, self.ffp, m, h)
            res = y["down"]
        s.rms_norm(xp[cur], self.out_norm, d, m, eps, xn, dres=res, dsum=xp[nxt], stream=h)
        self._prompt_head(xn, m, h)
        s.argmax(y["head"][m - 1], self.shapes["head"][0], 1, self.token, stream=h)
        return n + 3

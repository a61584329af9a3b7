"""End-to-end batched speculative step over a random-init Llama (config 4).

A caller of the verify path, not part of it: the model's dense layers are
plain library GEMMs (torch / cuBLAS) and elementwise torch ops, and every
step of the verify path runs on this library's kernels through the C ABI:

  kv_reserve (k+1 slots, shared by target and draft)
  draft loop, k times:   draft forward of one token per request
                         (rope_kv_write + verify_attention per layer)
                         -> sample_tokens (Philox stream 0)
  target verify forward: k+1 tokens per request at context_len + j
                         (rope_kv_write + verify_attention per layer)
  spec_accept (stochastic, temperature T) -> kv_commit (keeps accept_len + 1)

The layer follows the reference's `LlamaAttention::forward`
(src/model/llama.rs:62-119): q/k/v projections, RoPE at `index + i`
(theta 10000, src/model/llama.rs:45), K/V appended to the cache, attention,
o_proj; RMSNorm and a SwiGLU MLP around it (src/model/llama.rs:121-176).
The draft is a narrower stack of the same layer (2 layers, same width) that
shares the target's embedding and lm_head; it keeps its own paged K/V
caches over the same block table, since its tokens sit at the same
positions.

One simplification, documented where it matters: when every draft token is
accepted, the draft's own K/V row for the last draft token is not written
(the draft never ran on it).  The next step's draft attends over that slot
as it was; a serving draft would run two tokens on its next first step.
With random-init weights this changes values, not the work or its timing.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List

import numpy as np
import torch
import torch.nn.functional as F

from .verify import (Context, kv_commit, kv_reserve, rope_kv_write, sample_tokens, spec_accept,
                     verify_attention)


@dataclass
class LlamaShape:
    layers: int = 16
    hidden: int = 2048
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 64
    ffn: int = 8192
    vocab: int = 128256
    rope_theta: float = 10000.0
    eps: float = 1e-5


@dataclass
class E2EConfig:
    requests: int = 512
    k: int = 4
    temperature: float = 0.7
    ctx_median: int = 1024
    ctx_sigma: float = 1.0   # lognormal sigma (not stated by the benchmark; assumed)
    ctx_max: int = 16384
    block_size: int = 16
    draft_layers: int = 2
    # KV blocks per attention work item (0: the library's plan, 256 here).
    # The grid spans the block table's width, so short items mostly launch
    # empty CTAs: measured 445 us at 64 blocks against 308 us at 256 for the
    # target's 5 query rows
    kv_split_blocks: int = 0


CONFIG4 = E2EConfig()
CONFIG4_SHAPE = LlamaShape()


def context_lengths(cfg: E2EConfig, seed: int = 0) -> np.ndarray:
    """Lognormal context lengths (median cfg.ctx_median), clipped to [1, ctx_max]."""
    rng = np.random.default_rng(seed)
    x = rng.lognormal(math.log(cfg.ctx_median), cfg.ctx_sigma, size=cfg.requests)
    return np.clip(np.rint(x), 1, cfg.ctx_max).astype(np.int64)


class Layers:
    """Random-init weights of a stack of Llama layers (bf16)."""

    def __init__(self, shape: LlamaShape, n: int, device, gen: torch.Generator):
        h, d, hq, hkv, f = shape.hidden, shape.head_dim, shape.heads, shape.kv_heads, shape.ffn
        std = 0.02

        def w(*s):
            return (torch.randn(*s, generator=gen, device=device, dtype=torch.bfloat16) * std)

        self.wqkv = [w(h, (hq + 2 * hkv) * d) for _ in range(n)]
        self.wo = [w(hq * d, h) for _ in range(n)]
        self.wgu = [w(h, 2 * f) for _ in range(n)]
        self.wdown = [w(f, h) for _ in range(n)]
        self.norm1 = [torch.ones(h, device=device, dtype=torch.bfloat16) for _ in range(n)]
        self.norm2 = [torch.ones(h, device=device, dtype=torch.bfloat16) for _ in range(n)]
        self.n = n


class SpecModels:
    """Target and draft models with their paged K/V caches.

    K/V caches: one [num_blocks, Hkv, block_size, D] bf16 pair per layer
    (the reference's layout, src/model/attention_kernel.rs:52-57), filled
    with N(0, 1) to stand for the prefilled contexts."""

    def __init__(self, shape: LlamaShape, cfg: E2EConfig, num_blocks: int, device, seed: int = 0):
        g = torch.Generator(device=device).manual_seed(seed)
        self.shape, self.cfg, self.device = shape, cfg, device
        self.embed = torch.randn(shape.vocab, shape.hidden, generator=g, device=device,
                                 dtype=torch.bfloat16)
        self.lm_head = torch.randn(shape.hidden, shape.vocab, generator=g, device=device,
                                   dtype=torch.bfloat16) * 0.02
        self.final_norm = torch.ones(shape.hidden, device=device, dtype=torch.bfloat16)
        self.target = Layers(shape, shape.layers, device, g)
        self.draft = Layers(shape, cfg.draft_layers, device, g)
        cs = (num_blocks, shape.kv_heads, cfg.block_size, shape.head_dim)

        def cache():
            return torch.randn(cs, generator=g, device=device, dtype=torch.bfloat16)

        self.t_k = [cache() for _ in range(shape.layers)]
        self.t_v = [cache() for _ in range(shape.layers)]
        self.d_k = [cache() for _ in range(cfg.draft_layers)]
        self.d_v = [cache() for _ in range(cfg.draft_layers)]

    def forward(self, ctx: Context, layers: Layers, kc: List[torch.Tensor], vc: List[torch.Tensor],
                tokens: torch.Tensor, block_table: torch.Tensor, lens: torch.Tensor,
                ws_attn: torch.Tensor, logits: torch.Tensor, timer=None) -> torch.Tensor:
        """tokens int64 [B, n] at positions lens[b] + j -> fp32 logits, written
        by the lm_head GEMM into `logits` and returned as [B, n, V].  `logits`
        is [B * n, V], contiguous, or (n == 1) a [B, V] view with unit column
        stride, such as column i of a [B, k, V] buffer, which the GEMM writes
        in place.  Each layer stores its new K/V rows into slots lens[b] + j."""
        s = self.shape
        B, n = tokens.shape
        hq, hkv, d = s.heads, s.kv_heads, s.head_dim
        x = self.embed[tokens]  # [B, n, hidden]
        for i in range(layers.n):
            h = F.rms_norm(x, (s.hidden,), layers.norm1[i], s.eps)
            qkv = torch.matmul(h, layers.wqkv[i])  # [B, n, (hq + 2 hkv) d]
            q = qkv[..., :hq * d].reshape(B, n, hq, d).contiguous()
            kk = qkv[..., hq * d:(hq + hkv) * d].reshape(B, n, hkv, d).contiguous()
            vv = qkv[..., (hq + hkv) * d:].reshape(B, n, hkv, d).contiguous()
            rope_kv_write(ctx, q, kk, vv, block_table, lens, kc[i], vc[i], self.cfg.block_size,
                          theta=s.rope_theta, q_out=q)
            if timer is not None:
                timer.begin("attention")
            o = verify_attention(ctx, q, kc[i], vc[i], block_table, lens,
                                 kv_split_blocks=self.cfg.kv_split_blocks, workspace=ws_attn)
            if timer is not None:
                timer.end("attention")
            x = x + torch.matmul(o.view(B, n, hq * d), layers.wo[i])
            h = F.rms_norm(x, (s.hidden,), layers.norm2[i], s.eps)
            gu = torch.matmul(h, layers.wgu[i])
            x = x + torch.matmul(F.silu(gu[..., :s.ffn]) * gu[..., s.ffn:], layers.wdown[i])
        h = F.rms_norm(x, (s.hidden,), self.final_norm, s.eps)
        torch.mm(h.view(B * n, s.hidden), self.lm_head, out_dtype=torch.float32, out=logits)
        if logits.is_contiguous():
            return logits.view(B, n, s.vocab)
        return logits.unsqueeze(1)  # [B, 1, V], rows k * V apart


class SpecStep:
    """Buffers and the launch sequence of one batched speculative step."""

    def __init__(self, models: SpecModels, ctx_t: Context, ctx_d: Context, kv, seed: int = 0,
                 seq_offset: int = 0):
        self.m, self.ctx_t, self.ctx_d, self.kv = models, ctx_t, ctx_d, kv
        cfg, s = models.cfg, models.shape
        B, k, V, dev = kv.block_table.shape[0], cfg.k, s.vocab, models.device
        self.B, self.k, self.seed, self.seq_offset = B, k, seed, seq_offset
        self.last = torch.randint(0, V, (B,), device=dev, dtype=torch.int64,
                                  generator=torch.Generator(device=dev).manual_seed(seed + 7))
        self.drafts = torch.empty(B, k, dtype=torch.int32, device=dev)
        self.drf = torch.empty(B, k, V, dtype=torch.float32, device=dev)
        self.tgt = torch.empty(B, k + 1, V, dtype=torch.float32, device=dev)
        self.d_lens = torch.empty_like(kv.context_lens)
        self.ok = torch.empty(B, dtype=torch.int32, device=dev)
        self.acc = torch.empty(B, dtype=torch.int32, device=dev)
        self.toks = torch.empty(B, k + 1, dtype=torch.int32, device=dev)
        self.num = torch.empty(B, dtype=torch.int32, device=dev)
        self.tokens_in = torch.empty(B, k + 1, dtype=torch.int64, device=dev)
        from . import _lib
        import ctypes as C
        from .verify import attn_params
        L = _lib.load()

        def attn_ws(nq):
            q = torch.empty(B, nq, s.heads, s.head_dim, dtype=torch.bfloat16, device="meta")
            p = attn_params(q, models.t_k[0], kv.block_table,
                            kv_split_blocks=cfg.kv_split_blocks)
            return torch.empty(max(256, L.kyro_verify_attention_workspace_size(C.byref(p))),
                               dtype=torch.uint8, device=dev)

        self.ws_t, self.ws_d = attn_ws(k + 1), attn_ws(1)
        p = _lib.AcceptParams(B, k, V, _lib.ACCEPT_STOCHASTIC, cfg.temperature, 0, 0, 0)
        self.ws_acc = torch.empty(max(256, L.kyro_spec_accept_workspace_size(C.byref(p))),
                                  dtype=torch.uint8, device=dev)
        sp = _lib.SampleParams(B, 1, V, cfg.temperature, 0, 0, 0, 0)
        self.ws_smp = torch.empty(max(256, L.kyro_sample_workspace_size(C.byref(sp))),
                                  dtype=torch.uint8, device=dev)

    def __call__(self, step: int, timer=None):
        m, kv, cfg, k = self.m, self.kv, self.m.cfg, self.k
        V = m.shape.vocab
        bs = cfg.block_size
        kv_reserve(self.ctx_t, k + 1, kv.block_table, kv.context_lens, kv.free_stack, kv.free_top,
                   kv.ref_counts, bs, out_ok=self.ok)
        # draft loop: draft token i is sampled from the draft's logits at
        # position context_len + i; its Philox counter carries step*k + i
        if timer is not None:
            timer.begin("draft")
        tok = self.last.view(-1, 1)
        for i in range(k):
            torch.add(kv.context_lens, i, out=self.d_lens)
            # the lm_head GEMM writes position i's logits straight into
            # column i of the [B, k, V] draft buffer that acceptance reads
            logits = m.forward(self.ctx_d, m.draft, m.d_k, m.d_v, tok, kv.block_table, self.d_lens,
                               self.ws_d, self.drf[:, i])  # [B, 1, V] fp32, rows k * V apart
            t, _ = sample_tokens(self.ctx_d, logits, cfg.temperature, seed=self.seed,
                                 step=step * k + i, seq_offset=self.seq_offset,
                                 workspace=self.ws_smp)
            self.drafts[:, i] = t[:, 0]
            tok = t.long()
        if timer is not None:
            timer.end("draft")
            timer.begin("target")
        self.tokens_in[:, 0] = self.last
        self.tokens_in[:, 1:] = self.drafts
        m.forward(self.ctx_t, m.target, m.t_k, m.t_v, self.tokens_in, kv.block_table,
                  kv.context_lens, self.ws_t, self.tgt.view(self.B * (k + 1), V), timer=timer)
        if timer is not None:
            timer.end("target")
            timer.begin("accept")
        spec_accept(self.ctx_t, self.tgt, self.drf, self.drafts, temperature=cfg.temperature,
                    seed=self.seed, step=step, seq_offset=self.seq_offset,
                    out=(self.acc, self.toks, self.num, None), workspace=self.ws_acc)
        if timer is not None:
            timer.end("accept")
        kv_commit(self.ctx_t, k + 1, self.acc, kv.block_table, kv.context_lens, kv.free_stack,
                  kv.free_top, kv.ref_counts, bs)
        # the emitted token that ends the accepted run feeds the next step
        self.last.copy_(self.toks.gather(1, self.acc.long().view(-1, 1)).view(-1))

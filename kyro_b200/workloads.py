"""Seeded synthetic workloads with the shapes and value distributions of the
benchmark configurations of the verify step.

The reference publishes no benchmark data for this path, so every input is
synthetic:
  config 0  acceptance only: B=8, k=4, V=32000, fp32; target logits
            z ~ N(0, 3^2), draft logits z + N(0, 1^2), temperature 1.0,
            draft tokens sampled from softmax(draft logits).
  config 1  chain verify attention + accept, Llama-3-8B layer shape:
            Hq=32, Hkv=8, D=128, bf16 KV, block_size 16, B=64,
            context ~ U[512, 4096], k=5 (+1 bonus row), Q/K/V ~ N(0,1),
            block tables from a random permutation of 16384 blocks,
            V=128256 with the config-0 logit distribution.
The generators are deterministic in `seed`.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch


@dataclass
class ChainConfig:
    batch: int = 64
    k: int = 5
    num_heads: int = 32
    num_kv_heads: int = 8
    head_dim: int = 128
    block_size: int = 16
    num_blocks: int = 16384
    ctx_min: int = 512
    ctx_max: int = 4096
    vocab: int = 128256
    temperature: float = 1.0
    logit_std: float = 3.0
    draft_noise: float = 1.0
    # room for growth: the bench commits up to k+1 tokens per step
    headroom_tokens: int = 1024

    @property
    def num_query(self) -> int:
        return self.k + 1

    @property
    def max_blocks_per_seq(self) -> int:
        return -(-(self.ctx_max + self.headroom_tokens) // self.block_size)


CONFIG0 = dict(batch=8, k=4, vocab=32000)
CONFIG1 = ChainConfig()
# Config 2: tree verification, 64 query heads over 8 KV heads, context 8192,
# a 64-node tree (k + 1 = 64 positions), vocabulary 32000.
CONFIG2 = ChainConfig(batch=32, k=63, num_heads=64, num_kv_heads=8, head_dim=128,
                      num_blocks=17408, ctx_min=8192, ctx_max=8192, vocab=32000,
                      temperature=1.0, headroom_tokens=128)

# Config 3: vocabulary-sharded acceptance and KV commit on a 32768-block
# table (the table only: a one-head, 8-wide cache keeps the K/V arrays small;
# contexts U[256, 1800] fit 256 sequences plus growth in the pool).
CONFIG3 = ChainConfig(batch=256, k=8, num_heads=1, num_kv_heads=1, head_dim=8,
                      num_blocks=32768, ctx_min=256, ctx_max=1800, vocab=128256,
                      temperature=0.8, headroom_tokens=128)


def accept_inputs(batch: int, k: int, vocab: int, device, seed: int = 0, std: float = 3.0,
                  noise: float = 1.0):
    """Target logits [B,k+1,V] ~ N(0, std^2) and draft logits = target[:, :k] + N(0, noise^2)."""
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed)
    tgt = torch.randn(batch, k + 1, vocab, generator=g, device=dev) * std
    drf = tgt[:, :k] + torch.randn(batch, k, vocab, generator=g, device=dev) * noise
    return tgt.contiguous(), drf.contiguous()


@dataclass
class PagedState:
    q: torch.Tensor            # bf16 [B, nq, Hq, D]
    k_cache: torch.Tensor      # bf16 [NB, Hkv, bs, D]
    v_cache: torch.Tensor
    block_table: torch.Tensor  # int64 [B, max_blocks]
    context_lens: torch.Tensor  # int64 [B]
    free_stack: torch.Tensor   # int32 [NB]
    free_top: torch.Tensor     # int32 [1]
    ref_counts: torch.Tensor   # int32 [NB]


def paged_state(cfg: ChainConfig, device, seed: int = 0, ctx_lens: Optional[np.ndarray] = None,
                num_query: Optional[int] = None, fill_cache: bool = True) -> PagedState:
    """Paged KV cache and block tables.  The free list is a random
    permutation of the pool; each sequence's context blocks are popped from
    its back in batch order, as BlockManager admits prompts."""
    rng = np.random.default_rng(seed)
    B, bs, NB = cfg.batch, cfg.block_size, cfg.num_blocks
    nq = cfg.num_query if num_query is None else num_query
    if ctx_lens is None:
        ctx_lens = rng.integers(cfg.ctx_min, cfg.ctx_max + 1, size=B)
    ctx_lens = np.asarray(ctx_lens, dtype=np.int64)
    maxb = cfg.max_blocks_per_seq
    free = rng.permutation(NB).astype(np.int32)
    top = NB
    table = np.full((B, maxb), -1, dtype=np.int64)
    refs = np.zeros(NB, dtype=np.int32)
    for b in range(B):
        n = -(-int(ctx_lens[b]) // bs)
        if n > top or n > maxb:
            raise ValueError("KV pool too small for the requested contexts")
        for i in range(n):
            top -= 1
            table[b, i] = free[top]
            refs[free[top]] = 1
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed + 1)
    shape = (NB, cfg.num_kv_heads, bs, cfg.head_dim)
    if fill_cache:
        kc = torch.randn(shape, generator=g, device=dev, dtype=torch.bfloat16)
        vc = torch.randn(shape, generator=g, device=dev, dtype=torch.bfloat16)
    else:
        kc = torch.zeros(shape, dtype=torch.bfloat16, device=dev)
        vc = torch.zeros(shape, dtype=torch.bfloat16, device=dev)
    q = torch.randn(B, nq, cfg.num_heads, cfg.head_dim, generator=g, device=dev,
                    dtype=torch.bfloat16)
    return PagedState(
        q=q, k_cache=kc, v_cache=vc,
        block_table=torch.from_numpy(table).to(device),
        context_lens=torch.from_numpy(ctx_lens).to(device),
        free_stack=torch.from_numpy(free).to(device),
        free_top=torch.tensor([top], dtype=torch.int32, device=device),
        ref_counts=torch.from_numpy(refs).to(device))


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> numpy uint16 bit patterns (for the oracle)."""
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def chain_bytes_per_step(context_lens: np.ndarray, cfg: ChainConfig,
                         separate_rope: bool = False) -> dict:
    """Algorithmic bytes of one verify step, per unit:
      attention: every K and V element of the context plus the k+1 new
                 positions, once per KV head (2 * Hkv * D * 2 bytes per
                 token), plus Q read and O written (bf16);
      accept:    every target (k+1 rows) and draft (k rows) logit once (fp32);
      new_rows:  the store of the k+1 new K/V rows: read and written once
                 (4 * Hkv * D * 2 bytes per new token); with a separate RoPE
                 pass (separate_rope) also the rotated queries written and
                 read back (2 * Hq * D * 2).  RoPE inside the attention
                 launch reads the queries once, as part of attention."""
    toks = int(np.sum(context_lens + cfg.num_query))
    kv = toks * 2 * cfg.num_kv_heads * cfg.head_dim * 2
    qo = 2 * cfg.batch * cfg.num_query * cfg.num_heads * cfg.head_dim * 2
    logits = cfg.batch * (2 * cfg.k + 1) * cfg.vocab * 4
    new = cfg.batch * cfg.num_query * 4 * cfg.num_kv_heads * cfg.head_dim * 2
    if separate_rope:
        new += cfg.batch * cfg.num_query * 2 * cfg.num_heads * cfg.head_dim * 2
    return {"attention": kv + qo, "accept": logits, "new_rows": new,
            "total": kv + qo + logits + new}


def bfs_tree(num_nodes: int = 64, branching=(4, 4, 4)) -> np.ndarray:
    """Parents of a BFS-ordered draft tree: node 0 is the root, each level
    gives every node of the previous level `branching[d]` children, and the
    tree is cut at num_nodes (config 2: 4, 4, 4 cut to 64 = 1 + 4 + 16 + 43)."""
    parents = [-1]
    level = [0]
    for br in branching:
        nxt = []
        for u in level:
            for _ in range(br):
                if len(parents) == num_nodes:
                    break
                parents.append(u)
                nxt.append(len(parents) - 1)
        level = nxt
    return np.asarray(parents[:num_nodes], dtype=np.int32)


def tree_inputs(batch: int, parents: np.ndarray, vocab: int, seed: int = 0,
                std: float = 3.0, noise: float = 1.0, temperature: float = 1.0):
    """Target logits z ~ N(0, std^2) per (seq, node, vocab), draft logits
    z + N(0, noise^2), and node tokens: each child's token sampled from its
    parent's draft distribution softmax(draft / T) (numpy, seeded)."""
    rng = np.random.default_rng(seed)
    N = parents.size
    tgt = (rng.standard_normal((batch, N, vocab)) * std).astype(np.float32)
    drf = (tgt + rng.standard_normal((batch, N, vocab)) * noise).astype(np.float32)
    tok = np.zeros((batch, N), dtype=np.int32)
    for b in range(batch):
        for n in range(1, N):
            z = drf[b, parents[n]].astype(np.float64) / temperature
            q = np.exp(z - z.max())
            tok[b, n] = rng.choice(vocab, p=q / q.sum())
    return tgt, drf, tok


def tree_mask_bits(parents: np.ndarray) -> np.ndarray:
    """uint64-as-int64 ancestor masks: bit i of mask[j] is set iff node i is
    node j or one of its ancestors."""
    N = parents.size
    mask = np.zeros(N, dtype=np.uint64)
    for j in range(N):
        bits = np.uint64(0)
        n = j
        while n >= 0:
            bits |= np.uint64(1) << np.uint64(n)
            n = int(parents[n])
        mask[j] = bits
    return mask.view(np.int64)

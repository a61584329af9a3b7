"""PagedAttention with the reference's constructor and forward signature.

Mirrors ``PagedAttention`` of src/model/attention_kernel.rs:4-31:
``PagedAttention::new(block_size, num_heads, head_dim, num_kv_heads)`` and
``forward(query, key_cache, value_cache, block_table, context_lens)``, with
the layouts documented at :52-57.  The computation runs in the sm_100a
verify-attention kernel (kyro_verify_attention).

Two query layouts are accepted:
  * [B, Hq, D] -- the reference's single-query decode layout.  As in the
    reference, each query attends all context_lens[b] cached positions and a
    sequence with context 0 returns zeros (:77-84).  The result is fp32, the
    reference's output dtype (:114).
  * [B, num_query, Hq, D] -- multi-query verify: query j sits at position
    context_lens[b] + j (its K/V already in the cache) and attends the cached
    positions plus the new positions its mask allows (chain: i <= j; tree:
    bit i of tree_mask[b, j]).  The result is bf16.
"""
from __future__ import annotations

from typing import Optional

import torch

from .verify import Context, verify_attention


class PagedAttention:
    def __init__(self, block_size: int, num_heads: int, head_dim: int, num_kv_heads: int,
                 ctx: Optional[Context] = None):
        if num_heads % num_kv_heads:
            raise ValueError("num_heads must be a multiple of num_kv_heads")
        self.block_size = block_size
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.num_kv_heads = num_kv_heads
        self._ctx = ctx

    def _context(self, device) -> Context:
        if self._ctx is None or self._ctx.device != device:
            self._ctx = Context(device.index)
        return self._ctx

    def forward(self, query: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                block_table: torch.Tensor, context_lens: torch.Tensor,
                tree_mask: Optional[torch.Tensor] = None, kv_split_blocks: int = 0):
        if key_cache.shape[1] != self.num_kv_heads or key_cache.shape[2] != self.block_size:
            raise ValueError("key_cache must be [num_blocks, num_kv_heads, block_size, head_dim]")
        # The paged caches are the big operands: a dtype conversion here
        # would copy the whole cache on every call, so only bf16 caches are
        # taken (the reference's KVCacheManager holds f16,
        # src/model/kv_cache.rs:55-56; convert such a cache once, up front).
        for name, c in (("key_cache", key_cache), ("value_cache", value_cache)):
            if c.dtype != torch.bfloat16:
                raise TypeError(f"{name} must be bfloat16, got {c.dtype} (the verify kernel reads "
                                "bf16 caches; convert the cache once, not per call)")
            if not c.is_contiguous():
                raise ValueError(f"{name} must be contiguous")
        ctx = self._context(query.device)
        # queries are small ([B, n, Hq, D]); they are converted when needed
        q = query.to(torch.bfloat16)
        kc, vc = key_cache, value_cache
        bt = block_table.to(torch.int64).contiguous()
        cl = context_lens.to(torch.int64).contiguous()
        if q.dim() == 3:
            # reference decode layout: the query is the last cached token
            empty = cl <= 0
            cl_q = torch.clamp(cl - 1, min=0)
            out = verify_attention(ctx, q.unsqueeze(1).contiguous(), kc, vc, bt, cl_q,
                                   kv_split_blocks=kv_split_blocks)
            out = out.squeeze(1).float()
            return torch.where(empty[:, None, None], torch.zeros_like(out), out)
        return verify_attention(ctx, q.contiguous(), kc, vc, bt, cl, tree_mask=tree_mask,
                                kv_split_blocks=kv_split_blocks)

    __call__ = forward

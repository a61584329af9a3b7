"""Device-resident BlockManager state for the verify step.

Mirrors ``BlockManager`` (src/scheduler/block_manager.rs:15-30): a block
table, a LIFO free list initialised to 0..num_gpu_blocks and popped from
the back (:36, :92-98), and per-block reference counts (:29).  The state
lives in device tensors so the KV reserve / commit / rollback kernels
(kyro_kv_reserve, kyro_kv_commit, kyro_kv_commit_tree) update it without a
host round trip.
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch

from .verify import Context, kv_commit, kv_commit_tree, kv_reserve


class DeviceBlockManager:
    def __init__(self, block_size: int, num_gpu_blocks: int, max_seqs: int,
                 max_blocks_per_seq: int, device=None, free_order: Optional[torch.Tensor] = None,
                 ctx: Optional[Context] = None):
        self.block_size = block_size
        self.num_gpu_blocks = num_gpu_blocks
        self.ctx = ctx or Context(device)
        dev = self.ctx.device
        order = (torch.arange(num_gpu_blocks, dtype=torch.int32) if free_order is None
                 else free_order.to(torch.int32))
        self.free_stack = order.to(dev).contiguous()
        self.free_top = torch.tensor([num_gpu_blocks], dtype=torch.int32, device=dev)
        self.ref_counts = torch.zeros(num_gpu_blocks, dtype=torch.int32, device=dev)
        self.block_table = torch.full((max_seqs, max_blocks_per_seq), -1, dtype=torch.int64,
                                      device=dev)
        self.context_lens = torch.zeros(max_seqs, dtype=torch.int64, device=dev)

    def num_free_blocks(self) -> int:
        return int(self.free_top.item())

    def reserve(self, num_new: int) -> torch.Tensor:
        """Make room for num_new more tokens in every sequence (allocate,
        block_manager.rs:109-125).  Returns ok [B] (int32)."""
        return kv_reserve(self.ctx, num_new, self.block_table, self.context_lens, self.free_stack,
                          self.free_top, self.ref_counts, self.block_size)

    def commit(self, num_new: int, accept_len: torch.Tensor) -> None:
        """Keep accept_len+1 of the num_new reserved slots and release the
        blocks beyond them (free, block_manager.rs:129-153)."""
        kv_commit(self.ctx, num_new, accept_len.to(torch.int32).contiguous(), self.block_table,
                  self.context_lens, self.free_stack, self.free_top, self.ref_counts,
                  self.block_size)

    def commit_tree(self, num_nodes: int, path: torch.Tensor, path_len: torch.Tensor,
                    k_caches: Sequence[torch.Tensor], v_caches: Sequence[torch.Tensor]) -> None:
        kv_commit_tree(self.ctx, num_nodes, path.to(torch.int32).contiguous(),
                       path_len.to(torch.int32).contiguous(), k_caches, v_caches,
                       self.block_table, self.context_lens, self.free_stack, self.free_top,
                       self.ref_counts, self.block_size)

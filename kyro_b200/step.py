"""The batched verify step: SpeculativeDecoder::step's verify half
(src/speculative.rs:342-353) over a paged KV cache, on the library's kernels.

The reference verifies one sequence at a time: one target forward over the
k draft tokens, then an argmax compare per position with a host sync
(verify_drafts, src/speculative.rs:286-339), and its KV "commit" is a dense
concatenation that never rolls back (append_kv, src/model/kv_cache.rs:49-75).
Here one call runs, for a whole batch and with no host sync, the verify
path of one attention layer and the acceptance that follows the target's
lm_head:

  kv_reserve     k + 1 slots per sequence, popped from the device free list
                 (BlockManager::allocate semantics, block_manager.rs:109-125)
  verify_attention_rope  RoPE of the new queries and keys at context_len + j,
                 the paged store of the new K/V rows (LlamaAttention::forward,
                 src/model/llama.rs:73-82) and the attention of the k + 1
                 query rows against the paged cache, in one launch; or
                 kv_write + verify_attention for rows that are already
                 rotated
  spec_accept    accept lengths and emitted tokens from the target / draft
                 logits (stochastic, greedy, or the reference's greedy rule)
  kv_commit      keep accept_len + 1 slots, release the rest (one call with
                 the acceptance, kyro_spec_accept_commit: the commit runs
                 beside the acceptance's final pass)

In a decode loop the next step's reserve joins the commit (reserve_next):
call the first step with reserve=True, the later ones with reserve=False,
and every step with reserve_next=k+1.

The caller owns the KV state and the inputs; the step owns its outputs and
workspaces, allocated once, so a step can be captured in a CUDA graph and
replayed.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib
from .verify import (ACCEPT_STOCHASTIC, Context, attn_params, kv_reserve, kv_write,
                     rope_kv_write, spec_accept_commit, verify_attention, verify_attention_rope)


def tree_kernel_shape(num_heads: int, num_kv_heads: int, head_dim: int, block_size: int,
                      num_query: int) -> bool:
    """Whether kyro_verify_attention runs this shape on the tcgen05 tree kernel
    (128 query rows per KV head: head_dim 128, block 16, Hq/Hkv dividing 128
    and num_query a multiple of 128 / (Hq/Hkv), at most 64), which the fused
    RoPE entry point does not cover."""
    group = num_heads // num_kv_heads
    if head_dim != 128 or block_size != 16 or group > 128 or 128 % group:
        return False
    npt = 128 // group
    return npt <= num_query <= 64 and num_query % npt == 0


@dataclass
class KVState:
    """The caller's paged KV state: the block table, context lengths, free
    list and ref counts of the BlockManager mirror, and one layer's caches."""
    block_table: torch.Tensor   # int64 [B, max_blocks]
    context_lens: torch.Tensor  # int64 [B]
    free_stack: torch.Tensor    # int32 [num_blocks]
    free_top: torch.Tensor      # int32 [1]
    ref_counts: torch.Tensor    # int32 [num_blocks]
    k_cache: torch.Tensor       # bf16 [num_blocks, Hkv, block_size, D]
    v_cache: torch.Tensor


class VerifyStep:
    """One batched verify step with preallocated outputs and workspaces.

    batch, k, num_heads (Hq), vocab and block_size fix the shapes; the caches
    and block table passed to each call fix the rest.  rope_theta None skips
    the rotary embedding (the new rows are stored as given by kv_write)."""

    def __init__(self, ctx: Context, batch: int, k: int, num_heads: int, kv: KVState,
                 vocab: int, block_size: int, mode: int = ACCEPT_STOCHASTIC,
                 temperature: float = 1.0, seed: int = 0, seq_offset: int = 0,
                 rope_theta: Optional[float] = 10000.0):
        self.ctx, self.B, self.k, self.vocab = ctx, batch, k, vocab
        self.block_size, self.mode, self.temperature = block_size, mode, temperature
        self.seed, self.seq_offset, self.rope_theta = seed, seq_offset, rope_theta
        dev = ctx.device
        nq = k + 1
        d = kv.k_cache.shape[3]
        self.attn_out = torch.empty(batch, nq, num_heads, d, dtype=torch.bfloat16, device=dev)
        # RoPE runs inside the attention launch unless the shape takes the
        # tree kernel (then rope_kv_write writes the rotated queries here)
        self.fused_rope = rope_theta is not None and not tree_kernel_shape(
            num_heads, kv.k_cache.shape[1], d, block_size, nq)
        self.q_rot = (torch.empty_like(self.attn_out)
                      if rope_theta is not None and not self.fused_rope else None)
        self.ok = torch.empty(batch, dtype=torch.int32, device=dev)
        self.acc = torch.empty(batch, dtype=torch.int32, device=dev)
        self.toks = torch.empty(batch, nq, dtype=torch.int32, device=dev)
        self.num = torch.empty(batch, dtype=torch.int32, device=dev)
        L = _lib.load()
        p = attn_params(self.attn_out, kv.k_cache, kv.block_table)
        self.ws_attn = torch.empty(max(256, L.kyro_verify_attention_workspace_size(C.byref(p))),
                                   dtype=torch.uint8, device=dev)
        ap = _lib.AcceptParams(batch, k, vocab, mode, temperature, 0, 0, 0)
        self.ws_acc = torch.empty(max(256, L.kyro_spec_accept_workspace_size(C.byref(ap))),
                                  dtype=torch.uint8, device=dev)

    def __call__(self, kv: KVState, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                 target_logits: torch.Tensor, draft_logits: Optional[torch.Tensor],
                 draft_tokens: torch.Tensor, step: int, events: Optional[dict] = None,
                 reserve: bool = True, reserve_next: int = 0):
        """Run the step on the current stream.  q bf16 [B, k+1, Hq, D]; k_new /
        v_new bf16 [B, k+1, Hkv, D]; logits fp32 [B, k+1, V] / [B, k, V];
        draft_tokens int32 [B, k].  Returns (attention out, ok, accept_len,
        tokens, num_tokens), all owned by the step.  reserve: reserve this
        step's k + 1 slots first (False when the previous step's commit
        reserved them); reserve_next: slots the commit reserves for the next
        step (ok then reports that reserve).  `events`, if given, maps
        "attention" and "accept" to lists that get a (start, end) pair of CUDA
        events around those launches (events between launches break their
        programmatic chaining, so timed steps should pass None)."""
        ctx, bs, nq = self.ctx, self.block_size, self.k + 1

        def mark():
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            return e

        if reserve:
            kv_reserve(ctx, nq, kv.block_table, kv.context_lens, kv.free_stack, kv.free_top,
                       kv.ref_counts, bs, out_ok=self.ok)
        e0 = None
        if self.fused_rope:
            e0 = mark() if events is not None else None
            verify_attention_rope(ctx, q, k_new, v_new, kv.k_cache, kv.v_cache, kv.block_table,
                                  kv.context_lens, theta=self.rope_theta, out=self.attn_out,
                                  workspace=self.ws_attn)
        else:
            if self.rope_theta is not None:
                rope_kv_write(ctx, q, k_new, v_new, kv.block_table, kv.context_lens, kv.k_cache,
                              kv.v_cache, bs, theta=self.rope_theta, q_out=self.q_rot)
                qq = self.q_rot
            else:
                kv_write(ctx, k_new, v_new, kv.block_table, kv.context_lens, kv.k_cache,
                         kv.v_cache, bs)
                qq = q
            e0 = mark() if events is not None else None
            verify_attention(ctx, qq, kv.k_cache, kv.v_cache, kv.block_table, kv.context_lens,
                             out=self.attn_out, workspace=self.ws_attn)
        e1 = mark() if events is not None else None
        spec_accept_commit(ctx, target_logits, draft_logits, draft_tokens, kv.block_table,
                           kv.context_lens, kv.free_stack, kv.free_top, kv.ref_counts, bs,
                           num_new=nq, num_new_next=reserve_next, mode=self.mode,
                           temperature=self.temperature, seed=self.seed, step=step,
                           seq_offset=self.seq_offset, out=(self.acc, self.toks, self.num, None),
                           workspace=self.ws_acc, out_ok=self.ok if reserve_next else None)
        if events is not None:
            e2 = mark()
            events.setdefault("attention", []).append((e0, e1))
            events.setdefault("accept", []).append((e1, e2))
        return self.attn_out, self.ok, self.acc, self.toks, self.num

    def launches(self, reserve: bool = True) -> int:
        """Kernels one call launches: reserve (if asked), the kv write (unless
        RoPE is fused into the attention), attention, the acceptance's stats
        and decide kernels, the commit, and the final kernel (stochastic mode
        only)."""
        from .verify import ACCEPT_STOCHASTIC as S
        return (int(reserve) + int(not self.fused_rope) + 4
                + int(self.mode == S and self.temperature > 0))

"""Host-side operators of the speculative verify step, over the C ABI.

Each function validates its tensors, then calls one entry point of
include/kyro_spec.h through ctypes on the current torch CUDA stream.  torch
supplies device memory and streams only; all computation happens in the
sm_100a kernels of libkyro_spec.so.  There is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional, Sequence

import torch

from . import _lib
from ._lib import (ACCEPT_GREEDY, ACCEPT_GREEDY_REF, ACCEPT_STOCHASTIC, AcceptParams, AttnParams,
                   KVParams, SampleParams, check)

__all__ = [
    "Context", "spec_accept", "spec_accept_commit", "sample_tokens", "verify_attention", "kv_reserve", "kv_commit",
    "kv_commit_tree", "kv_write", "philox_uniforms", "ACCEPT_STOCHASTIC", "ACCEPT_GREEDY", "ACCEPT_GREEDY_REF",
]


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else C.c_void_p(t.data_ptr())


def _need(t: torch.Tensor, name: str, dtype, device, ndim=None):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if t.device != device:
        raise ValueError(f"{name} must be on {device}, got {t.device}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if ndim is not None and t.dim() != ndim:
        raise ValueError(f"{name} must have {ndim} dims, got shape {tuple(t.shape)}")


class Context:
    """One kyro_ctx per GPU: the device, the stream kernels go to, and a
    cached workspace buffer.  Calls enqueue on torch's current stream."""

    def __init__(self, device: Optional[int] = None):
        L = _lib.load()
        if device is None:
            device = torch.cuda.current_device()
        self.device = torch.device("cuda", device)
        self.index = device
        h = C.c_void_p()
        with torch.cuda.device(device):
            stream = torch.cuda.current_stream(device).cuda_stream
            check(L.kyro_ctx_create(device, C.c_void_p(stream), C.byref(h)))
        self._h = h
        self._ws: Optional[torch.Tensor] = None

    @property
    def handle(self):
        return self._h

    def bind_stream(self):
        stream = torch.cuda.current_stream(self.index).cuda_stream
        check(_lib.load().kyro_ctx_set_stream(self._h, C.c_void_p(stream)))

    def workspace(self, nbytes: int) -> torch.Tensor:
        """A caller-owned scratch buffer of at least nbytes (grown on demand)."""
        if nbytes <= 0:
            nbytes = 256
        if self._ws is None or self._ws.numel() < nbytes:
            self._ws = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        return self._ws

    def tp_init(self, unique_id: bytes, rank: int, world: int):
        """Join a tensor-parallel group (kyro_ctx_tp_init); blocks until all
        `world` ranks have joined.  unique_id comes from tp_unique_id() on
        rank 0, passed to the others by the caller's launcher."""
        if len(unique_id) != _lib.TP_UNIQUE_ID_BYTES:
            raise ValueError(f"unique_id must be {_lib.TP_UNIQUE_ID_BYTES} bytes")
        buf = C.create_string_buffer(bytes(unique_id), _lib.TP_UNIQUE_ID_BYTES)
        with torch.cuda.device(self.index):
            check(_lib.load().kyro_ctx_tp_init(self._h, buf, rank, world))
        self.tp_rank, self.tp_world = rank, world

    @property
    def tp_transport(self) -> str:
        """The exchange rounds' transport: "none", "nccl" or "peer" (NVLink
        peer memory)."""
        return ("none", "nccl", "peer")[_lib.load().kyro_ctx_tp_transport(self._h)]

    def set_wait_timeout(self, ms: int):
        """Bound of this context's waits on other ranks (kyro_ctx_set_wait_timeout)."""
        check(_lib.load().kyro_ctx_set_wait_timeout(self._h, int(ms)))

    def inject_skip(self, rounds: int = 1):
        """Fault injection: this rank skips its next `rounds` peer-memory
        exchange rounds (kyro_ctx_tp_inject_skip)."""
        check(_lib.load().kyro_ctx_tp_inject_skip(self._h, int(rounds)))

    def device_status(self, clear: bool = True) -> int:
        flags = C.c_uint32(0)
        check(_lib.load().kyro_ctx_device_status(self._h, C.byref(flags), int(clear)))
        return flags.value

    def close(self):
        if self._h is not None and self._h.value:
            _lib.load().kyro_ctx_destroy(self._h)
        self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def spec_accept(ctx: Context, target_logits: torch.Tensor, draft_logits: Optional[torch.Tensor],
                draft_tokens: torch.Tensor, mode: int = ACCEPT_STOCHASTIC,
                temperature: float = 1.0, seed: int = 0, step: int = 0, seq_offset: int = 0,
                want_probs: bool = False, out=None, workspace: Optional[torch.Tensor] = None):
    """kyro_spec_accept.  target_logits fp32 [B,k+1,V], draft_logits fp32 [B,k,V]
    (stochastic mode), draft_tokens int32 [B,k].

    Returns (accept_len [B], tokens [B,k+1], num_tokens [B], probs [B,k,2] or None).
    """
    dev = ctx.device
    _need(target_logits, "target_logits", torch.float32, dev, 3)
    B, k1, V = target_logits.shape
    k = k1 - 1
    _need(draft_tokens, "draft_tokens", torch.int32, dev)
    if draft_tokens.numel() != B * k:
        raise ValueError(f"draft_tokens must hold B*k = {B * k} entries")
    if draft_logits is not None:
        _need(draft_logits, "draft_logits", torch.float32, dev, 3)
        if tuple(draft_logits.shape) != (B, k, V):
            raise ValueError(f"draft_logits must be {(B, k, V)}, got {tuple(draft_logits.shape)}")
    if out is None:
        acc = torch.empty(B, dtype=torch.int32, device=dev)
        toks = torch.empty(B, k + 1, dtype=torch.int32, device=dev)
        num = torch.empty(B, dtype=torch.int32, device=dev)
        probs = torch.empty(B, k, 2, dtype=torch.float32, device=dev) if want_probs else None
    else:
        acc, toks, num, probs = out
    p = AcceptParams(B, k, V, mode, float(temperature), step & 0xFFFFFFFF,
                     seed & 0xFFFFFFFFFFFFFFFF, seq_offset)
    L = _lib.load()
    need = L.kyro_spec_accept_workspace_size(C.byref(p))
    ws = workspace if workspace is not None else ctx.workspace(need)
    ctx.bind_stream()
    check(L.kyro_spec_accept(ctx.handle, C.byref(p), _ptr(target_logits), _ptr(draft_logits),
                             _ptr(draft_tokens), _ptr(acc), _ptr(toks), _ptr(num), _ptr(probs),
                             _ptr(ws), ws.numel()))
    return acc, toks, num, probs


def spec_accept_commit(ctx: Context, target_logits: torch.Tensor,
                       draft_logits: Optional[torch.Tensor], draft_tokens: torch.Tensor,
                       block_table, context_lens, free_stack, free_top, ref_counts,
                       block_size: int, num_new: int, num_new_next: int = 0,
                       mode: int = ACCEPT_STOCHASTIC, temperature: float = 1.0, seed: int = 0,
                       step: int = 0, seq_offset: int = 0, out=None,
                       workspace: Optional[torch.Tensor] = None, out_ok=None):
    """kyro_spec_accept_commit: the acceptance, then the KV commit of the
    accepted slots (and the reserve of num_new_next slots for the next step)
    in one call; the commit runs beside the acceptance's final pass.
    Returns (accept_len, tokens, num_tokens, probs or None) like spec_accept."""
    dev = ctx.device
    _need(target_logits, "target_logits", torch.float32, dev, 3)
    B, k1, V = target_logits.shape
    k = k1 - 1
    _need(draft_tokens, "draft_tokens", torch.int32, dev)
    if draft_tokens.numel() != B * k:
        raise ValueError(f"draft_tokens must hold B*k = {B * k} entries")
    if draft_logits is not None:
        _need(draft_logits, "draft_logits", torch.float32, dev, 3)
        if tuple(draft_logits.shape) != (B, k, V):
            raise ValueError(f"draft_logits must be {(B, k, V)}, got {tuple(draft_logits.shape)}")
    _check_kv_state(ctx, block_table, context_lens, free_stack, free_top, ref_counts)
    if block_table.shape[0] != B:
        raise ValueError("block_table batch differs from the logits' batch")
    if out is None:
        out = (torch.empty(B, dtype=torch.int32, device=dev),
               torch.empty(B, k + 1, dtype=torch.int32, device=dev),
               torch.empty(B, dtype=torch.int32, device=dev), None)
    acc, toks, num, probs = out
    p = AcceptParams(B, k, V, mode, float(temperature), step & 0xFFFFFFFF,
                     seed & 0xFFFFFFFFFFFFFFFF, seq_offset)
    kvp = _kv_params(block_table, block_size, ref_counts.numel())
    L = _lib.load()
    need = L.kyro_spec_accept_workspace_size(C.byref(p))
    ws = workspace if workspace is not None else ctx.workspace(need)
    ctx.bind_stream()
    check(L.kyro_spec_accept_commit(ctx.handle, C.byref(p), _ptr(target_logits),
                                    _ptr(draft_logits), _ptr(draft_tokens), _ptr(acc), _ptr(toks),
                                    _ptr(num), _ptr(probs), _ptr(ws), ws.numel(), C.byref(kvp),
                                    int(num_new), int(num_new_next), _ptr(block_table),
                                    _ptr(context_lens), _ptr(free_stack), _ptr(free_top),
                                    _ptr(ref_counts), _ptr(out_ok)))
    return acc, toks, num, probs


def spec_accept_tree(ctx: Context, target_logits: torch.Tensor,
                     draft_logits: Optional[torch.Tensor], node_tokens: torch.Tensor,
                     parents: torch.Tensor, mode: int = ACCEPT_STOCHASTIC,
                     temperature: float = 1.0, seed: int = 0, step: int = 0,
                     seq_offset: int = 0):
    """kyro_spec_accept_tree.  target/draft logits fp32 [B,N,V]; node_tokens
    and parents int32 [B,N] (BFS order, parents[:,0] == -1).  Returns
    (path [B,N], path_len [B], tokens [B,N], num_tokens [B])."""
    from ._lib import TreeParams
    dev = ctx.device
    _need(target_logits, "target_logits", torch.float32, dev, 3)
    B, N, V = target_logits.shape
    _need(node_tokens, "node_tokens", torch.int32, dev, 2)
    _need(parents, "parents", torch.int32, dev, 2)
    if draft_logits is not None:
        _need(draft_logits, "draft_logits", torch.float32, dev, 3)
    path = torch.empty(B, N, dtype=torch.int32, device=dev)
    plen = torch.empty(B, dtype=torch.int32, device=dev)
    toks = torch.empty(B, N, dtype=torch.int32, device=dev)
    num = torch.empty(B, dtype=torch.int32, device=dev)
    p = TreeParams(B, N, V, mode, float(temperature), step & 0xFFFFFFFF,
                   seed & 0xFFFFFFFFFFFFFFFF, seq_offset)
    L = _lib.load()
    ws = ctx.workspace(L.kyro_spec_accept_tree_workspace_size(C.byref(p)))
    ctx.bind_stream()
    check(L.kyro_spec_accept_tree(ctx.handle, C.byref(p), _ptr(target_logits), _ptr(draft_logits),
                                  _ptr(node_tokens), _ptr(parents), _ptr(path), _ptr(plen),
                                  _ptr(toks), _ptr(num), _ptr(ws), ws.numel()))
    return path, plen, toks, num


def tp_unique_id() -> bytes:
    """An NCCL unique id for kyro_ctx_tp_init (call on rank 0)."""
    buf = C.create_string_buffer(_lib.TP_UNIQUE_ID_BYTES)
    check(_lib.load().kyro_tp_unique_id(buf))
    return buf.raw


def spec_accept_tp(ctx: Context, target_shard: torch.Tensor, draft_shard: Optional[torch.Tensor],
                   draft_tokens: torch.Tensor, vocab: int, mode: int = ACCEPT_STOCHASTIC,
                   temperature: float = 1.0, seed: int = 0, step: int = 0, seq_offset: int = 0,
                   want_probs: bool = False):
    """kyro_spec_accept_tp: this rank's vocabulary columns, target_shard fp32
    [B,k+1,V/R] and draft_shard fp32 [B,k,V/R]; draft_tokens int32 [B,k]
    hold global ids; vocab is the full V.  Every rank returns the same
    (accept_len [B], tokens [B,k+1], num_tokens [B], probs [B,k,2] or None)."""
    dev = ctx.device
    _need(target_shard, "target_shard", torch.float32, dev, 3)
    B, k1, _ = target_shard.shape
    k = k1 - 1
    _need(draft_tokens, "draft_tokens", torch.int32, dev)
    if draft_shard is not None:
        _need(draft_shard, "draft_shard", torch.float32, dev, 3)
    acc = torch.empty(B, dtype=torch.int32, device=dev)
    toks = torch.empty(B, k + 1, dtype=torch.int32, device=dev)
    num = torch.empty(B, dtype=torch.int32, device=dev)
    probs = torch.empty(B, k, 2, dtype=torch.float32, device=dev) if want_probs else None
    p = AcceptParams(B, k, vocab, mode, float(temperature), step & 0xFFFFFFFF,
                     seed & 0xFFFFFFFFFFFFFFFF, seq_offset)
    L = _lib.load()
    world = getattr(ctx, "tp_world", 1)
    need = L.kyro_spec_accept_tp_workspace_size(C.byref(p), world)
    if need == 0:
        raise ValueError(f"vocab {vocab} does not split over {world} ranks")
    ws = ctx.workspace(need)
    ctx.bind_stream()
    check(L.kyro_spec_accept_tp(ctx.handle, C.byref(p), _ptr(target_shard), _ptr(draft_shard),
                                _ptr(draft_tokens), _ptr(acc), _ptr(toks), _ptr(num),
                                _ptr(probs), _ptr(ws), ws.numel()))
    return acc, toks, num, probs


def sample_tokens(ctx: Context, logits: torch.Tensor, temperature: float, seed: int = 0,
                  step: int = 0, seq_offset: int = 0, workspace: Optional[torch.Tensor] = None):
    """kyro_sample_tokens.  logits fp32 [B,P,V] -> (tokens int32 [B,P], probs fp32 [B,P]).

    The rows of one sequence must be dense ([P, V] contiguous), but the
    sequences may sit further apart: logits[:, i:i+1] of a [B, k, V] buffer
    is taken as it is (seq_stride k), without a copy."""
    dev = ctx.device
    if not isinstance(logits, torch.Tensor):
        raise TypeError("logits must be a torch.Tensor")
    if logits.dim() != 3:
        raise ValueError(f"logits must have 3 dims, got shape {tuple(logits.shape)}")
    B, P, V = logits.shape
    st = logits.stride()
    seq_stride = 0
    if not logits.is_contiguous():
        if st[2] != 1 or (P > 1 and st[1] != V) or st[0] % V or st[0] // V < P:
            raise ValueError("logits rows must be dense within a sequence "
                             f"(strides {st} for shape {tuple(logits.shape)})")
        seq_stride = st[0] // V
    if logits.dtype != torch.float32 or logits.device != dev:
        raise TypeError(f"logits must be float32 on {dev}")
    toks = torch.empty(B, P, dtype=torch.int32, device=dev)
    probs = torch.empty(B, P, dtype=torch.float32, device=dev)
    p = SampleParams(B, P, V, float(temperature), step & 0xFFFFFFFF, seq_stride,
                     seed & 0xFFFFFFFFFFFFFFFF, seq_offset)
    L = _lib.load()
    need = L.kyro_sample_workspace_size(C.byref(p))
    ws = workspace if workspace is not None else ctx.workspace(need)
    ctx.bind_stream()
    check(L.kyro_sample_tokens(ctx.handle, C.byref(p), _ptr(logits), _ptr(toks), _ptr(probs),
                               _ptr(ws), ws.numel()))
    return toks, probs


def attn_params(q: torch.Tensor, k_cache: torch.Tensor, block_table: torch.Tensor,
                scale: Optional[float] = None, kv_split_blocks: int = 0) -> AttnParams:
    B, nq, hq, d = q.shape
    nb, hkv, bs, d2 = k_cache.shape
    return AttnParams(B, nq, hq, hkv, d, bs, block_table.shape[1], nb,
                      float(scale) if scale else 0.0, kv_split_blocks)


def verify_attention(ctx: Context, q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                     block_table: torch.Tensor, context_lens: torch.Tensor,
                     tree_mask: Optional[torch.Tensor] = None, scale: Optional[float] = None,
                     kv_split_blocks: int = 0, out: Optional[torch.Tensor] = None,
                     workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """kyro_verify_attention.  q bf16 [B,nq,Hq,D]; caches bf16 [NB,Hkv,bs,D];
    block_table int64 [B,max_blocks]; context_lens int64 [B]; tree_mask
    int64/uint64 [B,nq] or None (chain).  Returns bf16 [B,nq,Hq,D]."""
    dev = ctx.device
    _need(q, "q", torch.bfloat16, dev, 4)
    _need(k_cache, "k_cache", torch.bfloat16, dev, 4)
    _need(v_cache, "v_cache", torch.bfloat16, dev, 4)
    if k_cache.shape != v_cache.shape:
        raise ValueError("k_cache and v_cache shapes differ")
    _need(block_table, "block_table", torch.int64, dev, 2)
    _need(context_lens, "context_lens", torch.int64, dev, 1)
    B = q.shape[0]
    if block_table.shape[0] != B or context_lens.shape[0] != B:
        raise ValueError("block_table / context_lens batch mismatch")
    if tree_mask is not None:
        if tree_mask.dtype not in (torch.int64, torch.uint64):
            raise TypeError("tree_mask must be int64 or uint64")
        _need(tree_mask, "tree_mask", tree_mask.dtype, dev, 2)
    p = attn_params(q, k_cache, block_table, scale, kv_split_blocks)
    if out is None:
        out = torch.empty_like(q)
    L = _lib.load()
    need = L.kyro_verify_attention_workspace_size(C.byref(p))
    ws = workspace if workspace is not None else ctx.workspace(need)
    ctx.bind_stream()
    check(L.kyro_verify_attention(ctx.handle, C.byref(p), _ptr(q), _ptr(k_cache), _ptr(v_cache),
                                  _ptr(block_table), _ptr(context_lens), _ptr(tree_mask),
                                  _ptr(out), _ptr(ws), ws.numel()))
    return out


def verify_attention_rope(ctx: Context, q: torch.Tensor, k_new: torch.Tensor,
                          v_new: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                          block_table: torch.Tensor, context_lens: torch.Tensor,
                          theta: float = 10000.0, pos_offsets: Optional[torch.Tensor] = None,
                          tree_mask: Optional[torch.Tensor] = None, scale: Optional[float] = None,
                          kv_split_blocks: int = 0, out: Optional[torch.Tensor] = None,
                          workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """kyro_verify_attention_rope: the rotary embedding of q and k_new (bf16
    [B, nq, Hq or Hkv, D], unrotated), the store of the rotated keys and of
    v_new into the paged slots context_lens[b] + j, and the verify attention,
    in one launch.  Same result as rope_kv_write then verify_attention."""
    dev = ctx.device
    _need(q, "q", torch.bfloat16, dev, 4)
    _need(k_new, "k_new", torch.bfloat16, dev, 4)
    _need(v_new, "v_new", torch.bfloat16, dev, 4)
    _need(k_cache, "k_cache", torch.bfloat16, dev, 4)
    _need(v_cache, "v_cache", torch.bfloat16, dev, 4)
    if k_cache.shape != v_cache.shape:
        raise ValueError("k_cache and v_cache shapes differ")
    _need(block_table, "block_table", torch.int64, dev, 2)
    _need(context_lens, "context_lens", torch.int64, dev, 1)
    B, n, hq, d = q.shape
    hkv = k_cache.shape[1]
    if (tuple(k_new.shape) != (B, n, hkv, d) or tuple(v_new.shape) != (B, n, hkv, d)
            or k_cache.shape[3] != d):
        raise ValueError("q / k_new / v_new / cache shapes disagree")
    if block_table.shape[0] != B or context_lens.shape[0] != B:
        raise ValueError("block_table / context_lens batch mismatch")
    if pos_offsets is not None:
        _need(pos_offsets, "pos_offsets", torch.int32, dev, 1)
        if pos_offsets.numel() != n:
            raise ValueError("pos_offsets needs one entry per new token")
    if tree_mask is not None:
        if tree_mask.dtype not in (torch.int64, torch.uint64):
            raise TypeError("tree_mask must be int64 or uint64")
        _need(tree_mask, "tree_mask", tree_mask.dtype, dev, 2)
    p = attn_params(q, k_cache, block_table, scale, kv_split_blocks)
    if out is None:
        out = torch.empty_like(q)
    L = _lib.load()
    need = L.kyro_verify_attention_workspace_size(C.byref(p))
    ws = workspace if workspace is not None else ctx.workspace(need)
    ctx.bind_stream()
    check(L.kyro_verify_attention_rope(
        ctx.handle, C.byref(p), float(theta), _ptr(pos_offsets), _ptr(q), _ptr(k_new),
        _ptr(v_new), _ptr(k_cache), _ptr(v_cache), _ptr(block_table), _ptr(context_lens),
        _ptr(tree_mask), _ptr(out), _ptr(ws), ws.numel()))
    return out


def _kv_params(block_table: torch.Tensor, block_size: int, num_blocks: int) -> KVParams:
    return KVParams(block_table.shape[0], block_size, block_table.shape[1], num_blocks)


def _check_kv_state(ctx, block_table, context_lens, free_stack, free_top, ref_counts):
    dev = ctx.device
    _need(block_table, "block_table", torch.int64, dev, 2)
    _need(context_lens, "context_lens", torch.int64, dev, 1)
    _need(free_stack, "free_stack", torch.int32, dev, 1)
    _need(free_top, "free_top", torch.int32, dev)
    _need(ref_counts, "ref_counts", torch.int32, dev, 1)
    if free_stack.numel() != ref_counts.numel():
        raise ValueError("free_stack and ref_counts must both hold num_blocks entries")


def kv_reserve(ctx: Context, num_new: int, block_table, context_lens, free_stack, free_top,
               ref_counts, block_size: int, out_ok: Optional[torch.Tensor] = None):
    """kyro_kv_reserve (in place).  Returns out_ok int32 [B]."""
    _check_kv_state(ctx, block_table, context_lens, free_stack, free_top, ref_counts)
    if out_ok is None:
        out_ok = torch.empty(block_table.shape[0], dtype=torch.int32, device=ctx.device)
    p = _kv_params(block_table, block_size, ref_counts.numel())
    ctx.bind_stream()
    check(_lib.load().kyro_kv_reserve(ctx.handle, C.byref(p), num_new, _ptr(block_table),
                                      _ptr(context_lens), _ptr(free_stack), _ptr(free_top),
                                      _ptr(ref_counts), _ptr(out_ok)))
    return out_ok


def kv_commit(ctx: Context, num_new: int, accept_len: torch.Tensor, block_table, context_lens,
              free_stack, free_top, ref_counts, block_size: int):
    """kyro_kv_commit (in place)."""
    _check_kv_state(ctx, block_table, context_lens, free_stack, free_top, ref_counts)
    _need(accept_len, "accept_len", torch.int32, ctx.device, 1)
    p = _kv_params(block_table, block_size, ref_counts.numel())
    ctx.bind_stream()
    check(_lib.load().kyro_kv_commit(ctx.handle, C.byref(p), num_new, _ptr(accept_len),
                                     _ptr(block_table), _ptr(context_lens), _ptr(free_stack),
                                     _ptr(free_top), _ptr(ref_counts)))


def kv_commit_tree(ctx: Context, num_nodes: int, path: torch.Tensor, path_len: torch.Tensor,
                   k_caches: Sequence[torch.Tensor], v_caches: Sequence[torch.Tensor],
                   block_table, context_lens, free_stack, free_top, ref_counts, block_size: int):
    """kyro_kv_commit_tree (in place): move the accepted path's K/V rows in
    every layer's cache, then commit path_len slots."""
    _check_kv_state(ctx, block_table, context_lens, free_stack, free_top, ref_counts)
    _need(path, "path", torch.int32, ctx.device, 2)
    _need(path_len, "path_len", torch.int32, ctx.device, 1)
    if len(k_caches) != len(v_caches):
        raise ValueError("k_caches and v_caches differ in length")
    for c in list(k_caches) + list(v_caches):
        _need(c, "cache", torch.bfloat16, ctx.device, 4)
    nl = len(k_caches)
    kp = (C.c_void_p * max(nl, 1))(*[c.data_ptr() for c in k_caches])
    vp = (C.c_void_p * max(nl, 1))(*[c.data_ptr() for c in v_caches])
    hkv = k_caches[0].shape[1] if nl else 1
    d = k_caches[0].shape[3] if nl else 8
    p = _kv_params(block_table, block_size, ref_counts.numel())
    ctx.bind_stream()
    check(_lib.load().kyro_kv_commit_tree(ctx.handle, C.byref(p), num_nodes, _ptr(path),
                                          _ptr(path_len), nl, C.cast(kp, C.c_void_p),
                                          C.cast(vp, C.c_void_p), hkv, d, _ptr(block_table),
                                          _ptr(context_lens), _ptr(free_stack), _ptr(free_top),
                                          _ptr(ref_counts)))


def kv_reserve_cow(ctx: Context, num_new: int, k_caches: Sequence[torch.Tensor],
                   v_caches: Sequence[torch.Tensor], block_table, context_lens, free_stack,
                   free_top, ref_counts, block_size: int):
    """kyro_kv_reserve_cow (in place): kv_reserve, except that a sequence whose
    last block is partly filled and shared gets a private copy of it first
    (every layer's K/V).  Returns (ok [B] int32, cow [B, 2] int32: the
    (shared, fresh) block pair or -1)."""
    _check_kv_state(ctx, block_table, context_lens, free_stack, free_top, ref_counts)
    if len(k_caches) != len(v_caches):
        raise ValueError("k_caches and v_caches differ in length")
    for c in list(k_caches) + list(v_caches):
        _need(c, "cache", torch.bfloat16, ctx.device, 4)
    nl = len(k_caches)
    kp = (C.c_void_p * max(nl, 1))(*[c.data_ptr() for c in k_caches])
    vp = (C.c_void_p * max(nl, 1))(*[c.data_ptr() for c in v_caches])
    hkv = k_caches[0].shape[1] if nl else 1
    d = k_caches[0].shape[3] if nl else 8
    B = block_table.shape[0]
    ok = torch.empty(B, dtype=torch.int32, device=ctx.device)
    cow = torch.empty(B, 2, dtype=torch.int32, device=ctx.device)
    p = _kv_params(block_table, block_size, ref_counts.numel())
    ctx.bind_stream()
    check(_lib.load().kyro_kv_reserve_cow(ctx.handle, C.byref(p), num_new, nl,
                                          C.cast(kp, C.c_void_p), C.cast(vp, C.c_void_p), hkv, d,
                                          _ptr(block_table), _ptr(context_lens), _ptr(free_stack),
                                          _ptr(free_top), _ptr(ref_counts), _ptr(ok), _ptr(cow)))
    return ok, cow


def kv_write(ctx: Context, k_new: torch.Tensor, v_new: torch.Tensor, block_table, context_lens,
             k_cache: torch.Tensor, v_cache: torch.Tensor, block_size: int):
    """kyro_kv_write: k_new / v_new bf16 [B, num_new, Hkv, D] into the paged
    slots at context_lens[b] + j."""
    dev = ctx.device
    _need(k_new, "k_new", torch.bfloat16, dev, 4)
    _need(v_new, "v_new", torch.bfloat16, dev, 4)
    _need(k_cache, "k_cache", torch.bfloat16, dev, 4)
    _need(v_cache, "v_cache", torch.bfloat16, dev, 4)
    _need(block_table, "block_table", torch.int64, dev, 2)
    _need(context_lens, "context_lens", torch.int64, dev, 1)
    B, n, hkv, d = k_new.shape
    if tuple(v_new.shape) != (B, n, hkv, d) or k_cache.shape[1] != hkv or k_cache.shape[3] != d:
        raise ValueError("k_new / v_new / cache shapes disagree")
    p = _kv_params(block_table, block_size, k_cache.shape[0])
    ctx.bind_stream()
    check(_lib.load().kyro_kv_write(ctx.handle, C.byref(p), n, hkv, d, _ptr(k_new), _ptr(v_new),
                                    _ptr(block_table), _ptr(context_lens), _ptr(k_cache),
                                    _ptr(v_cache)))


def rope_kv_write(ctx: Context, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                  block_table, context_lens, k_cache: torch.Tensor, v_cache: torch.Tensor,
                  block_size: int, theta: float = 10000.0, pos_offsets=None,
                  q_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """kyro_rope_kv_write: rotary embedding of q [B, n, Hq, D] and k_new
    [B, n, Hkv, D] (bf16) at positions context_lens[b] + pos_offsets[j]
    (default j), rotated keys and the values into the paged slots
    context_lens[b] + j, rotated queries into q_out (default a new tensor;
    q itself is allowed)."""
    dev = ctx.device
    _need(q, "q", torch.bfloat16, dev, 4)
    _need(k_new, "k_new", torch.bfloat16, dev, 4)
    _need(v_new, "v_new", torch.bfloat16, dev, 4)
    _need(k_cache, "k_cache", torch.bfloat16, dev, 4)
    _need(v_cache, "v_cache", torch.bfloat16, dev, 4)
    _need(block_table, "block_table", torch.int64, dev, 2)
    _need(context_lens, "context_lens", torch.int64, dev, 1)
    B, n, hq, d = q.shape
    hkv = k_new.shape[2]
    if (tuple(k_new.shape) != (B, n, hkv, d) or tuple(v_new.shape) != (B, n, hkv, d)
            or k_cache.shape[1] != hkv or k_cache.shape[3] != d):
        raise ValueError("q / k_new / v_new / cache shapes disagree")
    if q_out is None:
        q_out = torch.empty_like(q)
    _need(q_out, "q_out", torch.bfloat16, dev, 4)
    if tuple(q_out.shape) != tuple(q.shape):
        raise ValueError("q_out shape disagrees with q")
    if pos_offsets is not None:
        _need(pos_offsets, "pos_offsets", torch.int32, dev, 1)
        if pos_offsets.numel() != n:
            raise ValueError("pos_offsets needs one entry per new token")
    p = _kv_params(block_table, block_size, k_cache.shape[0])
    ctx.bind_stream()
    check(_lib.load().kyro_rope_kv_write(
        ctx.handle, C.byref(p), n, hq, hkv, d, float(theta),
        None if pos_offsets is None else _ptr(pos_offsets), _ptr(q), _ptr(k_new), _ptr(v_new),
        _ptr(block_table), _ptr(context_lens), _ptr(q_out), _ptr(k_cache), _ptr(v_cache)))
    return q_out


def philox_uniforms(ctx: Context, seed: int, seq: int, pos0: int, stream: int, step: int,
                    n: int) -> torch.Tensor:
    out = torch.empty(n, dtype=torch.float32, device=ctx.device)
    ctx.bind_stream()
    check(_lib.load().kyro_philox_uniforms(ctx.handle, seed, seq, pos0, stream, step, n,
                                           _ptr(out)))
    return out


def selftest_exp(ctx: Context) -> tuple:
    """Mismatch counts of the kernels' two fast ky_exp forms against the
    contract's ky_exp over every fp32 input in [-100, 0] (both 0 when the
    kernels compute the contract's bits)."""
    counts = torch.zeros(2, dtype=torch.int64, device=ctx.device)
    ctx.bind_stream()
    check(_lib.load().kyro_selftest_exp(ctx.handle, _ptr(counts)))
    c = counts.cpu()
    return int(c[0]), int(c[1])

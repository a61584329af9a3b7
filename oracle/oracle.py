"""ctypes bindings to the CPU oracle (oracle/libkyro_oracle.so).

TEST INFRASTRUCTURE ONLY: the oracle checks the sm_100a kernels.  Only
tests/, __graft_entry__.smoke() and bench.py (cpu_baseline and
``--impl reference``) load it; the kyro_b200 package never does.

Each function takes and returns numpy arrays and mirrors one C entry point
of kyro_oracle.h; see that header for the reference lines each follows.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libkyro_oracle.so")
_lib = None

MODE_STOCHASTIC = 0
MODE_GREEDY = 1
MODE_GREEDY_REF = 2


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile; returns the library path."""
    if force or not os.path.exists(_LIB_PATH):
        subprocess.run(["make", "-s", "-C", _HERE] + (["-B"] if force else []), check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = C.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


def _p(a):
    return a.ctypes.data_as(C.c_void_p) if a is not None else None


def _declare(L):
    i32, i64, u32, u64, f32, vp = C.c_int32, C.c_int64, C.c_uint32, C.c_uint64, C.c_float, C.c_void_p
    L.ko_philox4x32_10.argtypes = [vp, u64, vp]
    L.ko_uniform.argtypes = [u64, u32, u32, u32, u32]
    L.ko_uniform.restype = f32
    L.ko_exp.argtypes = [f32]
    L.ko_exp.restype = f32
    L.ko_softmax_row.argtypes = [vp, i32, i32, f32, vp]
    L.ko_sample_tokens.argtypes = [i32, i32, i32, f32, u64, u32, i64, vp, vp, vp, i32]
    L.ko_spec_accept.argtypes = [i32, i32, i32, i32, f32, u64, u32, i64, i32, vp, vp, vp, vp, vp,
                                 vp, vp, i32]
    L.ko_spec_accept_tree.argtypes = [i32, i32, i32, i32, f32, u64, u32, i64, vp, vp, vp, vp, vp,
                                      vp, vp, vp, i32]
    f64 = C.c_double
    L.ko_tp_row_max.argtypes = [vp, i32, f32]
    L.ko_tp_row_max.restype = f32
    L.ko_tp_row_sum_part.argtypes = [vp, i32, f32, f32]
    L.ko_tp_row_sum_part.restype = f64
    L.ko_tp_entry.argtypes = [vp, i32, f32, i32, vp, vp]
    L.ko_tp_weight_totals.argtypes = [vp, vp, i32, f32, f32, f64, f32, f64, vp, vp]
    L.ko_tp_cut.argtypes = [vp, vp, i32, f32, f32, f64, f32, f64, i32, u64]
    L.ko_tp_cut.restype = i32
    L.ko_paged_attention.argtypes = [i32, i32, i32, i32, i32, i32, i32, f32, vp, vp, vp, vp, vp,
                                     vp, vp, i32]
    L.ko_kv_reserve.argtypes = [i32, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp]
    L.ko_kv_reserve_cow.argtypes = [i32, i32, i32, i32, i32, i32, vp, vp, i32, i32, vp, vp, vp,
                                    vp, vp, vp, vp]
    L.ko_kv_commit.argtypes = [i32, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp]
    L.ko_kv_write.argtypes = [i32, i32, i32, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp]
    L.ko_rope_kv_write.argtypes = [i32, i32, i32, i32, i32, i32, i32, i32, f32, vp, vp, vp, vp,
                                   vp, vp, vp, vp, vp]
    L.ko_kv_commit_tree.argtypes = [i32, i32, i32, i32, i32, vp, vp, i32, vp, vp, i32, i32, vp,
                                    vp, vp, vp, vp]


def philox4x32_10(ctr, key: int) -> np.ndarray:
    c = np.ascontiguousarray(ctr, dtype=np.uint32)
    out = np.zeros(4, dtype=np.uint32)
    lib().ko_philox4x32_10(_p(c), key, _p(out))
    return out


def uniform(seed: int, seq: int, pos: int, stream: int, step: int) -> float:
    return lib().ko_uniform(seed, seq, pos, stream, step)


def exp(x: float) -> float:
    return lib().ko_exp(x)


def softmax_row(row: np.ndarray, temperature: float = 1.0, num_shards: int = 1) -> np.ndarray:
    r = np.ascontiguousarray(row, dtype=np.float32)
    out = np.empty_like(r)
    lib().ko_softmax_row(_p(r), r.size, num_shards, temperature, _p(out))
    return out


def sample_tokens(logits: np.ndarray, temperature: float, seed: int, step: int = 0,
                  seq_offset: int = 0, nthreads: int = 1):
    """logits [B, P, V] -> (tokens [B, P] int32, probs [B, P] float32)."""
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    B, P, V = lg.shape
    toks = np.empty((B, P), dtype=np.int32)
    probs = np.empty((B, P), dtype=np.float32)
    lib().ko_sample_tokens(B, P, V, temperature, seed, step, seq_offset, _p(lg), _p(toks),
                           _p(probs), nthreads)
    return toks, probs


def spec_accept(target_logits, draft_logits, draft_tokens, mode=MODE_STOCHASTIC,
                temperature=1.0, seed=0, step=0, seq_offset=0, num_shards=1, nthreads=1):
    """Chain acceptance; returns (accept_len [B], tokens [B,k+1], num_tokens [B], probs [B,k,2])."""
    tg = np.ascontiguousarray(target_logits, dtype=np.float32)
    B, k1, V = tg.shape
    k = k1 - 1
    dr = None if draft_logits is None else np.ascontiguousarray(draft_logits, dtype=np.float32)
    dt = np.ascontiguousarray(draft_tokens, dtype=np.int32).reshape(B, k)
    acc = np.empty(B, dtype=np.int32)
    toks = np.empty((B, k + 1), dtype=np.int32)
    num = np.empty(B, dtype=np.int32)
    probs = np.zeros((B, k, 2), dtype=np.float32)
    lib().ko_spec_accept(B, k, V, mode, temperature, seed, step, seq_offset, num_shards, _p(tg),
                         _p(dr), _p(dt), _p(acc), _p(toks), _p(num), _p(probs), nthreads)
    return acc, toks, num, probs


def spec_accept_tree(target_logits, draft_logits, node_tokens, parents, mode=MODE_STOCHASTIC,
                     temperature=1.0, seed=0, step=0, seq_offset=0, nthreads=1):
    """Tree acceptance; target/draft logits [B, N, V] fp32, node_tokens and
    parents [B, N] int32.  Returns (path [B,N], path_len [B], tokens [B,N],
    num_tokens [B])."""
    tg = np.ascontiguousarray(target_logits, dtype=np.float32)
    B, N, V = tg.shape
    dr = None if draft_logits is None else np.ascontiguousarray(draft_logits, dtype=np.float32)
    nt = np.ascontiguousarray(node_tokens, dtype=np.int32).reshape(B, N)
    pa = np.ascontiguousarray(parents, dtype=np.int32).reshape(B, N)
    path = np.empty((B, N), dtype=np.int32)
    plen = np.empty(B, dtype=np.int32)
    toks = np.empty((B, N), dtype=np.int32)
    num = np.empty(B, dtype=np.int32)
    lib().ko_spec_accept_tree(B, N, V, mode, temperature, seed, step, seq_offset, _p(tg), _p(dr),
                              _p(nt), _p(pa), _p(path), _p(plen), _p(toks), _p(num), nthreads)
    return path, plen, toks, num


# ---- one rank's pieces of a vocabulary-sharded row (test infrastructure for
# the tensor-parallel exchange; rank order combination happens in the caller)

def _f32row(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def tp_row_max(shard, temperature: float) -> float:
    r = _f32row(shard)
    return float(lib().ko_tp_row_max(_p(r), r.size, temperature))


def tp_row_sum_part(shard, temperature: float, M: float) -> float:
    r = _f32row(shard)
    return float(lib().ko_tp_row_sum_part(_p(r), r.size, temperature, M))


def tp_entry(shard, temperature: float, idx: int):
    r = _f32row(shard)
    e, m = C.c_float(), C.c_float()
    lib().ko_tp_entry(_p(r), r.size, temperature, idx, C.byref(e), C.byref(m))
    return e.value, m.value


def tp_weight_totals(p_shard, q_shard, temperature, Mp, Sp, Mq, Sq):
    p = _f32row(p_shard)
    q = None if q_shard is None else _f32row(q_shard)
    a, b = C.c_uint64(), C.c_uint64()
    lib().ko_tp_weight_totals(_p(p), _p(q), p.size, temperature, Mp, Sp, Mq, Sq, C.byref(a),
                              C.byref(b))
    return a.value, b.value


def tp_cut(p_shard, q_shard, temperature, Mp, Sp, Mq, Sq, residual: bool, T: int) -> int:
    p = _f32row(p_shard)
    q = None if q_shard is None else _f32row(q_shard)
    return int(lib().ko_tp_cut(_p(p), _p(q), p.size, temperature, Mp, Sp, Mq, Sq, int(residual),
                               T))


def paged_attention(q_bits, k_bits, v_bits, block_table, context_lens, block_size, scale=None,
                    tree_mask=None, nthreads=1):
    """q_bits [B,nq,Hq,D] uint16 (bf16 bits); caches [NB,Hkv,bs,D] uint16 -> fp32 [B,nq,Hq,D]."""
    q = np.ascontiguousarray(q_bits, dtype=np.uint16)
    kc = np.ascontiguousarray(k_bits, dtype=np.uint16)
    vc = np.ascontiguousarray(v_bits, dtype=np.uint16)
    bt = np.ascontiguousarray(block_table, dtype=np.int64)
    cl = np.ascontiguousarray(context_lens, dtype=np.int64)
    tm = None if tree_mask is None else np.ascontiguousarray(tree_mask, dtype=np.uint64)
    B, nq, hq, d = q.shape
    hkv = kc.shape[1]
    if scale is None:
        scale = 1.0 / np.sqrt(d)
    out = np.empty((B, nq, hq, d), dtype=np.float32)
    lib().ko_paged_attention(B, nq, hq, hkv, d, block_size, bt.shape[1], scale, _p(q), _p(kc),
                             _p(vc), _p(bt), _p(cl), _p(tm), _p(out), nthreads)
    return out


def kv_reserve(num_new, block_table, context_lens, free_stack, free_top, ref_counts, block_size):
    """In-place on numpy arrays (free_top is a 1-element int32 array); returns ok [B]."""
    B, maxb = block_table.shape
    ok = np.empty(B, dtype=np.int32)
    lib().ko_kv_reserve(B, block_size, maxb, ref_counts.size, num_new, _p(block_table),
                        _p(context_lens), _p(free_stack), _p(free_top), _p(ref_counts), _p(ok))
    return ok


def kv_reserve_cow(num_new, k_caches, v_caches, block_table, context_lens, free_stack,
                   free_top, ref_counts, block_size):
    """kv_reserve with copy-on-write of shared, partly filled last blocks; in
    place on numpy arrays and the uint16 caches [NB,Hkv,bs,D] of every layer.
    Returns (ok [B], cow [B, 2])."""
    B, maxb = block_table.shape
    ok = np.empty(B, dtype=np.int32)
    cow = np.empty((B, 2), dtype=np.int32)
    L = len(k_caches)
    kp = (C.c_void_p * max(L, 1))(*[c.ctypes.data for c in k_caches])
    vp = (C.c_void_p * max(L, 1))(*[c.ctypes.data for c in v_caches])
    hkv, d = (k_caches[0].shape[1], k_caches[0].shape[3]) if L else (1, 8)
    lib().ko_kv_reserve_cow(B, block_size, maxb, ref_counts.size, num_new, L,
                            C.cast(kp, C.c_void_p), C.cast(vp, C.c_void_p), hkv, d,
                            _p(block_table), _p(context_lens), _p(free_stack), _p(free_top),
                            _p(ref_counts), _p(ok), _p(cow))
    return ok, cow


def kv_commit(num_new, accept_len, block_table, context_lens, free_stack, free_top, ref_counts,
              block_size):
    B, maxb = block_table.shape
    acc = np.ascontiguousarray(accept_len, dtype=np.int32)
    lib().ko_kv_commit(B, block_size, maxb, ref_counts.size, num_new, _p(acc), _p(block_table),
                       _p(context_lens), _p(free_stack), _p(free_top), _p(ref_counts))


def kv_commit_tree(num_nodes, path, path_len, k_caches, v_caches, block_table, context_lens,
                   free_stack, free_top, ref_counts, block_size):
    """k_caches / v_caches: lists of uint16 arrays [NB,Hkv,bs,D], modified in place."""
    B, maxb = block_table.shape
    pth = np.ascontiguousarray(path, dtype=np.int32)
    pl = np.ascontiguousarray(path_len, dtype=np.int32)
    L = len(k_caches)
    kp = (C.c_void_p * L)(*[c.ctypes.data for c in k_caches])
    vp = (C.c_void_p * L)(*[c.ctypes.data for c in v_caches])
    hkv, d = k_caches[0].shape[1], k_caches[0].shape[3]
    lib().ko_kv_commit_tree(B, block_size, maxb, ref_counts.size, num_nodes, _p(pth), _p(pl), L,
                            C.cast(kp, C.c_void_p), C.cast(vp, C.c_void_p), hkv, d,
                            _p(block_table), _p(context_lens), _p(free_stack), _p(free_top),
                            _p(ref_counts))


def kv_write(k_new, v_new, block_table, context_lens, k_cache, v_cache, block_size):
    """k_new / v_new uint16 [B, n, Hkv, D]; caches modified in place."""
    B, n, hkv, d = k_new.shape
    kn = np.ascontiguousarray(k_new, dtype=np.uint16)
    vn = np.ascontiguousarray(v_new, dtype=np.uint16)
    lib().ko_kv_write(B, block_size, block_table.shape[1], k_cache.shape[0], n, hkv, d, _p(kn),
                      _p(vn), _p(np.ascontiguousarray(block_table)),
                      _p(np.ascontiguousarray(context_lens)), _p(k_cache), _p(v_cache))


def rope_kv_write(q, k_new, v_new, block_table, context_lens, k_cache, v_cache, block_size,
                  theta=10000.0, pos_offsets=None):
    """Rotary embedding of q and k (layers.rs:37-61) + paged K/V store.
    q uint16 [B, n, Hq, D], k_new / v_new uint16 [B, n, Hkv, D]; returns the
    rotated q; the caches are modified in place."""
    B, n, hq, d = q.shape
    hkv = k_new.shape[2]
    qq = np.ascontiguousarray(q, dtype=np.uint16)
    kn = np.ascontiguousarray(k_new, dtype=np.uint16)
    vn = np.ascontiguousarray(v_new, dtype=np.uint16)
    q_out = np.empty_like(qq)
    po = None if pos_offsets is None else np.ascontiguousarray(pos_offsets, dtype=np.int32)
    lib().ko_rope_kv_write(B, block_size, block_table.shape[1], k_cache.shape[0], n, hq, hkv, d,
                           float(theta), None if po is None else _p(po), _p(qq), _p(kn), _p(vn),
                           _p(np.ascontiguousarray(block_table)),
                           _p(np.ascontiguousarray(context_lens)), _p(q_out), _p(k_cache),
                           _p(v_cache))
    return q_out


def verify_step(state: dict, q, k_new, v_new, target_logits, draft_logits, draft_tokens,
                block_size, mode=MODE_STOCHASTIC, temperature=1.0, seed=0, step=0,
                seq_offset=0, rope_theta=None, nthreads=1, reserve=True, reserve_next=0):
    """One batched verify step, composed from the restatements above in the
    order SpeculativeDecoder::step runs it (src/speculative.rs:342-353) with
    the paged cache of the verify path:

      kv_reserve (k + 1 slots, BlockManager::allocate semantics)
      -> rope_kv_write (rope_theta given: RoPE at context_len + j, llama.rs:73-82)
         or kv_write (append_kv, kv_cache.rs:49-75) of the new K/V rows
      -> paged attention of the k + 1 query rows (attention_kernel.rs:22-136)
      -> acceptance (verify_drafts, speculative.rs:286-339, or the
         stochastic rule) -> kv_commit of accept_len + 1 slots.

    `state` holds numpy arrays block_table, context_lens, free_stack,
    free_top, ref_counts and the uint16 caches k_cache, v_cache; all are
    modified in place.  q / k_new / v_new are uint16 bf16 bit patterns.
    reserve=False skips the first reserve (an earlier step reserved the
    slots); reserve_next > 0 reserves that many slots after the commit, and
    `ok` is then that reserve's result.
    Returns dict(attention fp32 [B, k+1, Hq, D], ok, accept_len, tokens,
    num_tokens, probs)."""
    nq = np.asarray(target_logits).shape[1]
    s = state
    ok = None
    if reserve:
        ok = kv_reserve(nq, s["block_table"], s["context_lens"], s["free_stack"],
                        s["free_top"], s["ref_counts"], block_size)
    if rope_theta is not None:
        qq = rope_kv_write(q, k_new, v_new, s["block_table"], s["context_lens"], s["k_cache"],
                           s["v_cache"], block_size, theta=rope_theta)
    else:
        kv_write(k_new, v_new, s["block_table"], s["context_lens"], s["k_cache"], s["v_cache"],
                 block_size)
        qq = q
    att = paged_attention(qq, s["k_cache"], s["v_cache"], s["block_table"], s["context_lens"],
                          block_size, nthreads=nthreads)
    acc, toks, num, probs = spec_accept(target_logits, draft_logits, draft_tokens, mode=mode,
                                        temperature=temperature, seed=seed, step=step,
                                        seq_offset=seq_offset, nthreads=nthreads)
    kv_commit(nq, acc, s["block_table"], s["context_lens"], s["free_stack"], s["free_top"],
              s["ref_counts"], block_size)
    if reserve_next:
        ok = kv_reserve(reserve_next, s["block_table"], s["context_lens"], s["free_stack"],
                        s["free_top"], s["ref_counts"], block_size)
    return {"attention": att, "ok": ok, "accept_len": acc, "tokens": toks, "num_tokens": num,
            "probs": probs}

"""The vocabulary-sharded exchange of kyro_spec_accept_tp, run as two gloo
ranks on the CPU.

Each rank holds only its columns of the target and draft rows (the shard
rule of src/distributed.rs:90-98) and computes its pieces with the oracle's
per-shard functions.  The pieces travel in the same three rounds the GPU
path uses (an all-gather of row maxima with the normaliser parts under
them and the owner's values at the draft tokens; an all-gather of weight
totals; a max-reduction of the token id) and are combined in rank order.  Both ranks must reach the decisions of
the single-process oracle over the same shards.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CASES = [
    # B, k, V, T, seed
    (4, 3, 4096, 0.8, 1),
    (3, 5, 3000, 1.0, 2),   # 1500 columns per rank: a ragged last chunk
    (2, 0, 2048, 1.0, 3),   # bonus only
]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(B, k, V, seed):
    rng = np.random.default_rng(seed)
    tgt = (rng.standard_normal((B, k + 1, V)) * 3.0).astype(np.float32)
    drf = (tgt[:, :k, :] + rng.standard_normal((B, k, V))).astype(np.float32)
    return tgt, drf


def _gather(x):
    import torch.distributed as dist
    t = torch.from_numpy(np.ascontiguousarray(x))
    out = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(out, t)
    return [o.numpy() for o in out]


def _protocol(O, rank, world, tgt, drf, drafts, T, seed):
    """One rank of the exchange; returns (accept_len, tokens, num_tokens)."""
    import torch.distributed as dist
    B, k1, V = tgt.shape
    k = k1 - 1
    R = 2 * k + 1
    Vs = V // world
    lo = rank * Vs
    ts, ds = tgt[:, :, lo:lo + Vs], drf[:, :, lo:lo + Vs]

    def row(b, r):
        return ts[b, r] if r <= k else ds[b, r - k - 1]

    def token_of_row(b, r):
        if r < k:
            return int(drafts[b, r])
        if r > k:
            return int(drafts[b, r - k - 1])
        return -1

    # round 1: each rank's row max, its normaliser part under that max, and
    # the owner's e and chunk max at the draft token
    m_loc = np.array([[O.tp_row_max(row(b, r), T) for r in range(R)] for b in range(B)],
                     dtype=np.float32)
    S_loc = np.zeros((B, R), dtype=np.float64)
    ex = np.zeros((B, R), dtype=np.float32)
    mcx = np.zeros((B, R), dtype=np.float32)
    for b in range(B):
        for r in range(R):
            S_loc[b, r] = O.tp_row_sum_part(row(b, r), T, float(m_loc[b, r]))
            x = token_of_row(b, r)
            if lo <= x < lo + Vs:
                ex[b, r], mcx[b, r] = O.tp_entry(row(b, r), T, x - lo)
    m_all, S_all, ex_all, mcx_all = _gather(m_loc), _gather(S_loc), _gather(ex), _gather(mcx)
    M = np.max(np.stack(m_all), axis=0)

    def shard_scale(mr, mm):  # ky_shard_scale
        return 1.0 if mr == mm else float(np.float64(O.exp(np.float32(mr) - np.float32(mm))))

    S = np.zeros((B, R), dtype=np.float64)
    for q in range(world):  # rank order
        for b in range(B):
            for r in range(R):
                S[b, r] = S[b, r] + S_all[q][b, r] * shard_scale(m_all[q][b, r], M[b, r])

    def scale(m_c, Mr, Sr):
        return np.float32(np.float64(O.exp(np.float32(m_c) - np.float32(Mr))) / Sr)

    acc = np.zeros(B, dtype=np.int32)
    toks = np.full((B, k + 1), -1, dtype=np.int32)
    num = np.zeros(B, dtype=np.int32)
    totals = np.zeros((B, 2), dtype=np.int64)
    for b in range(B):
        aa = k
        for j in range(k):
            x = int(drafts[b, j])
            owner = x // Vs
            p = np.float32(ex_all[owner][b, j]) * scale(mcx_all[owner][b, j], M[b, j], S[b, j])
            qv = np.float32(ex_all[owner][b, k + 1 + j]) * scale(mcx_all[owner][b, k + 1 + j],
                                                                M[b, k + 1 + j], S[b, k + 1 + j])
            u = np.float32(O.uniform(seed, b, j, 1, 0))
            if not (u < np.float32(p) / np.float32(qv)):
                aa = j
                break
        acc[b] = aa
        toks[b, :aa] = drafts[b, :aa]
        num[b] = aa + 1
        q_shard = ds[b, aa] if aa < k else None
        Mq = float(M[b, k + 1 + aa]) if aa < k else 0.0
        Sq = float(S[b, k + 1 + aa]) if aa < k else 1.0
        totals[b] = O.tp_weight_totals(ts[b, aa], q_shard, T, float(M[b, aa]), float(S[b, aa]),
                                       Mq, Sq)
    # round 2: weight totals; the owner rank of the cut point finds the token
    tot_all = _gather(totals)
    cand = np.full(B, -1, dtype=np.int64)
    for b in range(B):
        aa = int(acc[b])
        tw = sum(int(tot_all[q][b, 0]) for q in range(world))
        tp = sum(int(tot_all[q][b, 1]) for q in range(world))
        residual = aa < k and tw != 0
        col = 0 if residual else 1
        tot = tw if residual else tp
        if tot == 0:
            if rank == world - 1:
                cand[b] = V - 1
            continue
        odd = int(round(O.uniform(seed, b, aa, 2, 0) * (1 << 24)))
        thr = (odd * tot + (1 << 24) - 1) >> 24
        before = sum(int(tot_all[q][b, col]) for q in range(rank))
        mine = int(tot_all[rank][b, col])
        if before < thr <= before + mine:
            q_shard = ds[b, aa] if aa < k else None
            Mq = float(M[b, k + 1 + aa]) if aa < k else 0.0
            Sq = float(S[b, k + 1 + aa]) if aa < k else 1.0
            local = O.tp_cut(ts[b, aa], q_shard, T, float(M[b, aa]), float(S[b, aa]), Mq, Sq,
                             residual, thr - before)
            cand[b] = lo + local
    # round 3: the token id, from its owner
    t = torch.from_numpy(cand)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    for b in range(B):
        toks[b, int(acc[b])] = int(t[b])
    return acc, toks, num


def _rank_main(rank, world, port, q_out):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import torch.distributed as dist
    import oracle as O
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        res = []
        for (B, k, V, T, seed) in CASES:
            tgt, drf = _inputs(B, k, V, seed)
            drafts = (O.sample_tokens(drf, T, seed=seed)[0] if k > 0
                      else np.zeros((B, 0), dtype=np.int32))
            res.append(_protocol(O, rank, world, tgt, drf, drafts, T, seed))
        q_out.put((rank, res, None))
    except Exception as e:
        q_out.put((rank, None, repr(e)))
    finally:
        dist.destroy_process_group()


def test_tp_exchange_reproduces_sharded_oracle(oracle):
    import torch.multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q_out)) for r in range(world)]
    for p in procs:
        p.start()
    outs = {}
    try:
        for _ in range(world):
            rank, res, err = q_out.get(timeout=300)
            outs[rank] = (res, err)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for (B, k, V, T, seed), case_i in zip(CASES, range(len(CASES))):
        tgt, drf = _inputs(B, k, V, seed)
        drafts = (oracle.sample_tokens(drf, T, seed=seed)[0] if k > 0
                  else np.zeros((B, 0), dtype=np.int32))
        racc, rtoks, rnum, _ = oracle.spec_accept(tgt, drf, drafts, temperature=T, seed=seed,
                                                  num_shards=world)
        for rank in range(world):
            res, err = outs[rank]
            assert err is None, f"rank {rank}: {err}"
            acc, toks, num = res[case_i]
            assert np.array_equal(acc, racc), (rank, case_i, acc, racc)
            assert np.array_equal(toks, rtoks), (rank, case_i, toks, rtoks)
            assert np.array_equal(num, rnum), (rank, case_i)

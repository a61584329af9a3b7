"""Vocabulary-sharded acceptance (kyro_spec_accept_tp) on 2+ GPUs against
the oracle's sharded contract.

The shard rule is DistributedContext::shard_dim (src/distributed.rs:90-98):
rank r holds vocabulary columns [r*V/R, (r+1)*V/R).  Each rank is a spawned
process with its own GPU and kyro context; rank 0's NCCL unique id reaches
the others through a queue.  Every rank must return the oracle's results
for num_shards = R, bit for bit.  Skipped with fewer than two GPUs.
"""
import os
import sys
import time

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

pytestmark = pytest.mark.gpu

CASES = [
    # B, k, V, mode, T, seed
    (8, 4, 32000, 0, 0.8, 3),     # 16000 columns per rank: a ragged last chunk on each
    (6, 8, 128256, 0, 0.8, 11),   # config-3 rows (k 8, T 0.8), a small batch
    (5, 3, 32000, 0, 1.0, 5),
    (4, 4, 32000, 2, 1.0, 7),     # greedy, the reference rule
    (4, 0, 32000, 0, 1.0, 9),     # k = 0: bonus only
]


def _inputs(B, k, V, seed):
    g = torch.Generator().manual_seed(seed)
    tgt = torch.randn(B, k + 1, V, generator=g) * 3.0
    drf = tgt[:, :k, :] + torch.randn(B, k, V, generator=g)
    return tgt.contiguous(), drf.contiguous()


def _rank_main(rank, world, q_id, q_out, cases, transport="peer"):
    if transport == "nccl":
        os.environ["KYRO_TP_TRANSPORT"] = "nccl"
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    from kyro_b200.verify import Context, spec_accept_tp, sample_tokens, tp_unique_id
    torch.cuda.set_device(rank)
    ctx = Context(rank)
    try:
        if rank == 0:
            uid = tp_unique_id()
            for _ in range(world - 1):
                q_id.put(uid)
        else:
            uid = q_id.get(timeout=120)
        ctx.tp_init(uid, rank, world)
        if ctx.tp_transport != transport:
            raise RuntimeError(f"transport {ctx.tp_transport}, expected {transport}")
        dev = torch.device("cuda", rank)
        results = []
        for (B, k, V, mode, T, seed) in cases:
            tgt, drf = _inputs(B, k, V, seed)
            # the drafts every rank sees: sampled once from the full draft rows
            if k > 0:
                drafts = torch.from_numpy(O.sample_tokens(drf.numpy(), T, seed=seed)[0]).int()
            else:
                drafts = torch.zeros(B, 0, dtype=torch.int32)
            Vs = V // world
            ts = tgt[:, :, rank * Vs:(rank + 1) * Vs].contiguous().to(dev)
            ds = drf[:, :, rank * Vs:(rank + 1) * Vs].contiguous().to(dev)
            acc, toks, num, probs = spec_accept_tp(ctx, ts, ds if mode == 0 else None,
                                                   drafts.to(dev), V, mode=mode, temperature=T,
                                                   seed=seed, want_probs=mode == 0)
            torch.cuda.synchronize(dev)
            ref = O.spec_accept(tgt.numpy(), drf.numpy(), drafts.numpy(), mode=mode,
                                temperature=T, seed=seed, num_shards=world, nthreads=4)
            got = (acc.cpu().numpy(), toks.cpu().numpy(), num.cpu().numpy(),
                   None if probs is None else probs.cpu().numpy())
            results.append((got, ref))
        status = ctx.device_status()
        q_out.put((rank, results, status, None))
    except Exception as e:  # reported to the parent, which fails the test
        q_out.put((rank, None, None, repr(e)))
    finally:
        ctx.close()


@pytest.mark.parametrize("transport", ["peer", "nccl"])
def test_vocab_sharded_accept_matches_oracle(transport):
    """Both transports of the exchange rounds: NVLink peer-memory stores with
    per-sender flags (the default on B200 nodes) and NCCL collectives."""
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    if n < 2:
        pytest.skip("needs two GPUs")
    world = 2
    import torch.multiprocessing as mp
    mpc = mp.get_context("spawn")
    q_id, q_out = mpc.Queue(), mpc.Queue()
    procs = [mpc.Process(target=_rank_main, args=(r, world, q_id, q_out, CASES, transport))
             for r in range(world)]
    for p in procs:
        p.start()
    outs = {}
    try:
        for _ in range(world):
            rank, results, status, err = q_out.get(timeout=600)
            outs[rank] = (results, status, err)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank in range(world):
        results, status, err = outs[rank]
        assert err is None, f"rank {rank}: {err}"
        assert status == 0, f"rank {rank}: device status 0x{status:x}"
        for case, (got, ref) in zip(CASES, results):
            acc, toks, num, probs = got
            racc, rtoks, rnum, rprobs = ref
            assert np.array_equal(acc, racc), (rank, case, acc, racc)
            assert np.array_equal(toks, rtoks), (rank, case)
            assert np.array_equal(num, rnum), (rank, case)
            if probs is not None:
                assert np.array_equal(probs, rprobs), (rank, case)


def _skip_rank_main(rank, world, q_id, q_out):
    """Both ranks join a peer-memory group; rank 1 skips its first exchange
    round towards rank 0 (it stays alive and runs the rest of the call), so
    rank 0's first round must run into its 100 ms bound, flag
    KYRO_DEV_WAIT_TIMEOUT and return instead of hanging."""
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    sys.path.insert(0, ROOT)
    from kyro_b200 import _lib
    from kyro_b200.verify import Context, spec_accept_tp, tp_unique_id
    torch.cuda.set_device(rank)
    ctx = Context(rank)
    try:
        if rank == 0:
            uid = tp_unique_id()
            q_id.put(uid)
        else:
            uid = q_id.get(timeout=120)
        ctx.tp_init(uid, rank, world)
        if ctx.tp_transport != "peer":
            raise RuntimeError(f"transport {ctx.tp_transport}")
        # rank 0 gives up after 100 ms; rank 1's later rounds wait about that
        # long for rank 0 and keep a bound well above it
        ctx.set_wait_timeout(100 if rank == 0 else 3000)
        B, k, V = 4, 3, 32000
        tgt, drf = _inputs(B, k, V, 1)
        Vs = V // world
        dev = torch.device("cuda", rank)
        ts = tgt[:, :, rank * Vs:(rank + 1) * Vs].contiguous().to(dev)
        ds = drf[:, :, rank * Vs:(rank + 1) * Vs].contiguous().to(dev)
        drafts = torch.zeros(B, k, dtype=torch.int32, device=dev)
        if rank == 1:
            ctx.inject_skip(1)
        t0 = time.monotonic()
        spec_accept_tp(ctx, ts, ds, drafts, V, seed=1)
        status = ctx.device_status(clear=True)
        q_out.put((rank, status, time.monotonic() - t0, None))
    except Exception as e:
        q_out.put((rank, None, None, repr(e)))
    finally:
        ctx.close()


def test_skipped_round_times_out_on_the_peer():
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    if n < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    from kyro_b200._lib import DEV_WAIT_TIMEOUT
    mpc = mp.get_context("spawn")
    q_id, q_out = mpc.Queue(), mpc.Queue()
    procs = [mpc.Process(target=_skip_rank_main, args=(r, 2, q_id, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    outs = {}
    try:
        for _ in range(2):
            rank, status, dt, err = q_out.get(timeout=300)
            outs[rank] = (status, dt, err)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank in (0, 1):
        assert outs[rank][2] is None, outs
    assert outs[0][0] & DEV_WAIT_TIMEOUT, outs
    assert outs[0][1] < 10.0, outs
    # rank 1 skipped its own stores, but rank 0 raised every flag it waited for
    assert not (outs[1][0] & DEV_WAIT_TIMEOUT), outs

"""Failure detection on the host, without a GPU.

The reference bounds request lifetimes with deadlines
(src/scheduler/continuous_batching.rs:83-100) and logs worker errors
(src/main.rs:146-148).  The library's counterpart for the verify step's
collectives is a host watchdog (kyro_b200/csrc/watchdog.h): an NCCL
collective that has not completed within the context's wait bound gets its
communicator aborted.  These tests run that watchdog through
kyro_selftest_watchdog on probes made on the host: a probe that completes,
one that never does, and the async all-reduce of two gloo ranks one of which
joins late (the other rank's watchdog must fire) or in time (it must not).
"""
import os
import time

import pytest


@pytest.fixture(scope="module")
def lib():
    from kyro_b200 import _lib, build
    build.build()
    return _lib.load()


def _watch(lib, timeout_ms, poll):
    from kyro_b200 import _lib
    aborts = []
    pf = _lib.POLL_FN(lambda _u: 1 if poll() else 0)
    af = _lib.ABORT_FN(lambda _u: aborts.append(time.monotonic()))
    t0 = time.monotonic()
    st = lib.kyro_selftest_watchdog(timeout_ms, pf, af, None)
    return st, time.monotonic() - t0, aborts, t0


def test_watchdog_quiet_when_work_completes(lib):
    t_done = time.monotonic() + 0.05
    st, dt, aborts, _ = _watch(lib, 2000, lambda: time.monotonic() >= t_done)
    assert st == 0 and not aborts
    assert dt < 1.0


def test_watchdog_fires_once_on_stuck_work(lib):
    from kyro_b200 import _lib
    st, dt, aborts, t0 = _watch(lib, 100, lambda: False)
    assert st == _lib.KYRO_ERR_TIMEOUT
    assert len(aborts) == 1
    assert aborts[0] - t0 >= 0.1 and dt < 2.0
    assert "did not complete" in _lib.last_error()


def test_watchdog_rejects_bad_arguments(lib):
    from kyro_b200 import _lib
    pf = _lib.POLL_FN(lambda _u: 1)
    af = _lib.ABORT_FN(lambda _u: None)
    assert lib.kyro_selftest_watchdog(0, pf, af, None) == _lib.KYRO_ERR_INVALID_ARG
    assert lib.kyro_ctx_set_wait_timeout(None, 10) == _lib.KYRO_ERR_INVALID_ARG
    assert lib.kyro_ctx_tp_inject_skip(None, 1) == _lib.KYRO_ERR_INVALID_ARG


def _gloo_rank(rank, world, port, delay_s, bound_ms, q):
    import torch
    import torch.distributed as dist

    from kyro_b200 import _lib
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        t = torch.ones(4)
        if rank == 1:
            time.sleep(delay_s)  # the peer that stalls before the collective
            dist.all_reduce(t)
            q.put((rank, None, None))
        else:
            work = dist.all_reduce(t, async_op=True)
            st, dt, aborts, _ = _watch(_lib.load(), bound_ms, work.is_completed)
            work.wait()  # the late peer joins in the end: nothing is left in flight
            q.put((rank, st, len(aborts)))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent
        q.put((rank, "error", repr(e)))


def _run_pair(delay_s, bound_ms, port):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, delay_s, bound_ms, q))
             for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(2):
            rank, st, n = q.get(timeout=120)
            out[rank] = (st, n)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return out


@pytest.mark.parametrize("delay_s,bound_ms,fires", [(1.5, 300, True), (0.05, 5000, False)])
def test_watchdog_on_gloo_ranks(lib, delay_s, bound_ms, fires):
    """Rank 1 joins the all-reduce `delay_s` late; rank 0's watchdog bounds
    its wait by `bound_ms` and aborts exactly when the peer is too late."""
    from kyro_b200 import _lib
    out = _run_pair(delay_s, bound_ms, 29500 + int(delay_s * 10) + bound_ms % 97)
    assert out[1][0] is None, out
    st, n_aborts = out[0]
    if fires:
        assert st == _lib.KYRO_ERR_TIMEOUT and n_aborts == 1, out
    else:
        assert st == 0 and n_aborts == 0, out

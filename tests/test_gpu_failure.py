"""Bounded device-side waits on one GPU.

The exchange kernel of the tensor-parallel sampler waits for flags that
peers raise over NVLink.  Here it runs as a one-rank group that skips its own
round, so it waits for a flag that nothing sets: it must give up after the
context's wait bound, record KYRO_DEV_WAIT_TIMEOUT in the status word and
return, and the context must stay usable for the next call.  No fault, trap
or hang is involved; the wait bound is 50 ms.
"""
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_exchange_wait_times_out_and_context_survives(ctx, oracle):
    from kyro_b200 import _lib
    from kyro_b200.verify import sample_tokens, spec_accept
    from kyro_b200.workloads import accept_inputs
    region = torch.empty(8192, dtype=torch.uint8, device=ctx.device)
    assert ctx.device_status(clear=True) == 0
    ctx.set_wait_timeout(50)
    ctx.bind_stream()
    torch.cuda.synchronize()
    t0 = time.monotonic()
    _lib.check(_lib.load().kyro_selftest_exchange_timeout(ctx.handle, region.data_ptr(),
                                                          region.numel()))
    status = ctx.device_status(clear=True)
    dt = time.monotonic() - t0
    assert status & _lib.DEV_WAIT_TIMEOUT, hex(status)
    assert 0.045 <= dt < 1.5, dt
    # the context is still usable: one acceptance call, bit-exact
    tgt, drf = accept_inputs(4, 3, 32000, ctx.device, seed=11)
    drafts, _ = sample_tokens(ctx, drf, 1.0, seed=11)
    acc, toks, num, _ = spec_accept(ctx, tgt, drf, drafts, seed=11)
    oacc, otoks, onum, _ = oracle.spec_accept(tgt.cpu().numpy(), drf.cpu().numpy(),
                                              drafts.cpu().numpy(), seed=11)
    assert np.array_equal(acc.cpu().numpy(), oacc)
    assert np.array_equal(toks.cpu().numpy(), otoks)
    assert ctx.device_status() == 0
    ctx.set_wait_timeout(2000)


def test_wait_timeout_argument_checks(ctx):
    from kyro_b200 import _lib
    L = _lib.load()
    assert L.kyro_ctx_set_wait_timeout(ctx.handle, 0) == _lib.KYRO_ERR_INVALID_ARG
    assert L.kyro_ctx_set_wait_timeout(ctx.handle, 600001) == _lib.KYRO_ERR_INVALID_ARG
    # a context without a peer-memory group has no exchange to skip
    assert L.kyro_ctx_tp_inject_skip(ctx.handle, 1) == _lib.KYRO_ERR_INVALID_ARG
    small = torch.empty(1024, dtype=torch.uint8, device=ctx.device)
    assert L.kyro_selftest_exchange_timeout(ctx.handle, small.data_ptr(), 1024) == \
        _lib.KYRO_ERR_INVALID_ARG

"""The no-allocation acceptance entry point, kyro_spec_accept_static.

Some hosts own every byte of device memory themselves (a serving runtime
with a fixed arena, or a loop that may not call the allocator), so they
cannot hand the library a workspace.  kyro_spec_accept_static serves them
from a static device array inside the library.  These tests call it through
the C ABI and require exactly the outputs of kyro_spec_accept with a
caller-provided workspace, on two calls in a row (the second call starts
from whatever the first left in the shared scratch).

This file is named to be collected last, so a run that stops at the first
failure has already run every other test; it passes on its own in a fresh
process as well.
"""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _accept_static(ctx, tgt, drf, drafts, temperature, seed, step):
    from kyro_b200 import _lib
    B, k1, V = tgt.shape
    k = k1 - 1
    acc = torch.full((B,), -7, dtype=torch.int32, device=ctx.device)
    toks = torch.full((B, k + 1), -7, dtype=torch.int32, device=ctx.device)
    num = torch.full((B,), -7, dtype=torch.int32, device=ctx.device)
    probs = torch.full((B, k, 2), -7.0, dtype=torch.float32, device=ctx.device)
    p = _lib.AcceptParams(B, k, V, _lib.ACCEPT_STOCHASTIC, temperature, step, seed, 0)
    ctx.bind_stream()
    st = _lib.load().kyro_spec_accept_static(
        ctx.handle, C.byref(p), C.c_void_p(tgt.data_ptr()), C.c_void_p(drf.data_ptr()),
        C.c_void_p(drafts.data_ptr()), C.c_void_p(acc.data_ptr()), C.c_void_p(toks.data_ptr()),
        C.c_void_p(num.data_ptr()), C.c_void_p(probs.data_ptr()))
    _lib.check(st)
    return acc, toks, num, probs


@pytest.mark.parametrize("B,k,V,T", [(8, 4, 32000, 1.0), (64, 5, 128256, 0.7)])
def test_static_scratch_matches_workspace_entry_point(ctx, B, k, V, T):
    from kyro_b200.verify import sample_tokens, spec_accept
    from kyro_b200.workloads import accept_inputs
    tgt, drf = accept_inputs(B, k, V, ctx.device, seed=B + k)
    drafts, _ = sample_tokens(ctx, drf, T, seed=5)
    for step in (0, 1):  # two calls in a row share the static scratch
        want = spec_accept(ctx, tgt, drf, drafts, temperature=T, seed=5, step=step,
                           want_probs=True)
        got = _accept_static(ctx, tgt, drf, drafts, T, 5, step)
        for w, g in zip(want, got):
            assert torch.equal(w, g)
    assert ctx.device_status() == 0


def test_static_scratch_rejects_oversized_batches(ctx):
    from kyro_b200 import _lib
    p = _lib.AcceptParams(4096, 8, 128256, _lib.ACCEPT_STOCHASTIC, 1.0, 0, 0, 0)
    need = _lib.load().kyro_spec_accept_workspace_size(C.byref(p))
    assert need > _lib.ACCEPT_STATIC_SCRATCH_BYTES
    st = _lib.load().kyro_spec_accept_static(ctx.handle, C.byref(p), *([C.c_void_p(16)] * 7))
    assert st == _lib.KYRO_ERR_WORKSPACE
    assert "static scratch" in _lib.last_error()
    # nothing was launched, so the context is still clean
    assert ctx.device_status() == 0

"""The composed verify step on the GPU against the oracle's composition of
the same step (SpeculativeDecoder::step, src/speculative.rs:342-353):
reserve -> RoPE + paged K/V store -> verify attention -> acceptance ->
commit, two steps in a row on one KV state, so that every hand-off between
the kernels is checked: the block table the reserve extends is the one
attention reads, the accept lengths are the ones the commit keeps, and the
second step starts from the state the first one committed.

Bar: accept lengths, emitted tokens, the reserve's ok flags, the block
table, context lengths, free list, free top, ref counts and every cache
bit exact; attention within 2e-2 of the double-precision oracle.
"""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

NTHREADS = os.cpu_count() or 1
ATOL = 2e-2
STATE = ("block_table", "context_lens", "free_stack", "free_top", "ref_counts")


def _np(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("rope,mode,T,loop", [(True, 0, 1.0, False), (False, 0, 0.7, False),
                                               (True, 2, 1.0, False), (True, 0, 1.0, True),
                                               (True, 1, 1.0, True)])
def test_composed_step_matches_oracle(ctx, oracle, rope, mode, T, loop):
    """loop: the decode-loop form, where a step's commit also reserves the
    next step's slots (kyro_spec_accept_commit with num_new_next = k + 1)
    after one initial reserve."""
    from kyro_b200.step import KVState, VerifyStep
    from kyro_b200.workloads import ChainConfig, accept_inputs, bf16_bits, paged_state
    # config-1 layer and vocabulary, a smaller batch with config-1 context draws
    # plus the edges: an empty context, one token, a block boundary
    cfg = ChainConfig(batch=12, num_blocks=4096, headroom_tokens=64)
    rng = np.random.default_rng(21)
    lens = rng.integers(cfg.ctx_min, cfg.ctx_max + 1, size=cfg.batch)
    lens[:3] = [0, 1, 16]
    st = paged_state(cfg, ctx.device, seed=22, ctx_lens=lens)
    kv = KVState(st.block_table, st.context_lens, st.free_stack, st.free_top, st.ref_counts,
                 st.k_cache, st.v_cache)
    g = torch.Generator(device=ctx.device).manual_seed(23)
    shape = (cfg.batch, cfg.num_query, cfg.num_kv_heads, cfg.head_dim)
    k_new = torch.randn(shape, generator=g, device=ctx.device, dtype=torch.bfloat16)
    v_new = torch.randn(shape, generator=g, device=ctx.device, dtype=torch.bfloat16)
    tgt, drf = accept_inputs(cfg.batch, cfg.k, cfg.vocab, ctx.device, seed=24)
    drafts = oracle.sample_tokens(_np(drf), T, seed=25, nthreads=NTHREADS)[0]
    drafts_d = torch.from_numpy(drafts).to(ctx.device)
    host = {n: _np(getattr(st, n)).copy() for n in STATE}
    host["k_cache"], host["v_cache"] = bf16_bits(st.k_cache).copy(), bf16_bits(st.v_cache).copy()
    theta = 10000.0 if rope else None
    step = VerifyStep(ctx, cfg.batch, cfg.k, cfg.num_heads, kv, cfg.vocab, cfg.block_size,
                      mode=mode, temperature=T, seed=7, seq_offset=100, rope_theta=theta)
    drf_in = drf if mode == 0 else None
    nxt = cfg.num_query if loop else 0
    if loop:
        from kyro_b200.verify import kv_reserve
        kv_reserve(ctx, cfg.num_query, st.block_table, st.context_lens, st.free_stack,
                   st.free_top, st.ref_counts, cfg.block_size)
        oracle.kv_reserve(cfg.num_query, host["block_table"], host["context_lens"],
                          host["free_stack"], host["free_top"], host["ref_counts"],
                          cfg.block_size)
    for i in range(2):
        att, ok, acc, toks, num = step(kv, st.q, k_new, v_new, tgt, drf_in, drafts_d, step=i,
                                       reserve=not loop, reserve_next=nxt)
        ref = oracle.verify_step(host, bf16_bits(st.q), bf16_bits(k_new), bf16_bits(v_new),
                                 _np(tgt), None if drf_in is None else _np(drf), drafts,
                                 cfg.block_size, mode=mode, temperature=T, seed=7, step=i,
                                 seq_offset=100, rope_theta=theta, nthreads=NTHREADS,
                                 reserve=not loop, reserve_next=nxt)
        torch.cuda.synchronize()
        assert np.array_equal(_np(ok), ref["ok"]), i
        assert np.array_equal(_np(acc), ref["accept_len"]), (i, _np(acc), ref["accept_len"])
        assert np.array_equal(_np(toks), ref["tokens"]), i
        assert np.array_equal(_np(num), ref["num_tokens"]), i
        err = np.abs(att.float().cpu().numpy() - ref["attention"]).max()
        assert err < ATOL, (i, err)
        for n in STATE:
            assert np.array_equal(_np(getattr(st, n)), host[n]), (i, n)
        assert np.array_equal(bf16_bits(st.k_cache), host["k_cache"]), i
        assert np.array_equal(bf16_bits(st.v_cache), host["v_cache"]), i
    # the two steps grew every context by the tokens they committed
    assert (_np(st.context_lens) > lens).all()
    assert ctx.device_status() == 0

"""GPU parity of the acceptance sampler and the draft sampler against the
CPU oracle, through the C ABI.

Bar: accept lengths and emitted tokens bit-exact given identical uniforms;
p(x)/q(x) identical to the oracle and within 1e-5 relative of a torch fp32
softmax."""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

NTHREADS = os.cpu_count() or 1


def _np(t):
    return t.detach().cpu().numpy()


def test_device_philox_matches_oracle(ctx, oracle):
    from kyro_b200.verify import philox_uniforms
    for seed, seq, stream, step in [(0, 0, 1, 0), (12345678901234, 7, 2, 99), (2**64 - 1, 2**32 - 1, 0, 5)]:
        u = _np(philox_uniforms(ctx, seed, seq, 3, stream, step, 64))
        ref = np.array([oracle.uniform(seed, seq, 3 + i, stream, step) for i in range(64)],
                       dtype=np.float32)
        assert np.array_equal(u, ref)


def _sample_drafts(ctx, oracle, drf, T, seed, step=0):
    from kyro_b200.verify import sample_tokens
    toks, probs = sample_tokens(ctx, drf, T, seed=seed, step=step)
    otoks, oprobs = oracle.sample_tokens(_np(drf), T, seed=seed, step=step, nthreads=NTHREADS)
    assert np.array_equal(_np(toks), otoks)
    assert np.array_equal(_np(probs), oprobs)
    return toks


CASES = [
    # B, k, V, T, seed
    (8, 4, 32000, 1.0, 0),     # config 0
    (8, 4, 32000, 1.0, 1),
    (3, 1, 1000, 0.7, 2),      # one ragged chunk
    (5, 8, 4099, 0.8, 3),      # V % 4 != 0: scalar loads
    (2, 0, 2048, 1.0, 4),      # k = 0: bonus only
    (16, 5, 128256, 0.7, 5),   # config-1 vocabulary
]


@pytest.mark.parametrize("B,k,V,T,seed", CASES)
def test_stochastic_accept_matches_oracle(ctx, oracle, B, k, V, T, seed):
    from kyro_b200.verify import spec_accept
    from kyro_b200.workloads import accept_inputs
    tgt, drf = accept_inputs(B, k, V, ctx.device, seed=seed)
    drafts = (_sample_drafts(ctx, oracle, drf, T, seed) if k > 0
              else torch.zeros(B, 0, dtype=torch.int32, device=ctx.device))
    for step in (0, 1):
        acc, toks, num, probs = spec_accept(ctx, tgt, drf, drafts, temperature=T, seed=seed,
                                            step=step, want_probs=True)
        oacc, otoks, onum, oprobs = oracle.spec_accept(_np(tgt), _np(drf), _np(drafts),
                                                       temperature=T, seed=seed, step=step,
                                                       nthreads=NTHREADS)
        assert np.array_equal(_np(acc), oacc)
        assert np.array_equal(_np(num), onum)
        assert np.array_equal(_np(toks), otoks)
        assert np.array_equal(_np(probs), oprobs)
    assert ctx.device_status() == 0


@pytest.mark.parametrize("std", [25.0, 60.0])
def test_wide_logits_and_minus_inf_match_oracle(ctx, oracle, std):
    """Logit spreads above 87 within a chunk, and -inf entries, take the
    clamped exponential; chunks within 87 of their max skip the clamp.  Both
    must give the contract's bits."""
    from kyro_b200.verify import spec_accept
    from kyro_b200.workloads import accept_inputs
    B, k, V, T, seed = 6, 4, 32000, 1.0, 11
    tgt, drf = accept_inputs(B, k, V, ctx.device, seed=seed, std=std, noise=std / 3)
    g = torch.Generator(device=ctx.device).manual_seed(seed)
    holes = torch.rand(B, 1, V, generator=g, device=ctx.device) < 0.002
    tgt = tgt.masked_fill(holes, float("-inf")).contiguous()
    drf = drf.masked_fill(holes[:, :, :V].expand(B, k, V), float("-inf")).contiguous()
    drafts = _sample_drafts(ctx, oracle, drf, T, seed)
    acc, toks, num, probs = spec_accept(ctx, tgt, drf, drafts, temperature=T, seed=seed,
                                        want_probs=True)
    oacc, otoks, onum, oprobs = oracle.spec_accept(_np(tgt), _np(drf), _np(drafts),
                                                   temperature=T, seed=seed, step=0,
                                                   nthreads=NTHREADS)
    assert np.array_equal(_np(acc), oacc)
    assert np.array_equal(_np(toks), otoks)
    assert np.array_equal(_np(probs), oprobs)
    assert ctx.device_status() == 0


def test_probabilities_match_torch_softmax(ctx, oracle):
    """probabilities within 1e-5 relative (fp32) of softmax(z / T)."""
    from kyro_b200.verify import spec_accept
    from kyro_b200.workloads import accept_inputs
    B, k, V, T = 8, 4, 32000, 0.8
    tgt, drf = accept_inputs(B, k, V, ctx.device, seed=11)
    drafts = _sample_drafts(ctx, oracle, drf, T, 11)
    _, _, _, probs = spec_accept(ctx, tgt, drf, drafts, temperature=T, seed=11, want_probs=True)
    inv_t = np.float32(1.0 / T)
    p_ref = torch.softmax(tgt[:, :k].double() * float(inv_t), -1)
    q_ref = torch.softmax(drf.double() * float(inv_t), -1)
    idx = drafts.long().unsqueeze(-1)
    p_x = p_ref.gather(-1, idx).squeeze(-1)
    q_x = q_ref.gather(-1, idx).squeeze(-1)
    torch.testing.assert_close(probs[..., 0].double(), p_x, rtol=1e-5, atol=0)
    torch.testing.assert_close(probs[..., 1].double(), q_x, rtol=1e-5, atol=0)


@pytest.mark.parametrize("mode", [1, 2])
def test_greedy_modes_match_oracle(ctx, oracle, mode):
    from kyro_b200.verify import spec_accept
    from kyro_b200.workloads import accept_inputs
    B, k, V = 32, 5, 32000
    tgt, _ = accept_inputs(B, k, V, ctx.device, seed=21)
    top = tgt.argmax(-1).to(torch.int32)
    rng = np.random.default_rng(0)
    drafts = top[:, :k].clone()
    # sequence b mismatches at position b % (k+1) (k+1: all match)
    for b in range(B):
        j = b % (k + 1)
        if j < k:
            drafts[b, j] = int((top[b, j].item() + 1 + rng.integers(0, V - 1)) % V)
    acc, toks, num, _ = spec_accept(ctx, tgt, None, drafts.contiguous(), mode=mode)
    oacc, otoks, onum, _ = oracle.spec_accept(_np(tgt), None, _np(drafts), mode=mode)
    assert np.array_equal(_np(acc), oacc)
    assert np.array_equal(_np(toks), otoks)
    assert np.array_equal(_np(num), onum)
    assert list(oacc) == [b % (k + 1) for b in range(B)]


def test_reference_argmax_cases_on_device(ctx, oracle):
    """src/worker.rs:395-422: argmax at T = 0 through the device sampler."""
    import json
    from kyro_b200.verify import sample_tokens
    cases = json.load(open(os.path.join(os.path.dirname(__file__), "golden",
                                        "reference_known_answers.json")))["sample_token"]
    for c in cases:
        if not c["logits"] or "expect_token" not in c:
            continue
        lg = torch.tensor(c["logits"], dtype=torch.float32, device=ctx.device)[None, None]
        toks, _ = sample_tokens(ctx, lg.contiguous(), c["temperature"], seed=0)
        assert int(toks[0, 0]) == c["expect_token"], c["name"]


def test_out_of_range_draft_token_is_flagged_and_rejected(ctx, oracle):
    from kyro_b200.verify import spec_accept
    from kyro_b200.workloads import accept_inputs
    B, k, V = 4, 3, 4096
    tgt, drf = accept_inputs(B, k, V, ctx.device, seed=31)
    drafts = _sample_drafts(ctx, oracle, drf, 1.0, 31)
    drafts[1, 0] = V + 5
    drafts[2, 1] = -1
    ctx.device_status(clear=True)
    acc, toks, num, _ = spec_accept(ctx, tgt, drf, drafts, seed=31)
    from kyro_b200._lib import DEV_BAD_TOKEN
    assert ctx.device_status() & DEV_BAD_TOKEN
    oacc, otoks, onum, _ = oracle.spec_accept(_np(tgt), _np(drf), _np(drafts), seed=31)
    assert np.array_equal(_np(acc), oacc) and np.array_equal(_np(toks), otoks)
    assert oacc[1] == 0 and oacc[2] <= 1


def test_determinism(ctx, oracle):
    from kyro_b200.verify import spec_accept
    from kyro_b200.workloads import accept_inputs
    tgt, drf = accept_inputs(16, 5, 32000, ctx.device, seed=41)
    drafts = _sample_drafts(ctx, oracle, drf, 1.0, 41)
    a = spec_accept(ctx, tgt, drf, drafts, seed=41, want_probs=True)
    b = spec_accept(ctx, tgt, drf, drafts, seed=41, want_probs=True)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


def test_full_config1_accept_matches_oracle(ctx, oracle):
    """config 1 acceptance at full size: B=64, k=5, V=128256."""
    from kyro_b200.verify import spec_accept
    from kyro_b200.workloads import accept_inputs
    B, k, V = 64, 5, 128256
    tgt, drf = accept_inputs(B, k, V, ctx.device, seed=0)
    drafts = _sample_drafts(ctx, oracle, drf, 1.0, 0)
    acc, toks, num, probs = spec_accept(ctx, tgt, drf, drafts, seed=0, want_probs=True)
    oacc, otoks, onum, oprobs = oracle.spec_accept(_np(tgt), _np(drf), _np(drafts), seed=0,
                                                   nthreads=NTHREADS)
    assert np.array_equal(_np(acc), oacc)
    assert np.array_equal(_np(toks), otoks)
    assert np.array_equal(_np(probs), oprobs)
    # per-token acceptance probability E[min(1, p/q)]: BASELINE quotes ~0.6-0.8
    rate = np.minimum(1.0, oprobs[..., 0] / oprobs[..., 1]).mean()
    assert 0.5 < rate < 0.9, rate


@pytest.mark.gpu
def test_fast_exp_forms_match_contract(ctx):
    """The exponent-add and packed fp32x2 forms the kernels use give ky_exp's
    bits on every fp32 input in [-100, 0], -inf and NaN."""
    from kyro_b200 import verify
    assert verify.selftest_exp(ctx) == (0, 0)


@pytest.mark.parametrize("k,V,T", [(4, 32000, 0.7), (5, 4099, 1.0), (3, 1000, 0.0)])
def test_sampler_reads_strided_sequences(ctx, oracle, k, V, T):
    """Column i of a [B, k, V] draft buffer, sampled in place (seq_stride k),
    gives the tokens and probabilities of the same rows copied out densely,
    and both match the oracle."""
    from kyro_b200.verify import sample_tokens
    from kyro_b200.workloads import accept_inputs
    B = 6
    _, drf = accept_inputs(B, k, V, ctx.device, seed=40 + k)
    for i in range(k):
        col = drf[:, i:i + 1]
        assert not col.is_contiguous() or k == 1
        toks, probs = sample_tokens(ctx, col, T, seed=3, step=i, seq_offset=5)
        dense = col.contiguous()
        dtoks, dprobs = sample_tokens(ctx, dense, T, seed=3, step=i, seq_offset=5)
        otoks, oprobs = oracle.sample_tokens(_np(dense), T, seed=3, step=i, seq_offset=5,
                                             nthreads=NTHREADS)
        assert torch.equal(toks, dtoks) and torch.equal(probs, dprobs)
        assert np.array_equal(_np(toks), otoks)
        if T > 0:
            assert np.array_equal(_np(probs), oprobs)
    assert ctx.device_status() == 0


def test_accept_graph_replays_match_oracle(ctx, oracle):
    """kyro_spec_accept captured once in a CUDA graph and replayed on new
    inputs copied into the captured buffers: every replay must give the
    oracle's decisions.  (The acceptance kernel tags its records per call
    from a device-side count, so a replay must not read an earlier replay's
    records.)"""
    from kyro_b200.verify import spec_accept
    from kyro_b200.workloads import accept_inputs
    B, k, V, T = 24, 5, 128256, 1.0
    tgt, drf = accept_inputs(B, k, V, ctx.device, seed=90)
    drafts = torch.zeros(B, k, dtype=torch.int32, device=ctx.device)
    acc = torch.empty(B, dtype=torch.int32, device=ctx.device)
    toks = torch.empty(B, k + 1, dtype=torch.int32, device=ctx.device)
    num = torch.empty(B, dtype=torch.int32, device=ctx.device)
    ws = torch.empty(64 << 20, dtype=torch.uint8, device=ctx.device)
    side = torch.cuda.Stream(ctx.device)
    with torch.cuda.stream(side):
        spec_accept(ctx, tgt, drf, drafts, temperature=T, seed=3, out=(acc, toks, num, None),
                    workspace=ws)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            spec_accept(ctx, tgt, drf, drafts, temperature=T, seed=3,
                        out=(acc, toks, num, None), workspace=ws)
    torch.cuda.synchronize()
    for rep in range(4):
        t2, d2 = accept_inputs(B, k, V, ctx.device, seed=91 + rep)
        dr = oracle.sample_tokens(_np(d2), T, seed=rep, nthreads=NTHREADS)[0]
        tgt.copy_(t2)
        drf.copy_(d2)
        drafts.copy_(torch.from_numpy(dr))
        with torch.cuda.stream(side):
            g.replay()
        torch.cuda.synchronize()
        oacc, otoks, onum, _ = oracle.spec_accept(_np(t2), _np(d2), dr, temperature=T, seed=3,
                                                  nthreads=NTHREADS)
        assert np.array_equal(_np(acc), oacc), rep
        assert np.array_equal(_np(toks), otoks), rep
        assert np.array_equal(_np(num), onum), rep
    del g
    ctx.bind_stream()
    assert ctx.device_status() == 0

"""CPU tests of the oracle: pinned against published known answers and the
reference's own unit-test cases (tests/golden/), plus the distributional
property of the published rejection-sampling rule."""
import json
import math
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "reference_known_answers.json")


def golden():
    with open(GOLDEN) as f:
        return json.load(f)


# Random123 known-answer vectors for philox4x32-10 (counter, key, output).
PHILOX_KAT = [
    ([0, 0, 0, 0], 0, [0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8]),
    ([0xffffffff] * 4, 0xffffffffffffffff, [0x408f276d, 0x41c83b0e, 0xa20bc7c6, 0x6d5451fd]),
    ([0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344], (0x299f31d0 << 32) | 0xa4093822,
     [0xd16cfe09, 0x94fdcceb, 0x5001e420, 0x24126ea1]),
]


@pytest.mark.parametrize("ctr,key,expect", PHILOX_KAT)
def test_philox_known_answers(oracle, ctr, key, expect):
    assert list(oracle.philox4x32_10(ctr, key)) == expect


def test_uniform_range_and_form(oracle):
    us = np.array([oracle.uniform(0, s, p, 1, 0) for s in range(64) for p in range(8)])
    assert (us > 0).all() and (us < 1).all()
    odd = us * 2 ** 24
    assert np.all(odd == np.round(odd)) and np.all(np.round(odd) % 2 == 1)


def test_exp_accuracy(oracle):
    rng = np.random.default_rng(0)
    xs = np.concatenate([-rng.uniform(0, 86.9, 20000), -rng.uniform(0, 1, 5000),
                         [0.0, -1e-30, -0.3465, -0.3466, -86.9]]).astype(np.float32)
    got = np.array([oracle.exp(float(x)) for x in xs], dtype=np.float64)
    ref = np.exp(xs.astype(np.float64))
    ulp = np.abs(got - ref) / np.spacing(ref.astype(np.float32)).astype(np.float64)
    assert ulp.max() <= 6.0
    assert oracle.exp(0.0) == 1.0
    # below -87 (and -inf) behaves as -87
    assert oracle.exp(-87.5) == oracle.exp(-87.0) == oracle.exp(float("-inf")) < 2e-38


def test_exp_polynomial_constants():
    """The committed ky_exp coefficients: c0 is 1 (so ky_exp(0) == 1), the
    fit's relative error before rounding is the stated 9.3e-8, and the fit
    restated by oracle/exp_poly.py lands within that error class."""
    import exp_poly
    c = exp_poly.committed()
    assert c[0] == 1.0
    err = exp_poly.max_rel_error(c)
    assert err < 9.4e-8
    refit = exp_poly.lawson_fit()
    assert exp_poly.max_rel_error(refit) < 1e-7
    assert max(abs(a - b) / abs(b) for a, b in zip(refit[1:], c[1:])) < 1e-3


@pytest.mark.parametrize("V,shards", [(7, 1), (2048, 1), (32000, 1), (128256, 1), (128256, 2),
                                      (128256, 8)])
def test_softmax_contract_matches_float64(oracle, V, shards):
    rng = np.random.default_rng(V + shards)
    z = (rng.standard_normal(V) * 3).astype(np.float32)
    for T in (1.0, 0.7):
        p = oracle.softmax_row(z, temperature=T, num_shards=shards)
        s = z.astype(np.float64) * np.float64(np.float32(1.0 / T))
        ref = np.exp(s - s.max())
        ref /= ref.sum()
        rel = np.abs(p - ref) / ref
        assert rel.max() < 1e-5, rel.max()


def test_reference_sample_token_cases(oracle):
    """src/worker.rs:395-457 known answers through the oracle's draft sampler
    (T <= 0 -> argmax; peaked rows at T > 0 -> the peak)."""
    for case in golden()["sample_token"]:
        if not case["logits"]:
            continue  # empty rows are rejected by argument validation here
        lg = np.array(case["logits"], dtype=np.float32)[None, None, :]
        tok, _ = oracle.sample_tokens(lg, case["temperature"], seed=0)
        t = int(tok[0, 0])
        if "expect_token" in case:
            assert t == case["expect_token"], case["name"]
        elif "expect_one_of" in case:
            assert t in case["expect_one_of"], case["name"]


def test_reference_greedy_verify_rule(oracle):
    """verify_drafts (src/speculative.rs:286-339): accept while the draft
    equals the target argmax; on the first mismatch emit the argmax and
    stop; no bonus when all match; k == 0 emits one argmax."""
    rows = [c["logits"] for c in golden()["sample_token"][:3]]
    V = 8
    tgt = np.full((1, 4, V), -1.0, dtype=np.float32)
    for j, r in enumerate(rows):
        tgt[0, j, :len(r)] = r
    tgt[0, 3, 7] = 9.0
    tops = tgt[0].argmax(-1)  # [5, 2, 2, 7]
    # all match
    acc, toks, num, _ = oracle.spec_accept(tgt, None, tops[None, :3], mode=oracle.MODE_GREEDY_REF)
    assert acc[0] == 3 and num[0] == 3 and list(toks[0, :3]) == list(tops[:3])
    # GREEDY adds the bonus argmax
    acc, toks, num, _ = oracle.spec_accept(tgt, None, tops[None, :3], mode=oracle.MODE_GREEDY)
    assert acc[0] == 3 and num[0] == 4 and toks[0, 3] == 7
    # mismatch at position 1
    drafts = np.array([[5, 3, 2]], dtype=np.int32)
    acc, toks, num, _ = oracle.spec_accept(tgt, None, drafts, mode=oracle.MODE_GREEDY_REF)
    assert acc[0] == 1 and num[0] == 2 and list(toks[0, :2]) == [5, 2]
    # k == 0
    acc, toks, num, _ = oracle.spec_accept(tgt[:, :1], None, np.zeros((1, 0), np.int32),
                                           mode=oracle.MODE_GREEDY_REF)
    assert acc[0] == 0 and num[0] == 1 and toks[0, 0] == 5


def test_stochastic_rule_emits_target_distribution(oracle):
    """Leviathan et al. 2023, Thm. 1: the first emitted token is distributed
    as p whatever q is; the acceptance rate is sum(min(p, q))."""
    V, N = 8, 200_000
    rng = np.random.default_rng(1)
    zt = (rng.standard_normal(V) * 1.5).astype(np.float32)
    zd = (zt + rng.standard_normal(V)).astype(np.float32)
    tgt = np.broadcast_to(np.stack([zt, zt])[None], (N, 2, V)).copy()
    drf = np.broadcast_to(zd[None, None], (N, 1, V)).copy()
    drafts, _ = oracle.sample_tokens(drf, 1.0, seed=7, nthreads=8)
    acc, toks, num, _ = oracle.spec_accept(tgt, drf, drafts, temperature=1.0, seed=7, nthreads=8)
    p = oracle.softmax_row(zt)
    q = oracle.softmax_row(zd)
    counts = np.bincount(toks[:, 0], minlength=V)
    expected = p * N
    chi2 = ((counts - expected) ** 2 / expected).sum()
    assert chi2 < 35.0, (chi2, counts, expected)  # dof 7: p ~ 1e-5
    rate = (acc == 1).mean()
    assert abs(rate - np.minimum(p, q).sum()) < 4 * math.sqrt(0.25 / N)


def _star_tree(n_children):
    """root (node 0) with n_children leaf children"""
    par = np.full(n_children + 1, -1, dtype=np.int32)
    par[1:] = 0
    return par


def test_tree_rule_emits_target_distribution(oracle):
    """Multi-candidate rejection sampling (SpecInfer, Miao et al. 2023): with
    children drawn i.i.d. from q, the first emitted token is distributed as
    p at the root, whatever q is -- whether a child is accepted or the final
    residual is sampled."""
    V, N, C = 8, 120_000, 4
    rng = np.random.default_rng(11)
    zt = (rng.standard_normal(V) * 1.5).astype(np.float32)
    zd = (zt + rng.standard_normal(V) * 1.5).astype(np.float32)
    nodes = C + 1
    tgt = np.broadcast_to(zt[None, None], (N, nodes, V)).copy()
    drf = np.broadcast_to(zd[None, None], (N, nodes, V)).copy()
    par = np.broadcast_to(_star_tree(C)[None], (N, nodes)).copy()
    q = oracle.softmax_row(zd)
    p = oracle.softmax_row(zt)
    tok = np.zeros((N, nodes), dtype=np.int32)
    tok[:, 1:] = rng.choice(V, size=(N, C), p=q / q.sum())
    path, plen, toks, num = oracle.spec_accept_tree(tgt, drf, tok, par, seed=5, nthreads=8)
    counts = np.bincount(toks[:, 0], minlength=V)
    expected = p * N
    chi2 = ((counts - expected) ** 2 / expected).sum()
    assert chi2 < 35.0, (chi2, counts, expected)  # dof 7: p ~ 1e-5
    # more candidates accept more often than one
    assert (plen == 2).mean() > np.minimum(p, q).sum()


def test_tree_walk_structure(oracle):
    """Paths follow parent links from the root; emitted tokens are the path's
    node tokens then one sampled token; identical models accept the first
    child at every level down to a leaf, which adds the bonus token."""
    B, V = 4, 600
    rng = np.random.default_rng(12)
    par = np.array([-1, 0, 0, 1, 1, 2, 3], dtype=np.int32)  # depth 3 along 0-1-3-6
    N = par.size
    z = (rng.standard_normal((B, N, V)) * 3).astype(np.float32)
    tok = rng.integers(0, V, size=(B, N)).astype(np.int32)
    pars = np.broadcast_to(par[None], (B, N)).copy()
    path, plen, toks, num = oracle.spec_accept_tree(z, z + 1.0, tok, pars, seed=2)
    for b in range(B):
        L = plen[b]
        assert path[b, 0] == 0 and num[b] == L
        for i in range(1, L):
            assert par[path[b, i]] == path[b, i - 1]
            assert toks[b, i - 1] == tok[b, path[b, i]]
        assert (path[b, L:] == -1).all() and (toks[b, num[b]:] == -1).all()
    # identical target and draft: every first child is accepted (p/q == 1)
    for b in range(B):
        tok[b, 1] = rng.integers(0, V)
    path, plen, toks, num = oracle.spec_accept_tree(z, z, tok, pars, seed=4)
    assert (plen == 4).all() and (path[:, :4] == [0, 1, 3, 6]).all()
    # greedy: the first child whose token is the argmax
    top0 = z[:, 0].argmax(axis=1)
    tok2 = tok.copy()
    tok2[:, 1] = (top0 + 1) % V
    tok2[:, 2] = top0
    path, plen, toks, num = oracle.spec_accept_tree(z, None, tok2, pars, mode=oracle.MODE_GREEDY)
    assert (path[:, 1] == 2).all() and (toks[:, 0] == top0).all()


def test_stochastic_identical_models_accept_everything(oracle):
    V, B, k = 64, 32, 4
    rng = np.random.default_rng(2)
    z = (rng.standard_normal((B, k + 1, V)) * 3).astype(np.float32)
    drafts, _ = oracle.sample_tokens(z[:, :k].copy(), 1.0, seed=3)
    acc, toks, num, probs = oracle.spec_accept(z, z[:, :k].copy(), drafts, seed=3)
    assert (acc == k).all() and (num == k + 1).all()
    assert np.array_equal(probs[..., 0], probs[..., 1])


def test_sharded_normaliser_is_consistent(oracle):
    """Splitting the vocabulary into TP shards changes only the grouping of
    the double-precision normaliser; decisions agree on these inputs."""
    B, k, V = 8, 4, 32000
    rng = np.random.default_rng(4)
    z = (rng.standard_normal((B, k + 1, V)) * 3).astype(np.float32)
    d = (z[:, :k] + rng.standard_normal((B, k, V))).astype(np.float32)
    drafts, _ = oracle.sample_tokens(d, 1.0, seed=0)
    r1 = oracle.spec_accept(z, d, drafts, seed=0, num_shards=1)
    r4 = oracle.spec_accept(z, d, drafts, seed=0, num_shards=4)
    assert np.array_equal(r1[0], r4[0])
    np.testing.assert_allclose(r1[3], r4[3], rtol=1e-6)


def _numpy_attention(q, kc, vc, bt, cl, bs, mask=None):
    B, nq, hq, d = q.shape
    hkv = kc.shape[1]
    g = hq // hkv
    out = np.zeros((B, nq, hq, d))
    for b in range(B):
        total = cl[b] + nq
        pos = np.arange(total)
        blocks = bt[b, pos // bs]
        K = kc[blocks, :, pos % bs, :]  # [total, hkv, d]
        Vv = vc[blocks, :, pos % bs, :]
        for j in range(nq):
            m = mask[b, j] if mask is not None else (1 << (j + 1)) - 1
            allowed = (pos < cl[b]) | (((m >> np.maximum(pos - cl[b], 0)) & 1).astype(bool) &
                                       (pos >= cl[b]))
            for h in range(hq):
                s = K[:, h // g, :] @ q[b, j, h] / math.sqrt(d)
                s = np.where(allowed, s, -np.inf)
                w = np.exp(s - s.max())
                w /= w.sum()
                out[b, j, h] = w @ Vv[:, h // g, :]
    return out


def _bf16_bits(x):
    return (np.asarray(x, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def _from_bits(b):
    return (b.astype(np.uint32) << 16).view(np.float32)


@pytest.mark.parametrize("hq,hkv,nq,tree", [(8, 2, 3, False), (4, 4, 1, False), (8, 1, 5, True)])
def test_attention_oracle_vs_numpy(oracle, hq, hkv, nq, tree):
    rng = np.random.default_rng(hq * 10 + nq)
    B, d, bs, NB = 3, 32, 16, 40
    cl = np.array([0, 17, 40], dtype=np.int64)
    maxb = 8
    bt = np.stack([rng.permutation(NB)[:maxb] for _ in range(B)]).astype(np.int64)
    qb = _bf16_bits(rng.standard_normal((B, nq, hq, d)))
    kb = _bf16_bits(rng.standard_normal((NB, hkv, bs, d)))
    vb = _bf16_bits(rng.standard_normal((NB, hkv, bs, d)))
    mask = None
    if tree:
        parent = [-1] + [int(rng.integers(0, i)) for i in range(1, nq)]
        anc = []
        for j in range(nq):
            m, n = 0, j
            while n >= 0:
                m |= 1 << n
                n = parent[n]
            anc.append(m)
        mask = np.array([anc] * B, dtype=np.uint64)
    got = oracle.paged_attention(qb, kb, vb, bt, cl, bs, tree_mask=mask)
    ref = _numpy_attention(_from_bits(qb).astype(np.float64), _from_bits(kb).astype(np.float64),
                           _from_bits(vb).astype(np.float64), bt, cl, bs,
                           None if mask is None else mask.astype(object))
    np.testing.assert_allclose(got, ref, atol=1e-5)


def test_reference_attention_cases(oracle):
    """src/model/attention_kernel.rs:163-227: shapes [1, 8, 64]; with
    all-ones K/V the output is all ones; zero context gives zeros."""
    for c in golden()["paged_attention"]:
        hq, hkv, d, bs, nb = c["num_heads"], c["num_kv_heads"], c["head_dim"], c["block_size"], \
            c["num_blocks"]
        q = _bf16_bits(np.full((1, 1, hq, d), c["fill"], np.float32))
        kc = _bf16_bits(np.full((nb, hkv, bs, d), c["fill"], np.float32))
        bt = np.zeros((1, 4), np.int64)
        ctx = c["context_len"]
        if ctx == 0:
            out = np.zeros((1, hq, d), np.float32)  # the reference's zero-context branch
        else:
            out = oracle.paged_attention(q, kc, kc, bt, np.array([ctx - 1]), bs)[:, 0]
        assert list(out.shape) == c["expect_shape"]
        np.testing.assert_allclose(out, c["expect_value"], atol=1e-6)


def _fresh_pool(n, B, maxb):
    return (np.full((B, maxb), -1, np.int64), np.zeros(B, np.int64),
            np.arange(n, dtype=np.int32), np.array([n], np.int32), np.zeros(n, np.int32))


def _prefill(bt, cl, fs, top, rc, bs, lens):
    """Give each sequence blocks for lens[b] cached tokens, popping the free
    list from the back in batch order (prompt admission)."""
    for b, n in enumerate(lens):
        for i in range(-(-n // bs)):
            top[0] -= 1
            blk = fs[top[0]]
            rc[blk] = 1
            bt[b, i] = blk
        cl[b] = n


def test_reference_block_manager_cases(oracle):
    g = golden()["block_manager"]
    c = g[0]
    bt, cl, fs, top, rc = _fresh_pool(c["num_gpu_blocks"], 1, 8)
    ok = oracle.kv_reserve(c["tokens"], bt, cl, fs, top, rc, c["block_size"])
    assert ok[0] == 1 and (bt[0] >= 0).sum() == c["expect_blocks"]
    assert top[0] == c["expect_free_after"]
    # LIFO: the first block handed out is the last one in the free list (Vec::pop)
    assert bt[0, 0] == c["num_gpu_blocks"] - 1 and rc[bt[0, 0]] == 1
    c = g[1]
    bt, cl, fs, top, rc = _fresh_pool(c["num_gpu_blocks"], 1, 8)
    ok = oracle.kv_reserve(c["tokens"], bt, cl, fs, top, rc, c["block_size"])
    assert ok[0] == 0 and top[0] == 1 and (bt < 0).all()
    c = g[2]
    bt, cl, fs, top, rc = _fresh_pool(c["num_gpu_blocks"], 2, 8)
    ok = oracle.kv_reserve(4, bt, cl, fs, top, rc, c["block_size"])
    assert ok.all() and set(bt[0][bt[0] >= 0]).isdisjoint(bt[1][bt[1] >= 0])


def test_block_manager_reserve_commit_conserves_blocks(oracle):
    rng = np.random.default_rng(5)
    n, B, maxb, bs = 200, 16, 40, 4
    bt, cl, fs, top, rc = _fresh_pool(n, B, maxb)
    fs[:] = rng.permutation(n).astype(np.int32)
    for step in range(30):
        k = int(rng.integers(1, 7))
        ok = oracle.kv_reserve(k + 1, bt, cl, fs, top, rc, bs)
        acc = np.where(ok == 1, rng.integers(0, k + 1, B), -1).astype(np.int32)
        oracle.kv_commit(k + 1, acc, bt, cl, fs, top, rc, bs)
        held = bt[bt >= 0]
        assert len(set(held.tolist())) == held.size  # no block held twice
        assert held.size + top[0] == n  # nothing lost
        assert (rc[held] == 1).all()
        for b in range(B):
            assert (bt[b] >= 0).sum() == -(-cl[b] // bs)


def test_tree_commit_moves_path_rows(oracle):
    rng = np.random.default_rng(6)
    n, B, maxb, bs, hkv, d, nodes = 64, 2, 16, 4, 2, 8, 7
    bt, cl, fs, top, rc = _fresh_pool(n, B, maxb)
    _prefill(bt, cl, fs, top, rc, bs, [5, 9])
    oracle.kv_reserve(nodes, bt, cl, fs, top, rc, bs)
    kc = [rng.integers(0, 65535, (n, hkv, bs, d), dtype=np.uint16) for _ in range(2)]
    vc = [rng.integers(0, 65535, (n, hkv, bs, d), dtype=np.uint16) for _ in range(2)]
    saved = [(k.copy(), v.copy()) for k, v in zip(kc, vc)]
    bt0, ctx0 = bt.copy(), cl.copy()
    path = np.array([[0, 2, 5, 6, 0, 0, 0], [0, 1, 0, 0, 0, 0, 0]], np.int32)
    plen = np.array([4, 2], np.int32)
    top0 = int(top[0])
    oracle.kv_commit_tree(nodes, path, plen, kc, vc, bt, cl, fs, top, rc, bs)
    assert list(cl) == [ctx0[0] + 4, ctx0[1] + 2]

    def row(cache, table, b, pos):
        return cache[table[b, pos // bs], :, pos % bs]

    for (k0, v0), k1, v1 in zip(saved, kc, vc):
        for b in range(B):
            for i in range(plen[b]):
                src, dst = ctx0[b] + path[b, i], ctx0[b] + i
                assert np.array_equal(row(k1, bt, b, dst), row(k0, bt0, b, src))
                assert np.array_equal(row(v1, bt, b, dst), row(v0, bt0, b, src))
    # blocks wholly beyond the kept length went back to the free list
    released = sum((bt0[b] >= 0).sum() - (bt[b] >= 0).sum() for b in range(B))
    assert top[0] == top0 + released


def _bf16_to_f32(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def _f32_to_bf16(x):
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def _rope_state(rng, B, n, hq, hkv, d, bs, NB):
    maxb = 64
    lens = rng.integers(0, 700, B).astype(np.int64)
    table = np.full((B, maxb), -1, np.int64)
    perm = rng.permutation(NB)
    k = 0
    for b in range(B):
        for i in range(-(-(int(lens[b]) + n) // bs)):
            table[b, i] = perm[k]
            k += 1
    bits = lambda *s: _f32_to_bf16(rng.standard_normal(s).astype(np.float32))
    return lens, table, bits(B, n, hq, d), bits(B, n, hkv, d), bits(B, n, hkv, d), maxb


def test_rope_reference_known_answer(oracle):
    """layers.rs:82-89 applies RotaryEmbedding (dim 64) to ones at index 0:
    at position 0 cos = 1 and sin = 0, so the rotation returns its input."""
    B, n, hq, hkv, d, bs, NB = 1, 1, 4, 4, 64, 16, 4
    ones = np.full((B, n, hq, d), 0x3F80, np.uint16)  # bf16 1.0
    table = np.array([[0, 1, 2, 3]], np.int64)
    kc = np.zeros((NB, hkv, bs, d), np.uint16)
    vc = np.zeros_like(kc)
    q_out = oracle.rope_kv_write(ones, ones, ones, table, np.zeros(1, np.int64), kc, vc, bs)
    assert q_out.shape == ones.shape and np.array_equal(q_out, ones)
    assert np.array_equal(kc[0, :, 0, :], ones[0, 0]) and np.array_equal(vc[0, :, 0, :], ones[0, 0])


@pytest.mark.parametrize("theta,offsets", [(10000.0, None), (500000.0, None), (10000.0, "tree")])
def test_rope_oracle_vs_float64(oracle, theta, offsets):
    """The oracle's rotation (fp32 products and sums, bf16 out) against a
    float64 evaluation of RotaryEmbedding::apply (layers.rs:37-61) at the
    same fp32 angles: within one bf16 rounding step; the paged slots hold
    the rotated keys and the unchanged values."""
    rng = np.random.default_rng(11)
    B, n, hq, hkv, d, bs, NB = 5, 6, 8, 2, 128, 16, 400
    lens, table, q, k, v, maxb = _rope_state(rng, B, n, hq, hkv, d, bs, NB)
    po = None if offsets is None else np.array([0, 1, 1, 2, 2, 2], np.int32)
    kc = np.zeros((NB, hkv, bs, d), np.uint16)
    vc = np.zeros_like(kc)
    q_out = oracle.rope_kv_write(q, k, v, table, lens, kc, vc, bs, theta=theta, pos_offsets=po)
    half = d // 2
    inv = (1.0 / np.power(np.float64(theta), 2.0 * np.arange(half) / d)).astype(np.float32)

    def rot(x_bits, b, j):
        off = j if po is None else int(po[j])
        ang = (np.float32(lens[b] + off) * inv).astype(np.float64)  # fp32 product
        c, s = np.cos(ang), np.sin(ang)
        x = _bf16_to_f32(x_bits).astype(np.float64)
        x1, x2 = x[..., :half], x[..., half:]
        return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1)

    for b in range(B):
        for j in range(n):
            want = rot(q[b, j], b, j)
            got = _bf16_to_f32(q_out[b, j]).astype(np.float64)
            assert np.all(np.abs(got - want) <= 2.0 ** -7 * np.abs(want) + 1e-6)
            pos = lens[b] + j
            blk = table[b, pos // bs]
            wk = rot(k[b, j], b, j)
            gk = _bf16_to_f32(kc[blk, :, pos % bs, :]).astype(np.float64)
            assert np.all(np.abs(gk - wk) <= 2.0 ** -7 * np.abs(wk) + 1e-6)
            assert np.array_equal(vc[blk, :, pos % bs, :], v[b, j])


def _shared_prefix_pool(rng, n, maxb, bs, hkv, d, layers):
    """Four sequences: 0 and 1 hold the same prefix blocks (ref 2, the last
    one partly filled), 2 shares only full blocks with them, 3 is private."""
    bt, cl, fs, top, rc = _fresh_pool(n, 4, maxb)
    fs[:] = rng.permutation(n).astype(np.int32)
    _prefill(bt, cl, fs, top, rc, bs, [10, 0, 0, 7])
    bt[1, :3] = bt[0, :3]
    cl[1] = 10
    bt[2, :2] = bt[0, :2]
    cl[2] = 8
    rc[bt[0, :3]] += 1
    rc[bt[0, :2]] += 1
    kc = [rng.integers(0, 65535, (n, hkv, bs, d), dtype=np.uint16) for _ in range(layers)]
    vc = [rng.integers(0, 65535, (n, hkv, bs, d), dtype=np.uint16) for _ in range(layers)]
    return bt, cl, fs, top, rc, kc, vc


def test_reserve_cow_copies_shared_tail_block(oracle):
    """Copy-on-write at a shared, partly filled last block (prefix sharing,
    block_manager.rs:60-63): sequence 0 gets a private copy (the shared
    block's ref drops to 1), so sequence 1 -- now its only holder -- keeps
    it; full shared blocks and private tails are left alone."""
    rng = np.random.default_rng(12)
    n, maxb, bs, hkv, d = 64, 16, 4, 2, 8
    bt, cl, fs, top, rc, kc, vc = _shared_prefix_pool(rng, n, maxb, bs, hkv, d, 2)
    shared = int(bt[0, 2])
    before = [(k.copy(), v.copy()) for k, v in zip(kc, vc)]
    held0 = set(bt[bt >= 0].tolist())
    top0 = int(top[0])
    ok, cow = oracle.kv_reserve_cow(3, kc, vc, bt, cl, fs, top, rc, bs)
    assert ok.tolist() == [1, 1, 1, 1]
    fresh = int(fs[top0 - 1])  # the COW block is popped first
    assert cow.tolist() == [[shared, fresh], [-1, -1], [-1, -1], [-1, -1]]
    assert bt[0, 2] == fresh and bt[1, 2] == shared and rc[shared] == 1 and rc[fresh] == 1
    for (k0, v0), k1, v1 in zip(before, kc, vc):
        assert np.array_equal(k1[fresh], k0[shared]) and np.array_equal(v1[fresh], v0[shared])
        assert np.array_equal(k1[shared], k0[shared])
    # every block is held once per reference: the table's multiset matches ref counts
    held = bt[bt >= 0]
    counts = np.bincount(held, minlength=n)
    assert (counts[held] == rc[held]).all()
    assert len(set(held.tolist()) - held0) + int(top[0]) == top0


def test_reserve_cow_out_of_blocks(oracle):
    """A sequence that cannot get its COW block and its new blocks gets
    nothing, and the shared block keeps its ref count."""
    rng = np.random.default_rng(13)
    n, maxb, bs, hkv, d = 64, 16, 4, 2, 8
    bt, cl, fs, top, rc, kc, vc = _shared_prefix_pool(rng, n, maxb, bs, hkv, d, 1)
    shared = int(bt[0, 2])
    top[0] = 1  # one free block: sequences 0 and 1 need two each (COW + one new)
    ok, cow = oracle.kv_reserve_cow(3, kc, vc, bt, cl, fs, top, rc, bs)
    assert ok.tolist() == [0, 0, 1, 0] and (cow == -1).all()
    assert rc[shared] == 2 and bt[0, 2] == shared and bt[1, 2] == shared and top[0] == 0


def test_tp_golden_fixture_matches_oracle(oracle):
    """tests/golden/tp_accept_golden.json (read by bench.py --gpus N to check
    the sharded kernels) holds exactly the oracle's outputs at 1, 2, 4 and 8
    shards."""
    import json
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import make_tp_golden as G
    with open(G.OUT) as f:
        fixture = json.load(f)
    assert [tuple(c[n] for n in ("B", "k", "V", "mode", "T", "seed")) for c in fixture["cases"]] \
        == [tuple(c) for c in G.CASES]
    for case in fixture["cases"]:
        assert case["shards"] == G.expected(oracle, case)

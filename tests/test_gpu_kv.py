"""GPU parity of KV reserve / commit / tree commit against the oracle's
BlockManager restatement: every table, length, free-list and ref-count
entry must match exactly."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _host(st):
    return {k: v.cpu().numpy().copy() for k, v in st.items()}


def _device_state(rng, NB, B, maxb, bs, lens, device):
    free = rng.permutation(NB).astype(np.int32)
    top = NB
    table = np.full((B, maxb), -1, np.int64)
    refs = np.zeros(NB, np.int32)
    for b in range(B):
        for i in range(-(-int(lens[b]) // bs)):
            top -= 1
            table[b, i] = free[top]
            refs[free[top]] = 1
    st = {"block_table": table, "context_lens": np.asarray(lens, np.int64), "free_stack": free,
          "free_top": np.array([top], np.int32), "ref_counts": refs}
    return {k: torch.from_numpy(v.copy()).to(device) for k, v in st.items()}


def _assert_same(dev, host):
    d = _host(dev)
    top = int(host["free_top"][0])
    assert int(d["free_top"][0]) == top
    assert np.array_equal(d["free_stack"][:top], host["free_stack"][:top])
    for k in ("block_table", "context_lens", "ref_counts"):
        assert np.array_equal(d[k], host[k]), k


@pytest.mark.parametrize("B,NB,bs", [(64, 16384, 16), (512, 32768, 16), (7, 300, 4), (1500, 60000, 16)])
def test_reserve_commit_matches_oracle(ctx, oracle, B, NB, bs):
    from kyro_b200.verify import kv_commit, kv_reserve
    rng = np.random.default_rng(B)
    maxb = 300
    lens = rng.integers(0, NB * bs // B, B)  # about half the pool in use
    dev = _device_state(rng, NB, B, maxb, bs, lens, ctx.device)
    host = _host(dev)
    for step in range(6):
        k = int(rng.integers(0, 9))
        ok = kv_reserve(ctx, k + 1, dev["block_table"], dev["context_lens"], dev["free_stack"],
                        dev["free_top"], dev["ref_counts"], bs)
        hok = oracle.kv_reserve(k + 1, host["block_table"], host["context_lens"],
                                host["free_stack"], host["free_top"], host["ref_counts"], bs)
        assert np.array_equal(ok.cpu().numpy(), hok)
        _assert_same(dev, host)
        acc = np.where(hok == 1, rng.integers(0, k + 1, B), -1).astype(np.int32)
        kv_commit(ctx, k + 1, torch.from_numpy(acc).to(ctx.device), dev["block_table"],
                  dev["context_lens"], dev["free_stack"], dev["free_top"], dev["ref_counts"], bs)
        oracle.kv_commit(k + 1, acc, host["block_table"], host["context_lens"],
                         host["free_stack"], host["free_top"], host["ref_counts"], bs)
        _assert_same(dev, host)
    assert ctx.device_status() == 0


def test_reserve_out_of_blocks_is_first_fit(ctx, oracle):
    from kyro_b200.verify import kv_reserve
    rng = np.random.default_rng(1)
    B, NB, bs = 40, 120, 4
    lens = rng.integers(0, 10, B)
    dev = _device_state(rng, NB, B, 64, bs, lens, ctx.device)
    host = _host(dev)
    ok = kv_reserve(ctx, 9, dev["block_table"], dev["context_lens"], dev["free_stack"],
                    dev["free_top"], dev["ref_counts"], bs)
    hok = oracle.kv_reserve(9, host["block_table"], host["context_lens"], host["free_stack"],
                            host["free_top"], host["ref_counts"], bs)
    assert not hok.all() and hok.any()
    assert np.array_equal(ok.cpu().numpy(), hok)
    _assert_same(dev, host)


def test_commit_with_shared_blocks(ctx, oracle):
    """Blocks with ref_count > 1 (prefix sharing) are decremented but stay
    allocated; the sequential path handles them exactly like the oracle."""
    from kyro_b200.verify import kv_commit, kv_reserve
    rng = np.random.default_rng(2)
    B, NB, bs = 16, 400, 4
    lens = rng.integers(1, 30, B)
    dev = _device_state(rng, NB, B, 64, bs, lens, ctx.device)
    kv_reserve(ctx, 8, dev["block_table"], dev["context_lens"], dev["free_stack"],
               dev["free_top"], dev["ref_counts"], bs)
    # share the last reserved block of sequence 0 with an extra reference
    l0 = int(dev["context_lens"][0])
    blk = int(dev["block_table"][0, -(-(l0 + 8) // bs) - 1])
    dev["ref_counts"][blk] += 1
    host = _host(dev)
    acc = torch.zeros(B, dtype=torch.int32, device=ctx.device)
    kv_commit(ctx, 8, acc, dev["block_table"], dev["context_lens"], dev["free_stack"],
              dev["free_top"], dev["ref_counts"], bs)
    oracle.kv_commit(8, acc.cpu().numpy(), host["block_table"], host["context_lens"],
                     host["free_stack"], host["free_top"], host["ref_counts"], bs)
    _assert_same(dev, host)


def test_tree_commit_matches_oracle(ctx, oracle):
    from kyro_b200.verify import kv_commit_tree, kv_reserve
    from kyro_b200.workloads import bf16_bits
    rng = np.random.default_rng(3)
    B, NB, bs, hkv, d, nodes, layers = 6, 2048, 16, 8, 128, 64, 3
    lens = rng.integers(0, 500, B)
    dev = _device_state(rng, NB, B, 64, bs, lens, ctx.device)
    kv_reserve(ctx, nodes, dev["block_table"], dev["context_lens"], dev["free_stack"],
               dev["free_top"], dev["ref_counts"], bs)
    kc = [torch.randn(NB, hkv, bs, d, device=ctx.device).to(torch.bfloat16) for _ in range(layers)]
    vc = [torch.randn(NB, hkv, bs, d, device=ctx.device).to(torch.bfloat16) for _ in range(layers)]
    # random root-to-leaf paths in a BFS-ordered tree (parent index < child index)
    parent = [-1] + [int(rng.integers(max(0, i - 6), i)) for i in range(1, nodes)]
    path = np.zeros((B, nodes), np.int32)
    plen = np.zeros(B, np.int32)
    for b in range(B):
        leaf = int(rng.integers(0, nodes))
        chain = []
        while leaf >= 0:
            chain.append(leaf)
            leaf = parent[leaf]
        chain = chain[::-1][: int(rng.integers(1, 9))]
        path[b, :len(chain)] = chain
        plen[b] = len(chain)
    host = _host(dev)
    hk = [bf16_bits(c) for c in kc]
    hv = [bf16_bits(c) for c in vc]
    kv_commit_tree(ctx, nodes, torch.from_numpy(path).to(ctx.device),
                   torch.from_numpy(plen).to(ctx.device), kc, vc, dev["block_table"],
                   dev["context_lens"], dev["free_stack"], dev["free_top"], dev["ref_counts"], bs)
    oracle.kv_commit_tree(nodes, path, plen, hk, hv, host["block_table"], host["context_lens"],
                          host["free_stack"], host["free_top"], host["ref_counts"], bs)
    _assert_same(dev, host)
    for c, h in zip(kc + vc, hk + hv):
        assert np.array_equal(bf16_bits(c), h)


def test_kv_write_matches_oracle(ctx, oracle):
    from kyro_b200.verify import kv_reserve, kv_write
    from kyro_b200.workloads import bf16_bits
    rng = np.random.default_rng(4)
    B, NB, bs, hkv, d, n = 9, 1024, 16, 8, 128, 6
    lens = rng.integers(0, 700, B)
    dev = _device_state(rng, NB, B, 64, bs, lens, ctx.device)
    kv_reserve(ctx, n, dev["block_table"], dev["context_lens"], dev["free_stack"],
               dev["free_top"], dev["ref_counts"], bs)
    kc = torch.randn(NB, hkv, bs, d, device=ctx.device).to(torch.bfloat16)
    vc = torch.randn(NB, hkv, bs, d, device=ctx.device).to(torch.bfloat16)
    kn = torch.randn(B, n, hkv, d, device=ctx.device).to(torch.bfloat16)
    vn = torch.randn(B, n, hkv, d, device=ctx.device).to(torch.bfloat16)
    hk, hv = bf16_bits(kc), bf16_bits(vc)
    kv_write(ctx, kn, vn, dev["block_table"], dev["context_lens"], kc, vc, bs)
    oracle.kv_write(bf16_bits(kn), bf16_bits(vn), dev["block_table"].cpu().numpy(),
                    dev["context_lens"].cpu().numpy(), hk, hv, bs)
    assert np.array_equal(bf16_bits(kc), hk) and np.array_equal(bf16_bits(vc), hv)


@pytest.mark.parametrize("theta,tree,inplace", [(10000.0, False, False), (500000.0, True, True)])
def test_rope_kv_write_matches_oracle(ctx, oracle, theta, tree, inplace):
    """Rotary embedding of the new tokens' q and k (layers.rs:37-61) fused with
    the paged store: q_out and both caches bit-identical to the oracle."""
    from kyro_b200.verify import kv_reserve, rope_kv_write
    from kyro_b200.workloads import bf16_bits
    rng = np.random.default_rng(5)
    B, NB, bs, hq, hkv, d, n = 9, 1024, 16, 32, 8, 128, 6
    lens = rng.integers(0, 700, B)
    dev = _device_state(rng, NB, B, 64, bs, lens, ctx.device)
    kv_reserve(ctx, n, dev["block_table"], dev["context_lens"], dev["free_stack"],
               dev["free_top"], dev["ref_counts"], bs)
    kc = torch.randn(NB, hkv, bs, d, device=ctx.device).to(torch.bfloat16)
    vc = torch.randn(NB, hkv, bs, d, device=ctx.device).to(torch.bfloat16)
    q = (torch.randn(B, n, hq, d, device=ctx.device) * 3).to(torch.bfloat16)
    kn = torch.randn(B, n, hkv, d, device=ctx.device).to(torch.bfloat16)
    vn = torch.randn(B, n, hkv, d, device=ctx.device).to(torch.bfloat16)
    offs = np.array([0, 1, 1, 2, 2, 3], np.int32) if tree else None
    hq_bits, hk, hv = bf16_bits(q), bf16_bits(kc), bf16_bits(vc)
    want_q = oracle.rope_kv_write(hq_bits, bf16_bits(kn), bf16_bits(vn),
                                  dev["block_table"].cpu().numpy(),
                                  dev["context_lens"].cpu().numpy(), hk, hv, bs, theta=theta,
                                  pos_offsets=offs)
    po = None if offs is None else torch.from_numpy(offs).to(ctx.device)
    out = rope_kv_write(ctx, q, kn, vn, dev["block_table"], dev["context_lens"], kc, vc, bs,
                        theta=theta, pos_offsets=po, q_out=q if inplace else None)
    assert ctx.device_status() == 0
    assert np.array_equal(bf16_bits(out), want_q)
    assert np.array_equal(bf16_bits(kc), hk) and np.array_equal(bf16_bits(vc), hv)


def test_rope_kv_write_position_zero_is_identity(ctx):
    """At position 0 (empty context, first token) the rotation is the identity
    (the reference's RotaryEmbedding test applies it at index 0)."""
    from kyro_b200.verify import rope_kv_write
    bs, NB, hq, hkv, d = 16, 8, 4, 4, 64
    table = torch.tensor([[0, 1]], dtype=torch.int64, device=ctx.device)
    lens = torch.zeros(1, dtype=torch.int64, device=ctx.device)
    x = torch.randn(1, 1, hq, d, device=ctx.device).to(torch.bfloat16)
    kc = torch.zeros(NB, hkv, bs, d, device=ctx.device, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    out = rope_kv_write(ctx, x, x, x, table, lens, kc, vc, bs)
    assert torch.equal(out, x) and torch.equal(kc[0, :, 0], x[0, 0]) and torch.equal(vc[0, :, 0], x[0, 0])


@pytest.mark.parametrize("B,NB,free_left", [(40, 2048, None), (1500, 60000, None), (40, 2048, 9)])
def test_reserve_cow_matches_oracle(ctx, oracle, B, NB, free_left):
    """Copy-on-write reserve against the oracle: groups of sequences share
    prefix blocks (ref count = holders), some ending in a partly filled
    block; tables, ref counts, free list, ok / cow pairs and both layers'
    caches must match exactly (one-thread tiles where a shared tail occurs,
    parallel tiles elsewhere, and a pool that runs dry)."""
    from kyro_b200.verify import kv_reserve_cow
    rng = np.random.default_rng(21)
    bs, maxb, hkv, d, n_new, layers = 16, 48, 2, 64, 6, 2
    free = rng.permutation(NB).astype(np.int32)
    top = NB
    table = np.full((B, maxb), -1, np.int64)
    refs = np.zeros(NB, np.int32)
    lens = np.zeros(B, np.int64)
    b = 0
    while b < B:
        # a group of 1..3 holders of one prefix; only some groups start in the first tile
        g = int(rng.integers(1, 4)) if (b < 1024 or B < 1024 or rng.random() < 0.02) else 1
        g = min(g, B - b)
        plen = int(rng.integers(1, 300))
        nblk = -(-plen // bs)
        blks = [free[top - 1 - i] for i in range(nblk)]
        top -= nblk
        for m in range(g):
            table[b + m, :nblk] = blks
            lens[b + m] = plen
        refs[blks] += g
        b += g
    if free_left is not None:
        top = free_left
    st = {"block_table": table, "context_lens": lens, "free_stack": free,
          "free_top": np.array([top], np.int32), "ref_counts": refs}
    dev = {k: torch.from_numpy(v.copy()).to(ctx.device) for k, v in st.items()}
    host = {k: v.copy() for k, v in st.items()}
    kc = [torch.randn(NB, hkv, bs, d, device=ctx.device).to(torch.bfloat16) for _ in range(layers)]
    vc = [torch.randn(NB, hkv, bs, d, device=ctx.device).to(torch.bfloat16) for _ in range(layers)]
    from kyro_b200.workloads import bf16_bits
    hk = [bf16_bits(t) for t in kc]
    hv = [bf16_bits(t) for t in vc]
    ok, cow = kv_reserve_cow(ctx, n_new, kc, vc, dev["block_table"], dev["context_lens"],
                             dev["free_stack"], dev["free_top"], dev["ref_counts"], bs)
    hok, hcow = oracle.kv_reserve_cow(n_new, hk, hv, host["block_table"], host["context_lens"],
                                      host["free_stack"], host["free_top"], host["ref_counts"], bs)
    assert ctx.device_status() == 0
    assert (hcow[:, 0] >= 0).any()  # the case exercises copy-on-write
    assert np.array_equal(ok.cpu().numpy(), hok) and np.array_equal(cow.cpu().numpy(), hcow)
    _assert_same(dev, host)
    for t, h in zip(kc + vc, hk + hv):
        assert np.array_equal(bf16_bits(t), h)

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

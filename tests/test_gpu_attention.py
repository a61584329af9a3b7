"""GPU parity of paged verify attention against the CPU oracle (double
precision), through the C ABI.  Bar: 2e-2 absolute (bf16 output)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ATOL = 2e-2


def _setup(ctx, hq, hkv, d, nq, ctx_lens, seed, num_blocks=4096, tree=False):
    from kyro_b200.verify import kv_reserve
    from kyro_b200.workloads import ChainConfig, paged_state
    cfg = ChainConfig(batch=len(ctx_lens), k=nq - 1, num_heads=hq, num_kv_heads=hkv,
                      head_dim=d, num_blocks=num_blocks, ctx_max=int(max(ctx_lens)),
                      headroom_tokens=128)
    st = paged_state(cfg, ctx.device, seed=seed, ctx_lens=np.array(ctx_lens), num_query=nq)
    ok = kv_reserve(ctx, nq, st.block_table, st.context_lens, st.free_stack, st.free_top,
                    st.ref_counts, cfg.block_size)
    assert bool(ok.all())
    mask = None
    if tree:
        rng = np.random.default_rng(seed)
        anc = []
        parent = [-1] + [int(rng.integers(max(0, i - 8), i)) for i in range(1, nq)]
        for j in range(nq):
            m, n = 0, j
            while n >= 0:
                m |= 1 << n
                n = parent[n]
            anc.append(m)
        mask = torch.tensor(np.array([anc] * len(ctx_lens), dtype=np.uint64).view(np.int64),
                            device=ctx.device)
    return cfg, st, mask


def _oracle(oracle, st, cfg, mask):
    from kyro_b200.workloads import bf16_bits
    m = None if mask is None else mask.cpu().numpy().view(np.uint64)
    return oracle.paged_attention(bf16_bits(st.q), bf16_bits(st.k_cache), bf16_bits(st.v_cache),
                                  st.block_table.cpu().numpy(), st.context_lens.cpu().numpy(),
                                  cfg.block_size, tree_mask=m, nthreads=8)


@pytest.mark.parametrize("hq,hkv,d,nq,lens", [
    (32, 8, 128, 6, [0, 1, 15, 16, 17, 600, 2100]),   # config-1 layer shape
    (8, 8, 128, 1, [1, 33, 300]),                     # MHA, one query
    (64, 8, 128, 8, [40, 700]),                       # 64 rows per KV head: two row groups
    (32, 8, 64, 5, [10, 500]),                        # head_dim 64
    (32, 8, 64, 1, [0, 2, 47, 48, 49, 1700]),         # head_dim 64, one query (the draft)
    (16, 2, 128, 3, [255, 256, 257]),
])
def test_chain_attention_matches_oracle(ctx, oracle, hq, hkv, d, nq, lens):
    from kyro_b200.verify import verify_attention
    cfg, st, _ = _setup(ctx, hq, hkv, d, nq, lens, seed=hq + nq)
    out = verify_attention(ctx, st.q, st.k_cache, st.v_cache, st.block_table, st.context_lens)
    ref = _oracle(oracle, st, cfg, None)
    err = (out.float().cpu().numpy() - ref)
    assert np.abs(err).max() < ATOL, np.abs(err).max()
    assert ctx.device_status() == 0


@pytest.mark.parametrize("d,split", [(128, 4), (128, 8), (128, 16), (128, 0), (64, 7), (64, 0)])
def test_split_kv_merge(ctx, oracle, d, split):
    from kyro_b200.verify import verify_attention
    cfg, st, _ = _setup(ctx, 32, 8, d, 6, [3000, 47, 1500, 4096], seed=7)
    out = verify_attention(ctx, st.q, st.k_cache, st.v_cache, st.block_table, st.context_lens,
                           kv_split_blocks=split)
    ref = _oracle(oracle, st, cfg, None)
    assert np.abs(out.float().cpu().numpy() - ref).max() < ATOL


def test_tree_mask_attention(ctx, oracle):
    from kyro_b200.verify import verify_attention
    cfg, st, mask = _setup(ctx, 64, 8, 128, 64, [300, 1000], seed=9, tree=True)
    out = verify_attention(ctx, st.q, st.k_cache, st.v_cache, st.block_table, st.context_lens,
                           tree_mask=mask)
    ref = _oracle(oracle, st, cfg, mask)
    assert np.abs(out.float().cpu().numpy() - ref).max() < ATOL


def test_reference_layout_cases(ctx):
    """src/model/attention_kernel.rs:163-227 through the PagedAttention
    mirror: shape [1, 8, 64]; all-ones K/V gives all ones; context 0 gives
    zeros."""
    from kyro_b200.attention import PagedAttention
    for hkv, ctx_len, fill in [(2, 0, 0.0), (8, 8, 1.0), (8, 24, 1.0)]:
        attn = PagedAttention(16, 8, 64, hkv, ctx=ctx)
        q = torch.full((1, 8, 64), fill, device=ctx.device)
        kc = torch.full((4, hkv, 16, 64), fill, device=ctx.device, dtype=torch.bfloat16)
        bt = torch.zeros(1, 4, dtype=torch.int64, device=ctx.device)
        cl = torch.full((1,), ctx_len, dtype=torch.int64, device=ctx.device)
        out = attn.forward(q, kc, kc, bt, cl)
        assert tuple(out.shape) == (1, 8, 64) and out.dtype == torch.float32
        assert torch.allclose(out, torch.full_like(out, fill), atol=1e-6)


def test_attention_determinism(ctx):
    from kyro_b200.verify import verify_attention
    cfg, st, _ = _setup(ctx, 32, 8, 128, 6, [1234, 88], seed=3)
    a = verify_attention(ctx, st.q, st.k_cache, st.v_cache, st.block_table, st.context_lens)
    b = verify_attention(ctx, st.q, st.k_cache, st.v_cache, st.block_table, st.context_lens)
    assert torch.equal(a, b)


def test_bad_block_id_is_flagged(ctx):
    from kyro_b200._lib import DEV_BAD_BLOCK
    from kyro_b200.verify import verify_attention
    cfg, st, _ = _setup(ctx, 32, 8, 128, 6, [100], seed=5)
    st.block_table[0, 2] = cfg.num_blocks + 7
    ctx.device_status(clear=True)
    verify_attention(ctx, st.q, st.k_cache, st.v_cache, st.block_table, st.context_lens)
    assert ctx.device_status() & DEV_BAD_BLOCK

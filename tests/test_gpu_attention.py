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


def test_split_merge_graph_replays(ctx, oracle):
    """Replays of a captured call reuse its epoch: the merging split sets the
    ticket and the other splits' ready flags back to zero, so every replay
    merges afresh (64 splits of 4 blocks on the longest sequence)."""
    from kyro_b200.verify import verify_attention
    cfg, st, _ = _setup(ctx, 32, 8, 128, 6, [3000, 47, 1500, 4096], seed=11)
    ref = _oracle(oracle, st, cfg, None)
    out = torch.empty_like(st.q)
    side = torch.cuda.Stream(ctx.device)
    try:
        with torch.cuda.stream(side):
            ctx.bind_stream()
            verify_attention(ctx, st.q, st.k_cache, st.v_cache, st.block_table, st.context_lens,
                             out=out, kv_split_blocks=4)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side):
                verify_attention(ctx, st.q, st.k_cache, st.v_cache, st.block_table,
                                 st.context_lens, out=out, kv_split_blocks=4)
        for _ in range(3):
            with torch.cuda.stream(side):
                out.zero_()
                graph.replay()
            torch.cuda.synchronize()
            assert np.abs(out.float().cpu().numpy() - ref).max() < ATOL
        del graph
    finally:
        ctx.bind_stream()
    assert ctx.device_status() == 0


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


@pytest.mark.parametrize("hq,hkv,d,nq,lens,split,tree", [
    (32, 8, 128, 6, [0, 1, 15, 16, 17, 600, 2100], 0, False),       # config-1 layer shape
    (32, 8, 128, 6, [11, 12, 13, 58, 59, 60, 61, 250], 4, False),   # new slots across block
                                                                     # and split edges
    (64, 8, 128, 8, [40, 700], 0, False),    # two row groups store the same slots
    (32, 8, 64, 5, [10, 47, 500], 3, False),  # head_dim 64
    (16, 4, 128, 6, [30, 333], 0, True),      # tree depths as positions, tree mask
])
def test_fused_rope_attention_matches_separate_launches(ctx, hq, hkv, d, nq, lens, split, tree):
    """kyro_verify_attention_rope against kyro_rope_kv_write followed by
    kyro_verify_attention on a copy of the same state: the output and both
    caches bit for bit."""
    from kyro_b200.verify import rope_kv_write, verify_attention, verify_attention_rope
    cfg, st, mask = _setup(ctx, hq, hkv, d, nq, lens, seed=hq + 7 * nq + split, tree=tree)
    g = torch.Generator(device=ctx.device).manual_seed(nq + d)
    shape = (len(lens), nq, hkv, d)
    k_new = torch.randn(shape, generator=g, device=ctx.device, dtype=torch.bfloat16)
    v_new = torch.randn(shape, generator=g, device=ctx.device, dtype=torch.bfloat16)
    pos = None
    if tree:
        depth = [bin(int(m)).count("1") - 1 for m in mask[0].cpu().numpy().view(np.uint64)]
        pos = torch.tensor(depth, dtype=torch.int32, device=ctx.device)
    theta = 500000.0
    kc, vc = st.k_cache.clone(), st.v_cache.clone()
    q_rot = rope_kv_write(ctx, st.q, k_new, v_new, st.block_table, st.context_lens, kc, vc,
                          cfg.block_size, theta=theta, pos_offsets=pos)
    ref = verify_attention(ctx, q_rot, kc, vc, st.block_table, st.context_lens, tree_mask=mask,
                           kv_split_blocks=split)
    out = verify_attention_rope(ctx, st.q, k_new, v_new, st.k_cache, st.v_cache, st.block_table,
                                st.context_lens, theta=theta, pos_offsets=pos, tree_mask=mask,
                                kv_split_blocks=split)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
    assert torch.equal(st.k_cache.view(torch.int16), kc.view(torch.int16))
    assert torch.equal(st.v_cache.view(torch.int16), vc.view(torch.int16))
    assert ctx.device_status() == 0


def test_fused_rope_rejects_tree_kernel_shapes(ctx):
    """Shapes that take the tcgen05 tree kernel are refused, not run."""
    from kyro_b200.verify import verify_attention_rope
    from kyro_b200._lib import KyroError
    cfg, st, mask = _setup(ctx, 32, 8, 128, 32, [100], seed=3, tree=True)
    k_new = torch.zeros(1, 32, 8, 128, device=ctx.device, dtype=torch.bfloat16)
    with pytest.raises(KyroError):
        verify_attention_rope(ctx, st.q, k_new, k_new, st.k_cache, st.v_cache, st.block_table,
                              st.context_lens, tree_mask=mask)

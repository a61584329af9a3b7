"""The tensor-core (tcgen05) attention path, taken when a KV head's query
rows fill 128-row tiles (draft trees), against the double-precision oracle.
Bar: 2e-2 absolute (bf16 output)."""
import numpy as np
import pytest
import torch

from test_gpu_attention import ATOL, _oracle, _setup

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("hq,hkv,nq,lens,tree", [
    (64, 8, 64, [0, 1, 127, 128, 129, 300, 1000, 2047], True),   # config-2 heads, tile edges
    (64, 8, 16, [5, 200], False),                                 # chain mask, one row tile
    (32, 8, 64, [77, 640], True),                                 # group 4: 32 nodes per tile
    (128, 8, 16, [33, 500], True),                                # group 16: 8 nodes per tile
])
def test_tensor_core_attention_matches_oracle(ctx, oracle, hq, hkv, nq, lens, tree):
    from kyro_b200.verify import verify_attention
    cfg, st, mask = _setup(ctx, hq, hkv, 128, nq, lens, seed=hq + nq + len(lens), tree=tree)
    out = verify_attention(ctx, st.q, st.k_cache, st.v_cache, st.block_table, st.context_lens,
                           tree_mask=mask)
    ref = _oracle(oracle, st, cfg, mask)
    err = np.abs(out.float().cpu().numpy() - ref)
    assert ctx.device_status() == 0
    assert err.max() < ATOL, err.max()


def test_tensor_core_attention_long_context(ctx, oracle):
    """Config-2 length: 8192 cached tokens, 65 KV tiles."""
    from kyro_b200.verify import verify_attention
    cfg, st, mask = _setup(ctx, 64, 8, 128, 64, [8192], seed=3, num_blocks=1024, tree=True)
    out = verify_attention(ctx, st.q, st.k_cache, st.v_cache, st.block_table, st.context_lens,
                           tree_mask=mask)
    ref = _oracle(oracle, st, cfg, mask)
    assert ctx.device_status() == 0
    assert np.abs(out.float().cpu().numpy() - ref).max() < ATOL

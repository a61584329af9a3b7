"""Host-side pieces of the end-to-end speculative step (config 4): the
synthetic context lengths and the block budget the bench derives from them."""
import numpy as np


def test_context_lengths_are_seeded_lognormal_and_clipped():
    from kyro_b200.e2e_model import CONFIG4, context_lengths
    a = context_lengths(CONFIG4, seed=0)
    b = context_lengths(CONFIG4, seed=0)
    assert a.dtype == np.int64 and a.shape == (CONFIG4.requests,)
    assert np.array_equal(a, b)
    assert a.min() >= 1 and a.max() <= CONFIG4.ctx_max
    # median 1024 in distribution; 512 draws land within a few percent
    assert 900 <= np.median(a) <= 1150
    assert not np.array_equal(a, context_lengths(CONFIG4, seed=1))


def test_config4_shape_matches_the_benchmark():
    from kyro_b200.e2e_model import CONFIG4, CONFIG4_SHAPE
    s = CONFIG4_SHAPE
    assert (s.layers, s.hidden, s.heads, s.kv_heads, s.head_dim, s.ffn, s.vocab) == \
        (16, 2048, 32, 8, 64, 8192, 128256)
    assert (CONFIG4.requests, CONFIG4.k, CONFIG4.temperature, CONFIG4.draft_layers) == \
        (512, 4, 0.7, 2)
    assert s.heads * s.head_dim == s.hidden and s.heads % s.kv_heads == 0

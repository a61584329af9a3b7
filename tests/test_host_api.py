"""Host-side argument checks of the Python mirrors that need no GPU."""
import pytest
import torch


def test_paged_attention_rejects_non_bf16_caches():
    """A non-bf16 cache is refused before any device work: converting it
    inside forward() would copy the whole paged cache on every call."""
    from kyro_b200.attention import PagedAttention
    attn = PagedAttention(16, 8, 64, 2)
    q = torch.zeros(1, 8, 64)
    bt = torch.zeros(1, 4, dtype=torch.int64)
    cl = torch.zeros(1, dtype=torch.int64)
    for dt in (torch.float16, torch.float32):
        kc = torch.zeros(4, 2, 16, 64, dtype=dt)
        with pytest.raises(TypeError, match="bfloat16"):
            attn.forward(q, kc, kc, bt, cl)


def test_sample_tokens_rejects_rows_that_are_not_dense():
    from kyro_b200.verify import sample_tokens

    class FakeCtx:
        device = torch.device("cpu")

    x = torch.zeros(4, 3, 10)
    with pytest.raises(ValueError, match="dense"):
        sample_tokens(FakeCtx(), x[:, :, ::2], 1.0)

"""The end-to-end speculative step (random-init Llama target + draft) on the
library's kernels: two consecutive steps on a small model, checked for the
invariants of speculative decoding.  The kernels themselves are checked
against the oracle in the other GPU tests; this covers their composition
into the step a serving loop runs (draft loop -> target verify -> accept ->
commit)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_two_spec_steps_keep_the_invariants(ctx):
    from kyro_b200.e2e_model import E2EConfig, LlamaShape, SpecModels, SpecStep, context_lengths
    from kyro_b200.verify import Context
    from kyro_b200.workloads import ChainConfig, paged_state

    dev = ctx.device
    shape = LlamaShape(layers=2, hidden=256, heads=8, kv_heads=2, head_dim=64, ffn=512,
                       vocab=4096)
    cfg = E2EConfig(requests=12, k=4, temperature=0.7, ctx_median=100, ctx_max=700,
                    draft_layers=1, kv_split_blocks=16)
    lens = context_lengths(cfg, seed=3)
    kvcfg = ChainConfig(batch=cfg.requests, k=cfg.k, num_heads=1, num_kv_heads=1, head_dim=8,
                        num_blocks=int(sum(-(-(int(c) + 64) // 16) for c in lens)) + 16,
                        ctx_min=1, ctx_max=cfg.ctx_max, headroom_tokens=64)
    kv = paged_state(kvcfg, dev, seed=5, ctx_lens=lens, num_query=1, fill_cache=False)
    models = SpecModels(shape, cfg, kvcfg.num_blocks, dev, seed=9)
    ctx_d = Context(dev.index)
    spec = SpecStep(models, ctx, ctx_d, kv, seed=0)
    free0 = int(kv.free_top.item())
    for step in range(2):
        before = kv.context_lens.clone()
        spec(step)
        torch.cuda.synchronize()
        assert int(spec.ok.min().item()) == 1  # every reserve found blocks
        acc = spec.acc.cpu().numpy()
        assert ((acc >= 0) & (acc <= cfg.k)).all()
        assert (spec.num.cpu().numpy() == acc + 1).all()
        # contexts grow by the last token plus the accepted drafts
        grown = (kv.context_lens - before).cpu().numpy()
        assert (grown == acc + 1).all()
        # accepted drafts are emitted unchanged; the next input is the last emitted token
        toks, drafts = spec.toks.cpu().numpy(), spec.drafts.cpu().numpy()
        for b in range(cfg.requests):
            assert (toks[b, :acc[b]] == drafts[b, :acc[b]]).all()
            assert spec.last[b].item() == toks[b, acc[b]]
            assert 0 <= toks[b, acc[b]] < shape.vocab
        assert torch.isfinite(spec.tgt).all() and torch.isfinite(spec.drf).all()
    # blocks held = blocks the grown contexts need
    held = kvcfg.num_blocks - int(kv.free_top.item())
    need = int(sum(-(-int(c) // 16) for c in kv.context_lens.cpu().numpy()))
    assert held == need and held >= kvcfg.num_blocks - free0
    assert ctx.device_status() == 0 and ctx_d.device_status() == 0
    ctx_d.close()

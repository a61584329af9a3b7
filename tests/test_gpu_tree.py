"""Tree acceptance on the GPU (kyro_spec_accept_tree) against the oracle's
multi-candidate rejection sampling, bit for bit: paths, path lengths,
emitted tokens."""
import numpy as np
import pytest
import torch

from kyro_b200.workloads import bfs_tree, tree_inputs

pytestmark = pytest.mark.gpu

CASES = [
    # B, N, branching, V, mode, T, seed
    (4, 21, (4, 4), 2000, 0, 1.0, 1),
    (6, 64, (4, 4, 4), 32000, 0, 1.0, 2),     # config-2 tree and vocabulary
    (3, 64, (4, 4, 4), 32000, 0, 0.7, 3),
    (4, 40, (2, 3, 3, 2), 5000, 0, 1.0, 4),   # ragged last chunk, deeper tree
    (4, 64, (4, 4, 4), 32000, 1, 1.0, 5),     # greedy
]


@pytest.mark.parametrize("B,N,br,V,mode,T,seed", CASES)
def test_tree_accept_matches_oracle(ctx, oracle, B, N, br, V, mode, T, seed):
    from kyro_b200.verify import spec_accept_tree
    par = bfs_tree(N, br)
    tgt, drf, tok = tree_inputs(B, par, V, seed=seed, temperature=T)
    pars = np.broadcast_to(par[None], (B, N)).copy()
    dev = ctx.device
    path, plen, toks, num = spec_accept_tree(
        ctx, torch.from_numpy(tgt).to(dev), torch.from_numpy(drf).to(dev) if mode == 0 else None,
        torch.from_numpy(tok).to(dev), torch.from_numpy(pars).to(dev), mode=mode,
        temperature=T, seed=seed)
    rp, rl, rt, rn = oracle.spec_accept_tree(tgt, drf, tok, pars, mode=mode, temperature=T,
                                             seed=seed, nthreads=8)
    assert ctx.device_status() == 0
    assert np.array_equal(plen.cpu().numpy(), rl)
    assert np.array_equal(path.cpu().numpy(), rp)
    assert np.array_equal(toks.cpu().numpy(), rt)
    assert np.array_equal(num.cpu().numpy(), rn)


def test_tree_identical_models_reach_a_leaf(ctx, oracle):
    """p == q: the first child is accepted at every level, ending at a leaf."""
    from kyro_b200.verify import spec_accept_tree
    B, N, V = 4, 64, 32000
    par = bfs_tree(N)
    tgt, _, tok = tree_inputs(B, par, V, seed=9)
    pars = np.broadcast_to(par[None], (B, N)).copy()
    dev = ctx.device
    t = torch.from_numpy(tgt).to(dev)
    path, plen, toks, num = spec_accept_tree(ctx, t, t, torch.from_numpy(tok).to(dev),
                                             torch.from_numpy(pars).to(dev), seed=9)
    assert (plen.cpu().numpy() == 4).all()
    assert (path.cpu().numpy()[:, :4] == [0, 1, 5, 21]).all()

"""Regenerate tests/golden/tp_accept_golden.json: the oracle's accept
decisions for vocabulary-sharded rows at 1, 2, 4 and 8 shards.

The tensor-parallel acceptance (kyro_spec_accept_tp) takes the normaliser
contract over R shards (DistributedContext::shard_dim's contiguous split,
src/distributed.rs:90-98), so its outputs are defined per shard count.  This
file holds them for a few small cases, so that `bench.py --gpus N` (which
may not run the oracle) can check the sharded kernels on the N ranks it has,
and the GPU tests can check any group size without a CPU pass.

The inputs are regenerated from the seeds by `inputs()` (numpy's PCG64, the
same bits on every machine with this numpy), so the fixture stores only the
case parameters, the drafts and the expected outputs.

    python tests/golden/make_tp_golden.py
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "tp_accept_golden.json")

# B, k, V, mode (0 stochastic, 2 the reference's greedy rule), T, seed
CASES = [
    (6, 4, 32000, 0, 0.8, 31),    # 4000 columns per rank at 8 shards: ragged chunks
    (4, 8, 128256, 0, 0.8, 32),   # config-3 rows (k 8, T 0.8, V 128256)
    (5, 3, 32000, 0, 1.0, 33),
    (4, 4, 32000, 2, 1.0, 34),
    (3, 0, 32000, 0, 1.0, 35),    # k = 0: the bonus token only
]
SHARDS = (1, 2, 4, 8)


def inputs(B: int, k: int, V: int, seed: int):
    """Target logits [B, k+1, V] ~ N(0, 3^2) and draft logits = target[:, :k]
    + N(0, 1), fp32 (the config-0 distribution)."""
    rng = np.random.default_rng(seed)
    tgt = (rng.standard_normal((B, k + 1, V), dtype=np.float32) * np.float32(3.0))
    drf = tgt[:, :k] + rng.standard_normal((B, k, V), dtype=np.float32)
    return np.ascontiguousarray(tgt), np.ascontiguousarray(drf, dtype=np.float32)


def draft_tokens(O, tgt, drf, mode, T, seed):
    """Drafts sampled from the draft rows; for the greedy rule, sequence b's
    first b mod (k+1) drafts are the target's argmax instead, so that every
    accept length from 0 to k occurs."""
    B, k = drf.shape[0], drf.shape[1]
    if k == 0:
        return np.zeros((B, 0), dtype=np.int32)
    d = O.sample_tokens(drf, T, seed=seed)[0]
    if mode != 0:
        for b in range(B):
            m = b % (k + 1)
            d[b, :m] = np.argmax(tgt[b, :m], axis=1)
    return d


def expected(O, case):
    """The oracle's outputs of one case at every shard count."""
    B, k, V, mode, T, seed = (case[n] for n in ("B", "k", "V", "mode", "T", "seed"))
    tgt, drf = inputs(B, k, V, seed)
    drafts = np.asarray(case["drafts"], dtype=np.int32).reshape(B, k)
    res = {}
    for R in SHARDS:
        acc, toks, num, probs = O.spec_accept(tgt, drf if mode == 0 else None, drafts,
                                              mode=mode, temperature=T, seed=seed,
                                              num_shards=R, nthreads=os.cpu_count() or 1)
        res[str(R)] = {
            "accept_len": acc.tolist(), "tokens": toks.tolist(), "num_tokens": num.tolist(),
            # p and q at the drafts as fp32 bit patterns
            "probs_bits": probs.view(np.uint32).tolist() if mode == 0 else None}
    return res


def main():
    sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
    import oracle as O
    O.build()
    out = {"about": "oracle outputs of kyro_spec_accept_tp cases; regenerate with "
                    "tests/golden/make_tp_golden.py", "cases": []}
    for B, k, V, mode, T, seed in CASES:
        tgt, drf = inputs(B, k, V, seed)
        drafts = draft_tokens(O, tgt, drf, mode, T, seed)
        case = {"B": B, "k": k, "V": V, "mode": mode, "T": T, "seed": seed,
                "drafts": drafts.tolist()}
        case["shards"] = expected(O, case)
        out["cases"].append(case)
    with open(OUT, "w") as f:
        json.dump(out, f, separators=(",", ":"))
    print(OUT)


if __name__ == "__main__":
    main()

"""Utterance-parallel replicas (configs 1 and 3 across GPUs: independent
utterances, weights replicated, no collective on the data path).  CPU only:

- nrp_partition_utterances assigns every utterance to exactly one rank,
  deterministically, and its longest-first greedy split stays within 4/3 of
  the best split (brute force on small batches) and near-even on config 1's
  and config 3's length distributions;
- two gloo ranks that each run their share of a batch through the oracle's
  attention (RelPositionMultiHeadAttention::forward, attention.rs:446-573)
  and all-gather the rows reproduce the single-process forward exactly.
"""
import itertools

import numpy as np
import pytest

from conftest import rand_weights
from __graft_entry__ import load_package
from test_seq_split_host import _spawn


@pytest.fixture(scope="module")
def nrp():
    return load_package()


def cost(L, d=1024):
    L = np.asarray(L, np.float64)
    return L * L + 4.0 * d / 3.0 * L


def test_partition_covers_every_utterance_once(nrp):
    rng = np.random.default_rng(1)
    for n, k in [(16, 1), (16, 2), (16, 8), (32, 8), (5, 8), (0, 3), (1, 4)]:
        ln = rng.integers(1, 751, n).astype(np.int32)
        parts, c = nrp.partition_utterances(ln, k)
        assert len(parts) == k
        got = np.sort(np.concatenate(parts)) if n else np.array([], np.int64)
        assert np.array_equal(got, np.arange(n))
        assert np.allclose([cost(ln[p]).sum() for p in parts], c)
        again, _ = nrp.partition_utterances(ln, k)
        assert all(np.array_equal(a, b) for a, b in zip(parts, again))


def test_partition_within_four_thirds_of_best(nrp):
    rng = np.random.default_rng(2)
    for _ in range(20):
        n, k = int(rng.integers(2, 9)), int(rng.integers(2, 4))
        ln = rng.integers(1, 751, n).astype(np.int32)
        _, c = nrp.partition_utterances(ln, k)
        w = cost(ln)
        best = min(max(sum(w[i] for i in range(n) if a[i] == r) for r in range(k))
                   for a in itertools.product(range(k), repeat=n))
        assert c.max() <= 4.0 / 3.0 * best + 1e-6


@pytest.mark.parametrize("B,lo,hi,k", [(16, 375, 750, 2), (16, 375, 750, 8), (32, 250, 500, 8),
                                       (256, 250, 500, 8)])
def test_partition_balances_the_bench_batches(nrp, B, lo, hi, k):
    ln = np.random.default_rng(1234).integers(lo, hi + 1, B).astype(np.int32)
    _, c = nrp.partition_utterances(ln, k)
    # the spread is at most about one utterance's cost
    assert c.max() - c.min() <= cost(hi).item() + 1e-6


def _replica_forward(rank, world, B, T, D, H, seed):
    import torch
    import torch.distributed as dist
    from __graft_entry__ import load_package
    from oracle import oracle as orc
    nrp = load_package()
    rng = np.random.default_rng(seed)
    w = rand_weights(rng, D, H, scale=0.3)
    x = rng.standard_normal((B, T, D)).astype(np.float32)
    lengths = rng.integers(1, T + 1, B).astype(np.int32)
    parts, _ = nrp.partition_utterances(lengths, world, D)
    mine = parts[rank]
    pe = orc.get_encoding(D, 5000, T)
    out = np.zeros((B, T, D), np.float32)
    if len(mine):
        out[mine] = orc.mha_forward(np.ascontiguousarray(x[mine]), w, pe, H,
                                    lengths=lengths[mine])
    # rows of other ranks are zero here: summing the replicas gathers them
    t = torch.from_numpy(out)
    dist.all_reduce(t)
    full = orc.mha_forward(x, w, pe, H, lengths=lengths)
    valid = [np.abs(t.numpy()[b, :L] - full[b, :L]).max() for b, L in enumerate(lengths)]
    return float(max(valid))


def test_two_gloo_replicas_reproduce_the_batch():
    err = _spawn(_replica_forward, 2, 7, 24, 32, 2, 5)
    assert err[0] == 0.0 and err[1] == 0.0

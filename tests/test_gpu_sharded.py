"""Vocab-sharded sampling (select per shard, merge, full-row fallback) against
the oracle on the full rows.  The shards are emulated on one GPU: the columns
of each row are split into ranges and every range goes through
noel_sampler_shard_select as its own rank would; the all-gather becomes a
stack.  Ids, RNG states and probabilities must equal sampling the full row."""
import numpy as np
import pytest

from oracle.oracle import make_config as orc_config
from tests.golden.cases import _cfg, edge_cases, workload_cases

pytestmark = pytest.mark.gpu

PROB_RTOL = 1e-5


def run_sharded(device, cfgkw, logits, hist, rng, n_shards):
    import torch

    from noel_b200 import sampler as S
    from noel_b200.sharded import sample_vocab_sharded_local, shard_bounds

    if logits.dtype == np.uint16:
        lg = torch.from_numpy(logits.view(np.int16)).view(torch.bfloat16).to(device)
    else:
        lg = torch.from_numpy(logits).to(device)
    rng_t = torch.from_numpy(np.ascontiguousarray(rng).view(np.int64)).to(device)
    h = torch.from_numpy(np.ascontiguousarray(hist, np.int32)).to(device) if hist is not None else None
    bounds = shard_bounds(logits.shape[1], n_shards)
    ids, pr, n_full = sample_vocab_sharded_local(S.make_config(**cfgkw), lg, bounds, rng_t, history=h, probs=True)
    torch.cuda.synchronize()
    return ids.cpu().numpy(), pr.cpu().numpy(), rng_t.cpu().numpy().view(np.uint64), n_full


def check(name, cfgkw, logits, hist, rng, oracle, cuda, n_shards):
    o = oracle.sample_batch(orc_config(**cfgkw), logits, history=hist, rng=rng, n_list=1)
    ids, pr, rng_out, n_full = run_sharded(cuda, cfgkw, logits, hist, rng, n_shards)
    np.testing.assert_array_equal(ids, o.ids, err_msg=f"{name}/{n_shards}: ids")
    np.testing.assert_array_equal(rng_out, o.rng, err_msg=f"{name}/{n_shards}: rng states")
    greedy = o.diag["greedy"] == 1
    np.testing.assert_allclose(pr[~greedy], o.probs[~greedy], rtol=PROB_RTOL, err_msg=f"{name}/{n_shards}: probs")
    return n_full


@pytest.mark.parametrize("n_shards", [2, 3, 8])
@pytest.mark.parametrize("case", workload_cases(batch=24), ids=lambda c: c[0])
def test_sharded_workloads_gpu(cuda, oracle, case, n_shards):
    name, cfgkw, logits, hist, rng = case
    check(name, cfgkw, logits, hist, rng, oracle, cuda, n_shards)


@pytest.mark.parametrize("n_shards", [2, 5])
@pytest.mark.parametrize("case", [c for c in edge_cases() if c[2].shape[1] >= 10],
                         ids=lambda c: c[0])
def test_sharded_edge_cases_gpu(cuda, oracle, case, n_shards):
    name, cfgkw, logits, hist, rng = case
    check(name, cfgkw, logits, hist, rng, oracle, cuda, n_shards)


def test_sharded_full_row_fallback_gpu(cuda, oracle):
    """All-equal rows tie every weight: the merge cannot decide them from the
    gathered entries and samples them from their full rows."""
    logits = np.full((6, 4000), 0.25, np.float32)
    logits[3] = np.random.Generator(np.random.PCG64(3)).standard_normal(4000).astype(np.float32)
    from noel_b200.workloads import row_states

    rng = row_states(77, np.arange(6))
    n_full = check("all_equal", _cfg(k=40), logits, None, rng, oracle, cuda, 4)
    assert n_full == 5


def test_sharded_penalty_lands_in_its_shard_gpu(cuda, oracle):
    """History ids of every shard (and outside the vocabulary) penalise the
    right columns."""
    g = np.random.Generator(np.random.PCG64(9))
    V = 9001
    logits = g.standard_normal((8, V)).astype(np.float32)
    hist = g.integers(-50, V + 50, size=(8, 300)).astype(np.int32)
    hot = g.integers(0, V, size=(8, 4))
    for b in range(8):
        logits[b, hot[b]] = 9.0
        hist[b, :40] = np.repeat(hot[b], 10)
    from noel_b200.workloads import row_states

    rng = row_states(5, np.arange(8))
    for T in (0.0, 0.9):
        check(f"penalty T={T}", _cfg(T=T, k=8, rep=1.3), logits, hist, rng, oracle, cuda, 3)


@pytest.mark.parametrize("top_k", [0, 500, 1000])
def test_sharded_full_list_gpu(cuda, oracle, top_k):
    """Top-k off or above 120: every shard lists its candidates under its own
    maximum.  Heavy-tailed rows (few candidates) are decided by the merge;
    Gaussian rows (candidates everywhere) fall back to their full rows."""
    from noel_b200.workloads import WORKLOADS, generate_numpy

    w = WORKLOADS["nucleus_bf16"].resized(batch=24, vocab=64000)
    d = generate_numpy(w, seed=41)
    cfgkw = dict(w.config_kwargs(), top_k=top_k)
    n_full = check("heavy tail", cfgkw, d["logits"], None, d["rng"], oracle, cuda, 8)
    assert n_full < 24  # most rows decided from the lists
    w2 = WORKLOADS["vocab_sharded"].resized(batch=6, vocab=16000, history=64)
    d2 = generate_numpy(w2, seed=42)
    cfg2 = dict(w2.config_kwargs(), top_k=top_k)
    check("gaussian", cfg2, d2["logits"], d2["history"], d2["rng"], oracle, cuda, 4)


def test_sharded_list_len_gpu(cuda):
    from noel_b200 import sampler as S
    from noel_b200.sharded import CudaKernels

    k = CudaKernels()
    assert k.list_len(S.make_config(temperature=0.0)) == 1
    assert k.list_len(S.make_config(top_k=64)) == 72
    assert k.list_len(S.make_config(top_k=120)) == 128
    assert k.list_len(S.make_config(top_k=0)) == 256
    assert k.list_len(S.make_config(top_k=121)) == 256

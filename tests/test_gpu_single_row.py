"""noel_sampler_sample (the reference's single-row ABI) on full-vocabulary
rows, three steps each: ids, RNG states, the drawn-from list left in
candidates, and the penalised entries written back into the caller's host
row, against the oracle and the reference's in-place penalty
(sampler.c:87-103)."""
import numpy as np
import pytest

from oracle.oracle import make_config as orc_config

pytestmark = pytest.mark.gpu


def penalised(x, hist, rep, window):
    """sampler.c:87-103 in float32, in history order."""
    x = x.copy()
    H = len(hist)
    start = H - window if 0 < window < H else 0
    for t in hist[start:]:
        if 0 <= t < len(x):
            x[t] = np.float32(x[t] / np.float32(rep)) if x[t] > 0 else np.float32(x[t] * np.float32(rep))
    return x


def rows():
    g = np.random.Generator(np.random.PCG64(21))
    V = 151936
    base = (2.0 * g.standard_normal(V)).astype(np.float32)
    base[g.integers(0, V, 8)] += 8.0
    hist = g.integers(0, V, 64).astype(np.int32)
    hist[:6] = np.argsort(base)[-6:]  # penalise some of the largest
    out = [
        ("topk40_pen", dict(temperature=0.8, top_p=0.95, top_k=40, repetition_penalty=1.1, repetition_window=0),
         base, hist),
        ("greedy_pen", dict(temperature=0.0, top_p=0.9, top_k=40, repetition_penalty=1.3, repetition_window=32),
         base, hist),
        ("topk1", dict(temperature=1.0, top_p=1.0, top_k=1, repetition_penalty=1.0, repetition_window=0), base,
         None),
        ("topk100_pen", dict(temperature=0.7, top_p=0.9, top_k=100, repetition_penalty=1.2, repetition_window=0),
         base, hist),
        ("all_equal", dict(temperature=0.8, top_p=0.9, top_k=40, repetition_penalty=1.0, repetition_window=0),
         np.full(40000, 0.5, np.float32), None),
    ]
    nan0 = base.copy()
    nan0[0] = np.nan
    out.append(("nan_at_0", dict(temperature=0.8, top_p=0.95, top_k=40, repetition_penalty=1.1,
                                 repetition_window=0), nan0, hist))
    odd = (1.5 * g.standard_normal(40003)).astype(np.float32)
    out.append(("odd_vocab", dict(temperature=0.9, top_p=0.8, top_k=20, repetition_penalty=1.1,
                                  repetition_window=0), odd, hist % 40003))
    return out


@pytest.mark.parametrize("case", rows(), ids=lambda c: c[0])
def test_single_row_matches_oracle_gpu(cuda, oracle, case):
    from noel_b200 import sampler as S

    name, cfgkw, x0, hist = case
    cfgkw = dict(cfgkw, seed=99)
    V = len(x0)
    sm = S.Sampler(S.make_config(**cfgkw), V)
    st = np.array([list(sm.rng_state)], np.uint64)
    x = x0.copy()
    for step in range(3):
        o = oracle.sample_batch(orc_config(**cfgkw), x[None].copy(), history=None if hist is None else hist[None],
                                rng=st, n_list=64)
        want_after = x if hist is None or cfgkw["repetition_penalty"] <= 1.0 else \
            penalised(x, hist, cfgkw["repetition_penalty"], cfgkw["repetition_window"])
        got = sm.sample(x, None if hist is None else hist.copy())
        assert got == o.ids[0], f"{name} step {step}"
        st = o.rng
        assert sm.rng_state == (int(st[0, 0]), int(st[0, 1]))
        np.testing.assert_array_equal(x.view(np.uint32), want_after.view(np.uint32), err_msg=f"{name}: write-back")
        if o.diag["greedy"][0] != 1:
            n = int(o.diag["n_final"][0])
            cands = sm.candidates(min(n, 64))
            assert [c[0] for c in cands] == list(o.topn_ids[0, : len(cands)])
    sm.free()


def test_single_row_host_logits_device_history_gpu(cuda, oracle):
    """Host logits with a device history: the kernel penalises the staged row
    and the whole penalised row comes back into the caller's host buffer
    (sampler.c:87-103 mutates the caller's logits)."""
    import torch

    from noel_b200 import sampler as S

    name, cfgkw, x0, hist = rows()[0]
    cfgkw = dict(cfgkw, seed=77)
    sm = S.Sampler(S.make_config(**cfgkw), len(x0))
    st = np.array([list(sm.rng_state)], np.uint64)
    x = x0.copy()
    hd = torch.from_numpy(hist.copy()).to(cuda)
    for step in range(2):
        o = oracle.sample_batch(orc_config(**cfgkw), x[None].copy(), history=hist[None], rng=st, n_list=64)
        want_after = penalised(x, hist, cfgkw["repetition_penalty"], cfgkw["repetition_window"])
        got = sm.sample(x, hd)
        assert got == o.ids[0], f"step {step}"
        st = o.rng
        assert sm.rng_state == (int(st[0, 0]), int(st[0, 1]))
        np.testing.assert_array_equal(x.view(np.uint32), want_after.view(np.uint32), err_msg="write-back")
        n = int(o.diag["n_final"][0])
        cands = sm.candidates(min(n, 64))
        assert [c[0] for c in cands] == list(o.topn_ids[0, : len(cands)])
    sm.free()

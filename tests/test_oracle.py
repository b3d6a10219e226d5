"""The oracle (oracle/sampler_oracle.c) pinned to the reference sampler.

CPU only.  Three anchors, strongest first:
1. the reference's own known answers (tests/test_engine.c:700-748),
2. the committed golden fixtures made by the reference sampler itself
   (tests/golden/make_golden.py),
3. the reference compiled from its sources here (oracle/_ref), on seeded
   inputs, when the reference tree is present.
"""
import numpy as np
import pytest

from oracle.oracle import make_config, seed_states
from tests.golden.cases import all_small_cases, edge_cases
from tests.golden.make_golden import load as load_golden


def _kat_sequence(sample):
    """test_engine.c:700-748: three checks on one sampler, seed 42, V 1000."""
    V = 1000
    logits = np.zeros((1, V), np.float32)
    rng = seed_states([42])
    cfg = make_config(temperature=0.0, top_p=0.9, top_k=40, repetition_penalty=1.0, seed=42)
    logits[0, 250], logits[0, 500], logits[0, 750] = 5.0, 10.0, 2.0
    ids, rng = sample(cfg, logits, None, rng)
    assert ids[0] == 500                                          # :714-719
    cfg.repetition_penalty = 3.0
    ids, rng = sample(cfg, logits, np.array([[500]], np.int32), rng)
    assert ids[0] == 250                                          # :721-725
    assert logits[0, 500] == np.float32(10.0) / np.float32(3.0)   # mutated in place
    logits[:] = 0
    logits[0, 10], logits[0, 20], logits[0, 30] = 4.0, 3.0, 2.0
    cfg.temperature, cfg.top_k, cfg.repetition_penalty = 0.8, 3, 1.0
    got = []
    for _ in range(20):                                           # :737-743
        ids, rng = sample(cfg, logits, None, rng)
        got.append(int(ids[0]))
    assert set(got) <= {10, 20, 30}
    return got


def test_known_answers_oracle(oracle):
    def sample(cfg, logits, hist, rng):
        r = oracle.sample_batch(cfg, logits, history=hist, rng=rng, in_place=True)
        return r.ids, r.rng

    _kat_sequence(sample)


def test_known_answers_reference_and_oracle_agree(oracle, ref_sampler):
    def s_or(cfg, logits, hist, rng):
        r = oracle.sample_batch(cfg, logits, history=hist, rng=rng, in_place=True)
        return r.ids, r.rng

    def s_ref(cfg, logits, hist, rng):
        r = ref_sampler.sample_batch(cfg, logits, history=hist, rng=rng, in_place=True)
        return r.ids, r.rng

    assert _kat_sequence(s_or) == _kat_sequence(s_ref)


def test_golden_fixtures(oracle):
    g = load_golden()
    assert len(g) >= 30
    for name, d in g.items():
        cfg = make_config(**d["cfg"])
        r = oracle.sample_batch(cfg, d["logits"], history=d["history"], rng=d["rng_in"], n_list=64)
        np.testing.assert_array_equal(r.ids, d["ids"], err_msg=name)
        np.testing.assert_array_equal(r.rng, d["rng_out"], err_msg=name)
        greedy = r.diag["greedy"] == 1
        np.testing.assert_array_equal(r.diag["num_cands"][~greedy], d["num_cands"][~greedy], err_msg=name)
        # the reference's sorted candidate list: ids and unnormalised weights
        for b in np.where(~greedy)[0]:
            n = min(int(r.diag["n_final"][b]), 64)
            np.testing.assert_array_equal(r.topn_ids[b, :n], d["cand_ids"][b, :n], err_msg=name)
            w = r.topn_probs[b, :n] * r.diag["total_mass"][b]
            np.testing.assert_allclose(w, d["cand_vals"][b, :n], rtol=2e-6, err_msg=name)


@pytest.mark.parametrize("case", [c for c in all_small_cases()], ids=lambda c: c[0])
def test_oracle_matches_reference_build(oracle, ref_sampler, case):
    name, cfgkw, logits, hist, rng = case
    cfg = make_config(**cfgkw)
    a = oracle.sample_batch(cfg, logits, history=hist, rng=rng, n_list=128)
    b = ref_sampler.sample_batch(cfg, logits, history=hist, rng=rng, n_list=128)
    np.testing.assert_array_equal(a.ids, b.ids)
    np.testing.assert_array_equal(a.rng, b.rng)
    greedy = a.diag["greedy"] == 1
    np.testing.assert_array_equal(a.diag["num_cands"][~greedy], b.num_cands[~greedy])


def test_oracle_matches_reference_full_vocab(oracle, ref_sampler):
    """Full-size rows (V = 151,936 / 152,064 / 256,000), a few per workload."""
    from noel_b200.workloads import WORKLOADS, generate_numpy

    for name in ["single_row", "greedy_penalty", "nucleus_bf16", "large_k"]:
        w = WORKLOADS[name].resized(batch=2)
        d = generate_numpy(w, seed=21)
        cfg = make_config(**w.config_kwargs())
        a = oracle.sample_batch(cfg, d["logits"], history=d["history"], rng=d["rng"])
        b = ref_sampler.sample_batch(cfg, d["logits"], history=d["history"], rng=d["rng"])
        np.testing.assert_array_equal(a.ids, b.ids, err_msg=name)
        np.testing.assert_array_equal(a.rng, b.rng, err_msg=name)


def test_qsort_ties_keep_ascending_ids(ref_sampler):
    """The oracle's (weight desc, id asc) order is the reference's qsort order
    on this libc: all-equal weights come back in ascending id order."""
    cfg = make_config(temperature=1.0, top_p=1.0, top_k=0, repetition_penalty=1.0)
    logits = np.zeros((1, 3000), np.float32)
    r = ref_sampler.sample_batch(cfg, logits, n_list=3000)
    np.testing.assert_array_equal(r.topn_ids[0], np.arange(3000))


def test_edge_cases_nonempty():
    assert len(edge_cases()) >= 25

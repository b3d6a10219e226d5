"""The pipeline-sampler oracle (oracle/aux_oracle.c) pinned to the
reference's own pipeline_stages.c (compiled into oracle/_ref): the returned
ids and the rows each call leaves behind (temperature-scaled and normalised
in place) must agree bit for bit, with the uniforms the reference draws from
rand() replayed from the same srand seed."""
import numpy as np
import pytest

from oracle.oracle import PostreqParams, RefAux, rand_uniforms


def postreq_rows(B=48, V=32000, seed=0):
    g = np.random.Generator(np.random.PCG64(seed))
    x = (g.standard_normal((B, V)) * 2.0).astype(np.float32)
    x[3, 0] = np.nan          # NaN at id 0
    x[4, :] = np.nan          # no number: id -1
    x[5, :] = -np.inf
    x[6, 100] = np.inf        # inf - inf: NaN probabilities
    x[7, :] = 0.5             # all tied
    x[8, 123] = 40.0          # one certain token
    x[9, :] = -1e9            # the grammar mask's fill value
    return x


CONFIGS = [(0.7, 0.9, 50), (1.0, 0.95, 0), (0.5, 1.0, 300), (0.0, 0.9, 50), (1.2, 0.5, 1), (0.9, 0.0, 256)]


@pytest.fixture(scope="module")
def ref_aux():
    if not RefAux.available():
        pytest.skip("oracle/_ref not built (reference sources absent)")
    return RefAux()


@pytest.mark.parametrize("T,p,k", CONFIGS)
def test_postreq_oracle_matches_reference(oracle, ref_aux, T, p, k):
    x = postreq_rows(seed=int(T * 10) + k)
    ri, rx = ref_aux.postreq_sample(x, PostreqParams(T, p, k, 1.0, 0, False), seed=77)
    u = rand_uniforms(77, x.shape[0]) if T > 1e-4 else np.zeros(x.shape[0], np.float32)
    oi, ox = oracle.postreq_sample(x, T, p, k, u)
    np.testing.assert_array_equal(oi, ri)
    np.testing.assert_array_equal(ox.view(np.uint32), rx.view(np.uint32))


def test_postreq_penalties_and_grammar_match_reference(oracle, ref_aux):
    x = postreq_rows(seed=5)
    g = np.random.Generator(np.random.PCG64(6))
    h = g.integers(-5, x.shape[1] + 5, size=(x.shape[0], 300)).astype(np.int32)
    h[:, :60] = h[:, :1]  # one id repeated: the penalty compounds per occurrence
    for window in (0, 64, 300, 1000):
        a = oracle.postreq_penalties(x, h, 1.15, window)
        b = ref_aux.postreq_penalties(x, h, 1.15, window)
        np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
    st = np.arange(x.shape[0]) % 3
    np.testing.assert_array_equal(oracle.postreq_grammar(x, st).view(np.uint32),
                                  ref_aux.postreq_grammar(x, st).view(np.uint32))

"""The MoE router oracle (oracle/aux_oracle.c) pinned to the reference's
aether_route_top_k (src/sparsity.c:46-79, compiled into oracle/_ref): its
known-answer test and seeded rows with ties, NaN, -inf, values at or below
the -1e9 slot sentinel, and fewer experts than slots must agree bit for bit."""
import numpy as np
import pytest

from oracle.oracle import Oracle, RefAux


def router_rows(T=3000, E=64, seed=0):
    g = np.random.Generator(np.random.PCG64(seed))
    x = (g.standard_normal((T, E)) * 3.0).astype(np.float32)
    c = lambda j: j % E  # columns that exist for any E
    x[::5, c(7)] = x[::5, c(2)]      # exact ties: lower id first
    x[::11, c(3)] = np.nan           # NaN never enters (sparsity.c:58)
    x[::13, c(4)] = -np.inf
    x[::17, :] = -2e9                # nothing above the sentinel: all (-1, -1e9) slots
    x[::19, c(9)] = -1e9             # equal to the sentinel: not above it
    x[::23, c(1)] = np.inf
    x[::29, :] = 0.0
    x[::29, ::2] = -0.0              # signed zeros tie
    return x


def test_router_known_answer(oracle):
    """tests/test_engine.c:128-142: top-2 of eight logits are experts 3 and 7,
    weights summing to 1."""
    x = np.array([[1.0, 5.0, 0.5, 8.0, 2.0, 3.0, 0.0, 7.0]], np.float32)
    ids, w = oracle.route_top_k(x, 2)
    assert ids.tolist() == [[3, 7]]
    assert abs(float(w.sum()) - 1.0) < 1e-5


@pytest.mark.parametrize("E,top_k", [(64, 8), (64, 2), (8, 2), (3, 8), (256, 64), (37, 1)])
def test_router_oracle_matches_reference(oracle, E, top_k):
    if not RefAux.available():
        pytest.skip("oracle/_ref not built (reference sources absent)")
    x = router_rows(E=E, seed=E + top_k)
    a = oracle.route_top_k(x, top_k)
    b = RefAux().route_top_k(x, top_k)
    np.testing.assert_array_equal(a[0], b[0])
    np.testing.assert_array_equal(a[1].view(np.uint32), b[1].view(np.uint32))

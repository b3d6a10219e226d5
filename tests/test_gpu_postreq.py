"""The pipeline's sibling sampler on the GPU (noel_postreq_*) against the
oracle (pipeline_stages.c:64-189 restated): token ids equal, the rows left
behind (probabilities) within 1e-5 relative, penalties and the grammar mask
bit-exact; and the single-row drop-in, which draws rand() itself, against the
reference's own aether_postreq_sample from the same srand seed."""
import numpy as np
import pytest

from oracle.oracle import LIBC, PostreqParams, RefAux, rand_uniforms
from tests.test_postreq import CONFIGS, postreq_rows

pytestmark = pytest.mark.gpu

P_RTOL = 1e-5


def _same(a, b):
    """bit-equal, any NaN equal to any NaN (the GPU's NaN is the canonical
    one, the host keeps a payload)"""
    nan = np.isnan(a) & np.isnan(b)
    np.testing.assert_array_equal(np.where(nan, 0, a.view(np.uint32)), np.where(nan, 0, b.view(np.uint32)))


def _close(a, b):
    nan = np.isnan(a) & np.isnan(b)
    np.testing.assert_allclose(np.where(nan, 0, a), np.where(nan, 0, b), rtol=P_RTOL, atol=1e-30)


@pytest.mark.parametrize("V", [32000, 152064, 1000])
@pytest.mark.parametrize("T,p,k", CONFIGS)
def test_postreq_batch_matches_oracle_gpu(cuda, oracle, T, p, k, V):
    import torch

    from noel_b200 import sampler as S

    x = postreq_rows(B=24, V=V, seed=V + k)
    u = rand_uniforms(5 + k, x.shape[0])
    lg = torch.from_numpy(x).to(cuda)
    ids = S.postreq_sample_batch(lg, S.postreq_params(T, p, k), torch.from_numpy(u).to(cuda))
    torch.cuda.synchronize()
    oi, ox = oracle.postreq_sample(x, T, p, k, u)
    np.testing.assert_array_equal(ids.cpu().numpy(), oi)
    _close(lg.cpu().numpy(), ox)


def test_postreq_penalties_and_grammar_gpu(cuda, oracle):
    import torch

    from noel_b200 import sampler as S

    x = postreq_rows(seed=9)
    g = np.random.Generator(np.random.PCG64(10))
    h = g.integers(-5, x.shape[1] + 5, size=(x.shape[0], 2048)).astype(np.int32)
    h[:, :200] = h[:, :1]
    for window in (0, 64, 2048):
        lg = torch.from_numpy(x).to(cuda)
        S.postreq_apply_penalties_batch(lg, torch.from_numpy(h).to(cuda), 1.15, window)
        torch.cuda.synchronize()
        _same(lg.cpu().numpy(), oracle.postreq_penalties(x, h, 1.15, window))
    st = (np.arange(x.shape[0]) % 3).astype(np.int32)
    lg = torch.from_numpy(x).to(cuda)
    S.postreq_grammar_mask_batch(lg, torch.from_numpy(st).to(cuda))
    torch.cuda.synchronize()
    _same(lg.cpu().numpy(), oracle.postreq_grammar(x, st))


def test_postreq_single_row_dropin_gpu(cuda):
    """noel_postreq_sample draws rand() itself: a sequence of calls on host
    rows equals the reference's sequence after the same srand."""
    import torch

    from noel_b200 import sampler as S

    if not RefAux.available():
        pytest.skip("oracle/_ref not built")
    ref = RefAux()
    x = postreq_rows(B=12, V=32000, seed=21)
    for T, p, k in CONFIGS:
        prm = PostreqParams(T, p, k, 1.15, 2048, False)
        ri, rx = ref.postreq_sample(x, prm, seed=1234)
        LIBC.srand(1234)
        rows = [x[b].copy() for b in range(x.shape[0])]
        gi = np.array([S.postreq_sample(r, S.postreq_params(T, p, k)) for r in rows], np.int32)
        np.testing.assert_array_equal(gi, ri)
        _close(np.stack(rows), rx)
        dev = torch.from_numpy(x[2].copy()).to(cuda)  # a device row is modified in place
        LIBC.srand(99)
        S.postreq_sample(dev, S.postreq_params(T, p, k))

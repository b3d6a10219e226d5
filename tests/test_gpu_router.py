"""The MoE router kernel (noel_moe_route_top_k) against the oracle
(sparsity.c:46-79 restated): expert ids bit-exact, weights within 1e-5
relative (the kernel uses CUDA's single-precision expf, within 2 units in
the last place of the C library's)."""
import numpy as np
import pytest

from tests.test_router import router_rows

pytestmark = pytest.mark.gpu

W_RTOL = 1e-5


@pytest.mark.parametrize("E,top_k", [(64, 8), (64, 2), (8, 2), (3, 8), (256, 64), (37, 1), (128, 32)])
def test_router_matches_oracle_gpu(cuda, oracle, E, top_k):
    import torch

    from noel_b200 import sampler as S

    x = router_rows(T=5000, E=E, seed=100 + E + top_k)
    ids, w = S.route_top_k(torch.from_numpy(x).to(cuda), top_k)
    torch.cuda.synchronize()
    oi, ow = oracle.route_top_k(x, top_k)
    np.testing.assert_array_equal(ids.cpu().numpy(), oi)
    gw = w.cpu().numpy()
    both_nan = np.isnan(gw) & np.isnan(ow)
    np.testing.assert_allclose(np.where(both_nan, 0, gw), np.where(both_nan, 0, ow), rtol=W_RTOL, atol=0)


def test_router_strided_rows_and_limits_gpu(cuda, oracle):
    import torch

    from noel_b200 import sampler as S

    x = router_rows(T=777, E=96, seed=7)
    big = torch.zeros(777, 128, device=cuda)
    big[:, :96] = torch.from_numpy(x).to(cuda)
    ids, w = S.route_top_k(big[:, :96], 8)  # row stride 128
    torch.cuda.synchronize()
    np.testing.assert_array_equal(ids.cpu().numpy(), oracle.route_top_k(x, 8)[0])
    with pytest.raises(S.NoelSamplerError):
        S.route_top_k(torch.zeros(4, 300, device=cuda), 8)   # more than 256 experts
    with pytest.raises(S.NoelSamplerError):
        S.route_top_k(torch.zeros(4, 64, device=cuda), 65)   # more than 64 slots

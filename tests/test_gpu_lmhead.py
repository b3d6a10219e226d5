"""The LM head feeding the sampler on the GPU (noel_lmhead_sample): the
logits equal the oracle's GEMV (the reference's summation order) bit for
bit, and the sampled ids, RNG states and probabilities equal the oracle
sampler's on those logits."""
import numpy as np
import pytest

from oracle.oracle import make_config as orc_config
from tests.test_lmhead import head_inputs

pytestmark = pytest.mark.gpu

PROB_RTOL = 1e-5


def _torch_weight(w, wtype, dev):
    import torch

    if wtype == 0:
        return torch.from_numpy(w).to(dev)
    t = torch.from_numpy(w.view(np.int16)).to(dev)
    return t.view(torch.bfloat16 if wtype == 30 else torch.float16)


@pytest.mark.parametrize("B", [1, 3, 8, 13])
@pytest.mark.parametrize("wtype", [0, 1, 30])
def test_lmhead_logits_and_samples_gpu(cuda, oracle, wtype, B):
    import torch

    from noel_b200 import sampler as S
    from noel_b200.workloads import row_states

    ws, x = head_inputs(rows=20000, cols=1024, B=B, seed=B * 7 + wtype)
    w = ws[wtype]
    g = np.random.Generator(np.random.PCG64(B))
    hist = g.integers(0, 20000, size=(B, 64)).astype(np.int32)
    rng = row_states(11, np.arange(B))
    cfgkw = dict(temperature=0.8, top_p=0.95, top_k=40, repetition_penalty=1.1, repetition_window=0)
    rng_t = torch.from_numpy(rng.view(np.int64).copy()).to(cuda)
    ids, logits, pr = S.lmhead_sample(_torch_weight(w, wtype, cuda), torch.from_numpy(x).to(cuda), rng_t,
                                      S.make_config(**cfgkw), history=torch.from_numpy(hist).to(cuda), probs=True)
    torch.cuda.synchronize()
    want = oracle.gemv(w, wtype, x)
    np.testing.assert_array_equal(logits.cpu().numpy().view(np.uint32), want.view(np.uint32))
    o = oracle.sample_batch(orc_config(**cfgkw), want, history=hist, rng=rng, n_list=1)
    np.testing.assert_array_equal(ids.cpu().numpy(), o.ids)
    np.testing.assert_array_equal(rng_t.cpu().numpy().view(np.uint64), o.rng)
    np.testing.assert_allclose(pr.cpu().numpy(), o.probs, rtol=PROB_RTOL)


def test_lmhead_rejects_ragged_width_gpu(cuda):
    import torch

    from noel_b200 import sampler as S

    w = torch.zeros(100, 12, device=cuda)
    rng = torch.ones(1, 2, dtype=torch.int64, device=cuda)
    with pytest.raises(S.NoelSamplerError):
        S.lmhead_sample(w, torch.zeros(1, 12, device=cuda), rng, S.make_config())

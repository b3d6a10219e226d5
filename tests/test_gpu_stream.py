"""The persistent streaming kernel: the bounded device-side waits, and rows
that cycle through both row sets of every CTA many times, against the oracle.

The failure-detection case makes no GPU fault: a 20 ms wait limit and the
stall hook (the kernel issues no row loads) make every wait run out; the
kernel returns, noel_sampler_cuda_sync_check reports NOEL_ERR_DEVICE_WAIT,
and the next call on the same context is exact again."""
import numpy as np
import pytest

from oracle.oracle import make_config as orc_config
from tests.test_gpu_parity import assert_parity, run_gpu

pytestmark = pytest.mark.gpu

NOEL_ERR_DEVICE_WAIT = -6


def test_wait_limit_reports_device_wait_gpu(cuda, oracle):
    import torch

    from noel_b200 import sampler as S
    from noel_b200.workloads import WORKLOADS, generate_numpy

    w = WORKLOADS["nucleus_bf16"].resized(batch=8, vocab=40000)
    d = generate_numpy(w, seed=5)
    cfgkw = w.config_kwargs()
    lg = torch.from_numpy(d["logits"].view(np.int16)).to(cuda).view(torch.bfloat16)
    h = None
    rng = torch.from_numpy(d["rng"].view(np.int64)).to(cuda)
    s = torch.cuda.current_stream()
    assert S.sync_check(s) == 0
    S.set_wait_limit(20_000_000, stall_next_call=True)
    try:
        S.sample_batch(lg, rng.clone(), S.make_config(**cfgkw), history=h)
        assert S.sync_check(s) == NOEL_ERR_DEVICE_WAIT
        assert S.sync_check(s) == 0  # the check clears the flag
    finally:
        S.set_wait_limit(0)
    # the context is still usable and the next call exact
    o = oracle.sample_batch(orc_config(**cfgkw), d["logits"], history=d["history"], rng=d["rng"], n_list=64)
    g = run_gpu(cuda, cfgkw, d["logits"], d["history"], d["rng"])
    assert_parity("after a stalled call", g, o)
    assert S.sync_check(s) == 0


@pytest.mark.parametrize("name", ["batch1024", "greedy_penalty", "nucleus_bf16", "large_k_small", "vocab_sharded"])
def test_many_rows_per_cta_gpu(cuda, oracle, name):
    """900 rows of a 20,000-token vocabulary: every CTA streams 6-7 rows
    back to back through one ring, alternating row sets."""
    from noel_b200.workloads import WORKLOADS, generate_numpy

    if name == "large_k_small":  # the large_k distribution, a 1024-id Zipf history, top-k 100
        w = WORKLOADS["large_k"].resized(batch=900, vocab=20000, history=1024)
        cfgkw = dict(w.config_kwargs(), top_k=100)
    else:
        w = WORKLOADS[name].resized(batch=900, vocab=20000)
        cfgkw = w.config_kwargs()
    d = generate_numpy(w, seed=23)
    o = oracle.sample_batch(orc_config(**cfgkw), d["logits"], history=d["history"], rng=d["rng"], n_list=64)
    g = run_gpu(cuda, cfgkw, d["logits"], d["history"], d["rng"])
    assert_parity(f"{name}/900x20000", g, o)

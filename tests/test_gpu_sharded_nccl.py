"""Vocab-sharded sampling across real ranks: one process per GPU (two, or up
to four when more GPUs are visible), NCCL over NVLink, each rank holding only
its columns of every row.  Every rank's ids, RNG states and probabilities
must equal the oracle's on the full rows; rows the merge cannot decide go
through the full-row gather.  Skipped with fewer than two GPUs."""
import datetime
import os
import socket

import numpy as np
import pytest

from oracle.oracle import make_config as orc_config

pytestmark = pytest.mark.gpu

PROB_RTOL = 1e-5


def _cases():
    """(name, config, logits [B, V], history or None, rng [B, 2] u64)"""
    from noel_b200.workloads import WORKLOADS, generate_numpy

    out = []
    w = WORKLOADS["vocab_sharded"].resized(batch=96, vocab=32000)
    d = generate_numpy(w, seed=61)
    out.append(("topk64", w.config_kwargs(), d["logits"], d["history"], d["rng"]))
    out.append(("greedy", dict(w.config_kwargs(), temperature=0.0), d["logits"], d["history"], d["rng"]))
    out.append(("topk500", dict(w.config_kwargs(), top_k=500), d["logits"][:8], d["history"][:8], d["rng"][:8]))
    wn = WORKLOADS["nucleus_bf16"].resized(batch=64, vocab=64000)
    dn = generate_numpy(wn, seed=62)
    out.append(("nucleus_bf16", wn.config_kwargs(), dn["logits"], None, dn["rng"]))
    eq = np.full((5, 8000), 0.5, np.float32)  # every weight ties: full-row fallback
    out.append(("all_equal", dict(w.config_kwargs(), top_k=40), eq, None, d["rng"][:5]))
    return out


def _rank_main(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist

    from noel_b200 import sampler as S
    from noel_b200.sharded import NcclGather, sample_vocab_sharded, shard_bounds

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        gather = NcclGather()
        for name, cfgkw, logits, hist, rng in _cases():
            b, wdt = shard_bounds(logits.shape[1], world)[rank]
            if logits.dtype == np.uint16:
                full = torch.from_numpy(logits.view(np.int16)).view(torch.bfloat16)
            else:
                full = torch.from_numpy(logits)
            shard = full[:, b:b + wdt].contiguous().to(dev)
            rng_t = torch.from_numpy(np.ascontiguousarray(rng).view(np.int64)).to(dev)
            h = torch.from_numpy(np.ascontiguousarray(hist, np.int32)).to(dev) if hist is not None else None
            ids, pr, n_full = sample_vocab_sharded(S.make_config(**cfgkw), shard, b, logits.shape[1], rng_t,
                                                   history=h, gather=gather, probs=True)
            torch.cuda.synchronize()
            np.savez(os.path.join(out_dir, f"{name}_r{rank}.npz"), ids=ids.cpu().numpy(), probs=pr.cpu().numpy(),
                     rng=rng_t.cpu().numpy().view(np.uint64), n_full=n_full)
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.timeout(600)
def test_vocab_sharded_nccl_ranks_gpu(oracle, tmp_path):
    import torch
    import torch.multiprocessing as mp

    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two GPUs")
    world = min(n, 4)
    env = dict(os.environ)
    os.environ["NCCL_NVLS_ENABLE"] = "0"  # plain NVLink transfers; no multicast objects
    try:
        mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                           start_method="spawn")
    finally:
        os.environ.clear()
        os.environ.update(env)
    for name, cfgkw, logits, hist, rng in _cases():
        o = oracle.sample_batch(orc_config(**cfgkw), logits, history=hist, rng=rng, n_list=1)
        greedy = o.diag["greedy"] == 1
        for r in range(world):
            g = np.load(tmp_path / f"{name}_r{r}.npz")
            np.testing.assert_array_equal(g["ids"], o.ids, err_msg=f"{name}: ids on rank {r}")
            np.testing.assert_array_equal(g["rng"], o.rng, err_msg=f"{name}: rng states on rank {r}")
            np.testing.assert_allclose(g["probs"][~greedy], o.probs[~greedy], rtol=PROB_RTOL,
                                       err_msg=f"{name}: probs on rank {r}")
        if name == "all_equal":
            assert int(g["n_full"]) == logits.shape[0]

"""The collective plumbing of vocab-sharded sampling on two gloo ranks (CPU).

The GPU kernels are replaced by small CPU stand-ins defined here (select: a
shard's top-K by (value desc, id asc) after a toy penalty, with the trailer of
its maximum; merge: the largest gathered value, leaving undecided every row
whose winner has an id divisible by 3; full row: the argmax of the full row).
What is checked is the host logic of noel_b200/sharded.py: the all-to-all of
row blocks (including a short last block), the rank-ordered all-gather of the
results, unequal shard widths, the reconstruction of the undecided rows from
every rank's columns, RNG states advanced once per row whichever path decided
it, and identical results on every rank.
"""
import os
import socket

import numpy as np
import pytest
import torch

B, V, K, H = 13, 1001, 4, 6


def _logits_history():
    g = np.random.Generator(np.random.PCG64(123))
    x = g.standard_normal((B, V)).astype(np.float32)
    hist = g.integers(0, V, size=(B, H)).astype(np.int32)
    for b in range(B):  # the row's largest value sits in its history half the time
        top = int(np.argmax(x[b]))
        if b % 2:
            hist[b, 0] = top
    return x, hist


def _penalised(x, v_begin, hist):
    x = x.copy()
    W = x.shape[1]
    for b in range(x.shape[0]):
        for t in hist[b]:
            if v_begin <= t < v_begin + W:
                x[b, t - v_begin] -= 10.0
    return x


class FakeKernels:
    def select(self, cfg, logits_shard, v_begin, history):
        x = _penalised(logits_shard.numpy(), v_begin, history.numpy())
        Bn, W = x.shape
        lists = np.full((Bn, K + 1, 2), -1, np.int32)
        for b in range(Bn):
            order = np.lexsort((np.arange(W), -x[b]))[:K]
            lists[b, : len(order), 0] = order + v_begin
            lists[b, : len(order), 1] = x[b, order].view(np.int32)
            lists[b, K, 0] = np.float32(x[b].max()).view(np.int32)
            lists[b, K, 1] = 0
        return torch.from_numpy(lists)

    def merge(self, cfg, lists, rng, probs):
        n, Bn = lists.shape[0], lists.shape[1]
        ids = torch.zeros(Bn, dtype=torch.int32)
        status = torch.zeros(Bn, dtype=torch.int32)
        e = lists.numpy()
        for b in range(Bn):
            cand = [(e[s, b, j, 1].view(np.float32), -e[s, b, j, 0]) for s in range(n) for j in range(K)
                    if e[s, b, j, 0] >= 0]
            best = -max(cand)[1]
            if best % 3 == 0:
                status[b] = 1
                continue
            ids[b] = best
            rng[b] += 1
        return ids, status, None

    def full(self, cfg, rows, rng, history, probs):
        x = _penalised(rows.numpy(), 0, history.numpy())
        rng += 1
        return torch.from_numpy(np.argmax(x, axis=1).astype(np.int32)), None


def _rank_main(rank, world, port, out_dir):
    import torch.distributed as dist

    from noel_b200.sharded import NcclGather, sample_vocab_sharded, shard_bounds

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x, hist = _logits_history()
        b, w = shard_bounds(V, world)[rank]
        rng = torch.zeros(B, 2, dtype=torch.int64)
        ids, _, n_full = sample_vocab_sharded(None, torch.from_numpy(x[:, b : b + w].copy()), b, V, rng,
                                              history=torch.from_numpy(hist), gather=NcclGather(),
                                              kernels=FakeKernels())
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), ids=ids.numpy(), rng=rng.numpy(), n_full=n_full)
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shard_bounds_cover_the_vocabulary():
    from noel_b200.sharded import shard_bounds

    for vocab, world in [(1001, 2), (256000, 8), (7, 3), (5, 5)]:
        bd = shard_bounds(vocab, world)
        assert bd[0][0] == 0 and sum(w for _, w in bd) == vocab
        assert all(bd[i][0] + bd[i][1] == bd[i + 1][0] for i in range(world - 1))
        assert max(w for _, w in bd) - min(w for _, w in bd) <= 1


@pytest.mark.timeout(300)
def test_sharded_plumbing_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp

    mp.start_processes(_rank_main, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn")
    x, hist = _logits_history()
    want = np.argmax(_penalised(x, 0, hist), axis=1)
    r0, r1 = np.load(tmp_path / "r0.npz"), np.load(tmp_path / "r1.npz")
    for r in (r0, r1):
        np.testing.assert_array_equal(r["ids"], want)
        assert (r["rng"][:, 0] == 1).all()  # one step per row, merged or full-row
        assert int(r["n_full"]) == int((want % 3 == 0).sum()) > 0

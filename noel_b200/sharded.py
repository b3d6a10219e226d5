"""Vocab-sharded sampling: the vocabulary split into column ranges, one per GPU.

The reference samples whole rows on the host (Sain-Kai/noel
src/sampler.c:80-192).  When a row's logits are produced by a vocab-parallel
LM head, each GPU holds only its columns; this module samples such rows
without moving them:

  1. ``noel_sampler_shard_select`` on every rank: per row, a list of the
     shard's best entries (global id, penalised logit) and a trailer (its
     largest penalised logit, flags);
  2. one all-to-all (NCCL over NVLink): rank r receives every shard's lists
     of its block of rows;
  3. ``noel_sampler_shard_merge`` on every rank, for its block of rows only;
  4. one all-gather of the blocks' results (ids, status, RNG states and
     optionally probabilities), so every rank holds every row's result and the
     replicated RNG states stay identical;
  5. the rare rows the merge cannot decide (a weight tie at the top-k boundary
     reaching below the gathered entries, or a full-list shard that left out
     elements within the row's cut) are gathered whole and sampled by
     ``noel_sampler_sample_batch`` on every rank.

Every rank takes the same collective steps in the same order.  Step 5 needs
the undecided-row count on the host: one 4-byte read per call.
"""
from __future__ import annotations

import ctypes as C

from . import sampler as S


class CudaKernels:
    """The library's kernels for each step (the product path)."""

    def list_len(self, cfg) -> int:
        return S.lib().noel_sampler_shard_list_len(C.byref(cfg))

    def select(self, cfg, logits_shard, v_begin: int, history=None):
        """Lists [B, L + 1, 2] int32 of the shard's columns."""
        import torch

        assert logits_shard.is_cuda and logits_shard.dim() == 2 and logits_shard.stride(1) == 1
        B, Vs = logits_shard.shape
        L = self.list_len(cfg)
        lists = torch.empty(B, L + 1, 2, dtype=torch.int32, device=logits_shard.device)
        dtype = {torch.float32: S.F32, torch.bfloat16: S.BF16}[logits_shard.dtype]
        if history is not None:
            hp, H, hld = history.data_ptr(), history.shape[1], history.stride(0)
        else:
            hp, H, hld = None, 0, 0
        s = torch.cuda.current_stream(logits_shard.device)
        S._check(S.lib().noel_sampler_shard_select(C.byref(cfg), logits_shard.data_ptr(), dtype, B, Vs,
                                                   logits_shard.stride(0), v_begin, hp, H, hld, lists.data_ptr(),
                                                   C.c_void_p(s.cuda_stream)))
        return lists

    def merge(self, cfg, lists, rng, probs: bool = False):
        """lists [n_shards, b, L + 1, 2]; rng [b, 2] int64 advanced in place."""
        import torch

        n, b = lists.shape[0], lists.shape[1]
        dev = lists.device
        assert rng.is_contiguous() and rng.shape[0] == b
        ids = torch.empty(b, dtype=torch.int32, device=dev)
        status = torch.empty(b, dtype=torch.int32, device=dev)
        pr = torch.empty(b, dtype=torch.float32, device=dev) if probs else None
        s = torch.cuda.current_stream(dev)
        S._check(S.lib().noel_sampler_shard_merge(C.byref(cfg), n, b, lists.contiguous().data_ptr(), rng.data_ptr(),
                                                  ids.data_ptr(), pr.data_ptr() if pr is not None else None,
                                                  status.data_ptr(), C.c_void_p(s.cuda_stream)))
        return ids, status, pr

    def full(self, cfg, rows, rng, history=None, probs: bool = False):
        out = S.sample_batch(rows, rng, cfg, history=history, probs=probs)
        return out["ids"], out.get("probs")


class NcclGather:
    """Rank-ordered collectives over a torch.distributed group (NCCL on GPUs)."""

    def __init__(self, group=None):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def all_gather(self, t):
        import torch

        t = t.contiguous()
        if self.dist.get_backend(self.group) == "nccl":
            out = torch.empty((self.world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
            self.dist.all_gather_into_tensor(out, t, group=self.group)
            return out
        parts = [torch.empty_like(t) for _ in range(self.world)]
        self.dist.all_gather(parts, t, group=self.group)
        return torch.stack(parts)

    def all_to_all(self, t, send_rows, recv_rows):
        """Rows of t split by send_rows go to ranks 0, 1, ...; returns the rows
        received, in rank order (recv_rows from each)."""
        import torch

        t = t.contiguous()
        out = torch.empty((sum(recv_rows),) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        self.dist.all_to_all_single(out, t, list(recv_rows), list(send_rows), group=self.group)
        return out

    def full_rows(self, logits_shard, rows, v_begin: int, vocab: int):
        """The full rows ``rows`` (same index tensor on every rank)."""
        import torch

        part = logits_shard.index_select(0, rows)
        meta = self.all_gather(torch.tensor([v_begin, part.shape[1]], dtype=torch.int64, device=part.device)).cpu()
        width = int(meta[:, 1].max())
        pad = torch.zeros(part.shape[0], width, dtype=part.dtype, device=part.device)
        pad[:, : part.shape[1]] = part
        parts = self.all_gather(pad)
        full = torch.empty(part.shape[0], vocab, dtype=part.dtype, device=part.device)
        for r in range(self.world):
            b, w = int(meta[r, 0]), int(meta[r, 1])
            full[:, b : b + w] = parts[r, :, :w]
        return full


def shard_bounds(vocab: int, world: int):
    """Contiguous, near-equal column ranges [(v_begin, width)] in rank order."""
    base, extra = divmod(vocab, world)
    out, b = [], 0
    for r in range(world):
        w = base + (1 if r < extra else 0)
        out.append((b, w))
        b += w
    return out


def _fallback(cfg, ids, pr, status, rng, history, full_rows, kernels, probs):
    """Rows with status 1, sampled from their full rows (identical on every rank)."""
    rows = status.nonzero().flatten()
    if rows.numel():
        rng_sub = rng.index_select(0, rows).contiguous()
        hist_sub = history.index_select(0, rows).contiguous() if history is not None else None
        fid, fpr = kernels.full(cfg, full_rows(rows), rng_sub, hist_sub, probs)
        ids[rows] = fid
        rng[rows] = rng_sub
        if probs:
            pr[rows] = fpr
    return int(rows.numel())


def sample_vocab_sharded(cfg, logits_shard, v_begin: int, vocab: int, rng, history=None, gather=None,
                         probs: bool = False, kernels=None):
    """Sample B rows whose columns [v_begin, v_begin + width) live on this rank.

    logits_shard [B, width] (fp32 or bf16, unit column stride); rng [B, 2]
    int64 replicated on every rank and advanced in place; history [B, H]
    int32 global ids (replicated) or None.  Returns (ids [B] int32, probs or
    None, number of rows sampled from their full rows)."""
    import torch

    kernels = kernels or CudaKernels()
    gather = gather or NcclGather()
    world, rank = gather.world, gather.rank
    B = logits_shard.shape[0]
    lists = kernels.select(cfg, logits_shard, v_begin, history)  # [B, L + 1, 2]
    nb = -(-B // world)  # rows merged per rank (the last block may be short)
    blocks = [(min(r * nb, B), min((r + 1) * nb, B)) for r in range(world)]
    r0, r1 = blocks[rank]
    mine = gather.all_to_all(lists, [e - b for b, e in blocks], [r1 - r0] * world)
    rng_mine = rng[r0:r1].contiguous()
    ids_m, status_m, pr_m = kernels.merge(cfg, mine.view(world, r1 - r0, *lists.shape[1:]), rng_mine, probs)
    # one packed row per sampled row: id, status, RNG state (4 x int32), probability bits
    cols = [ids_m.view(-1, 1), status_m.view(-1, 1), rng_mine.view(torch.int32).view(-1, 4)]
    if probs:
        cols.append(pr_m.view(torch.int32).view(-1, 1))
    packed = torch.zeros(nb, 7 if probs else 6, dtype=torch.int32, device=lists.device)
    packed[: r1 - r0] = torch.cat(cols, dim=1)
    allp = gather.all_gather(packed).view(world * nb, -1)[:B]
    ids = allp[:, 0].contiguous()
    status = allp[:, 1]
    rng.copy_(allp[:, 2:6].contiguous().view(torch.int64).view(B, 2))
    pr = allp[:, 6].contiguous().view(torch.float32) if probs else None
    n_full = _fallback(cfg, ids, pr, status, rng, history,
                       lambda rows: gather.full_rows(logits_shard, rows, v_begin, vocab), kernels, probs)
    return ids, pr, n_full


def sample_vocab_sharded_local(cfg, logits, bounds, rng, history=None, probs: bool = False, kernels=None):
    """All shards on one GPU (columns of ``logits`` split by ``bounds``): the
    same select / merge / fallback steps with the exchange replaced by a
    stack and every row merged at once, for parity tests and single-GPU use."""
    import torch

    kernels = kernels or CudaKernels()
    lists = torch.stack([kernels.select(cfg, logits[:, b : b + w], b, history) for b, w in bounds])
    ids, status, pr = kernels.merge(cfg, lists, rng, probs)
    n_full = _fallback(cfg, ids, pr, status, rng, history, lambda rows: logits.index_select(0, rows).contiguous(),
                       kernels, probs)
    return ids, pr, n_full

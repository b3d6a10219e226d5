"""Vocab-sharded sampling: the vocabulary split into column ranges, one per GPU.

The reference samples whole rows on the host (Sain-Kai/noel
src/sampler.c:80-192).  When a row's logits are produced by a vocab-parallel
LM head, each GPU holds only its columns; this module samples such rows
without moving them:

  1. ``noel_sampler_shard_select`` on every rank: per row, the shard's K best
     (global id, penalised logit), its largest penalised logit and flags;
  2. one all-gather (NCCL over NVLink) of those lists, in rank order;
  3. ``noel_sampler_shard_merge`` on every rank (identical results): the
     row's sample, equal to the reference's on the full row;
  4. the rare rows the merge cannot decide (a weight tie at the top-k boundary
     reaching below the gathered entries) are gathered whole and sampled by
     ``noel_sampler_sample_batch``.

Every rank takes the same collective steps in the same order.  The per-row
RNG states are replicated on every rank and advance identically.
"""
from __future__ import annotations

import ctypes as C

from . import sampler as S


class CudaKernels:
    """The library's kernels for each step (the product path)."""

    def kprime(self, cfg) -> int:
        return S.lib().noel_sampler_shard_kprime(C.byref(cfg))

    def select(self, cfg, logits_shard, v_begin: int, history=None):
        import torch

        assert logits_shard.is_cuda and logits_shard.dim() == 2 and logits_shard.stride(1) == 1
        B, Vs = logits_shard.shape
        K = self.kprime(cfg)
        if K <= 0:
            raise S.NoelSamplerError(-3, "vocab-sharded sampling needs greedy or 0 < top_k <= 120")
        dev = logits_shard.device
        entries = torch.empty(B, K, 2, dtype=torch.int32, device=dev)
        maxes = torch.empty(B, dtype=torch.float32, device=dev)
        flags = torch.empty(B, dtype=torch.int32, device=dev)
        dtype = {torch.float32: S.F32, torch.bfloat16: S.BF16}[logits_shard.dtype]
        if history is not None:
            hp, H, hld = history.data_ptr(), history.shape[1], history.stride(0)
        else:
            hp, H, hld = None, 0, 0
        s = torch.cuda.current_stream(dev)
        S._check(S.lib().noel_sampler_shard_select(C.byref(cfg), logits_shard.data_ptr(), dtype, B, Vs,
                                                   logits_shard.stride(0), v_begin, hp, H, hld,
                                                   entries.data_ptr(), maxes.data_ptr(), flags.data_ptr(),
                                                   C.c_void_p(s.cuda_stream)))
        return entries, maxes, flags

    def merge(self, cfg, entries, maxes, flags, rng, probs: bool = False):
        import torch

        n, B = maxes.shape
        dev = maxes.device
        ids = torch.empty(B, dtype=torch.int32, device=dev)
        status = torch.empty(B, dtype=torch.int32, device=dev)
        pr = torch.empty(B, dtype=torch.float32, device=dev) if probs else None
        s = torch.cuda.current_stream(dev)
        S._check(S.lib().noel_sampler_shard_merge(C.byref(cfg), n, B, entries.data_ptr(), maxes.data_ptr(),
                                                  flags.data_ptr(), rng.data_ptr(), ids.data_ptr(),
                                                  pr.data_ptr() if pr is not None else None, status.data_ptr(),
                                                  C.c_void_p(s.cuda_stream)))
        return ids, status, pr

    def full(self, cfg, rows, rng, history=None, probs: bool = False):
        out = S.sample_batch(rows, rng, cfg, history=history, probs=probs)
        return out["ids"], out.get("probs")


class NcclGather:
    """Rank-ordered all-gathers over a torch.distributed group (NCCL on GPUs)."""

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


def _finish(cfg, entries, maxes, flags, rng, history, full_rows, kernels, probs):
    ids, status, pr = kernels.merge(cfg, entries, maxes, flags, rng, probs)
    rows = status.nonzero().flatten()
    if rows.numel():  # identical on every rank: the merge is deterministic
        rng_sub = rng.index_select(0, rows).contiguous()
        hist_sub = history.index_select(0, rows).contiguous() if history is not None else None
        fid, fpr = kernels.full(cfg, full_rows(rows), rng_sub, hist_sub, probs)
        ids[rows] = fid
        rng[rows] = rng_sub
        if probs:
            pr[rows] = fpr
    return ids, pr, int(rows.numel())


def sample_vocab_sharded(cfg, logits_shard, v_begin: int, vocab: int, rng, history=None, gather=None,
                         probs: bool = False, kernels=None):
    """Sample B rows whose columns [v_begin, v_begin + width) live on this rank.

    logits_shard [B, width] (fp32 or bf16, unit column stride); rng [B, 2]
    int64 replicated on every rank and advanced in place; history [B, H]
    int32 global ids (replicated) or None.  Returns (ids [B] int32, probs or
    None, number of rows sampled from their full rows)."""
    kernels = kernels or CudaKernels()
    gather = gather or NcclGather()
    e, m, f = kernels.select(cfg, logits_shard, v_begin, history)
    E, M, F = gather.all_gather(e), gather.all_gather(m), gather.all_gather(f)
    return _finish(cfg, E, M, F, rng, history, lambda rows: gather.full_rows(logits_shard, rows, v_begin, vocab),
                   kernels, probs)


def sample_vocab_sharded_local(cfg, logits, bounds, rng, history=None, probs: bool = False, kernels=None):
    """All shards on one GPU (columns of ``logits`` split by ``bounds``): the
    same select / merge / fallback steps with the all-gather replaced by a
    stack, for parity tests and single-GPU use."""
    import torch

    kernels = kernels or CudaKernels()
    parts = [kernels.select(cfg, logits[:, b : b + w], b, history) for b, w in bounds]
    E = torch.stack([p[0] for p in parts])
    M = torch.stack([p[1] for p in parts])
    F = torch.stack([p[2] for p in parts])
    return _finish(cfg, E, M, F, rng, history, lambda rows: logits.index_select(0, rows).contiguous(), kernels,
                   probs)

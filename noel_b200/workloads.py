"""Seeded synthetic sampling workloads (logits rows, histories, parameters).

The shapes, value distributions and sampling parameters are the named
workloads of this path; there is no dataset behind them.  Two generators
produce the same distributions: numpy (``PCG64``; used for parity cases and
fixtures, exactly reproducible on any host) and torch on the device (used by
the benchmark, whose inputs are too large to build on the host every run).

Workloads (B rows x V vocab):

* ``single_row``      B=1,    V=151936 fp32 N(0,2^2), 8 ids +8.0; H=64 uniform;
                      rep 1.1, T 0.8, top-k 40, top-p 0.95
* ``greedy_penalty``  B=256,  V=152064 fp32 N(0,3^2); H=1024 Zipf(1.1);
                      rep 1.2, T 1.0, top-k 1, top-p 1.0
* ``nucleus_bf16``    B=1024, V=256000 bf16 2.5*Student-t(3); no penalty;
                      T 1.0, top-k off, top-p 0.9
* ``vocab_sharded``   B=4096, V=256000 fp32 N(0,2^2) as 8 shards of 32000;
                      H=256 uniform; rep 1.1, T 0.7, top-k 64, top-p 0.9
* ``large_k``         B=8192, V=152064 fp32 mixture 0.95 N(0,1.5^2) + 0.05
                      N(6,1); H=4096 Zipf(1.0); rep 1.05, T 0.9, top-k 1000,
                      top-p 0.98 (batch-sharded)
* ``batch1024``       B=1024, V=152064 fp32 with the single_row distribution
                      and parameters: the throughput workload.

Histories are token ids; a Zipf(s) history draws ranks r in [1, V] from the
finite law P(r) ~ r^-s (s = 1.0 has no numpy sampler, so both exponents use
the explicit CDF) and maps rank r to id r-1.  Row b's RNG state is the
reference seeding of seed = seed_base + b + 1 (never 0).
"""
from __future__ import annotations

from dataclasses import dataclass, field, replace

import numpy as np


@dataclass(frozen=True)
class Workload:
    name: str
    batch: int
    vocab: int
    dtype: str                  # "f32" | "bf16"
    dist: str                   # "normal" | "student_t" | "mixture"
    scale: float
    boost_ids: int = 0          # ids per row raised by boost_value
    boost_value: float = 8.0
    history: int = 0
    history_dist: str = "uniform"   # "uniform" | "zipf"
    zipf_s: float = 1.0
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = 0
    repetition_penalty: float = 1.0
    repetition_window: int = 0
    shards: int = 1
    extra: dict = field(default_factory=dict)

    def config_kwargs(self) -> dict:
        return dict(temperature=self.temperature, top_p=self.top_p, top_k=self.top_k,
                    repetition_penalty=self.repetition_penalty,
                    repetition_window=self.repetition_window, seed=0)

    def resized(self, batch: int | None = None, vocab: int | None = None,
                history: int | None = None) -> "Workload":
        return replace(self, batch=self.batch if batch is None else batch,
                       vocab=self.vocab if vocab is None else vocab,
                       history=self.history if history is None else history)

    def bytes_per_row(self) -> int:
        """Algorithmic HBM bytes per row: the row once, the history ids,
        the RNG state in and out (16 B), the sampled id and probability (8 B)."""
        el = 4 if self.dtype == "f32" else 2
        return self.vocab * el + 4 * self.history + 24


WORKLOADS = {
    "single_row": Workload("single_row", 1, 151936, "f32", "normal", 2.0, boost_ids=8,
                           history=64, temperature=0.8, top_p=0.95, top_k=40,
                           repetition_penalty=1.1),
    "greedy_penalty": Workload("greedy_penalty", 256, 152064, "f32", "normal", 3.0,
                               history=1024, history_dist="zipf", zipf_s=1.1,
                               temperature=1.0, top_p=1.0, top_k=1, repetition_penalty=1.2),
    "nucleus_bf16": Workload("nucleus_bf16", 1024, 256000, "bf16", "student_t", 2.5,
                             temperature=1.0, top_p=0.9, top_k=0),
    "vocab_sharded": Workload("vocab_sharded", 4096, 256000, "f32", "normal", 2.0,
                              history=256, temperature=0.7, top_p=0.9, top_k=64,
                              repetition_penalty=1.1, shards=8),
    "large_k": Workload("large_k", 8192, 152064, "f32", "mixture", 1.5, history=4096,
                        history_dist="zipf", zipf_s=1.0, temperature=0.9, top_p=0.98,
                        top_k=1000, repetition_penalty=1.05),
    "batch1024": Workload("batch1024", 1024, 152064, "f32", "normal", 2.0, boost_ids=8,
                          history=64, temperature=0.8, top_p=0.95, top_k=40,
                          repetition_penalty=1.1),
}


def _zipf_cdf(V: int, s: float) -> np.ndarray:
    w = np.arange(1, V + 1, dtype=np.float64) ** (-s)
    c = np.cumsum(w)
    return c / c[-1]


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16, returned as uint16 bit patterns."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = np.isnan(x)
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def row_states(seed_base: int, rows) -> np.ndarray:
    """Reference seeding (sampler.c:42-47) of seed = seed_base + row + 1."""
    seeds = np.asarray(rows, dtype=np.uint64) + np.uint64(seed_base + 1)
    st = np.empty((seeds.size, 2), dtype=np.uint64)
    st[:, 0] = seeds
    st[:, 1] = seeds ^ np.uint64(0x9E3779B97F4A7C15)
    return st


def generate_numpy(w: Workload, seed: int = 0, row0: int = 0, rows: int | None = None):
    """Rows [row0, row0+rows) of the workload, reproducible per row.

    Returns dict(logits=[rows, V] float32 or uint16 (bf16 bits),
    history=[rows, H] int32 or None, rng=[rows, 2] uint64).
    """
    rows = w.batch if rows is None else rows
    V = w.vocab
    logits = np.empty((rows, V), np.float32)
    hist = np.empty((rows, w.history), np.int32) if w.history else None
    cdf = _zipf_cdf(V, w.zipf_s) if (w.history and w.history_dist == "zipf") else None
    for i in range(rows):
        g = np.random.Generator(np.random.PCG64([seed, row0 + i]))
        if w.dist == "normal":
            x = g.standard_normal(V, dtype=np.float32) * np.float32(w.scale)
        elif w.dist == "student_t":
            x = (g.standard_t(3, V) * w.scale).astype(np.float32)
        elif w.dist == "mixture":
            hi = g.random(V) < 0.05
            x = np.where(hi, 6.0 + g.standard_normal(V), 1.5 * g.standard_normal(V)).astype(np.float32)
        else:
            raise ValueError(w.dist)
        if w.boost_ids:
            b = g.choice(V, size=w.boost_ids, replace=False)
            x[b] += np.float32(w.boost_value)
        logits[i] = x
        if hist is not None:
            if w.history_dist == "zipf":
                hist[i] = np.searchsorted(cdf, g.random(w.history), side="right").clip(0, V - 1)
            else:
                hist[i] = g.integers(0, V, size=w.history)
    if w.dtype == "bf16":
        logits = f32_to_bf16_bits(logits)
    return dict(logits=logits, history=hist, rng=row_states(seed, np.arange(row0, row0 + rows)))


def generate_torch(w: Workload, device, seed: int = 0, rows: int | None = None, row0: int = 0):
    """Device-side generator with the same distributions (not the same values
    as ``generate_numpy``).  Returns dict of torch tensors on ``device``."""
    import torch

    rows = w.batch if rows is None else rows
    V = w.vocab
    g = torch.Generator(device=device)
    g.manual_seed(seed * 1000003 + row0)
    if w.dist == "normal":
        x = torch.randn(rows, V, generator=g, device=device) * w.scale
    elif w.dist == "student_t":
        # Student-t(3) = N / sqrt(chi2_3 / 3), chi2_3 = sum of 3 squared normals
        n = torch.randn(rows, V, generator=g, device=device)
        c = torch.randn(3, rows, V, generator=g, device=device).square_().sum(0)
        x = n / torch.sqrt(c / 3.0) * w.scale
        del n, c
    elif w.dist == "mixture":
        hi = torch.rand(rows, V, generator=g, device=device) < 0.05
        a = torch.randn(rows, V, generator=g, device=device)
        x = torch.where(hi, 6.0 + a, 1.5 * a)
        del hi, a
    else:
        raise ValueError(w.dist)
    if w.boost_ids:
        idx = torch.argsort(torch.rand(rows, V, generator=g, device=device), dim=1)[:, : w.boost_ids]
        x.scatter_add_(1, idx, torch.full(idx.shape, w.boost_value, device=device))
    hist = None
    if w.history:
        if w.history_dist == "zipf":
            cdf = torch.from_numpy(_zipf_cdf(V, w.zipf_s)).to(device)
            u = torch.rand(rows, w.history, generator=g, device=device, dtype=torch.float64)
            hist = torch.searchsorted(cdf, u, right=True).clamp_(0, V - 1).to(torch.int32)
        else:
            hist = torch.randint(0, V, (rows, w.history), generator=g, device=device, dtype=torch.int32)
    x = x.to(torch.bfloat16) if w.dtype == "bf16" else x.float()
    rng = torch.from_numpy(row_states(seed, np.arange(row0, row0 + rows)).view(np.int64)).to(device)
    return dict(logits=x.contiguous(), history=hist, rng=rng)

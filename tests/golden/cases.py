"""Parity cases shared by the golden-fixture generator and the tests.

Each case is (name, config kwargs, logits [B, V] float32 or uint16-bf16,
history [B, H] int32 or None, rng [B, 2] uint64).  Workload cases are the
named workloads shrunk in batch (and vocab where marked); the edge cases
cover what the reference's sampler has to handle: the known answers of its
own test (tests/test_engine.c:700-748), NaN / +-inf logits, all-equal rows,
top-k >= vocab, top-p at 0 and 1, the greedy threshold, history ids outside
[0, V), duplicate-heavy histories, a window shorter than the history, V = 1,
exact ties at the top-k boundary, and weights that collapse to equal values.
"""
from __future__ import annotations

import numpy as np

from noel_b200.workloads import WORKLOADS, generate_numpy, row_states


def _cfg(T=0.8, p=0.95, k=40, rep=1.1, window=0):
    return dict(temperature=T, top_p=p, top_k=k, repetition_penalty=rep, repetition_window=window, seed=0)


def workload_cases(batch=4, vocab_small=None, seed=11):
    out = []
    for name in ["single_row", "greedy_penalty", "nucleus_bf16", "vocab_sharded", "large_k", "batch1024"]:
        w = WORKLOADS[name].resized(batch=min(batch, WORKLOADS[name].batch),
                                    vocab=vocab_small if vocab_small else None)
        if vocab_small and w.history:
            w = w.resized(history=min(w.history, 4 * vocab_small))
        d = generate_numpy(w, seed=seed)
        out.append((f"wl_{name}", w.config_kwargs(), d["logits"], d["history"], d["rng"]))
    return out


def edge_cases(seed=5):
    g = np.random.Generator(np.random.PCG64(seed))
    cases = []

    def add(name, cfg, logits, hist=None, rows=None):
        logits = np.ascontiguousarray(logits)
        B = logits.shape[0]
        cases.append((name, cfg, logits, None if hist is None else np.ascontiguousarray(hist, np.int32),
                      row_states(seed * 1000 + len(cases), np.arange(B))))

    V = 1000
    z = np.zeros((1, V), np.float32)
    z[0, 250], z[0, 500], z[0, 750] = 5.0, 10.0, 2.0
    add("kat_greedy", _cfg(T=0.0, p=0.9, k=40, rep=1.0), z)
    z2 = z.copy()
    add("kat_penalty", _cfg(T=0.0, p=0.9, k=40, rep=3.0), z2, np.array([[500]]))
    z3 = np.zeros((4, V), np.float32)
    z3[:, 10], z3[:, 20], z3[:, 30] = 4.0, 3.0, 2.0
    add("kat_topk3", _cfg(T=0.8, p=0.9, k=3, rep=1.0), z3)

    add("all_equal", _cfg(T=0.8, p=0.9, k=40), np.full((3, 257), 1.5, np.float32))
    add("all_equal_full", _cfg(T=0.8, p=0.5, k=0), np.full((2, 300), -2.0, np.float32))
    x = g.standard_normal((3, 777)).astype(np.float32)
    x[:, 0] = np.nan
    add("nan_at_0", _cfg(), x)
    x = g.standard_normal((3, 777)).astype(np.float32)
    x[:, [3, 100, 500]] = np.nan
    add("nan_inside", _cfg(k=0, p=0.9), x)
    x = g.standard_normal((2, 600)).astype(np.float32)
    x[:, 7] = np.inf
    add("pos_inf", _cfg(), x)
    add("all_neg_inf", _cfg(), np.full((2, 64), -np.inf, np.float32))
    x = g.standard_normal((2, 600)).astype(np.float32)
    x[:, 9] = -np.inf
    add("neg_inf_one", _cfg(k=0, p=1.0), x)
    add("topk_ge_vocab", _cfg(k=5000, p=0.9), g.standard_normal((3, 1000)).astype(np.float32) * 3)
    add("topp_zero", _cfg(k=50, p=0.0), g.standard_normal((3, 1000)).astype(np.float32) * 2)
    add("topp_one", _cfg(k=50, p=1.0), g.standard_normal((3, 1000)).astype(np.float32) * 2)
    add("temp_at_greedy_edge", _cfg(T=1e-4, k=40), g.standard_normal((3, 1000)).astype(np.float32))
    add("temp_above_greedy_edge", _cfg(T=1.0001e-4, k=40), g.standard_normal((3, 1000)).astype(np.float32))
    add("temp_negative", _cfg(T=-1.0), g.standard_normal((2, 1000)).astype(np.float32))
    h = np.array([[-5, 1000, 1003, 3, 3, 3, 7, 2 ** 31 - 1, -2 ** 31]] * 2, np.int32)
    add("hist_out_of_range", _cfg(rep=1.3), g.standard_normal((2, 1000)).astype(np.float32) * 2, h)
    x = g.standard_normal((3, 2000)).astype(np.float32) * 2
    hh = np.repeat(np.argmax(x, axis=1)[:, None], 64, axis=1).astype(np.int32)
    add("hist_one_id_x64", _cfg(rep=1.2), x, hh)
    add("window_8_of_32", _cfg(rep=1.5, window=8), g.standard_normal((3, 500)).astype(np.float32) * 2,
        g.integers(0, 500, (3, 32)))
    add("window_ge_history", _cfg(rep=1.5, window=64), g.standard_normal((2, 500)).astype(np.float32) * 2,
        g.integers(0, 500, (2, 32)))
    add("penalty_le_one", _cfg(rep=1.0), g.standard_normal((2, 500)).astype(np.float32),
        g.integers(0, 500, (2, 32)))
    add("vocab_1", _cfg(), g.standard_normal((3, 1)).astype(np.float32))
    add("vocab_1_greedy", _cfg(T=0.0), g.standard_normal((2, 1)).astype(np.float32))
    x = np.round(g.standard_normal((3, 3000)) * 4).astype(np.float32)  # many exact ties
    add("ties_at_boundary", _cfg(k=40, p=0.95), x)
    add("ties_at_boundary_k1", _cfg(k=1, p=1.0, T=1.0), x)
    base = np.float32(0.01)
    x = np.full((2, 4000), -30.0, np.float32)
    x[:, ::97] = base - np.arange(x[:, ::97].shape[1], dtype=np.float32) * np.float32(1e-9)
    add("weights_collapse", _cfg(k=8, p=0.99, T=1.0), x)
    add("ascending_row", _cfg(k=40, p=0.9), np.tile(np.linspace(-5, 5, 5000, dtype=np.float32), (2, 1)))
    add("descending_row", _cfg(k=40, p=0.9), np.tile(np.linspace(5, -5, 5000, dtype=np.float32), (2, 1)))
    add("flat_full_many", _cfg(k=0, p=0.9, T=2.0), g.standard_normal((2, 6000)).astype(np.float32) * 0.5)
    add("negative_zero", _cfg(k=4, p=1.0, T=1.0),
        np.array([[-0.0, 0.0, -0.0, 0.0, -1.0, -0.0]], np.float32))
    add("large_k_small_vocab", _cfg(k=1000, p=0.98, T=0.9), g.standard_normal((2, 3000)).astype(np.float32))
    return cases


def all_small_cases():
    return workload_cases(batch=4, vocab_small=4096) + edge_cases()

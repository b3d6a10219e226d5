"""Parity of the CUDA path with the oracle and the reference's golden fixtures.

Every call goes through the C ABI of libnoel_sampler_cuda.so.  The bar:
sampled ids, RNG states, list lengths and the drawn-from list are
bit-exact; probabilities agree within 1e-5 relative (they are computed with
the reference's own fp32 operations, so they are in fact exact).
"""
import numpy as np
import pytest

from oracle.oracle import make_config as orc_config
from tests.golden.cases import edge_cases, workload_cases
from tests.golden.make_golden import load as load_golden

pytestmark = pytest.mark.gpu

PROB_RTOL = 1e-5


def _to_torch(logits, device, ld=None):
    import torch

    B, V = logits.shape
    ld = V if ld is None else ld
    if logits.dtype == np.uint16:
        buf = np.zeros((B, ld), np.uint16)
        buf[:, :V] = logits
        t = torch.from_numpy(buf.view(np.int16)).view(torch.bfloat16).to(device)
    else:
        buf = np.zeros((B, ld), np.float32)
        buf[:, :V] = logits
        t = torch.from_numpy(buf).to(device)
    return t[:, :V]


def run_gpu(device, cfgkw, logits, hist, rng, list_len=64, ld=None, write_back=False):
    import torch

    from noel_b200 import sampler as S

    lg = _to_torch(logits, device, ld)
    rng_t = torch.from_numpy(np.ascontiguousarray(rng).view(np.int64)).to(device)
    h = torch.from_numpy(np.ascontiguousarray(hist, np.int32)).to(device) if hist is not None else None
    out = S.sample_batch(lg, rng_t, S.make_config(**cfgkw), history=h, probs=True, list_len=list_len,
                         stats=True, write_back=write_back)
    torch.cuda.synchronize()
    res = {k: v.cpu().numpy() for k, v in out.items()}
    res["rng"] = rng_t.cpu().numpy().view(np.uint64)
    res["logits_after"] = lg
    return res


def assert_parity(name, g, o, list_len=64):
    """g: GPU result dict; o: oracle BatchResult (n_list >= list_len)."""
    np.testing.assert_array_equal(g["ids"], o.ids, err_msg=f"{name}: ids")
    np.testing.assert_array_equal(g["rng"], o.rng, err_msg=f"{name}: rng states")
    greedy = o.diag["greedy"] == 1
    st = g["stats"]
    np.testing.assert_array_equal(st[~greedy, 1], o.diag["n_topk"][~greedy], err_msg=f"{name}: n_topk")
    np.testing.assert_array_equal(st[~greedy, 2], o.diag["n_final"][~greedy], err_msg=f"{name}: n_final")
    known = (~greedy) & (st[:, 0] >= 0)
    np.testing.assert_array_equal(st[known, 0], o.diag["num_cands"][known], err_msg=f"{name}: num_cands")
    np.testing.assert_allclose(g["probs"][~greedy], o.probs[~greedy], rtol=PROB_RTOL, err_msg=f"{name}: probs")
    for b in np.where(~greedy)[0]:
        n = min(int(o.diag["n_final"][b]), list_len)
        np.testing.assert_array_equal(g["list_ids"][b, :n], o.topn_ids[b, :n], err_msg=f"{name}: list row {b}")
        np.testing.assert_allclose(g["list_probs"][b, :n], o.topn_probs[b, :n], rtol=PROB_RTOL,
                                   err_msg=f"{name}: list probs row {b}")
        assert (g["list_ids"][b, n:] == -1).all() or n == list_len


def test_golden_fixtures_gpu(cuda):
    g = load_golden()
    for name, d in g.items():
        r = run_gpu(cuda, d["cfg"], d["logits"], d["history"], d["rng_in"])
        np.testing.assert_array_equal(r["ids"], d["ids"], err_msg=name)
        np.testing.assert_array_equal(r["rng"], d["rng_out"], err_msg=name)
        st = r["stats"]
        greedy = (st[:, 3] & 1) == 1
        known = (~greedy) & (st[:, 0] >= 0)
        np.testing.assert_array_equal(st[known, 0], d["num_cands"][known], err_msg=name)
        for b in np.where(~greedy)[0]:
            n = min(int(st[b, 2]), 64)
            np.testing.assert_array_equal(r["list_ids"][b, :n], d["cand_ids"][b, :n], err_msg=name)


@pytest.mark.parametrize("case", edge_cases(), ids=lambda c: c[0])
def test_edge_cases_gpu(cuda, oracle, case):
    name, cfgkw, logits, hist, rng = case
    o = oracle.sample_batch(orc_config(**cfgkw), logits, history=hist, rng=rng, n_list=64)
    g = run_gpu(cuda, cfgkw, logits, hist, rng)
    assert_parity(name, g, o)


@pytest.mark.parametrize("case", workload_cases(batch=48), ids=lambda c: c[0])
def test_workloads_full_vocab_gpu(cuda, oracle, case):
    """Named workloads at their full vocab (151,936 / 152,064 / 256,000)."""
    name, cfgkw, logits, hist, rng = case
    o = oracle.sample_batch(orc_config(**cfgkw), logits, history=hist, rng=rng, n_list=64)
    g = run_gpu(cuda, cfgkw, logits, hist, rng)
    assert_parity(name, g, o)


@pytest.mark.parametrize("name,batch", [("batch1024", 1024), ("batch1024", 560), ("greedy_penalty", 560),
                                        ("nucleus_bf16", 560)])
def test_workloads_full_occupancy_gpu(cuda, oracle, name, batch):
    """Batches that give every CTA of the streaming kernel several rows, so
    both row sets of each CTA are reused; 1024 rows is the throughput
    workload itself."""
    from noel_b200.workloads import WORKLOADS, generate_numpy

    w = WORKLOADS[name].resized(batch=batch)
    d = generate_numpy(w, seed=13)
    cfgkw = w.config_kwargs()
    o = oracle.sample_batch(orc_config(**cfgkw), d["logits"], history=d["history"], rng=d["rng"], n_list=64)
    g = run_gpu(cuda, cfgkw, d["logits"], d["history"], d["rng"])
    assert_parity(f"{name}/{batch}", g, o)


@pytest.mark.parametrize("top_k,T", [(500, 0.9), (40, 0.8), (1, 0.0), (0, 1.0)])
def test_heavy_penalty_gpu(cuda, oracle, top_k, T):
    """Histories that repeat the row's largest ids ten times or more (each
    occurrence divides again, sampler.c:96-100), so the penalty moves most of
    the row's top entries below the rest: greedy, top-k in the single-pass and
    block kernels, and the full list."""
    from noel_b200.workloads import row_states

    g = np.random.Generator(np.random.PCG64(31))
    B, V = 6, 30000
    logits = (2.0 * g.standard_normal((B, V))).astype(np.float32)
    hist = np.zeros((B, 3900), np.int32)
    for b in range(B):
        top = np.argsort(-logits[b])[:1200]
        hist[b] = np.concatenate([np.repeat(top[:300], 10), top[300:1200]])
        g.shuffle(hist[b])
    logits[:, 0] = np.abs(logits[:, 0]) + 30.0  # id 0: large raw value, in every window 10 times
    hist[:, :10] = 0
    cfgkw = dict(temperature=T, top_p=0.95, top_k=top_k, repetition_penalty=3.0, repetition_window=0, seed=0)
    rng = row_states(17, np.arange(B))
    o = oracle.sample_batch(orc_config(**cfgkw), logits, history=hist, rng=rng, n_list=64)
    r = run_gpu(cuda, cfgkw, logits, hist, rng)
    assert_parity(f"heavy_penalty k={top_k} T={T}", r, o)


@pytest.mark.parametrize("pad", [1, 3, 7])
def test_unaligned_rows_gpu(cuda, oracle, pad):
    """Row stride ld = V + pad puts every row at a different alignment."""
    for name, cfgkw, logits, hist, rng in workload_cases(batch=6, vocab_small=5003):
        o = oracle.sample_batch(orc_config(**cfgkw), logits, history=hist, rng=rng, n_list=64)
        g = run_gpu(cuda, cfgkw, logits, hist, rng, ld=logits.shape[1] + pad)
        assert_parity(f"{name}+{pad}", g, o)


def test_write_back_gpu(cuda, oracle):
    """The penalised entries land in the caller's fp32 logits (sampler.c:96-100)."""
    for name, cfgkw, logits, hist, rng in workload_cases(batch=4, vocab_small=8192):
        if hist is None or logits.dtype != np.float32 or cfgkw["repetition_penalty"] <= 1.0:
            continue
        mutated = logits.copy()
        o = oracle.sample_batch(orc_config(**cfgkw), mutated, history=hist, rng=rng, n_list=64, in_place=True)
        g = run_gpu(cuda, cfgkw, logits, hist, rng, write_back=True)
        assert_parity(name, g, o)
        after = g["logits_after"].cpu().numpy()
        np.testing.assert_array_equal(after, mutated, err_msg=f"{name}: written-back logits")


def test_exact_pass_rows_gpu(cuda, oracle):
    """Rows the single-pass kernel hands on to the two-pass kernel: a candidate
    set larger than shared memory (top-k off, flat logits) and ties at the
    top-k boundary."""
    rng_np = np.random.Generator(np.random.PCG64(7))
    from noel_b200.workloads import row_states

    flat = (rng_np.standard_normal((6, 60000)) * 0.5).astype(np.float32)
    cfgkw = dict(temperature=1.0, top_p=0.9, top_k=0, repetition_penalty=1.0, repetition_window=0, seed=0)
    st = row_states(3, np.arange(6))
    o = oracle.sample_batch(orc_config(**cfgkw), flat, rng=st, n_list=64)
    g = run_gpu(cuda, cfgkw, flat, None, st)
    assert (g["stats"][:, 3] & 2).all(), "expected the two-pass kernel"
    assert_parity("flat_full", g, o)

    ties = np.round(rng_np.standard_normal((6, 30000)) * 2).astype(np.float32)
    cfgkw = dict(temperature=1.0, top_p=0.95, top_k=50, repetition_penalty=1.0, repetition_window=0, seed=0)
    o = oracle.sample_batch(orc_config(**cfgkw), ties, rng=st, n_list=64)
    g = run_gpu(cuda, cfgkw, ties, None, st)
    assert_parity("ties", g, o)


def _warm_sample_vectors(V, f32, wide, block):
    """Vector indices the warm-up sample reads in a row starting on a 32-byte
    boundary: the single-pass kernel's 4 warps x 32 lanes x U slots, or the
    block kernel's (top-k above 120) 256 threads x U slots, spread evenly
    over the row's 32-byte vectors."""
    if block:
        ns = 256 * (4 if f32 else 2)
    else:
        ns = 4 * 32 * (2 if f32 else 1) * (4 if wide else 1)
    nvec = V // (8 if f32 else 16)
    return np.arange(ns, dtype=np.int64) * nvec // ns


@pytest.mark.parametrize("B,dtype,top_k", [(6, "f32", 40), (300, "f32", 40), (6, "bf16", 40), (300, "bf16", 40),
                                           (6, "f32", 500), (6, "bf16", 500)])
def test_warm_filter_bet_lost_gpu(cuda, oracle, B, dtype, top_k):
    """The single-pass and block kernels start a top-k row with a filter at a
    rank below K' of a sample spread over the row.  Rows whose largest
    elements all lie on the sampled vectors leave fewer than K' elements
    above it; they must go to the two-pass kernel and still match the
    oracle."""
    from noel_b200.workloads import f32_to_bf16_bits, row_states

    V = 32768
    f32 = dtype == "f32"
    g = np.random.Generator(np.random.PCG64(11))
    x = g.standard_normal((B, V)).astype(np.float32)
    vec = 8 if f32 else 16
    vi = _warm_sample_vectors(V, f32, wide=B <= 296, block=top_k > 120)
    cols = (vi[:, None] * vec + np.arange(vec)[None, :]).ravel()
    x[:, cols] += 10.0
    hist = np.concatenate([cols[g.integers(0, cols.size, (B, 16))], g.integers(0, V, (B, 16))], axis=1)
    hist = hist.astype(np.int32)
    logits = x if f32 else f32_to_bf16_bits(x)
    cfgkw = dict(temperature=0.8, top_p=0.95, top_k=top_k, repetition_penalty=1.3, repetition_window=32, seed=0)
    st = row_states(5, np.arange(B))
    o = oracle.sample_batch(orc_config(**cfgkw), logits, history=hist, rng=st, n_list=64)
    r = run_gpu(cuda, cfgkw, logits, hist, st)
    assert (r["stats"][:, 3] & 2).all(), "expected every row in the two-pass kernel"
    assert_parity(f"warm_bet_{dtype}_{B}_k{top_k}", r, o)


def test_single_row_abi_known_answers_gpu(cuda):
    """tests/test_engine.c:700-748 through the unchanged sampler.h ABI."""
    from noel_b200 import sampler as S

    V = 1000
    sm = S.Sampler(S.make_config(temperature=0.0, top_p=0.9, top_k=40, repetition_penalty=1.0, seed=42), V)
    logits = np.zeros(V, np.float32)
    logits[250], logits[500], logits[750] = 5.0, 10.0, 2.0
    assert sm.sample(logits) == 500
    sm.s.config.repetition_penalty = 3.0
    assert sm.sample(logits, np.array([500], np.int32)) == 250
    assert logits[500] == np.float32(10.0) / np.float32(3.0)
    logits[:] = 0
    logits[10], logits[20], logits[30] = 4.0, 3.0, 2.0
    sm.s.config.temperature, sm.s.config.top_k, sm.s.config.repetition_penalty = 0.8, 3, 1.0
    for _ in range(20):
        assert sm.sample(logits) in (10, 20, 30)
    sm.free()


def test_single_row_abi_matches_oracle_gpu(cuda, oracle):
    """Single-row calls (host and device logits) advance the sampler's state
    exactly like the reference and leave the drawn-from list in candidates."""
    import torch

    from noel_b200 import sampler as S
    from noel_b200.workloads import WORKLOADS, generate_numpy

    w = WORKLOADS["single_row"]
    d = generate_numpy(w, seed=4)
    cfgkw = w.config_kwargs()
    cfgkw["seed"] = 1234
    sm = S.Sampler(S.make_config(**cfgkw), w.vocab)
    st = np.array([list(sm.rng_state)], np.uint64)
    x = d["logits"].copy()
    h = d["history"]
    for step in range(3):
        o = oracle.sample_batch(orc_config(**cfgkw), x.copy(), history=h, rng=st, n_list=64)
        xs = x[0].copy()
        if step == 1:  # device pointers
            xd = torch.from_numpy(xs).to(cuda)
            hd = torch.from_numpy(h[0].copy()).to(cuda)
            got = sm.sample(xd, hd)
        else:
            got = sm.sample(xs, h[0].copy())
        assert got == o.ids[0]
        st = o.rng
        assert sm.rng_state == (int(st[0, 0]), int(st[0, 1]))
        n = int(o.diag["n_final"][0])
        cands = sm.candidates(min(n, 64))
        assert [c[0] for c in cands] == list(o.topn_ids[0, : len(cands)])
    sm.free()


def test_host_batch_api_gpu(cuda, oracle):
    from noel_b200 import sampler as S

    for name, cfgkw, logits, hist, rng in workload_cases(batch=8, vocab_small=20000):
        o = oracle.sample_batch(orc_config(**cfgkw), logits, history=hist, rng=rng)
        r = rng.copy()
        ids, pr = S.sample_batch_host(S.make_config(**cfgkw), np.ascontiguousarray(logits), r, history=hist,
                                      probs=True)
        np.testing.assert_array_equal(ids, o.ids, err_msg=name)
        np.testing.assert_array_equal(r, o.rng, err_msg=name)
        np.testing.assert_allclose(pr, o.probs, rtol=PROB_RTOL, err_msg=name)


def test_expf_domain_checksums_gpu(cuda, oracle):
    """The device exp weights equal the C library's expf on every float of
    (-15, 0] (about 1.1e9 inputs), compared as per-chunk checksums."""
    from noel_b200 import sampler as S

    dev = S.expf_checksums(24)
    host = oracle.expf_domain_checksums(24)
    bad = np.where(dev != host)[0]
    assert bad.size == 0, f"chunks differing: {bad[:10]}"


def test_invalid_arguments_gpu(cuda):
    import ctypes as C

    import torch

    from noel_b200 import sampler as S

    L = S.lib()
    cfg = S.make_config()
    x = torch.zeros(2, 10, device=cuda)
    rng = torch.ones(2, 2, dtype=torch.int64, device=cuda)
    ids = torch.empty(2, dtype=torch.int32, device=cuda)
    st = L.noel_sampler_sample_batch(C.byref(cfg), x.data_ptr(), 0, 2, 10, 5, None, 0, 0, rng.data_ptr(),
                                     ids.data_ptr(), None, None)
    assert st == -1 and L.noel_sampler_cuda_last_error() == -1   # ld < vocab
    st = L.noel_sampler_sample_batch(C.byref(cfg), x.data_ptr(), 7, 2, 10, 10, None, 0, 0, rng.data_ptr(),
                                     ids.data_ptr(), None, None)
    assert st == -1                                                # dtype
    st = L.noel_sampler_sample_batch(C.byref(cfg), x.data_ptr() + 2, 0, 2, 9, 10, None, 0, 0, rng.data_ptr(),
                                     ids.data_ptr(), None, None)
    assert st == -1                                                # misaligned base
    sm = S.Sampler(cfg, 10)
    assert L.noel_sampler_sample(C.byref(sm.s), None, 10, None, 0) == 0   # sampler.c:85
    assert L.noel_sampler_random_f32(None) == 0.0

"""The allocation-free entry point (noel_sampler_sample_batch_noalloc).

It exists for callers that cannot allocate device memory after start-up: it
keeps its scratch in a static device array of the library.  This file runs
last (pytest collects files in name order) and must pass both alone in a
fresh process and after every other test.  It checks, through the C ABI,
that the allocation-free entry point returns the same ids, RNG states and
probabilities as the regular noel_sampler_sample_batch on the same inputs,
for two calls in a row (fp32 and bf16 rows), including rows that go through
the two-pass kernel whose scratch is the static array; that the device's
free memory does not change across its first call in a fresh process; and
that sizes beyond the array are refused before anything runs.
"""
import ctypes as C
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

PROB_RTOL = 1e-5


def _cases():
    from noel_b200.workloads import WORKLOADS, generate_numpy, row_states

    out = []
    w = WORKLOADS["batch1024"].resized(batch=64)
    d = generate_numpy(w, seed=8)
    out.append(("batch1024x64", w.config_kwargs(), d["logits"], d["history"], d["rng"]))
    g = np.random.Generator(np.random.PCG64(9))
    flat = (g.standard_normal((8, 40000)) * 0.5).astype(np.float32)  # candidate set too big: two-pass rows
    cfg = dict(temperature=1.0, top_p=0.9, top_k=0, repetition_penalty=1.0, repetition_window=0, seed=0)
    out.append(("two_pass_rows", cfg, flat, None, row_states(4, np.arange(8))))
    wb = WORKLOADS["nucleus_bf16"].resized(batch=32)
    d = generate_numpy(wb, seed=10)
    out.append(("nucleus_bf16x32", wb.config_kwargs(), d["logits"], d["history"], d["rng"]))
    return out


def _call(fn, cfg, logits, hist, rng):
    import torch

    from noel_b200 import sampler as S

    dev = torch.device("cuda:0")
    bf16 = logits.dtype == np.uint16
    lg = torch.from_numpy(logits.view(np.int16)).to(dev).view(torch.bfloat16) if bf16 else \
        torch.from_numpy(logits).to(dev)
    r = torch.from_numpy(rng.view(np.int64).copy()).to(dev)
    h = torch.from_numpy(hist).to(dev) if hist is not None else None
    B, V = lg.shape
    ids = torch.empty(B, dtype=torch.int32, device=dev)
    pr = torch.empty(B, dtype=torch.float32, device=dev)
    st = fn(C.byref(S.make_config(**cfg)), lg.data_ptr(), 1 if bf16 else 0, B, V, V,
            h.data_ptr() if h is not None else None,
            h.shape[1] if h is not None else 0, h.shape[1] if h is not None else 0, r.data_ptr(), ids.data_ptr(),
            pr.data_ptr(), C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0, S.lib().noel_sampler_cuda_last_error_message()
    torch.cuda.synchronize()
    return ids.cpu().numpy(), pr.cpu().numpy(), r.cpu().numpy().view(np.uint64)


@pytest.mark.parametrize("case", _cases(), ids=lambda c: c[0])
def test_noalloc_matches_regular_entry_point(case):
    import torch

    from noel_b200 import sampler as S

    assert torch.cuda.is_available()
    L = S.lib()
    L.noel_sampler_sample_batch_noalloc.restype = C.c_int
    L.noel_sampler_sample_batch_noalloc.argtypes = L.noel_sampler_sample_batch.argtypes
    name, cfg, logits, hist, rng = case
    rng_a, rng_b = rng.copy(), rng.copy()
    for call in range(2):  # two calls in a row: the static scratch keeps the last call's contents
        ids_a, p_a, rng_a = _call(L.noel_sampler_sample_batch, cfg, logits, hist, rng_a)
        ids_b, p_b, rng_b = _call(L.noel_sampler_sample_batch_noalloc, cfg, logits, hist, rng_b)
        np.testing.assert_array_equal(ids_b, ids_a, err_msg=f"{name} call {call}: ids")
        np.testing.assert_array_equal(rng_b, rng_a, err_msg=f"{name} call {call}: rng states")
        np.testing.assert_allclose(p_b, p_a, rtol=PROB_RTOL, err_msg=f"{name} call {call}: probs")


def test_noalloc_rejects_oversize():
    import torch

    from noel_b200 import sampler as S

    assert torch.cuda.is_available()
    L = S.lib()
    L.noel_sampler_sample_batch_noalloc.restype = C.c_int
    L.noel_sampler_sample_batch_noalloc.argtypes = L.noel_sampler_sample_batch.argtypes
    x = torch.zeros(1, 8, device="cuda")
    ids = torch.empty(1, dtype=torch.int32, device="cuda")
    rng = torch.ones(1, 2, dtype=torch.int64, device="cuda")
    st = L.noel_sampler_sample_batch_noalloc(C.byref(S.make_config()), x.data_ptr(), 0, 8193, 8, 8, None, 0, 0,
                                             rng.data_ptr(), ids.data_ptr(), None, None)
    assert st == -4  # NOEL_ERR_TOO_LARGE, before touching any memory
    assert b"at most 8192 rows" in L.noel_sampler_cuda_last_error_message()


def test_noalloc_rejects_vocab_beyond_the_array():
    import torch

    from noel_b200 import sampler as S

    assert torch.cuda.is_available()
    L = S.lib()
    L.noel_sampler_sample_batch_noalloc.restype = C.c_int
    L.noel_sampler_sample_batch_noalloc.argtypes = L.noel_sampler_sample_batch.argtypes
    x = torch.zeros(1, 8, device="cuda")
    ids = torch.empty(1, dtype=torch.int32, device="cuda")
    rng = torch.ones(1, 2, dtype=torch.int64, device="cuda")
    # vocab 262145 > the array's 262144 tokens: refused from the sizes alone (no row is read)
    st = L.noel_sampler_sample_batch_noalloc(C.byref(S.make_config()), x.data_ptr(), 0, 1, 262145, 262145, None,
                                             0, 0, rng.data_ptr(), ids.data_ptr(), None, None)
    assert st == -4
    assert b"262144 tokens" in L.noel_sampler_cuda_last_error_message()


_FRESH = r"""
import ctypes as C, sys
import numpy as np, torch
sys.path.insert(0, sys.argv[1])
from noel_b200 import sampler as S
from noel_b200.workloads import row_states
dev = torch.device("cuda:0")
torch.cuda.init()
L = S.lib()
L.noel_sampler_sample_batch_noalloc.restype = C.c_int
L.noel_sampler_sample_batch_noalloc.argtypes = L.noel_sampler_sample_batch.argtypes
g = np.random.Generator(np.random.PCG64(12))
top = torch.from_numpy((2.0 * g.standard_normal((16, 30000))).astype(np.float32)).to(dev)
flat = torch.from_numpy((0.5 * g.standard_normal((4, 30000))).astype(np.float32)).to(dev)
ids = torch.empty(16, dtype=torch.int32, device=dev)
rng = torch.from_numpy(row_states(3, np.arange(16)).view(np.int64)).to(dev)
cfg_top = S.make_config(temperature=0.8, top_p=0.95, top_k=40, repetition_penalty=1.0)
cfg_full = S.make_config(temperature=1.0, top_p=0.9, top_k=0, repetition_penalty=1.0)
s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
def call(fn, cfg, x):
    B, V = x.shape
    assert fn(C.byref(cfg), x.data_ptr(), 0, B, V, V, None, 0, 0, rng.data_ptr(), ids.data_ptr(), None, s) == 0
# the kernels' first launches (module and local-memory set-up by the driver) through the regular entry point
call(L.noel_sampler_sample_batch, cfg_top, top)
call(L.noel_sampler_sample_batch, cfg_full, flat)
torch.cuda.synchronize()
free0 = torch.cuda.mem_get_info()[0]
call(L.noel_sampler_sample_batch_noalloc, cfg_top, top)     # the entry point's first call (its set-up)
torch.cuda.synchronize()
free1 = torch.cuda.mem_get_info()[0]
call(L.noel_sampler_sample_batch_noalloc, cfg_full, flat)   # two-pass rows through the static array
torch.cuda.synchronize()
free2 = torch.cuda.mem_get_info()[0]
print("FREE", free0, free1, free2)
"""


def test_noalloc_first_call_allocates_nothing():
    """In a fresh process: the device's free memory is the same before the
    entry point's first call, after it, and after a call whose rows take the
    two-pass kernel.  The process loads its kernels eagerly
    (CUDA_MODULE_LOADING=EAGER): with lazy loading the driver reserves a
    kernel's code memory at its first use, which the entry point's one-time
    set-up (it looks up every kernel it may launch) would trigger."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, CUDA_MODULE_LOADING="EAGER")
    r = subprocess.run([sys.executable, "-c", _FRESH, root], capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stdout + r.stderr
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("FREE")][-1]
    free0, free1, free2 = (int(v) for v in line.split()[1:])
    assert free1 == free0 and free2 == free0, (free0, free1, free2)

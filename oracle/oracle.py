"""ctypes front end of the CPU checkers (test infrastructure only).

* ``Oracle`` wraps ``oracle/liboracle.so``: the restatement of the reference
  sampler (Sain-Kai/noel src/sampler.c:8-192) in ``sampler_oracle.c``.
* ``RefSampler`` wraps ``oracle/_ref/libsampler_ref.so``: the reference
  sampler itself, compiled from its own sources by ``oracle/Makefile``.

Only tests/, ``__graft_entry__.smoke()`` and the cpu_baseline leg of
bench.py import this module; the library under ``noel_b200`` never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libsampler_ref.so")
REF_AUX_SO = os.path.join(HERE, "_ref", "libaux_ref.so")


class SamplerConfig(C.Structure):
    """Byte-compatible with noel_sampler_config_t (include/sampler.h:12-19)."""

    _fields_ = [
        ("temperature", C.c_float),
        ("top_p", C.c_float),
        ("top_k", C.c_int),
        ("repetition_penalty", C.c_float),
        ("repetition_window", C.c_int),
        ("seed", C.c_uint64),
    ]


DIAG_DTYPE = np.dtype(
    [
        ("id", np.int32),
        ("greedy", np.int32),
        ("num_cands", np.int32),
        ("n_topk", np.int32),
        ("n_final", np.int32),
        ("pos", np.int32),
        ("max_val", np.float32),
        ("total_mass", np.float32),
        ("u", np.float32),
        ("r", np.float32),
    ]
)


def make_config(temperature=0.7, top_p=0.9, top_k=40, repetition_penalty=1.1,
                repetition_window=64, seed=0) -> SamplerConfig:
    return SamplerConfig(float(temperature), float(top_p), int(top_k),
                         float(repetition_penalty), int(repetition_window), int(seed))


def reference_root() -> str:
    """The reference tree whose src/sampler.c oracle/_ref is built from:
    $NOEL_REFERENCE_ROOT, else a directory named ``reference`` beside the
    repository (absent on hosts that only run the prebuilt _ref/)."""
    env = os.environ.get("NOEL_REFERENCE_ROOT")
    if env:
        return env
    return os.path.abspath(os.path.join(HERE, "..", "..", "reference"))


def build(quiet: bool = True) -> None:
    """Compile the checkers (``make -C oracle``)."""
    out = subprocess.run(["make", "-C", HERE, f"REF_ROOT={reference_root()}"], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)
    if not quiet:
        print(out.stdout)


def _ptr(a, ctype):
    return None if a is None else a.ctypes.data_as(C.POINTER(ctype))


def seed_states(seeds) -> np.ndarray:
    """Per-row xorshift128+ states for non-zero seeds (sampler.c:42-47)."""
    seeds = np.asarray(seeds, dtype=np.uint64)
    st = np.empty((seeds.size, 2), dtype=np.uint64)
    st[:, 0] = seeds
    st[:, 1] = seeds ^ np.uint64(0x9E3779B97F4A7C15)
    zero = (st[:, 0] == 0) & (st[:, 1] == 0)
    st[zero, 0] = 123456789
    st[zero, 1] = 987654321
    return st


@dataclass
class BatchResult:
    ids: np.ndarray
    rng: np.ndarray
    probs: np.ndarray | None = None
    diag: np.ndarray | None = None
    topn_ids: np.ndarray | None = None
    topn_probs: np.ndarray | None = None
    num_cands: np.ndarray | None = None
    cand_vals: np.ndarray | None = None


class Oracle:
    """The restatement (sampler_oracle.c)."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build()
        self.lib = C.CDLL(path)
        L = self.lib
        L.orc_sample_batch.restype = None
        L.orc_sample_batch.argtypes = [
            C.POINTER(SamplerConfig), C.POINTER(C.c_float), C.c_int, C.c_int, C.c_size_t,
            C.POINTER(C.c_int32), C.c_int, C.c_size_t, C.POINTER(C.c_uint64),
            C.POINTER(C.c_int32), C.POINTER(C.c_float), C.c_void_p,
            C.POINTER(C.c_int32), C.POINTER(C.c_float), C.c_int, C.c_int, C.c_int,
        ]
        L.orc_sample_batch_bf16.restype = None
        L.orc_sample_batch_bf16.argtypes = [
            C.POINTER(SamplerConfig), C.POINTER(C.c_uint16), C.c_int, C.c_int, C.c_size_t,
            C.POINTER(C.c_int32), C.c_int, C.c_size_t, C.POINTER(C.c_uint64),
            C.POINTER(C.c_int32), C.POINTER(C.c_float), C.c_void_p,
            C.POINTER(C.c_int32), C.POINTER(C.c_float), C.c_int, C.c_int,
        ]
        L.orc_route_top_k.restype = None
        L.orc_route_top_k.argtypes = [C.POINTER(C.c_float), C.c_int, C.c_int, C.c_size_t, C.c_int,
                                      C.POINTER(C.c_int32), C.POINTER(C.c_float)]
        L.orc_postreq_sample_batch.restype = None
        L.orc_postreq_sample_batch.argtypes = [C.POINTER(C.c_float), C.c_int, C.c_int, C.c_size_t, C.c_float,
                                               C.c_float, C.c_int, C.POINTER(C.c_float), C.POINTER(C.c_int32)]
        L.orc_postreq_apply_penalties.restype = None
        L.orc_postreq_apply_penalties.argtypes = [C.POINTER(C.c_float), C.c_int, C.POINTER(C.c_int32), C.c_int,
                                                  C.c_float, C.c_int]
        L.orc_postreq_grammar_mask.restype = None
        L.orc_postreq_grammar_mask.argtypes = [C.POINTER(C.c_float), C.c_int, C.c_int]
        L.orc_gemv.restype = None
        L.orc_gemv.argtypes = [C.c_int, C.c_void_p, C.c_size_t, C.POINTER(C.c_float), C.c_size_t, C.c_int, C.c_int,
                               C.c_int, C.POINTER(C.c_float), C.c_size_t]
        L.orc_random_f32.restype = C.c_float
        L.orc_random_f32.argtypes = [C.POINTER(C.c_uint64)]
        L.orc_expf_range.restype = None
        L.orc_expf_range.argtypes = [C.c_uint32, C.c_uint32, C.POINTER(C.c_float)]
        L.orc_expf_domain_checksums.restype = None
        L.orc_expf_domain_checksums.argtypes = [C.c_int, C.POINTER(C.c_uint64), C.c_int, C.c_int]

    def sample_batch(self, cfg: SamplerConfig, logits: np.ndarray, vocab: int | None = None,
                     history: np.ndarray | None = None, rng: np.ndarray | None = None,
                     n_list: int = 0, nthreads: int = 0, in_place: bool = False) -> BatchResult:
        """logits: [B, ld] float32, or uint16 holding bf16 bits."""
        B, ld = logits.shape
        V = ld if vocab is None else vocab
        rng = np.ascontiguousarray(rng.copy() if rng is not None else seed_states(np.arange(1, B + 1)),
                                   dtype=np.uint64)
        assert rng.shape == (B, 2)
        ids = np.empty(B, np.int32)
        probs = np.empty(B, np.float32)
        diag = np.empty(B, DIAG_DTYPE)
        tn_ids = np.empty((B, max(n_list, 1)), np.int32) if n_list else None
        tn_p = np.empty((B, max(n_list, 1)), np.float32) if n_list else None
        if history is not None:
            history = np.ascontiguousarray(history, dtype=np.int32)
            H, hld = history.shape[1], history.shape[1]
        else:
            H, hld = 0, 0
        if logits.dtype == np.uint16:
            lg = np.ascontiguousarray(logits)
            self.lib.orc_sample_batch_bf16(C.byref(cfg), _ptr(lg, C.c_uint16), B, V, ld,
                                           _ptr(history, C.c_int32), H, hld, _ptr(rng, C.c_uint64),
                                           _ptr(ids, C.c_int32), _ptr(probs, C.c_float),
                                           diag.ctypes.data, _ptr(tn_ids, C.c_int32),
                                           _ptr(tn_p, C.c_float), n_list, nthreads)
        else:
            lg = logits if in_place else np.ascontiguousarray(logits, dtype=np.float32)
            assert lg.dtype == np.float32 and lg.flags.c_contiguous
            self.lib.orc_sample_batch(C.byref(cfg), _ptr(lg, C.c_float), B, V, ld,
                                      _ptr(history, C.c_int32), H, hld, _ptr(rng, C.c_uint64),
                                      _ptr(ids, C.c_int32), _ptr(probs, C.c_float), diag.ctypes.data,
                                      _ptr(tn_ids, C.c_int32), _ptr(tn_p, C.c_float), n_list,
                                      1 if in_place else 0, nthreads)
        return BatchResult(ids=ids, rng=rng, probs=probs, diag=diag, topn_ids=tn_ids, topn_probs=tn_p)

    def route_top_k(self, logits: np.ndarray, top_k: int):
        """sparsity.c:46-79 for every row of logits [T, E]: (ids [T, top_k],
        weights [T, top_k])."""
        x = np.ascontiguousarray(logits, dtype=np.float32)
        T, E = x.shape
        ids = np.empty((T, top_k), np.int32)
        w = np.empty((T, top_k), np.float32)
        self.lib.orc_route_top_k(_ptr(x, C.c_float), T, E, E, top_k, _ptr(ids, C.c_int32), _ptr(w, C.c_float))
        return ids, w

    def postreq_sample(self, logits: np.ndarray, temperature: float, top_p: float, top_k: int, r: np.ndarray):
        """pipeline_stages.c:103-189 on every row with uniforms r: (ids, the
        rows as the reference leaves them)."""
        x = np.array(logits, dtype=np.float32, copy=True, order="C")
        B, V = x.shape
        r = np.ascontiguousarray(r, dtype=np.float32)
        ids = np.empty(B, np.int32)
        self.lib.orc_postreq_sample_batch(_ptr(x, C.c_float), B, V, V, temperature, top_p, top_k, _ptr(r, C.c_float),
                                          _ptr(ids, C.c_int32))
        return ids, x

    def postreq_penalties(self, logits: np.ndarray, history: np.ndarray, penalty: float, window: int):
        x = np.array(logits, dtype=np.float32, copy=True, order="C")
        h = np.ascontiguousarray(history, dtype=np.int32)
        for b in range(x.shape[0]):
            self.lib.orc_postreq_apply_penalties(x[b].ctypes.data_as(C.POINTER(C.c_float)), x.shape[1],
                                                 h[b].ctypes.data_as(C.POINTER(C.c_int32)), h.shape[1], penalty,
                                                 window)
        return x

    def postreq_grammar(self, logits: np.ndarray, states) -> np.ndarray:
        x = np.array(logits, dtype=np.float32, copy=True, order="C")
        for b in range(x.shape[0]):
            self.lib.orc_postreq_grammar_mask(x[b].ctypes.data_as(C.POINTER(C.c_float)), x.shape[1], int(states[b]))
        return x

    def gemv(self, weight: np.ndarray, wtype: int, x: np.ndarray) -> np.ndarray:
        """dequant.c:412-470 restated: logits [B, rows] of weight [rows, cols]
        (float32, or uint16 bf16 / f16 bits for wtype 30 / 1) and x [B, cols]."""
        w = np.ascontiguousarray(weight)
        x = np.ascontiguousarray(x, dtype=np.float32)
        rows, cols = w.shape
        B = x.shape[0]
        y = np.empty((B, rows), np.float32)
        self.lib.orc_gemv(wtype, w.ctypes.data, cols, _ptr(x, C.c_float), cols, B, rows, cols, _ptr(y, C.c_float), rows)
        return y

    def expf(self, x: np.ndarray) -> np.ndarray:
        """glibc expf on an arbitrary float32 array (via contiguous bit ranges)."""
        x = np.ascontiguousarray(x, np.float32).ravel()
        out = np.empty_like(x)
        buf = np.empty(1, np.float32)
        for i, b in enumerate(x.view(np.uint32)):
            self.lib.orc_expf_range(int(b), 1, _ptr(buf, C.c_float))
            out[i] = buf[0]
        return out

    def expf_range(self, lo_bits: int, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        self.lib.orc_expf_range(lo_bits, n, _ptr(out, C.c_float))
        return out

    def expf_domain_checksums(self, chunk_log2: int = 24, nthreads: int = 0) -> np.ndarray:
        n = -(-(0xC1700000 - 0x80000000) // (1 << chunk_log2))
        out = np.empty(n, np.uint64)
        self.lib.orc_expf_domain_checksums(chunk_log2, _ptr(out, C.c_uint64), n, nthreads)
        return out


class RefSampler:
    """The reference sampler itself (oracle/_ref/libsampler_ref.so)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.lib = C.CDLL(path)
        L = self.lib
        L.ref_sample_batch.restype = None
        L.ref_sample_batch.argtypes = [
            C.POINTER(SamplerConfig), C.POINTER(C.c_float), C.c_int, C.c_int, C.c_size_t,
            C.POINTER(C.c_int32), C.c_int, C.c_size_t, C.POINTER(C.c_uint64),
            C.POINTER(C.c_int32), C.POINTER(C.c_int32), C.POINTER(C.c_int32),
            C.POINTER(C.c_float), C.c_int, C.c_int, C.c_int,
        ]
        L.ref_max_threads.restype = C.c_int
        L.ref_sampler_sizeof.restype = C.c_int
        L.ref_config_sizeof.restype = C.c_int
        L.ref_init_state.restype = None
        L.ref_init_state.argtypes = [C.POINTER(SamplerConfig), C.c_int, C.POINTER(C.c_uint64),
                                     C.POINTER(SamplerConfig)]
        # the reference ABI itself, for single-call known-answer tests
        L.noel_sampler_sample.restype = C.c_int32
        L.noel_sampler_random_f32.restype = C.c_float

    @staticmethod
    def available(path: str = REF_SO) -> bool:
        return os.path.exists(path)

    def max_threads(self) -> int:
        return self.lib.ref_max_threads()

    def sample_batch(self, cfg: SamplerConfig, logits: np.ndarray, vocab: int | None = None,
                     history: np.ndarray | None = None, rng: np.ndarray | None = None,
                     n_list: int = 0, nthreads: int = 0, in_place: bool = False) -> BatchResult:
        B, ld = logits.shape
        V = ld if vocab is None else vocab
        if logits.dtype == np.uint16:  # bf16 bits: upcast exactly
            logits = (logits.astype(np.uint32) << 16).view(np.float32)
        lg = logits if in_place else np.ascontiguousarray(logits, dtype=np.float32)
        rng = np.ascontiguousarray(rng.copy() if rng is not None else seed_states(np.arange(1, B + 1)),
                                   dtype=np.uint64)
        ids = np.empty(B, np.int32)
        nc = np.empty(B, np.int32)
        ci = np.empty((B, max(n_list, 1)), np.int32) if n_list else None
        cv = np.empty((B, max(n_list, 1)), np.float32) if n_list else None
        if history is not None:
            history = np.ascontiguousarray(history, dtype=np.int32)
            H, hld = history.shape[1], history.shape[1]
        else:
            H, hld = 0, 0
        self.lib.ref_sample_batch(C.byref(cfg), _ptr(lg, C.c_float), B, V, ld,
                                  _ptr(history, C.c_int32), H, hld, _ptr(rng, C.c_uint64),
                                  _ptr(ids, C.c_int32), _ptr(nc, C.c_int32), _ptr(ci, C.c_int32),
                                  _ptr(cv, C.c_float), n_list, 1 if in_place else 0, nthreads)
        return BatchResult(ids=ids, rng=rng, num_cands=nc, topn_ids=ci, cand_vals=cv)


class RoutingEntry(C.Structure):
    """moe_routing_t (reference include/sparsity.h:12-15)."""

    _fields_ = [("expert_id", C.c_int32), ("weight", C.c_float)]


class PostreqParams(C.Structure):
    """aether_sampling_params_t (reference include/pipeline_stages.h:13-20)."""

    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("top_k", C.c_int),
                ("repetition_penalty", C.c_float), ("repetition_window", C.c_int),
                ("grammar_enforce_json", C.c_bool)]


LIBC = C.CDLL(None)
LIBC.rand.restype = C.c_int
LIBC.srand.argtypes = [C.c_uint]
RAND_MAX = 2147483647


def rand_uniforms(seed: int, n: int) -> np.ndarray:
    """The uniforms aether_postreq_sample draws (pipeline_stages.c:180):
    (float)rand() / (float)RAND_MAX after srand(seed), from this process's C
    library, the one the reference build links."""
    LIBC.srand(seed)
    return np.array([np.float32(LIBC.rand()) / np.float32(RAND_MAX) for _ in range(n)], np.float32)


class RefAux:
    """The reference's router and pipeline samplers themselves
    (oracle/_ref/libaux_ref.so: src/sparsity.c, src/pipeline_stages.c)."""

    def __init__(self, path: str = REF_AUX_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.lib = C.CDLL(path)
        self.lib.aether_route_top_k.restype = None
        self.lib.aether_route_top_k.argtypes = [C.POINTER(C.c_float), C.c_int, C.c_int, C.POINTER(RoutingEntry)]
        for f in ("aether_postreq_apply_penalties", "aether_postreq_grammar_mask"):
            getattr(self.lib, f).restype = None
        self.lib.aether_postreq_apply_penalties.argtypes = [C.POINTER(C.c_float), C.c_int, C.POINTER(C.c_int32),
                                                            C.c_int, C.c_float, C.c_int]
        self.lib.aether_postreq_grammar_mask.argtypes = [C.POINTER(C.c_float), C.c_int, C.c_int]
        self.lib.aether_postreq_sample.restype = C.c_int32
        self.lib.aether_postreq_sample.argtypes = [C.POINTER(C.c_float), C.c_int, C.POINTER(PostreqParams)]
        self.lib.noel_gemv_quantized.restype = None
        self.lib.noel_gemv_quantized.argtypes = [C.c_int, C.POINTER(C.c_float), C.c_void_p, C.POINTER(C.c_float),
                                                 C.c_int, C.c_int, C.c_int]
        self.lib.ref_route_batch.restype = None
        self.lib.ref_route_batch.argtypes = [C.POINTER(C.c_float), C.c_int, C.c_int, C.c_size_t, C.c_int,
                                             C.c_void_p, C.c_int]

    @staticmethod
    def available(path: str = REF_AUX_SO) -> bool:
        return os.path.exists(path)

    def route_top_k(self, logits: np.ndarray, top_k: int):
        x = np.ascontiguousarray(logits, dtype=np.float32)
        T, E = x.shape
        ids = np.empty((T, top_k), np.int32)
        w = np.empty((T, top_k), np.float32)
        out = (RoutingEntry * top_k)()
        for t in range(T):
            self.lib.aether_route_top_k(x[t].ctypes.data_as(C.POINTER(C.c_float)), E, top_k, out)
            ids[t] = [e.expert_id for e in out]
            w[t] = [e.weight for e in out]
        return ids, w

    def route_batch(self, logits: np.ndarray, top_k: int, nthreads: int = 0):
        """ref_route_batch (aux_driver.c): the reference router over every row
        with OpenMP; returns (ids, weights)."""
        x = np.ascontiguousarray(logits, dtype=np.float32)
        T, E = x.shape
        out = np.empty((T, top_k, 2), np.int32)
        self.lib.ref_route_batch(x.ctypes.data_as(C.POINTER(C.c_float)), T, E, E, top_k, out.ctypes.data, nthreads)
        return out[:, :, 0].copy(), out[:, :, 1].copy().view(np.float32)

    def postreq_sample(self, logits: np.ndarray, params: PostreqParams, seed: int):
        """The reference's aether_postreq_sample on every row, after
        srand(seed) (it draws rand() itself): (ids, rows after the calls)."""
        x = np.array(logits, dtype=np.float32, copy=True, order="C")
        LIBC.srand(seed)
        ids = np.array([self.lib.aether_postreq_sample(x[b].ctypes.data_as(C.POINTER(C.c_float)), x.shape[1],
                                                       C.byref(params)) for b in range(x.shape[0])], np.int32)
        return ids, x

    def postreq_penalties(self, logits: np.ndarray, history: np.ndarray, penalty: float, window: int):
        x = np.array(logits, dtype=np.float32, copy=True, order="C")
        h = np.ascontiguousarray(history, dtype=np.int32)
        for b in range(x.shape[0]):
            self.lib.aether_postreq_apply_penalties(x[b].ctypes.data_as(C.POINTER(C.c_float)), x.shape[1],
                                                    h[b].ctypes.data_as(C.POINTER(C.c_int32)), h.shape[1], penalty,
                                                    window)
        return x

    def postreq_grammar(self, logits: np.ndarray, states) -> np.ndarray:
        x = np.array(logits, dtype=np.float32, copy=True, order="C")
        for b in range(x.shape[0]):
            self.lib.aether_postreq_grammar_mask(x[b].ctypes.data_as(C.POINTER(C.c_float)), x.shape[1], int(states[b]))
        return x

    def gemv(self, weight: np.ndarray, wtype: int, x: np.ndarray, nthreads: int = 0) -> np.ndarray:
        """The reference's noel_gemv_quantized (dequant.c:412) for each row of x."""
        w = np.ascontiguousarray(weight)
        x = np.ascontiguousarray(x, dtype=np.float32)
        rows, cols = w.shape
        y = np.empty((x.shape[0], rows), np.float32)
        for b in range(x.shape[0]):
            self.lib.noel_gemv_quantized(wtype, y[b].ctypes.data_as(C.POINTER(C.c_float)), w.ctypes.data,
                                         x[b].ctypes.data_as(C.POINTER(C.c_float)), rows, cols,
                                         nthreads or os.cpu_count())
        return y

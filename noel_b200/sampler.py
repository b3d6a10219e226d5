"""Python front end of libnoel_sampler_cuda.so (ctypes over the C ABI).

Mirrors the reference sampler's interface (Sain-Kai/noel include/sampler.h):
``Sampler`` wraps ``noel_sampler_t`` with the same init / set_config / sample
/ random_f32 / free semantics, and ``sample_batch`` exposes the batched
device entry point for torch tensors already on the GPU.  There is no CPU
path: loading fails loudly if the library has not been built.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from .build import LIB

F32, BF16 = 0, 1

STAT_NUM_CANDS, STAT_N_TOPK, STAT_N_FINAL, STAT_FLAGS = range(4)
ROW_GREEDY, ROW_EXACT_PASS, ROW_FALLBACK = 1, 2, 4


class SamplerConfig(C.Structure):
    """noel_sampler_config_t (include/sampler.h; reference include/sampler.h:12-19)."""

    _fields_ = [
        ("temperature", C.c_float),
        ("top_p", C.c_float),
        ("top_k", C.c_int),
        ("repetition_penalty", C.c_float),
        ("repetition_window", C.c_int),
        ("seed", C.c_uint64),
    ]


class TokenProb(C.Structure):
    _fields_ = [("id", C.c_int32), ("val", C.c_float)]


class SamplerStruct(C.Structure):
    """noel_sampler_t (reference include/sampler.h:26-31)."""

    _fields_ = [
        ("config", SamplerConfig),
        ("rng_state", C.c_uint64 * 2),
        ("candidates", C.POINTER(TokenProb)),
        ("candidate_capacity", C.c_int),
    ]


class Extras(C.Structure):
    _fields_ = [
        ("d_probs", C.c_void_p),
        ("d_list_ids", C.c_void_p),
        ("d_list_probs", C.c_void_p),
        ("list_len", C.c_int),
        ("list_weights", C.c_int),
        ("d_stats", C.c_void_p),
        ("write_back", C.c_int),
    ]


class NoelSamplerError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"noel sampler status {status}: {message}")
        self.status = status


_lib = None


def lib() -> C.CDLL:
    """Load the in-tree library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB):
        raise FileNotFoundError(f"{LIB} is missing: run `python -m noel_b200.build`")
    L = C.CDLL(LIB)
    L.noel_sampler_init.restype = None
    L.noel_sampler_init.argtypes = [C.POINTER(SamplerStruct), C.POINTER(SamplerConfig), C.c_int]
    L.noel_sampler_free.restype = None
    L.noel_sampler_free.argtypes = [C.POINTER(SamplerStruct)]
    L.noel_sampler_set_config.restype = None
    L.noel_sampler_set_config.argtypes = [C.POINTER(SamplerStruct), C.POINTER(SamplerConfig)]
    L.noel_sampler_sample.restype = C.c_int32
    L.noel_sampler_sample.argtypes = [C.POINTER(SamplerStruct), C.c_void_p, C.c_int, C.c_void_p, C.c_int]
    L.noel_sampler_random_f32.restype = C.c_float
    L.noel_sampler_random_f32.argtypes = [C.POINTER(SamplerStruct)]
    L.noel_sampler_sample_batch.restype = C.c_int
    L.noel_sampler_sample_batch.argtypes = [
        C.POINTER(SamplerConfig), C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_size_t, C.c_void_p,
        C.c_int, C.c_size_t, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
    ]
    L.noel_sampler_sample_batch_ex.restype = C.c_int
    L.noel_sampler_sample_batch_ex.argtypes = [
        C.POINTER(SamplerConfig), C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_size_t, C.c_void_p,
        C.c_int, C.c_size_t, C.c_void_p, C.c_void_p, C.POINTER(Extras), C.c_void_p,
    ]
    L.noel_sampler_sample_batch_host.restype = C.c_int
    L.noel_sampler_sample_batch_host.argtypes = [
        C.POINTER(SamplerConfig), C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_size_t, C.c_void_p,
        C.c_int, C.c_size_t, C.c_void_p, C.c_void_p, C.c_void_p,
    ]
    L.noel_sampler_shard_list_len.restype = C.c_int
    L.noel_sampler_shard_list_len.argtypes = [C.POINTER(SamplerConfig)]
    L.noel_sampler_shard_select.restype = C.c_int
    L.noel_sampler_shard_select.argtypes = [
        C.POINTER(SamplerConfig), C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_size_t, C.c_int,
        C.c_void_p, C.c_int, C.c_size_t, C.c_void_p, C.c_void_p,
    ]
    L.noel_sampler_shard_merge.restype = C.c_int
    L.noel_sampler_shard_merge.argtypes = [
        C.POINTER(SamplerConfig), C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
        C.c_void_p, C.c_void_p,
    ]
    L.noel_postreq_sample_batch.restype = C.c_int
    L.noel_postreq_sample_batch.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_size_t, C.c_void_p,
                                            C.c_void_p, C.c_void_p]
    L.noel_postreq_apply_penalties_batch.restype = C.c_int
    L.noel_postreq_apply_penalties_batch.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_size_t, C.c_void_p, C.c_int,
                                                     C.c_size_t, C.c_float, C.c_int, C.c_void_p]
    L.noel_postreq_grammar_mask_batch.restype = C.c_int
    L.noel_postreq_grammar_mask_batch.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_size_t, C.c_void_p, C.c_int,
                                                  C.c_void_p]
    L.noel_postreq_sample.restype = C.c_int32
    L.noel_postreq_sample.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
    L.noel_lmhead_sample.restype = C.c_int
    L.noel_lmhead_sample.argtypes = [C.POINTER(SamplerConfig), C.c_void_p, C.c_int, C.c_size_t, C.c_void_p,
                                     C.c_size_t, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_size_t,
                                     C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
    L.noel_moe_route_top_k.restype = C.c_int
    L.noel_moe_route_top_k.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_size_t, C.c_int, C.c_void_p, C.c_void_p]
    L.noel_sampler_cuda_last_error.restype = C.c_int
    L.noel_sampler_cuda_last_error_message.restype = C.c_char_p
    L.noel_sampler_cuda_status_string.restype = C.c_char_p
    L.noel_sampler_cuda_status_string.argtypes = [C.c_int]
    L.noel_sampler_cuda_expf_table_size.restype = C.c_int
    L.noel_sampler_cuda_profile_events.restype = C.c_int
    L.noel_sampler_cuda_profile_events.argtypes = [C.c_void_p, C.c_void_p]
    L.noel_sampler_cuda_expf_checksums.restype = C.c_int
    L.noel_sampler_cuda_expf_checksums.argtypes = [C.c_int, C.c_void_p, C.c_void_p]
    L.noel_sampler_cuda_sync_check.restype = C.c_int
    L.noel_sampler_cuda_sync_check.argtypes = [C.c_void_p]
    L.noel_sampler_cuda_set_wait_limit.restype = C.c_int
    L.noel_sampler_cuda_set_wait_limit.argtypes = [C.c_longlong, C.c_int]
    _lib = L
    return L


def _check(status: int) -> None:
    if status != 0:
        msg = lib().noel_sampler_cuda_last_error_message().decode(errors="replace")
        raise NoelSamplerError(status, msg)


def make_config(temperature=0.7, top_p=0.9, top_k=40, repetition_penalty=1.1,
                repetition_window=64, seed=0) -> SamplerConfig:
    return SamplerConfig(float(temperature), float(top_p), int(top_k), float(repetition_penalty),
                         int(repetition_window), int(seed))


class Sampler:
    """One noel_sampler_t, driven through the reference ABI."""

    def __init__(self, cfg: SamplerConfig | None = None, max_vocab: int = 1024):
        self.s = SamplerStruct()
        lib().noel_sampler_init(C.byref(self.s), C.byref(cfg) if cfg is not None else None, max_vocab)

    @property
    def config(self) -> SamplerConfig:
        return self.s.config

    @property
    def rng_state(self) -> tuple[int, int]:
        return (self.s.rng_state[0], self.s.rng_state[1])

    @rng_state.setter
    def rng_state(self, st) -> None:
        self.s.rng_state[0], self.s.rng_state[1] = int(st[0]), int(st[1])

    def set_config(self, cfg: SamplerConfig) -> None:
        lib().noel_sampler_set_config(C.byref(self.s), C.byref(cfg))

    def random_f32(self) -> float:
        return lib().noel_sampler_random_f32(C.byref(self.s))

    def sample(self, logits, history=None) -> int:
        """logits: float32 numpy array (host, modified in place when the
        penalty applies) or a CUDA torch tensor; history: int32 array/tensor."""
        lp, V = _ptr_len(logits)
        hp, H = _ptr_len(history) if history is not None else (None, 0)
        r = lib().noel_sampler_sample(C.byref(self.s), lp, V, hp, H)
        st = lib().noel_sampler_cuda_last_error()
        if st != 0:
            _check(st)
        return int(r)

    def candidates(self, n: int) -> list[tuple[int, float]]:
        return [(self.s.candidates[i].id, self.s.candidates[i].val) for i in range(n)]

    def free(self) -> None:
        lib().noel_sampler_free(C.byref(self.s))

    def __del__(self):
        try:
            if self.s.candidates:
                self.free()
        except Exception:
            pass


def _ptr_len(a):
    if a is None:
        return None, 0
    if isinstance(a, np.ndarray):
        assert a.flags.c_contiguous
        return a.ctypes.data, a.size
    return a.data_ptr(), a.numel()  # torch tensor


def sample_batch(logits, rng, cfg: SamplerConfig, history=None, probs: bool = True,
                 list_len: int = 0, list_weights: bool = False, stats: bool = False,
                 write_back: bool = False, vocab: int | None = None, stream=None):
    """Batched device sampling of torch tensors on the current CUDA device.

    logits: [B, ld] float32 or bfloat16 (row stride ld >= vocab, unit column
    stride); rng: [B, 2] int64 xorshift128+ states, advanced in place;
    history: [B, hld] int32 or None.  Returns a dict of torch tensors:
    ids [B] int32, and as requested probs [B], list_ids/list_probs
    [B, list_len], stats [B, 4].
    """
    import torch

    assert logits.is_cuda and logits.dim() == 2 and logits.stride(1) == 1
    B, ld = logits.shape[0], logits.stride(0)
    V = logits.shape[1] if vocab is None else vocab
    dtype = {torch.float32: F32, torch.bfloat16: BF16}[logits.dtype]
    assert rng.dtype == torch.int64 and rng.shape == (B, 2) and rng.is_contiguous()
    dev = logits.device
    out = {"ids": torch.empty(B, dtype=torch.int32, device=dev)}
    ex = Extras()
    if probs:
        out["probs"] = torch.empty(B, dtype=torch.float32, device=dev)
        ex.d_probs = out["probs"].data_ptr()
    if list_len:
        out["list_ids"] = torch.empty(B, list_len, dtype=torch.int32, device=dev)
        out["list_probs"] = torch.empty(B, list_len, dtype=torch.float32, device=dev)
        ex.d_list_ids = out["list_ids"].data_ptr()
        ex.d_list_probs = out["list_probs"].data_ptr()
        ex.list_len = list_len
        ex.list_weights = 1 if list_weights else 0
    if stats:
        out["stats"] = torch.empty(B, 4, dtype=torch.int32, device=dev)
        ex.d_stats = out["stats"].data_ptr()
    ex.write_back = 1 if write_back else 0
    if history is not None:
        assert history.is_cuda and history.dtype == torch.int32 and history.stride(1) == 1
        hp, H, hld = history.data_ptr(), history.shape[1], history.stride(0)
    else:
        hp, H, hld = None, 0, 0
    s = stream if stream is not None else torch.cuda.current_stream(dev)
    _check(lib().noel_sampler_sample_batch_ex(C.byref(cfg), logits.data_ptr(), dtype, B, V, ld, hp, H, hld,
                                              rng.data_ptr(), out["ids"].data_ptr(), C.byref(ex),
                                              C.c_void_p(s.cuda_stream)))
    return out


def sample_batch_raw(cfg: SamplerConfig, logits_ptr: int, dtype: int, B: int, V: int, ld: int,
                     hist_ptr, H: int, hld: int, rng_ptr: int, ids_ptr: int, probs_ptr, stream_ptr) -> None:
    """Thin pass-through to noel_sampler_sample_batch (pointers as ints)."""
    _check(lib().noel_sampler_sample_batch(C.byref(cfg), logits_ptr, dtype, B, V, ld, hist_ptr, H, hld,
                                           rng_ptr, ids_ptr, probs_ptr, C.c_void_p(stream_ptr)))


def sample_batch_host(cfg: SamplerConfig, logits: np.ndarray, rng: np.ndarray, history: np.ndarray | None = None,
                      probs: bool = False, vocab: int | None = None):
    """Host-buffer batched sampling (noel_sampler_sample_batch_host).
    logits: [B, ld] float32, or uint16 holding bf16 bits; rng [B, 2] uint64
    (advanced in place).  Returns ids (and probs)."""
    B, ld = logits.shape
    V = ld if vocab is None else vocab
    dtype = BF16 if logits.dtype == np.uint16 else F32
    assert logits.flags.c_contiguous and rng.flags.c_contiguous and rng.dtype == np.uint64
    ids = np.empty(B, np.int32)
    pr = np.empty(B, np.float32) if probs else None
    if history is not None:
        assert history.dtype == np.int32 and history.flags.c_contiguous
        hp, H, hld = history.ctypes.data, history.shape[1], history.shape[1]
    else:
        hp, H, hld = None, 0, 0
    _check(lib().noel_sampler_sample_batch_host(C.byref(cfg), logits.ctypes.data, dtype, B, V, ld, hp, H, hld,
                                                rng.ctypes.data, ids.ctypes.data,
                                                pr.ctypes.data if pr is not None else None))
    return (ids, pr) if probs else ids


def profile_events(before=None, after=None) -> None:
    """Record torch.cuda.Event ``before``/``after`` around the single-pass
    kernel of later batched calls on this thread (None, None to stop)."""
    for ev in (before, after):
        if ev is not None and not ev.cuda_event:
            ev.record()  # torch creates the CUDA event on its first record
    lib().noel_sampler_cuda_profile_events(before.cuda_event if before is not None else None,
                                           after.cuda_event if after is not None else None)


def sync_check(stream=None) -> int:
    """Wait for ``stream`` (default: the current one) and return the status of
    the device-side waits of the calls made on it (0, or NOEL_ERR_DEVICE_WAIT)."""
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return int(lib().noel_sampler_cuda_sync_check(C.c_void_p(s.cuda_stream)))


def set_wait_limit(wait_ns: int = 0, stall_next_call: bool = False) -> None:
    """Limit of the device-side waits of this thread's later batched calls
    (0: the default, 2 s); ``stall_next_call`` makes the next call's kernel
    issue no row loads so that its waits run out (failure-detection tests)."""
    _check(lib().noel_sampler_cuda_set_wait_limit(int(wait_ns), 1 if stall_next_call else 0))


def expf_table_size() -> int:
    return lib().noel_sampler_cuda_expf_table_size()


def expf_checksums(chunk_log2: int = 24):
    """Device exp-weight checksums over (-15, 0] (see include/noel_sampler_cuda.h)."""
    import torch

    n = -(-(0xC1700000 - 0x80000000) // (1 << chunk_log2))
    out = torch.empty(n, dtype=torch.int64, device="cuda")
    s = torch.cuda.current_stream()
    _check(lib().noel_sampler_cuda_expf_checksums(chunk_log2, out.data_ptr(), C.c_void_p(s.cuda_stream)))
    s.synchronize()
    return out.cpu().numpy().view(np.uint64)


def route_top_k(gate_logits, top_k: int):
    """MoE routing of every row of gate_logits (a CUDA float32 tensor [T, E],
    unit column stride): the reference's aether_route_top_k per token.
    Returns (expert ids [T, top_k] int32, weights [T, top_k] float32)."""
    import torch

    assert gate_logits.is_cuda and gate_logits.dtype == torch.float32 and gate_logits.stride(1) == 1
    T, E = gate_logits.shape
    out = torch.empty(T, top_k, 2, dtype=torch.int32, device=gate_logits.device)
    s = torch.cuda.current_stream(gate_logits.device)
    _check(lib().noel_moe_route_top_k(gate_logits.data_ptr(), T, E, gate_logits.stride(0), top_k, out.data_ptr(),
                                      C.c_void_p(s.cuda_stream)))
    return out[:, :, 0], out[:, :, 1].view(torch.float32)


class PostreqParams(C.Structure):
    """noel_postreq_params_t (include/noel_postreq.h; the reference's
    aether_sampling_params_t, include/pipeline_stages.h:13-20)."""

    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("top_k", C.c_int),
                ("repetition_penalty", C.c_float), ("repetition_window", C.c_int),
                ("grammar_enforce_json", C.c_bool)]


def postreq_params(temperature=0.7, top_p=0.9, top_k=50, repetition_penalty=1.15, repetition_window=2048,
                   grammar_enforce_json=False) -> PostreqParams:
    return PostreqParams(temperature, top_p, top_k, repetition_penalty, repetition_window, grammar_enforce_json)


def postreq_sample_batch(logits, params: PostreqParams, uniforms):
    """aether_postreq_sample on every row of logits (CUDA float32 [B, V],
    unit column stride; modified in place as the reference modifies its row)
    with the rows' uniforms (CUDA float32 [B]).  Returns ids [B] int32."""
    import torch

    assert logits.is_cuda and logits.dtype == torch.float32 and logits.stride(1) == 1
    B, V = logits.shape
    ids = torch.empty(B, dtype=torch.int32, device=logits.device)
    s = torch.cuda.current_stream(logits.device)
    _check(lib().noel_postreq_sample_batch(C.byref(params), logits.data_ptr(), B, V, logits.stride(0),
                                           uniforms.data_ptr() if uniforms is not None else None, ids.data_ptr(),
                                           C.c_void_p(s.cuda_stream)))
    return ids


def postreq_apply_penalties_batch(logits, history, penalty: float, window: int) -> None:
    import torch

    B, V = logits.shape
    s = torch.cuda.current_stream(logits.device)
    _check(lib().noel_postreq_apply_penalties_batch(logits.data_ptr(), B, V, logits.stride(0), history.data_ptr(),
                                                    history.shape[1], history.stride(0), penalty, window,
                                                    C.c_void_p(s.cuda_stream)))


def postreq_grammar_mask_batch(logits, states=None, state: int = 0) -> None:
    import torch

    B, V = logits.shape
    s = torch.cuda.current_stream(logits.device)
    _check(lib().noel_postreq_grammar_mask_batch(logits.data_ptr(), B, V, logits.stride(0),
                                                 states.data_ptr() if states is not None else None, state,
                                                 C.c_void_p(s.cuda_stream)))


def postreq_sample(logits, params: PostreqParams) -> int:
    """The drop-in single-row call (host numpy float32 row or CUDA tensor),
    drawing rand() where the reference does."""
    lp, V = _ptr_len(logits)
    r = lib().noel_postreq_sample(lp, V, C.byref(params))
    st = lib().noel_sampler_cuda_last_error()
    if st != 0:
        _check(st)
    return int(r)


HEAD_F32, HEAD_F16, HEAD_BF16 = 0, 1, 30


def lmhead_sample(weight, hidden, rng, cfg: SamplerConfig, history=None, probs: bool = False):
    """The LM head then the sampler (include/noel_lmhead.h): weight [V, D]
    CUDA float32 / float16 / bfloat16 (unit column stride), hidden [B, D]
    CUDA float32, rng [B, 2] int64 advanced in place, history [B, H] int32 or
    None.  Returns (ids [B] int32, logits [B, V] float32, probs or None)."""
    import torch

    wt = {torch.float32: HEAD_F32, torch.float16: HEAD_F16, torch.bfloat16: HEAD_BF16}[weight.dtype]
    assert weight.is_cuda and hidden.is_cuda and hidden.dtype == torch.float32
    V, D = weight.shape
    B = hidden.shape[0]
    dev = weight.device
    logits = torch.empty(B, V, dtype=torch.float32, device=dev)
    ids = torch.empty(B, dtype=torch.int32, device=dev)
    pr = torch.empty(B, dtype=torch.float32, device=dev) if probs else None
    if history is not None:
        hp, H, hld = history.data_ptr(), history.shape[1], history.stride(0)
    else:
        hp, H, hld = None, 0, 0
    s = torch.cuda.current_stream(dev)
    _check(lib().noel_lmhead_sample(C.byref(cfg), weight.data_ptr(), wt, weight.stride(0), hidden.data_ptr(),
                                    hidden.stride(0), B, D, V, hp, H, hld, rng.data_ptr(), ids.data_ptr(),
                                    pr.data_ptr() if pr is not None else None, logits.data_ptr(),
                                    C.c_void_p(s.cuda_stream)))
    return ids, logits, pr

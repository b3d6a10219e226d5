"""The drop-in boundary without a GPU: the library loads, exports every
function include/*.h declares (unmangled, C linkage), keeps the reference's
struct layouts, and its host-only entry points (init / free / set_config /
random_f32, and the invalid-argument returns of sample) behave as the
reference's own build (oracle/_ref, compiled from src/sampler.c) does."""
import ctypes as C
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", h) for h in ("sampler.h", "noel_sampler_cuda.h")]


@pytest.fixture(scope="module")
def lib():
    from noel_b200 import build, sampler

    build.build()
    return sampler.lib()


def declared_functions():
    names = []
    for h in HEADERS:
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        for m in re.finditer(r"^[A-Za-z_][\w \t\*]*?\b(noel_\w+)\s*\(", text, flags=re.M):
            if not text[m.start():m.end()].lstrip().startswith(("typedef", "#")):
                names.append(m.group(1))
    return sorted(set(names))


def test_headers_declare_the_reference_abi():
    names = declared_functions()
    for f in ["noel_sampler_init", "noel_sampler_free", "noel_sampler_set_config", "noel_sampler_sample",
              "noel_sampler_random_f32"]:
        assert f in names
    assert len(names) >= 15


def test_library_exports_every_declared_function(lib):
    so = lib._name
    out = subprocess.run(["nm", "-D", "--defined-only", so], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    missing = [f for f in declared_functions() if f not in exported]
    assert not missing, f"declared but not exported: {missing}"
    for f in declared_functions():
        assert hasattr(lib, f)


def test_struct_layouts_match_the_reference():
    from noel_b200.sampler import SamplerConfig, SamplerStruct, TokenProb

    assert C.sizeof(SamplerConfig) == 32  # sampler.h:12-19
    assert C.sizeof(TokenProb) == 8
    assert SamplerStruct.rng_state.offset == 32 and SamplerStruct.candidates.offset == 48
    assert C.sizeof(SamplerStruct) == 64


def _ref_lib(ref_sampler):
    from noel_b200.sampler import SamplerConfig, SamplerStruct

    L = ref_sampler.lib
    L.noel_sampler_init.argtypes = [C.POINTER(SamplerStruct), C.POINTER(SamplerConfig), C.c_int]
    L.noel_sampler_free.argtypes = [C.POINTER(SamplerStruct)]
    L.noel_sampler_set_config.argtypes = [C.POINTER(SamplerStruct), C.POINTER(SamplerConfig)]
    L.noel_sampler_random_f32.restype = C.c_float
    L.noel_sampler_random_f32.argtypes = [C.POINTER(SamplerStruct)]
    L.noel_sampler_sample.restype = C.c_int32
    L.noel_sampler_sample.argtypes = [C.POINTER(SamplerStruct), C.c_void_p, C.c_int, C.c_void_p, C.c_int]
    return L


def test_default_config_and_candidate_buffer(lib, ref_sampler):
    from noel_b200.sampler import SamplerStruct

    ref = _ref_lib(ref_sampler)
    for L in (lib, ref):
        s = SamplerStruct()
        L.noel_sampler_init(C.byref(s), None, 151936)
        c = s.config
        assert (round(c.temperature, 6), round(c.top_p, 6), c.top_k, round(c.repetition_penalty, 6),
                c.repetition_window, c.seed) == (0.7, 0.9, 40, 1.1, 64, 0)
        assert s.candidate_capacity == 151936 and bool(s.candidates)
        t = SamplerStruct()
        L.noel_sampler_init(C.byref(t), None, 10)
        assert t.candidate_capacity == 1024  # sampler.c:49-51
        L.noel_sampler_free(C.byref(s))
        L.noel_sampler_free(C.byref(t))
        assert not s.candidates and s.candidate_capacity == 0


def test_seeding_reseeding_and_random_stream(lib, ref_sampler):
    from noel_b200.sampler import SamplerConfig, SamplerStruct

    ref = _ref_lib(ref_sampler)
    runs = []
    for L in (lib, ref):
        s = SamplerStruct()
        cfg = SamplerConfig(0.8, 0.95, 40, 1.1, 0, 42)
        L.noel_sampler_init(C.byref(s), C.byref(cfg), 1000)
        seq = [tuple(s.rng_state)]
        seq += [L.noel_sampler_random_f32(C.byref(s)) for _ in range(2000)]
        L.noel_sampler_set_config(C.byref(s), C.byref(SamplerConfig(1.0, 0.5, 5, 1.0, 0, 0)))  # seed 0: keep
        seq.append(tuple(s.rng_state))
        L.noel_sampler_set_config(C.byref(s), C.byref(SamplerConfig(1.0, 0.5, 5, 1.0, 0, 7)))  # reseed
        seq.append(tuple(s.rng_state))
        seq += [L.noel_sampler_random_f32(C.byref(s)) for _ in range(100)]
        z = SamplerStruct()
        L.noel_sampler_init(C.byref(z), C.byref(SamplerConfig(0.8, 0.95, 40, 1.1, 0, 0x9E3779B97F4A7C15)), 1)
        seq.append(tuple(z.rng_state))  # seed ^ constant == 0 is not the both-zero state
        L.noel_sampler_free(C.byref(s))
        L.noel_sampler_free(C.byref(z))
        runs.append(seq)
    assert runs[0] == runs[1]
    assert all(0.0 <= u < 1.0 for u in runs[0][1:2001])


def test_invalid_arguments_return_zero(lib, ref_sampler):
    from noel_b200.sampler import SamplerStruct

    ref = _ref_lib(ref_sampler)
    for L in (lib, ref):
        assert L.noel_sampler_random_f32(None) == 0.0
        assert L.noel_sampler_sample(None, None, 10, None, 0) == 0
        s = SamplerStruct()
        L.noel_sampler_init(C.byref(s), None, 16)
        assert L.noel_sampler_sample(C.byref(s), None, 10, None, 0) == 0
        buf = (C.c_float * 4)()
        assert L.noel_sampler_sample(C.byref(s), buf, 0, None, 0) == 0
        L.noel_sampler_free(C.byref(s))
        L.noel_sampler_init(None, None, 10)
        L.noel_sampler_free(None)
        L.noel_sampler_set_config(None, None)
    assert lib.noel_sampler_cuda_last_error() == -1  # NOEL_ERR_INVALID_ARG on the side channel

"""Generate the golden fixtures from the reference sampler itself.

    python tests/golden/make_golden.py

Runs every case of tests/golden/cases.py through the reference's own
src/sampler.c (compiled from the reference sources into
oracle/_ref/libsampler_ref.so by oracle/Makefile) and stores inputs and
outputs in tests/golden/golden_cases.npz:

    <case>/logits, <case>/history (if any), <case>/rng_in, <case>/cfg
    <case>/ids, <case>/rng_out, <case>/num_cands,
    <case>/cand_ids, <case>/cand_vals   (the reference's sorted candidate
                                         list after the call, first 64)
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle.oracle import RefSampler, build, make_config  # noqa: E402
from tests.golden.cases import all_small_cases  # noqa: E402

N_LIST = 64
OUT = os.path.join(HERE, "golden_cases.npz")


def main() -> None:
    build()
    ref = RefSampler()
    arrays = {}
    names = []
    for name, cfgkw, logits, hist, rng in all_small_cases():
        cfg = make_config(**cfgkw)
        r = ref.sample_batch(cfg, logits, history=hist, rng=rng, n_list=N_LIST)
        names.append(name)
        arrays[f"{name}/logits"] = logits
        if hist is not None:
            arrays[f"{name}/history"] = hist
        arrays[f"{name}/rng_in"] = rng
        arrays[f"{name}/cfg"] = np.frombuffer(json.dumps(cfgkw).encode(), dtype=np.uint8)
        arrays[f"{name}/ids"] = r.ids
        arrays[f"{name}/rng_out"] = r.rng
        arrays[f"{name}/num_cands"] = r.num_cands
        arrays[f"{name}/cand_ids"] = r.topn_ids
        arrays[f"{name}/cand_vals"] = r.cand_vals
    arrays["__names__"] = np.frombuffer(json.dumps(names).encode(), dtype=np.uint8)
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT}: {len(names)} cases, {os.path.getsize(OUT) / 1e3:.0f} kB")


def load():
    """{name: dict(cfg, logits, history, rng_in, ids, rng_out, num_cands, cand_ids, cand_vals)}"""
    z = np.load(OUT)
    names = json.loads(bytes(z["__names__"]).decode())
    out = {}
    for n in names:
        d = {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(n + "/")}
        d["cfg"] = json.loads(bytes(d["cfg"]).decode())
        d.setdefault("history", None)
        out[n] = d
    return out


if __name__ == "__main__":
    main()

"""Generate ``sampler_golden.json`` by running miniserve's own sampler.

Run where the reference source tree is available (it is not on the GPU box):

    MINISERVE_REF=/path/to/miniserve python tests/golden/make_golden.py

It imports ``miniserve.sampler.Sampler`` and ``JSONLogitsProcessor`` from the
reference, feeds them the seeded rows of ``tests/golden/cases.py`` and the
first rows of each benchmark configuration (``miniserve_b200/workloads.py``),
and records the returned token (or the exception the reference raised).  The
tests pin both oracle restatements and the CUDA path to these tokens.
"""
from __future__ import annotations

import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(HERE))

import cases  # noqa: E402
import golden_util  # noqa: E402
from miniserve_b200 import workloads  # noqa: E402


def _ref_sampler():
    ref = golden_util.reference_root()
    sys.path.insert(0, ref)
    from miniserve.sampler import Sampler  # type: ignore
    return Sampler()


def _run(sampler, row, T, k, p, seed):
    """Call the reference; it draws ``random.Random(seed).random()`` itself."""
    try:
        return int(sampler.sample([float(v) for v in row], temperature=float(T), top_k=int(k),
                                  top_p=float(p), seed=seed))
    except ZeroDivisionError:
        return "ZeroDivisionError"


def main():
    sampler = _ref_sampler()
    out = {"python": sys.version.split()[0], "kat": [], "small": [], "configs": []}
    for c in cases.kat_cases():
        tok = _run(sampler, c["logits"], c["temperature"], c["top_k"], c["top_p"], seed=0)
        assert tok == c["token"], (c, tok)
        out["kat"].append({**c, "ref_token": tok})

    # Small groups: the reference draws its own uniform from the row seed,
    # which is the uniform cases.group hands to the oracles and the GPU.
    for V in cases.SMALL_VOCABS:
        x, T, k, p, u, seeds = cases.group(V, 11)
        toks = [_run(sampler, x[b], T[b], k[b], p[b], seed=seeds[b]) for b in range(x.shape[0])]
        out["small"].append({"V": V, "case_seed": 11, "ref_tokens": toks, "uniforms": list(map(float, u))})

    def cfg(name, batch, rows, gen_args):
        t0 = time.time()
        toks = []
        for b in rows:
            row = batch.logits[b]
            if batch.bf16:
                row = workloads.bf16_bits_to_f32(row)
            toks.append(_run(sampler, row, batch.temperature[b], batch.top_k[b], batch.top_p[b],
                             seed=int(batch.seeds[b])))
        out["configs"].append({"name": name, "gen": gen_args, "rows": list(rows), "ref_tokens": toks})
        print(f"{name}: {len(rows)} rows in {time.time() - t0:.1f}s", flush=True)

    cfg("config1", workloads.config1(1), range(8), {"fn": "config1", "seed": 1})
    cfg("config1_greedy", workloads.config1(1, greedy=True), range(8),
        {"fn": "config1", "seed": 1, "greedy": True})
    cfg("config2_fp32", workloads.config2(2), range(16), {"fn": "config2", "seed": 2})
    cfg("config2_bf16", workloads.config2(2, bf16=True), range(16),
        {"fn": "config2", "seed": 2, "bf16": True})
    cfg("config3", workloads.config3(3), range(512), {"fn": "config3", "seed": 3})  # the whole north-star batch
    cfg("config5", workloads.config5(5, B=4), range(4), {"fn": "config5", "seed": 5, "B": 4})

    with open(os.path.join(HERE, "sampler_golden.json"), "w") as f:
        json.dump(out, f, indent=1)
    print("wrote sampler_golden.json")


if __name__ == "__main__":
    main()

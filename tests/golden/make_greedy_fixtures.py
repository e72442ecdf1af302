"""Generates the full-depth greedy fixtures tests/golden/greedy_<model>.json.

For each seeded prompt the CPU oracle (oracle/c2s_oracle.c, the scalar
reference's statement order) runs the reference's generate loop
(c2slm.go:144-211: penalty 1.15 over 64 positions, strict-> argmax from
index 0) free-running for `steps` greedy steps after IngestFrom of the
prompt.  Recorded per prompt: the ids, every step's top-1 / top-2 margin
relative to max|logit|, and the first step at which the reference's AVX2
build (restated in the oracle: c2o_model_set_simd_order) leaves the scalar
build's sequence -- the reference's own build-to-build envelope, which the
GPU test holds the CUDA path to.

Prompts: prompt s has `plen` ids drawn by numpy's default_rng(1000 + s)
uniform in [0, 151643), the model is c2slm_b200.synth's preset (seeded).

Run (CPU only; config 1 takes ~20 s per prompt and build on 8 threads,
config 2 ~6 min):
  python tests/golden/make_greedy_fixtures.py qwen05b --prompts 24 --plen 32 --steps 96
  python tests/golden/make_greedy_fixtures.py qwen15b --prompts 6 --plen 1024 --steps 80
--cache DIR keeps (and reuses) each oracle run as DIR/<model>_<plen>[_simd].json,
so an interrupted run resumes.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

SEED_BASE = 1000
VOCAB_DRAW = 151643


def prompt_of(seed: int, plen: int) -> np.ndarray:
    return np.random.default_rng(SEED_BASE + seed).integers(0, VOCAB_DRAW, plen).astype(np.int32)


def oracle_runs(model: str, path: str, prompts: int, plen: int, steps: int, simd: bool, cache: str | None,
                threads: int) -> dict:
    from oracle import oracle as O
    cpath = os.path.join(cache, f"{model}_{plen}{'_simd' if simd else ''}.json") if cache else None
    res = json.load(open(cpath)) if cpath and os.path.exists(cpath) else {}
    todo = [s for s in range(prompts) if str(s) not in res or len(res[str(s)]["ids"]) < steps]
    if todo:
        with O.OracleModel(path, max_tokens=plen + steps + 8, nthreads=threads, simd_order=simd) as o:
            for s in todo:
                o.reset()
                nx = o.ingest_from(0, prompt_of(s, plen))
                ids, m, mx = o.generate(nx, steps, stop_on_special=False)
                res[str(s)] = {"ids": [int(i) for i in ids], "margin": [float(v) for v in m],
                               "maxabs": [float(v) for v in mx]}
                if cpath:
                    os.makedirs(cache, exist_ok=True)
                    json.dump(res, open(cpath, "w"))
                print(f"{model} {'avx2' if simd else 'scalar'} prompt {s} done", flush=True)
    return res


def main() -> None:
    from c2slm_b200 import synth
    ap = argparse.ArgumentParser()
    ap.add_argument("model")
    ap.add_argument("--prompts", type=int, default=24)
    ap.add_argument("--plen", type=int, default=32)
    ap.add_argument("--steps", type=int, default=96)
    ap.add_argument("--threads", type=int, default=os.cpu_count() or 1)
    ap.add_argument("--cache")
    a = ap.parse_args()
    path = synth.cached_model(a.model)
    sc = oracle_runs(a.model, path, a.prompts, a.plen, a.steps, False, a.cache, a.threads)
    av = oracle_runs(a.model, path, a.prompts, a.plen, a.steps, True, a.cache, a.threads)
    out = {"model": a.model, "layers": synth.get_config(a.model).layers, "seed_base": SEED_BASE,
           "plen": a.plen, "steps": a.steps, "penalty": 1.15, "window": 64, "prompts": []}
    for s in range(a.prompts):
        ids = sc[str(s)]["ids"][:a.steps]
        rel = [m / x if x > 0 else 0.0 for m, x in zip(sc[str(s)]["margin"], sc[str(s)]["maxabs"])][:a.steps]
        avx = av[str(s)]["ids"][:a.steps]
        same = next((i for i in range(a.steps) if avx[i] != ids[i]), a.steps)
        out["prompts"].append({"seed": s, "ids": ids, "rel_margin": [float(f"{v:.3e}") for v in rel],
                               "avx2_same_steps": same})
    dst = os.path.join(HERE, f"greedy_{a.model}.json")
    json.dump(out, open(dst, "w"), separators=(",", ":"))
    print("wrote", dst)


if __name__ == "__main__":
    main()

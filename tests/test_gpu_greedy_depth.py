"""Full-depth free-running greedy decode on the GPU against the reference's
greedy ids (BASELINE configs 1 and 2 at every layer; the oracle's ids and
margins are committed fixtures, tests/golden/make_greedy_fixtures.py).

At full depth on these seeded random-weight models, exact identity of long
free-running sequences is not a property the reference itself has: it
quantises every SwiGLU output to Q8_K before ffn_down, so a last-bit f32
difference anywhere upstream can move an int8 across a rounding boundary,
and the residual stream then differs by ~1e-2 of max|logit| -- above most
top-1/top-2 margins (median ~1e-4 of max|logit| here).  Its AVX2 build and
its scalar build (both restated in the oracle) part ways within 64 steps on
about half of the prompts.  The GPU path is held to that build-to-build
envelope, prompt set by prompt set:
  * as many prompts with >= 64 identical steps as the AVX2 build has, less
    a statistical allowance of about two standard deviations of the
    difference of two such counts (8 of 48 prompts, 2 of 6 at the 1.5B
    shape);
  * the first step identical on every prompt.
The AVX2 build shares the scalar build's Q5_0 matvecs and RMSNorm (they
have no SIMD path, tensor/ops.go:40-74,207-218), which the 0.5B model uses
for six of its seven projections; the GPU sums every dot product and norm
in its own order, so it is expected to sit at the edge of that envelope.
The per-prompt counts are printed (and recorded in the design notes).
"""
import json
import os

import numpy as np
import pytest

import c2slm_b200 as K
from c2slm_b200 import synth

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def fixture(model):
    p = os.path.join(GOLDEN, f"greedy_{model}.json")
    if not os.path.exists(p):
        pytest.skip(f"no fixture {p}")
    return json.load(open(p))


@pytest.mark.slow
@pytest.mark.parametrize("model,allowance", [("qwen05b", 8), ("qwen15b", 2)])
def test_full_depth_greedy_within_reference_build_envelope(model_cache, model, allowance):
    fx = fixture(model)
    assert fx["layers"] == synth.get_config(model).layers
    plen, steps = fx["plen"], fx["steps"]
    path = synth.cached_model(model, cache_dir=model_cache)
    gpu, avx = [], []
    with K.Engine(path, max_tokens=plen + steps + 16) as e:
        for p in fx["prompts"]:
            prompt = np.random.default_rng(fx["seed_base"] + p["seed"]).integers(0, 151643, plen).astype(np.int32)
            e.reset()
            e.ingest_from(0, prompt)
            got = e.generate(steps, penalty=fx["penalty"], window=fx["window"], stop_on_special=False)
            want = p["ids"]
            same = next((i for i in range(steps) if got[i] != want[i]), steps)
            gpu.append(same)
            avx.append(p["avx2_same_steps"])
    print(f"{model}: identical greedy steps per prompt, gpu {gpu}; reference avx2 build {avx}")
    g64, a64 = sum(s >= 64 for s in gpu), sum(s >= 64 for s in avx)
    print(f"{model}: prompts with >= 64 identical steps: gpu {g64}/{len(gpu)}, avx2 build {a64}/{len(avx)}")
    assert min(gpu) >= 1
    assert g64 >= a64 - allowance

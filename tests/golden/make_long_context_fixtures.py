"""Generates tests/golden/long_context.json: CPU-oracle results of two long
IngestFrom cases that the GPU suite compares with directly (the oracle takes
minutes on them, too long to run inside the GPU test):

  attn4096     7B shape (28 query heads, 4 kv heads, head_dim 128) at 2
               layers, a 4096-token prompt (numpy default_rng(9), ids in
               [0, 151643)), KV capacity 4160: the last NormX (attention
               over 4096 positions in 33 splits on the GPU), the first
               greedy ids and their top-1 / top-2 margins.
  prefill2048  1.5B shape at 2 layers, a 2048-token prompt
               (default_rng(7)), capacity 2112: the last NormX (the GPU
               ingests it with the tensor-core prefill), K and V rows of
               both layers and kv heads at positions 0, 1024 and 2047, the
               first greedy ids and margins.

Run (CPU, a few minutes on 8 threads):
  python tests/golden/make_long_context_fixtures.py
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

CASES = {
    "attn4096": {"model": "qwen7b", "layers": 2, "seed": 9, "n": 4096, "max_tokens": 4160, "gen": 6, "kv_pos": []},
    "prefill2048": {"model": "qwen15b", "layers": 2, "seed": 7, "n": 2048, "max_tokens": 2112, "gen": 4,
                    "kv_pos": [0, 1024, 2047]},
}


def run(name: str, c: dict, threads: int) -> dict:
    from c2slm_b200 import synth
    from oracle import oracle as O
    path = synth.cached_model(c["model"], layers=c["layers"])
    prompt = np.random.default_rng(c["seed"]).integers(0, 151643, c["n"]).astype(np.int32)
    with O.OracleModel(path, max_tokens=c["max_tokens"], nthreads=threads) as o:
        nx = o.ingest_from(0, prompt)
        kv = []
        for layer in range(c["layers"]):
            for g in range(synth.get_config(c["model"]).kv_heads):
                for p in c["kv_pos"]:
                    kv.append({"layer": layer, "kv_head": g, "pos": p,
                               "k": [float(v) for v in o.kv_get(0, layer, g, p)],
                               "v": [float(v) for v in o.kv_get(1, layer, g, p)]})
        ids, m, mx = o.generate(nx, c["gen"], stop_on_special=False)
    out = dict(c)
    out.update({"normx": [float(v) for v in nx], "kv": kv, "ids": [int(i) for i in ids],
                "rel_margin": [float(a / b) if b > 0 else 0.0 for a, b in zip(m, mx)]})
    print(name, "done", flush=True)
    return out


def main() -> None:
    threads = os.cpu_count() or 1
    res = {name: run(name, c, threads) for name, c in CASES.items()}
    dst = os.path.join(HERE, "long_context.json")
    json.dump(res, open(dst, "w"), separators=(",", ":"))
    print("wrote", dst)


if __name__ == "__main__":
    main()

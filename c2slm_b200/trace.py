"""Per-phase timing of the persistent decode kernel (c2s_trace_decode).

    python -m c2slm_b200.trace --model qwen05b --ctx 32
    python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 --master-addr 127.0.0.1 \\
        --master-port 29502 -m c2slm_b200.trace --model qwen7b --ctx 1024      # tensor parallel

Opens the seeded synthetic model (c2slm_b200.synth), ingests a uniform-random
prompt of --ctx tokens, decodes a few steps with the phase trace on and
prints one JSON line (rank 0): per phase kind, the critical-path time (from
the last CTA's end of the previous phase to the last CTA's end of this one),
the median CTA's busy time and its prologue (phase start to inputs ready),
medians over layers and steps, in microseconds.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import numpy as np

KINDS = ("qkv", "attn", "oproj", "gateup", "down", "logits")


def phase_table(tr: np.ndarray) -> dict:
    """tr: [steps, phases, ctas, 8] from Engine.trace_decode (fields 0..3 are
    %globaltimer ns at phase start, inputs ready, chunks done, end)."""
    tr = tr.astype(np.int64)
    S, NP, _, _ = tr.shape
    kinds = ["logits"] + ["qkv", "attn", "oproj", "gateup", "down"] * ((NP - 1) // 5)
    first = tr[..., 0].min(axis=2)
    last_end = tr[..., 3].max(axis=2)
    out = {}
    for k in KINDS:
        idx = [i for i, n in enumerate(kinds) if n == k]
        crit = [last_end[s, i] - (last_end[s, i - 1] if i > 0 else first[s, i]) for s in range(S) for i in idx]
        busy = [np.median(tr[s, i, :, 3] - tr[s, i, :, 0]) for s in range(S) for i in idx]
        row = {"crit_us": round(float(np.median(crit)) / 1e3, 2), "busy_med_us": round(float(np.median(busy)) / 1e3, 2)}
        if k != "attn":
            pro = [np.median(tr[s, i, :, 1] - tr[s, i, :, 0]) for s in range(S) for i in idx]
            row["prologue_med_us"] = round(float(np.median(pro)) / 1e3, 2)
        out[k] = row
    return out


def main() -> None:
    import c2slm_b200 as K
    import c2slm_b200.engine as KE
    from c2slm_b200 import synth
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen05b")
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--ctx", type=int, default=32)
    ap.add_argument("--steps", type=int, default=8)
    a = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = nid = None
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
        if rank == 0:
            synth.cached_model(a.model, layers=a.layers)
        dist.barrier()
        obj = [KE.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nid = obj[0]
    path = synth.cached_model(a.model, layers=a.layers)
    with K.Engine(path, device=local, max_tokens=a.ctx + a.steps + 64,
                  tp=(rank, world, nid) if world > 1 else None) as e:
        e.ingest_from(0, np.random.default_rng(2).integers(0, 151643, a.ctx).astype(np.int32))
        tr = e.trace_decode(a.steps + 2, 1.15, 64)[2:]
    if rank == 0:
        res = {"model": a.model, "world": world, "ctx": a.ctx, "phases": phase_table(tr)}
        print(json.dumps(res), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

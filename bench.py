#!/usr/bin/env python
"""Batch-1 greedy decode throughput of the c2slm token loop on B200.

Workload: Qwen2.5-0.5B-shaped Q4_K_M-style GGUF with
seeded random weights (Q5_0 q/k/v/o/gate/up, Q4_K/Q6_K ffn_down, Q8_0 tied
vocabulary projection of 151,936 rows), a 32-token uniform-random prompt,
then greedy decode with the reference's repetition penalty (1.15 over 64).
One step = one decoded token = logits + penalty + argmax + Forward of the
chosen token.  Decoding stays at config 1's positions (32..159): every 128
steps SeqLen is rewound to the prompt (KVCache.Rewind), so any --steps K
measures the same workload.

  value  device-resident decode (one launch of the persistent decode kernel,
         inputs in HBM), CUDA events on the engine's stream, max over ranks.
  e2e    the public C ABI driven from the host one token per call
         (c2s_decode_step: host token in, next token out, synchronised).
--impl reference times the reference's algorithm on the host cores instead
(the CPU port in oracle/, with the WorkerPool's row split; Go is absent).

Multi-GPU (torchrun): one independent request stream per GPU (data
parallel, no collective on the data path), weak scaling.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PERIOD = 128          # decode steps per request (config 1)
PROMPT = 32           # prompt tokens (config 1)
PENALTY, WINDOW = 1.15, 64
METRIC = "batch-1 greedy decode tokens/s (Qwen2.5-0.5B-shaped Q4_K_M, config 1)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=8192)
    ap.add_argument("--warmup", type=int, default=64)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--model", default="qwen05b")
    ap.add_argument("--layers", type=int, default=None,
                    help="decoder depth of the headline model (profiling captures of a shallower copy)")
    ap.add_argument("--profile-steps", type=int, default=8)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-tp7b", action="store_true", help="skip the 7B tensor-parallel line (config 3)")
    ap.add_argument("--tp-ctx", type=int, default=4096, help="config 3 context length before decoding")
    ap.add_argument("--tp-steps", type=int, default=256, help="config 3 decode steps")
    ap.add_argument("--no-prefill", action="store_true", help="skip the tensor-core prefill line (config 4)")
    ap.add_argument("--prefill-tokens", type=int, default=2048, help="config 4 prompt length")
    ap.add_argument("--no-config0", action="store_true", help="skip the single-op matvec line (config 0)")
    ap.add_argument("--no-config2", action="store_true", help="skip the 1.5B decode line (config 2)")
    ap.add_argument("--no-serving", action="store_true", help="skip the data-parallel serving line (config 4)")
    return ap.parse_args()


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def stage_bytes(path: str) -> dict:
    """Algorithmic bytes per decoded token by stage, from the GGUF tensor table."""
    from c2slm_b200 import gguf
    out = {"qkv": 0, "o_proj": 0, "gate_up": 0, "down": 0, "logits": 0, "attention": 0}
    with gguf.File(path) as f:
        T = f.tensor_map
        L = f.get_uint32("qwen2.block_count")[0]
        H = f.get_uint32("qwen2.embedding_length")[0]
        for l in range(L):
            p = f"blk.{l}."
            for n in ("attn_norm.weight", "attn_q.weight", "attn_k.weight", "attn_v.weight",
                      "attn_q.bias", "attn_k.bias", "attn_v.bias"):
                if p + n in T:
                    out["qkv"] += len(T[p + n].data)
            out["o_proj"] += len(T[p + "attn_output.weight"].data)
            out["gate_up"] += sum(len(T[p + n].data) for n in ("ffn_norm.weight", "ffn_gate.weight", "ffn_up.weight"))
            out["down"] += len(T[p + "ffn_down.weight"].data)
            for n in ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"):
                d = T[p + n + ".weight"].dimensions
                out["proj_weights"] = out.get("proj_weights", 0) + int(d[0]) * int(d[1])
        te = T["token_embd.weight"]
        out["qkv"] += len(te.data) // int(te.dimensions[1])  # one embedding row
        ow = T.get("output.weight", te)
        out["logits"] = len(ow.data) + len(T["output_norm.weight"].data)
        kvh = f.get_uint32("qwen2.attention.head_count_kv")[0]
        hd = H // f.get_uint32("qwen2.attention.head_count")[0]
        out["kv_per_pos"] = 2 * L * kvh * hd * 4  # fp32 K and V read per position
        out["layers"] = L
    return out


def phase_table(tr, sb: dict, mean_pos: float) -> dict:
    """Per-phase time of the persistent decode kernel from its trace
    ([step, phase, cta, 8]): a phase lasts from the first CTA's start to the
    first CTA's start of the next phase (grid barrier included); summed over
    layers, median over steps; bytes are the phase's algorithmic bytes."""
    import numpy as np
    tr = tr.astype(np.int64)
    S, NP, G, _ = tr.shape
    first = tr[..., 0].min(axis=2).reshape(-1)              # phase starts, in order
    dur = np.diff(first).astype(np.float64)
    dur = np.append(dur, np.nan).reshape(S, NP)
    kinds = ["logits"] + ["qkv", "attention", "o_proj", "gate_up", "down"] * ((NP - 1) // 5)
    out = {}
    for k in ("qkv", "attention", "o_proj", "gate_up", "down", "logits"):
        idx = [i for i, n in enumerate(kinds) if n == k]
        per_step = np.nansum(dur[:, idx], axis=1)[:-1] / 1000.0  # us; the last step lacks an end
        b = sb["kv_per_pos"] * (mean_pos + 1) if k == "attention" else sb[k]
        if len(per_step) == 0:
            out[k] = {"us_per_step": None, "bytes_per_step": int(b), "gbs": None}
            continue
        us = float(np.median(per_step))
        out[k] = {"us_per_step": round(us, 2), "bytes_per_step": int(b), "gbs": round(b / (us * 1e-6) / 1e9, 1)}
    return out


class Clocks:
    """nvidia-smi sampler running during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.index)], stdout=self.tmp,
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.tmp.flush()
        rows = [r.split(",") for r in open(self.tmp.name).read().strip().splitlines() if r.strip()]
        os.unlink(self.tmp.name)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [x.strip() for x in r]
            try:
                sm.append(float(r[1]))
                smax.append(float(r[2]))
            except (ValueError, IndexError):
                continue
            for n, v in zip(names, r[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_decode_rate(path: str, prompt, warmup: int, max_steps: int, budget_s: float, threads: int):
    """The reference algorithm on the host cores (oracle port, WorkerPool split)."""
    from oracle import oracle as O
    with O.OracleModel(path, max_tokens=PROMPT + PERIOD + 8, nthreads=threads) as o:
        nx = o.ingest_from(0, prompt)
        done = 0
        o.generate(nx, warmup, penalty=PENALTY, window=WINDOW, stop_on_special=False)
        t0 = time.perf_counter()
        while done < max_steps and time.perf_counter() - t0 < budget_s:
            if o.seq_len >= PROMPT + PERIOD:
                o.seq_len = PROMPT  # same rewind as the GPU arm
            # one decode step: logits + penalty + argmax + Forward (c2slm.go:148-223)
            o.generate(nx, 1, penalty=PENALTY, window=WINDOW, stop_on_special=False)
            done += 1
        t_total = time.perf_counter() - t0
    return done / t_total, done, t_total


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from c2slm_b200 import synth
    import numpy as np
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle")], check=True)
    path = synth.cached_model(args.model, layers=args.layers)
    prompt = np.random.default_rng(0).integers(0, 151643, PROMPT).astype(np.int32)
    threads = min(os.cpu_count() or 1, 32)  # engine/pool.go:47-53
    max_steps = min(args.steps, 256)
    rate, done, secs = cpu_decode_rate(path, prompt, min(args.warmup, 2), max_steps, 120.0, threads)
    sample = (f"{done} decode steps (of --steps {args.steps}) at positions {PROMPT}..{PROMPT + PERIOD - 1} "
              f"after a {PROMPT}-token prompt, {secs:.1f} s")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(rate, 3), "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1000.0 / rate, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 (int8 dot for K-quants)", "data": "synthetic",
        "config": {"workload": "config 1: qwen2.5-0.5b-shaped Q4_K_M, 32-token prompt, greedy decode",
                   "model": args.model},
        "cpu_baseline": {"value": round(rate, 3), "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(rate, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "hazyhaar/c2slm is Go (GOEXPERIMENT=simd, Go 1.27); no Go toolchain on this image, so the "
                "reference's scalar algorithm is timed through its C restatement in oracle/",
    }
    print(json.dumps(line), flush=True)


def run_ours(args) -> None:
    import numpy as np
    import torch
    import c2slm_b200 as K
    from c2slm_b200 import synth

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    if rank == 0:
        path = synth.cached_model(args.model, layers=args.layers)
    barrier()
    path = synth.cached_model(args.model, layers=args.layers)
    eng = K.Engine(path, device=local, max_tokens=1024)
    prompt = np.random.default_rng(rank).integers(0, 151643, PROMPT).astype(np.int32)
    eng.ingest_from(0, prompt)

    # ---- value: device-resident decode ---------------------------------
    eng.bench_decode_timed(max(args.warmup, 3), PENALTY, WINDOW, period=PERIOD)
    eng.seq_len = PROMPT
    clocks = Clocks(local)
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    ms = eng.bench_decode_timed(args.steps, PENALTY, WINDOW, period=PERIOD)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms_max = max_over_ranks(ms)
    value = world * args.steps / (ms_max / 1000.0)

    # ---- e2e: host-driven, one public call per token ---------------------
    eng.seq_len = PROMPT - 1
    tok = int(prompt[-1])
    e2e_steps = min(args.steps, 4096)
    for _ in range(8):
        tok = eng.decode_step(tok, PENALTY, WINDOW)
    eng.seq_len = PROMPT - 1
    tok = int(prompt[-1])
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        if eng_seq_wrap(i):
            eng.seq_len = PROMPT - 1
        tok = eng.decode_step(tok, PENALTY, WINDOW)
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    e2e = world * e2e_steps / e2e_s

    # ---- roofline of the dominant kernel and the per-phase breakdown ------
    sb = stage_bytes(path)
    peak, peak_kind = measured_peaks()
    per_token = sum(sb[k] for k in ("qkv", "o_proj", "gate_up", "down", "logits")) + \
        sb["kv_per_pos"] * (PROMPT + PERIOD / 2.0 + 1)
    step_ms = ms_max / args.steps
    launches = eng.decode_launches(args.steps)
    traffic = None
    tp = os.path.join(ROOT, "profiles", "traffic.json")
    if launches == 1:
        # one persistent launch ran the whole timed region: its algorithmic
        # bytes are the weights + KV rows of every step
        kernel = "k_persistent"
        bytes_per_launch = per_token * args.steps
        achieved = bytes_per_launch / (ms / 1000.0) / 1e9
        if os.path.exists(tp):
            t = json.load(open(tp)).get(kernel)
            if t and t.get("dram_bytes_per_step"):
                traffic = int(t["dram_bytes_per_step"] * args.steps)
        eng.seq_len = PROMPT
        phases = phase_table(eng.trace_decode(args.profile_steps + 2, PENALTY, WINDOW)[2:], sb,
                             PROMPT + 2 + args.profile_steps / 2.0)
    else:
        eng.seq_len = PROMPT
        prof = eng.profile_step(args.profile_steps, PENALTY, WINDOW)
        sb["attention"] = sb["kv_per_pos"] * (PROMPT + args.profile_steps / 2.0 + 1)
        phases = {}
        for name, d in prof.items():
            if d["launches"]:
                per_launch = sb[name] * args.profile_steps / d["launches"]
                phases[name] = {"us_per_step": round(1000 * d["ms"] / args.profile_steps, 2),
                                "launches": d["launches"], "bytes_per_launch": int(per_launch),
                                "gbs": round(per_launch / (d["ms"] / d["launches"] / 1000.0) / 1e9, 1)}
        kernel = max(phases, key=lambda k: phases[k]["us_per_step"])
        bytes_per_launch = phases[kernel]["bytes_per_launch"]
        achieved = phases[kernel]["gbs"]
        if os.path.exists(tp):
            t = json.load(open(tp)).get(kernel)
            traffic = t.get("dram_bytes_per_launch") if isinstance(t, dict) else t

    # ---- CPU baseline (rank 0, N=1) ---------------------------------------
    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        threads = min(os.cpu_count() or 1, 32)
        rate, done, secs = cpu_decode_rate(path, prompt, 1, 64, 20.0, threads)
        cpu = {"value": round(rate, 3), "unit": "tokens/s", "cores": threads, "kind": "port",
               "sample": f"{done} decode steps at positions {PROMPT}.. after a {PROMPT}-token prompt, {secs:.1f} s"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 activations; int8 dp4a for K-quant x Q8_K", "data": "synthetic",
            "config": {"workload": "config 1: qwen2.5-0.5b-shaped Q4_K_M (Q5_0/Q4_K/Q6_K/Q8_0), 32-token prompt, "
                                   "greedy decode at positions 32..159 (rewound every 128 steps)",
                       "model": args.model, "global_batch": world, "parallelism": f"dp{world}",
                       "l2": "inputs larger than L2 (%.0f MB of weights streamed per step)" % (per_token / 1e6),
                       "bytes_per_token": int(per_token),
                       "step_hbm_frac": round(per_token / (step_ms / 1000.0) / 1e9 / peak, 4)},
            "roofline": {"bound": "hbm", "kernel": kernel, "achieved": round(achieved, 1), "peak": peak,
                         "peak_kind": f"{peak_kind} hbm_gbs", "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": traffic, "bytes_per_launch": int(bytes_per_launch)},
            "phases": phases,
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e, 2), "unit": "tokens/s", "h2d_bytes_per_step": 36, "d2h_bytes_per_step": 4,
                    "api": "c2s_decode_step"},
            "gpu_launches": launches,
            "clocks": clk,
        }
    eng.close()
    tp7b = None
    if not args.no_tp7b:
        tp7b = run_tp7b(args, world, rank, local, dist)
    prefill = None
    if not args.no_prefill and rank == 0:
        prefill = run_prefill(args, local)
    serving = None
    if not args.no_serving:
        serving = run_serving(args, world, rank, local, dist)
    config0 = config2 = None
    if rank == 0 and not args.no_config0:
        config0 = run_config0(local)
    if rank == 0 and not args.no_config2:
        config2 = run_config2(args, local)
    if rank == 0:
        if tp7b is not None:
            line["tp7b"] = tp7b
        if prefill is not None:
            line["prefill"] = prefill
        if serving is not None:
            line["serving"] = serving
        if config0 is not None:
            line["config0"] = config0
        if config2 is not None:
            line["config2"] = config2
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_tp7b(args, world: int, rank: int, local: int, dist) -> dict:
    """the 7B-shaped model tensor-parallel over the run's
    GPUs (one rank per GPU; one GPU runs the whole model), context prefilled
    to --tp-ctx positions from a uniform-random prompt (seed 2), then
    --tp-steps greedy decode steps timed on the device (max over ranks).
    Strong scaling: one request stream whatever the GPU count."""
    import numpy as np
    import torch
    import c2slm_b200 as K
    import c2slm_b200.engine as KE
    from c2slm_b200 import synth

    if rank == 0:
        synth.cached_model("qwen7b")
    nid = None
    if world > 1:
        dist.barrier()
        obj = [KE.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nid = obj[0]
    path = synth.cached_model("qwen7b")
    ctx, steps = args.tp_ctx, args.tp_steps
    eng = K.Engine(path, device=local, max_tokens=ctx + steps + 16, tp=(rank, world, nid) if world > 1 else None)
    prompt = np.random.default_rng(2).integers(0, 151643, ctx).astype(np.int32)
    t0 = time.perf_counter()
    eng.ingest_from(0, prompt)
    prefill_s = time.perf_counter() - t0
    eng.bench_decode_timed(3, PENALTY, WINDOW, period=0)
    eng.seq_len = ctx
    torch.cuda.synchronize()
    ms = eng.bench_decode_timed(steps, PENALTY, WINDOW, period=steps)
    launches = eng.decode_launches(steps)
    eng.close()
    if dist is not None:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    sb = stage_bytes(path)
    per_token = sum(sb[k] for k in ("qkv", "o_proj", "gate_up", "down", "logits")) + \
        sb["kv_per_pos"] * (ctx + steps / 2.0 + 1)
    peak, kind = measured_peaks()
    tok_s = steps / (ms / 1000.0)
    per_gpu = per_token * tok_s / world / 1e9
    return {"metric": "batch-1 greedy decode tokens/s, Qwen2.5-7B-shaped Q4_K_M (config 3), tensor parallel",
            "value": round(tok_s, 2), "unit": "tokens/s", "n_gpus": world, "scaling": "strong",
            "ms_per_step": round(ms / steps, 4), "context": ctx, "steps": steps,
            "bytes_per_token": int(per_token), "achieved_gbs_per_gpu": round(per_gpu, 1),
            "frac_per_gpu": round(per_gpu / peak, 4), "peak_kind": f"{kind} hbm_gbs",
            "gpu_launches": launches, "prefill_s": round(prefill_s, 1),
            "decode": "persistent kernel, partial sums exchanged over NVLink peer memory" if launches == 1
                      else "per-phase kernels with NCCL collectives"}


INT8_NOMINAL_TOPS = 4500.0  # B200 dense int8 (nominal; 8.1k MACs/clk/SM measured with tcgen05 kind::i8)


def run_prefill(args, local: int) -> dict:
    """Config 4's prefill: a uniform-random prompt of --prefill-tokens ids
    ingested by a Qwen2.5-1.5B-shaped Q4_K_M model (all projections K-quant)
    through IngestFrom -- K-quant x Q8_K projections as tcgen05 int8 GEMMs.
    Timed end to end through the public API (host ids in, NormX back), after
    one warm-up ingest that also builds the weight planes."""
    import numpy as np
    import c2slm_b200 as K
    from c2slm_b200 import synth
    n = args.prefill_tokens
    path = synth.cached_model("qwen15b")
    prompt = np.random.default_rng(3).integers(0, 151643, n).astype(np.int32)
    eng = K.Engine(path, device=local, max_tokens=n + 64)
    eng.ingest_from(0, prompt[:256])
    eng.sync()
    times = []
    for _ in range(3):
        eng.reset()
        t0 = time.perf_counter()
        eng.ingest_from(0, prompt)
        eng.sync()
        times.append(time.perf_counter() - t0)
    eng.close()
    dt = statistics.median(times)
    sb = stage_bytes(path)
    macs = sb.get("proj_weights")  # multiply-adds of the layer projections per token
    out = {"metric": "prefill tokens/s (config 4: Qwen2.5-1.5B-shaped Q4_K_M, uniform-random prompt)",
           "value": round(n / dt, 1), "unit": "tokens/s", "tokens": n, "ms": round(dt * 1000.0, 2),
           "api": "c2s_ingest_from (host ids in, NormX out)",
           "kernels": "tcgen05 kind::i8 GEMM per K-quant projection (128 rows x 128 tokens per CTA); "
                      "tcgen05 kind::tf32 causal attention (f32 operands split hi + lo; 128 queries x 64-key "
                      "tiles, key splits)"}
    if macs:
        tops = 2.0 * macs * n / dt / 1e12
        out.update({"int8_tops_projections": round(tops, 1), "int8_nominal_tops": INT8_NOMINAL_TOPS,
                    "frac_of_nominal_int8": round(tops / INT8_NOMINAL_TOPS, 4)})
    return out


def run_config0(local: int) -> dict:
    """one Q4_K x Q8_K matvec of the ffn_down shape (896
    rows x 4864 columns, seed 0; x ~ N(0,1) quantised to Q8_K inside the op),
    10,000 repetitions through c2s_bench_gemv (device pointers, one CUDA graph
    of 1000 launches per replay): L2-hot (one weight copy) and HBM-cold (128
    rotated copies, 314 MB > L2).  The reference's counterpart is
    BenchmarkGEMVQ4_K_Q8_K_Cols896 (tensor/ops_test.go:143-156)."""
    import numpy as np
    import torch
    import c2slm_b200.engine as KE
    from c2slm_b200 import synth
    rows, cols, reps, copies = 896, 4864, 10000, 128
    rng = np.random.default_rng(0)
    w = synth.gen_blocks(rng, KE.Q4_K, rows, cols)
    x = rng.normal(0, 1, cols).astype(np.float32)
    stride = (w.nbytes + 255) // 256 * 256
    dev = torch.device("cuda", local)
    dw = torch.zeros(stride * copies + 256, dtype=torch.uint8, device=dev)
    one = torch.from_numpy(w).to(dev)
    for k in range(copies):
        dw[k * stride:k * stride + w.nbytes].copy_(one)
    dx = torch.from_numpy(x).to(dev)
    dy = torch.zeros(rows, dtype=torch.float32, device=dev)
    torch.cuda.synchronize()
    algo = w.nbytes + cols * 4 + rows * 4  # weights + f32 x + f32 y per matvec
    peak, kind = measured_peaks()
    out = {"metric": "single-op Q4_K x Q8_K matvec (config 0: 896 x 4864, ffn_down shape)", "unit": "us/op",
           "higher_is_better": False, "reps": reps, "bytes_per_op": algo,
           "api": "c2s_bench_gemv (c2s_gemv_device launches in a CUDA graph, Q8_K of x inside each launch)"}
    for name, n in (("l2_hot", 1), ("hbm_cold", copies)):
        ms = KE.bench_gemv(local, KE.Q4_K, dw.data_ptr(), stride, n, dx.data_ptr(), dy.data_ptr(), rows, cols, reps)
        us = ms * 1000.0 / reps
        gbs = algo / (us * 1e-6) / 1e9
        out[name] = {"value": round(us, 3), "unit": "us/op", "copies": n, "achieved_gbs": round(gbs, 1)}
        if n > 1:
            out[name]["roofline"] = {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                                     "frac": round(gbs / peak, 4), "peak_kind": f"{kind} hbm_gbs"}
    out["value"] = out["hbm_cold"]["value"]
    return out


def run_config2(args, local: int) -> dict:
    """the 1.5B-shaped Q4_K_M model (Q4_K/Q6_K, tied Q6_K
    vocabulary projection), KV cache prefilled to 1024 positions from a
    1024-token uniform-random prompt (seed 1, tensor-core prefill), then 256
    greedy decode steps in one persistent launch, timed with CUDA events."""
    import numpy as np
    import c2slm_b200 as K
    from c2slm_b200 import synth
    ctx, steps = 1024, 256
    path = synth.cached_model("qwen15b")
    prompt = np.random.default_rng(1).integers(0, 151643, ctx).astype(np.int32)
    eng = K.Engine(path, device=local, max_tokens=ctx + steps + 16)
    eng.ingest_from(0, prompt)
    eng.bench_decode_timed(3, PENALTY, WINDOW, period=0)
    eng.seq_len = ctx
    ms = eng.bench_decode_timed(steps, PENALTY, WINDOW, period=steps)
    launches = eng.decode_launches(steps)
    eng.close()
    sb = stage_bytes(path)
    per_token = sum(sb[k] for k in ("qkv", "o_proj", "gate_up", "down", "logits")) + \
        sb["kv_per_pos"] * (ctx + steps / 2.0 + 1)
    peak, kind = measured_peaks()
    tok_s = steps / (ms / 1000.0)
    gbs = per_token * tok_s / 1e9
    return {"metric": "batch-1 greedy decode tokens/s (config 2: Qwen2.5-1.5B-shaped Q4_K_M, 1024-token context)",
            "value": round(tok_s, 2), "unit": "tokens/s", "ms_per_step": round(ms / steps, 4), "context": ctx,
            "steps": steps, "bytes_per_token": int(per_token), "gpu_launches": launches,
            "roofline": {"bound": "hbm", "kernel": "k_persistent", "achieved": round(gbs, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(gbs / peak, 4), "peak_kind": f"{kind} hbm_gbs"}}


SERVING_STREAMS, SERVING_PROMPT, SERVING_STEPS, SERVING_PENALTY = 8, 512, 256, 1.1


def run_serving(args, world: int, rank: int, local: int, dist) -> dict | None:
    """BASELINE config 4's serving mode: 8 independent request streams of the
    1.5B-shaped model (seeds 3..10), stream s on rank s % world (one per GPU
    at 8 GPUs).  Each stream: IngestFrom of a 512-token uniform-random prompt
    (tensor-core prefill), then 256 greedy steps with repetition penalty 1.1
    over the last 64 tokens (stop tokens do not end a stream, so every stream
    decodes 256 tokens).  Timed end to end through the public API on the host
    (ids in, ids out), max over ranks; no collective on the data path."""
    import numpy as np
    import torch
    import c2slm_b200 as K
    from c2slm_b200 import synth
    if rank == 0:
        synth.cached_model("qwen15b")
    if dist is not None:
        dist.barrier()
    path = synth.cached_model("qwen15b")
    eng = K.Engine(path, device=local, max_tokens=SERVING_PROMPT + SERVING_STEPS + 16)
    warm = np.random.default_rng(99).integers(0, 151643, SERVING_PROMPT).astype(np.int32)
    eng.ingest_from(0, warm)
    eng.generate(8, penalty=SERVING_PENALTY, window=WINDOW, stop_on_special=False)
    mine = [s for s in range(SERVING_STREAMS) if s % world == rank]
    pre_s = dec_s = 0.0
    n_dec = 0
    torch.cuda.synchronize()
    for s in mine:
        prompt = np.random.default_rng(3 + s).integers(0, 151643, SERVING_PROMPT).astype(np.int32)
        eng.reset()
        t0 = time.perf_counter()
        eng.ingest_from(0, prompt)
        eng.sync()
        t1 = time.perf_counter()
        toks = eng.generate(SERVING_STEPS, penalty=SERVING_PENALTY, window=WINDOW, stop_on_special=False)
        t2 = time.perf_counter()
        pre_s += t1 - t0
        dec_s += t2 - t1
        n_dec += len(toks)
    eng.close()
    tot = torch.tensor([pre_s, dec_s, float(n_dec)], dtype=torch.float64, device="cuda")
    if dist is not None:
        mx = tot.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
        pre_s, dec_s = float(mx[0].item()), float(mx[1].item())
        n_dec = int(tot[2].item())
    if rank != 0:
        return None
    sb = stage_bytes(path)
    per_token = sum(sb[k] for k in ("qkv", "o_proj", "gate_up", "down", "logits")) + \
        sb["kv_per_pos"] * (SERVING_PROMPT + SERVING_STEPS / 2.0 + 1)
    peak, kind = measured_peaks()
    dec_rate = n_dec / dec_s
    per_gpu_gbs = per_token * dec_rate / min(world, SERVING_STREAMS) / 1e9
    return {"metric": "aggregate decode tokens/s (config 4 serving: 8 streams of the 1.5B shape, 512-token prompts, "
                      "256 greedy steps, penalty 1.1 over 64)",
            "value": round(dec_rate, 1), "unit": "tokens/s", "n_gpus": world, "streams": SERVING_STREAMS,
            "scaling": "strong", "decode_tokens": n_dec,
            "prefill_tokens_per_s": round(SERVING_STREAMS * SERVING_PROMPT / pre_s, 1),
            "timing": "host wall clock around c2s_ingest_from / c2s_generate (ids in, ids out), max over ranks",
            "roofline": {"bound": "hbm", "achieved": round(per_gpu_gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(per_gpu_gbs / peak, 4), "peak_kind": f"{kind} hbm_gbs",
                         "per": "GPU, decode"}}


def eng_seq_wrap(i: int) -> bool:
    return i > 0 and i % PERIOD == 0


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

"""Seeded synthetic Qwen2.5-shaped GGUF models (random weights, native blocks).

The reference measures on a real Qwen2.5-0.5B-Instruct Q4_K_M file; no
checkpoint is available here, so these files stand in for it: the same
architecture, tensor names, GGML block layouts and metadata keys that
engine/model.go:58-210 reads, filled with seeded random values drawn from the
distributions stated for each benchmark configuration.

Block encodings (tensor/ops.go:11-22, 342-424):
  Q5_0 22 B: fp16 d, u32 qh, 16 B qs          d ~ U[1e-3, 5e-3]
  Q8_0 34 B: fp16 d, 32 x int8               d ~ U[1e-3, 5e-3]
  Q4_K 144 B: fp16 d, fp16 dmin, 12 B 6-bit scales/mins, 128 B nibbles
             d, dmin ~ U[1e-4, 2e-3], scales/mins ~ U{0..63}
  Q6_K 210 B: ql[128], qh[64], int8 sc[16], fp16 d
             sc ~ U{-32..31}, d ~ U[1e-4, 1e-3]
Biases ~ N(0, 0.02^2); norm weights = 1 + N(0, 0.05^2).

Usage: python -m c2slm_b200.synth qwen05b /tmp/m.gguf [--layers N] [--seed S]
"""
from __future__ import annotations

import argparse
import math
import os
import struct
from dataclasses import dataclass, replace

import numpy as np

from . import gguf as G

ALIGN = 32


@dataclass(frozen=True)
class Config:
    name: str
    embd: int
    layers: int
    heads: int
    kv_heads: int
    ffn: int
    vocab: int
    tied: bool
    # quant types per tensor family
    attn_type: int          # q, k, o
    v_type: int             # attn_v (ordinary layers)
    v_more: int             # attn_v on "more bits" layers
    gate_up_type: int
    down_type: int
    down_more: int
    embd_type: int
    output_type: int        # used only when untied
    seed: int = 0
    rope_base: float = 1e6
    eps: float = 1e-6
    with_bias: bool = True
    qk_norm: bool = False   # Qwen3 per-head q/k RMSNorm weights

    @property
    def head_dim(self) -> int:
        return self.embd // self.heads


# BASELINE configs 1..3 (config 0 is a single-op case, config 4 reuses 1.5B)
PRESETS = {
    "qwen05b": Config("qwen05b", 896, 24, 14, 2, 4864, 151936, True,
                      G.Q5_0, G.Q5_0, G.Q8_0, G.Q5_0, G.Q4_K, G.Q6_K, G.Q8_0, G.Q8_0, seed=0),
    "qwen15b": Config("qwen15b", 1536, 28, 12, 2, 8960, 151936, True,
                      G.Q4_K, G.Q4_K, G.Q6_K, G.Q4_K, G.Q4_K, G.Q6_K, G.Q6_K, G.Q6_K, seed=1),
    "qwen7b": Config("qwen7b", 3584, 28, 28, 4, 18944, 152064, False,
                     G.Q4_K, G.Q4_K, G.Q6_K, G.Q4_K, G.Q4_K, G.Q6_K, G.Q4_K, G.Q6_K, seed=2),
    # small models with the same type mixes, for fast CPU-oracle parity runs
    "tiny05": Config("tiny05", 256, 3, 4, 2, 512, 2048, True,
                     G.Q5_0, G.Q5_0, G.Q8_0, G.Q5_0, G.Q4_K, G.Q6_K, G.Q8_0, G.Q8_0, seed=5),
    "tiny15": Config("tiny15", 512, 3, 4, 2, 768, 2048, True,
                     G.Q4_K, G.Q4_K, G.Q6_K, G.Q4_K, G.Q4_K, G.Q6_K, G.Q6_K, G.Q6_K, seed=6),
    "tiny7": Config("tiny7", 512, 3, 4, 2, 1024, 3000, False,
                    G.Q4_K, G.Q4_K, G.Q6_K, G.Q4_K, G.Q4_K, G.Q6_K, G.Q4_K, G.Q6_K, seed=7),
    # K-quant projections with 64-wide heads (the tensor-core prefill's HD = 64 path)
    "tiny64": Config("tiny64", 512, 2, 8, 2, 1024, 2048, True,
                     G.Q4_K, G.Q4_K, G.Q6_K, G.Q4_K, G.Q4_K, G.Q6_K, G.Q6_K, G.Q6_K, seed=9),
    "tiny3": Config("tiny3", 256, 2, 4, 2, 512, 1024, False,
                    G.Q5_0, G.Q8_0, G.Q8_0, G.Q5_0, G.Q4_K, G.Q6_K, G.Q5_0, G.Q4_K, seed=8,
                    qk_norm=True),
}


def more_bits(i: int, n: int) -> bool:
    """Q4_K_M "more bits" layers: {0..a} U {L-b..L-1} U every third between.
    (a, L-b) = (2, 21) at 24 layers and (3, 24) at 28 layers."""
    k = -(-n // 8)  # ceil(n/8)
    a, hi = k - 1, n - k
    return i <= a or i >= hi or (i - a - 1) % 3 == 2


def _fp16_bytes(v: np.ndarray) -> np.ndarray:
    return v.astype(np.float16).view(np.uint8).reshape(-1, 2)


def gen_blocks(rng: np.random.Generator, t: int, rows: int, cols: int) -> np.ndarray:
    """Random tensor data (rows x cols) in GGML block layout t, as uint8."""
    if t == G.Q5_0:
        nb = rows * (cols // 32)
        out = np.empty((nb, 22), np.uint8)
        out[:, 0:2] = _fp16_bytes(rng.uniform(1e-3, 5e-3, nb))
        out[:, 2:22] = rng.integers(0, 256, (nb, 20), dtype=np.uint8)
        return out.reshape(-1)
    if t == G.Q8_0:
        nb = rows * (cols // 32)
        out = np.empty((nb, 34), np.uint8)
        out[:, 0:2] = _fp16_bytes(rng.uniform(1e-3, 5e-3, nb))
        out[:, 2:34] = rng.integers(0, 256, (nb, 32), dtype=np.uint8)
        return out.reshape(-1)
    if t == G.Q4_K:
        nb = rows * (cols // 256)
        out = np.empty((nb, 144), np.uint8)
        out[:, 0:2] = _fp16_bytes(rng.uniform(1e-4, 2e-3, nb))
        out[:, 2:4] = _fp16_bytes(rng.uniform(1e-4, 2e-3, nb))
        sc = rng.integers(0, 64, (nb, 8), dtype=np.uint8)
        mn = rng.integers(0, 64, (nb, 8), dtype=np.uint8)
        s = np.empty((nb, 12), np.uint8)  # inverse of tensor/ops.go:354-361
        s[:, 0:4] = sc[:, 0:4] | ((sc[:, 4:8] >> 4) << 6)
        s[:, 4:8] = mn[:, 0:4] | ((mn[:, 4:8] >> 4) << 6)
        s[:, 8:12] = (sc[:, 4:8] & 15) | ((mn[:, 4:8] & 15) << 4)
        out[:, 4:16] = s
        out[:, 16:144] = rng.integers(0, 256, (nb, 128), dtype=np.uint8)
        return out.reshape(-1)
    if t == G.Q6_K:
        nb = rows * (cols // 256)
        out = np.empty((nb, 210), np.uint8)
        out[:, 0:192] = rng.integers(0, 256, (nb, 192), dtype=np.uint8)
        out[:, 192:208] = rng.integers(-32, 32, (nb, 16)).astype(np.int8).view(np.uint8)
        out[:, 208:210] = _fp16_bytes(rng.uniform(1e-4, 1e-3, nb))
        return out.reshape(-1)
    raise ValueError(f"unsupported type {t}")


class _Writer:
    """Streams a GGUF v3 file: header, metadata, tensor infos, aligned data."""

    def __init__(self):
        self.kv: list[bytes] = []
        self.infos: list[tuple] = []  # (name, dims, type, nbytes, producer)

    @staticmethod
    def _s(s: str) -> bytes:
        b = s.encode()
        return struct.pack("<Q", len(b)) + b

    def add_u32(self, k, v):
        self.kv.append(self._s(k) + struct.pack("<II", 4, v))

    def add_f32(self, k, v):
        self.kv.append(self._s(k) + struct.pack("<If", 6, v))

    def add_str(self, k, v):
        self.kv.append(self._s(k) + struct.pack("<I", 8) + self._s(v))

    def add_str_array(self, k, arr):
        parts = [self._s(k), struct.pack("<IIQ", 9, 8, len(arr))]
        parts += [self._s(s) for s in arr]
        self.kv.append(b"".join(parts))

    def add_tensor(self, name, dims, t, producer):
        self.infos.append((name, list(dims), t, G.tensor_byte_size(t, dims), producer))

    def write(self, path: str) -> None:
        with open(path, "wb") as f:
            f.write(struct.pack("<IIQQ", G.GGUF_MAGIC, 3, len(self.infos), len(self.kv)))
            for kv in self.kv:
                f.write(kv)
            off = 0
            offs = []
            for name, dims, t, nb, _ in self.infos:
                offs.append(off)
                f.write(self._s(name) + struct.pack("<I", len(dims)))
                f.write(struct.pack("<%dQ" % len(dims), *dims))
                f.write(struct.pack("<IQ", t, off))
                off += nb
                off += (-off) % ALIGN
            pos = f.tell()
            f.write(b"\0" * ((-pos) % ALIGN))
            base = f.tell()
            for (name, dims, t, nb, producer), o in zip(self.infos, offs):
                cur = f.tell() - base
                if cur < o:
                    f.write(b"\0" * (o - cur))
                data = producer()
                assert data.nbytes == nb, (name, data.nbytes, nb)
                f.write(data.tobytes())


def token_strings(vocab: int) -> list[str]:
    """Placeholder vocabulary; specials where Qwen2.5 keeps them (151643-151645)
    or, for small test vocabularies, in the last three ids."""
    toks = [f"t{i}" for i in range(vocab)]
    base = 151643 if vocab > 151646 else vocab - 3
    toks[base] = "<|endoftext|>"
    toks[base + 1] = "<|im_start|>"
    toks[base + 2] = "<|im_end|>"
    return toks


def write_model(cfg: Config, path: str) -> str:
    """Writes cfg as a GGUF file; returns path."""
    rng_master = np.random.default_rng(cfg.seed)
    seeds = rng_master.integers(0, 2**63 - 1, 10_000)
    counter = [0]

    def rng():
        s = int(seeds[counter[0]])
        counter[0] += 1
        return np.random.default_rng(s)

    w = _Writer()
    w.add_str("general.architecture", "qwen2")
    w.add_str("general.name", f"synthetic-{cfg.name}")
    w.add_u32("general.alignment", ALIGN)
    w.add_u32("qwen2.context_length", 32768)
    w.add_u32("qwen2.embedding_length", cfg.embd)
    w.add_u32("qwen2.block_count", cfg.layers)
    w.add_u32("qwen2.attention.head_count", cfg.heads)
    w.add_u32("qwen2.attention.head_count_kv", cfg.kv_heads)
    w.add_u32("qwen2.feed_forward_length", cfg.ffn)
    w.add_f32("qwen2.rope.freq_base", cfg.rope_base)
    w.add_f32("qwen2.attention.layer_norm_rms_epsilon", cfg.eps)
    w.add_str("tokenizer.ggml.model", "gpt2")
    w.add_str_array("tokenizer.ggml.tokens", token_strings(cfg.vocab))

    H, F, hd, kvd = cfg.embd, cfg.ffn, cfg.head_dim, cfg.kv_heads * cfg.head_dim

    def blocks(t, rows, cols):
        r = rng()
        return lambda: gen_blocks(r, t, rows, cols)

    def norm(n):
        r = rng()
        return lambda: (1.0 + r.normal(0, 0.05, n)).astype(np.float32)

    def bias(n):
        r = rng()
        return lambda: r.normal(0, 0.02, n).astype(np.float32)

    w.add_tensor("token_embd.weight", [H, cfg.vocab], cfg.embd_type, blocks(cfg.embd_type, cfg.vocab, H))
    w.add_tensor("output_norm.weight", [H], G.F32, norm(H))
    if not cfg.tied:
        w.add_tensor("output.weight", [H, cfg.vocab], cfg.output_type, blocks(cfg.output_type, cfg.vocab, H))
    for i in range(cfg.layers):
        mb = more_bits(i, cfg.layers)
        vt = cfg.v_more if mb else cfg.v_type
        dt = cfg.down_more if mb else cfg.down_type
        p = f"blk.{i}."
        w.add_tensor(p + "attn_norm.weight", [H], G.F32, norm(H))
        w.add_tensor(p + "attn_q.weight", [H, H], cfg.attn_type, blocks(cfg.attn_type, H, H))
        w.add_tensor(p + "attn_k.weight", [H, kvd], cfg.attn_type, blocks(cfg.attn_type, kvd, H))
        w.add_tensor(p + "attn_v.weight", [H, kvd], vt, blocks(vt, kvd, H))
        if cfg.with_bias:
            w.add_tensor(p + "attn_q.bias", [H], G.F32, bias(H))
            w.add_tensor(p + "attn_k.bias", [kvd], G.F32, bias(kvd))
            w.add_tensor(p + "attn_v.bias", [kvd], G.F32, bias(kvd))
        if cfg.qk_norm:
            w.add_tensor(p + "attn_q_norm.weight", [hd], G.F32, norm(hd))
            w.add_tensor(p + "attn_k_norm.weight", [hd], G.F32, norm(hd))
        w.add_tensor(p + "attn_output.weight", [H, H], cfg.attn_type, blocks(cfg.attn_type, H, H))
        w.add_tensor(p + "ffn_norm.weight", [H], G.F32, norm(H))
        w.add_tensor(p + "ffn_gate.weight", [H, F], cfg.gate_up_type, blocks(cfg.gate_up_type, F, H))
        w.add_tensor(p + "ffn_up.weight", [H, F], cfg.gate_up_type, blocks(cfg.gate_up_type, F, H))
        w.add_tensor(p + "ffn_down.weight", [F, H], dt, blocks(dt, H, F))
    w.write(path)
    return path


def get_config(name: str, layers: int | None = None, seed: int | None = None) -> Config:
    cfg = PRESETS[name]
    if layers is not None:
        cfg = replace(cfg, layers=layers)
    if seed is not None:
        cfg = replace(cfg, seed=seed)
    return cfg


def cached_model(name: str, layers: int | None = None, seed: int | None = None,
                 cache_dir: str | None = None) -> str:
    """Writes (once) and returns the path of a synthetic model in cache_dir."""
    cfg = get_config(name, layers, seed)
    cache_dir = cache_dir or os.environ.get("C2S_MODEL_CACHE", "/tmp/c2s_models")
    os.makedirs(cache_dir, exist_ok=True)
    path = os.path.join(cache_dir, f"{cfg.name}_L{cfg.layers}_s{cfg.seed}.gguf")
    if not os.path.exists(path):
        tmp = path + f".tmp{os.getpid()}"
        write_model(cfg, tmp)
        os.replace(tmp, path)
    return path


def weight_bytes(path: str) -> dict:
    """Per-token algorithmic bytes of a model file: every quantised matrix is
    read once per decoded token, plus norms/biases; the tied or separate vocab
    projection is counted once."""
    with G.File(path) as f:
        total = 0
        logits = 0
        for ti in f.tensors:
            if ti.name == "token_embd.weight":
                continue  # one row per token; the (tied) projection is counted below
            total += len(ti.data)
        out = f.tensor_map.get("output.weight") or f.tensor_map["token_embd.weight"]
        if "output.weight" not in f.tensor_map:
            total += len(out.data)
        logits = len(out.data)
        embd_row = len(f.tensor_map["token_embd.weight"].data) // int(f.tensor_map["token_embd.weight"].dimensions[1])
    return {"weights": total + embd_row, "logits": logits}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("preset", choices=sorted(PRESETS))
    ap.add_argument("out")
    ap.add_argument("--layers", type=int)
    ap.add_argument("--seed", type=int)
    a = ap.parse_args()
    write_model(get_config(a.preset, a.layers, a.seed), a.out)
    print(a.out, os.path.getsize(a.out), "bytes")


if __name__ == "__main__":
    main()

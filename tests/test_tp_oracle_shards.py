"""Tensor-parallel shard arithmetic on the CPU, world size 2 over gloo.

Each rank runs its c2s_tp_plan shard of the decoder step through the CPU
oracle's kernels (the reference's scalar arithmetic): q/k/v rows of its
query heads and the kv heads they use, attention over its own KV shard,
attn_output on its columns (whole 256-column superblocks), gate/up rows and
ffn_down columns of its FFN superblocks, vocabulary rows of its split.  The
o-proj and ffn_down partial rows are summed over the ranks (all_reduce)
before the residual add (engine/forward.go:112-114,129-131 add the full
sums), the logits are all-gathered.  Rank 0 checks NormX and the logits
against the one-rank oracle (engine/forward.go:54-212) at the north_star
tolerance, 1e-3 of max|ref|.  No GPU: this is the host-side contract the
GPU tensor-parallel engine (tests/test_gpu_tp.py) implements.
"""
import os
import socket

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TOL = 1e-3


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class Shard:
    """One rank's share of the model, sliced out of the GGUF tensors."""

    def __init__(self, path, rank, world):
        import c2slm_b200.engine as KE
        from c2slm_b200 import gguf
        from oracle import oracle as O
        self.O = O
        self.f = gguf.File(path)
        T = self.f.tensor_map
        g = lambda k: self.f.get_uint32(k)[0]
        self.H, self.L = g("qwen2.embedding_length"), g("qwen2.block_count")
        self.NH, self.KVH = g("qwen2.attention.head_count"), g("qwen2.attention.head_count_kv")
        self.F = g("qwen2.feed_forward_length")
        self.hd = self.H // self.NH
        self.eps = float(self.f.get_float32("qwen2.attention.layer_norm_rms_epsilon")[0])
        theta = float(self.f.get_float32("qwen2.rope.freq_base")[0])
        self.V = int(T["token_embd.weight"].dimensions[1])
        d = KE.ModelDesc()
        d.embd, d.n_layers, d.n_heads, d.n_kv_heads, d.ffn, d.vocab = self.H, self.L, self.NH, self.KVH, self.F, self.V
        d.head_dim = 0
        self.p = KE.tp_plan(d, rank, world)
        self.T = T
        self.max_len = 64
        self.rope = O.rope_table(self.max_len, self.hd, theta)
        nkv = self.p["g1"] - self.p["g0"]
        self.kc = np.zeros((self.L, nkv, self.max_len, self.hd), np.float32)
        self.vc = np.zeros_like(self.kc)

    def t(self, name):
        ti = self.T[name]
        return ti.type, np.frombuffer(ti.data, np.uint8), [int(x) for x in ti.dimensions]

    def rows(self, name, r0, r1):
        """rows [r0, r1) of a 2-D tensor"""
        typ, data, dims = self.t(name)
        rb = data.size // dims[1]
        return typ, data[r0 * rb:r1 * rb], dims[0]

    def cols(self, name, c0, c1):
        """columns [c0, c1) of every row (whole blocks)"""
        typ, data, dims = self.t(name)
        cols, nrows = dims[0], dims[1]
        rb = data.size // nrows
        blk = {6: 32, 8: 32, 12: 256, 14: 256}[typ]
        bb = rb // (cols // blk)
        m = data.reshape(nrows, rb)[:, (c0 // blk) * bb:(c1 // blk) * bb]
        return typ, np.ascontiguousarray(m).reshape(-1), c1 - c0, nrows

    def vec(self, name, a=None, b=None):
        v = np.frombuffer(self.T[name].data, np.float32)
        return v if a is None else v[a:b]

    def gemv_rows(self, name, r0, r1, x):
        typ, w, cols = self.rows(name, r0, r1)
        return self.O.gemv(typ, w, x, r1 - r0, cols)

    def gemv_cols(self, name, c0, c1, x):
        typ, w, ncols, nrows = self.cols(name, c0, c1)
        return self.O.gemv(typ, w, x, nrows, ncols)

    def forward(self, tok, pos, allreduce):
        O, p, hd = self.O, self.p, self.hd
        typ, data, dims = self.t("token_embd.weight")
        rb = data.size // dims[1]
        X = O.dequant_row(typ, data[tok * rb:(tok + 1) * rb], self.H)
        qpk = self.NH // self.KVH
        nh = p["h1"] - p["h0"]
        scale = np.float32(1.0 / np.sqrt(np.float64(hd)))
        for l in range(self.L):
            b = f"blk.{l}."
            xn = O.rmsnorm(X, self.vec(b + "attn_norm.weight"), self.eps)
            q0, q1 = p["h0"] * hd, p["h1"] * hd
            k0, k1 = p["g0"] * hd, p["g1"] * hd
            q = self.gemv_rows(b + "attn_q.weight", q0, q1, xn) + self.vec(b + "attn_q.bias", q0, q1)
            k = self.gemv_rows(b + "attn_k.weight", k0, k1, xn) + self.vec(b + "attn_k.bias", k0, k1)
            v = self.gemv_rows(b + "attn_v.weight", k0, k1, xn) + self.vec(b + "attn_v.bias", k0, k1)
            q = O.rope_apply(self.rope, self.max_len, hd, q, nh, pos)
            k = O.rope_apply(self.rope, self.max_len, hd, k, p["g1"] - p["g0"], pos)
            for j in range(p["g1"] - p["g0"]):
                self.kc[l, j, pos] = k[j * hd:(j + 1) * hd]
                self.vc[l, j, pos] = v[j * hd:(j + 1) * hd]
            att = np.zeros(nh * hd, np.float32)
            for i in range(nh):
                j = (p["h0"] + i) // qpk - p["g0"]
                s = O.attn_qk(q[i * hd:(i + 1) * hd], self.kc[l, j].reshape(-1), pos, hd, scale, hd)
                att[i * hd:(i + 1) * hd] = O.attn_av(O.softmax(s), self.vc[l, j].reshape(-1), pos, hd, hd)
            X = (X + allreduce(self.gemv_cols(b + "attn_output.weight", q0, q1, att))).astype(np.float32)
            xn = O.rmsnorm(X, self.vec(b + "ffn_norm.weight"), self.eps)
            f0, f1 = p["f0"] * 256, p["f1"] * 256
            h = O.swiglu(self.gemv_rows(b + "ffn_gate.weight", f0, f1, xn), self.gemv_rows(b + "ffn_up.weight", f0, f1, xn))
            X = (X + allreduce(self.gemv_cols(b + "ffn_down.weight", f0, f1, h))).astype(np.float32)
        return O.rmsnorm(X, self.vec("output_norm.weight"), self.eps)

    def logits(self, normx):
        name = "output.weight" if "output.weight" in self.T else "token_embd.weight"
        return self.gemv_rows(name, self.p["v0"], self.p["v1"], normx)


def rank_main(rank, world, port, path, toks, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)

    def allreduce(v):
        t = torch.from_numpy(np.ascontiguousarray(v, np.float32))
        dist.all_reduce(t)
        return t.numpy()

    sh = Shard(path, rank, world)
    nxs = [sh.forward(int(t), pos, allreduce) for pos, t in enumerate(toks)]
    lg = torch.from_numpy(np.ascontiguousarray(sh.logits(nxs[-1]), np.float32))
    sizes = torch.tensor([lg.numel()])
    all_sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(all_sizes, sizes)
    parts = [torch.zeros(int(s.item())) for s in all_sizes]
    dist.all_gather(parts, lg)
    if rank == 0:
        np.save(os.path.join(out_dir, "normx.npy"), np.stack(nxs))
        np.save(os.path.join(out_dir, "logits.npy"), torch.cat(parts).numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("name", ["tiny7", "tiny15"])
def test_two_rank_shards_match_one_rank_oracle(tmp_path, model_cache, name):
    import torch.multiprocessing as mp
    from c2slm_b200 import synth
    from oracle import oracle as O
    path = synth.cached_model(name, cache_dir=model_cache)
    toks = np.array([5, 17, 301, 999, 42, 7], np.int32)
    mp.spawn(rank_main, args=(2, free_port(), path, toks, str(tmp_path)), nprocs=2, join=True)
    nx_tp = np.load(tmp_path / "normx.npy")
    lg_tp = np.load(tmp_path / "logits.npy")
    with O.OracleModel(path, max_tokens=64) as o:
        for pos, t in enumerate(toks):
            ref = o.forward(int(t), pos)
            err = np.abs(nx_tp[pos] - ref).max() / np.abs(ref).max()
            assert err <= TOL, (pos, err)
        lref = o.compute_logits(ref)
    err = np.abs(lg_tp - lref).max() / np.abs(lref).max()
    assert err <= TOL, err

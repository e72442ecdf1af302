"""Model-level GPU parity: engine.Forward / ComputeLogits / generate against the
CPU oracle on seeded synthetic models (the reference's integration tests,
c2slm_test.go and engine/forward_test.go, need a real checkpoint; synthetic
GGUFs with the same layouts stand in for it).

Bars: NormX within 1e-3 of max|ref|; the vocabulary projection of identical
NormX within 1e-5; greedy ids identical on the small models, where a
divergence is accepted only at a step whose oracle top-1/top-2 margin is below
1e-3 * max|logit| (a tolerance tie).  At full 0.5B size the reference's Q8_K
activation quantisation amplifies last-bit differences (its own AVX2 and
scalar builds disagree), so that model is held to the envelope of the
reference's build-to-build differences.
"""
import numpy as np
import pytest

import c2slm_b200 as K
from c2slm_b200 import synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-3


def rel(got, ref):
    ref = np.asarray(ref, np.float64)
    return float(np.abs(np.asarray(got, np.float64) - ref).max() / max(np.abs(ref).max(), 1e-30))


def assert_greedy_parity(got, want, margins, maxabs, min_steps):
    n = min(len(got), len(want))
    for i in range(n):
        if got[i] != want[i]:
            tie = margins[i] < 1e-3 * maxabs[i]
            assert tie, f"step {i}: gpu {got[i]} != oracle {want[i]} (margin {margins[i]:.3e}, max {maxabs[i]:.3e})"
            return i
    assert len(got) == len(want)
    assert n >= min_steps
    return n


@pytest.fixture(scope="module")
def models(model_cache):
    return {name: synth.cached_model(name, cache_dir=model_cache) for name in ("tiny05", "tiny15", "tiny7", "tiny3")}


@pytest.mark.parametrize("name", ["tiny05", "tiny15", "tiny7", "tiny3"])
def test_forward_and_logits_match_oracle(models, name):
    path = models[name]
    with K.Engine(path, max_tokens=256) as e, O.OracleModel(path, max_tokens=256, nthreads=4) as o:
        rng = np.random.default_rng(7)
        toks = rng.integers(0, e.desc.vocab, 40).astype(np.int32)
        for p, t in enumerate(toks):
            g = e.forward(int(t), p)
            w = o.forward(int(t), p)
            assert rel(g, w) <= TOL, (p, rel(g, w))
        # the vocabulary projection on identical NormX (K-quant outputs quantise
        # NormX to Q8_K: identical input -> identical int8 -> f32-order tolerance)
        lg = e.compute_logits()
        lw = o.compute_logits(g)
        assert rel(lg, lw) <= 1e-5, rel(lg, lw)
        # caller-supplied NormX path
        lg2 = e.compute_logits(normx=w)
        assert rel(lg2, o.compute_logits(w)) <= 1e-5
        # KV cache contents (KVCache.GetKey/GetValue)
        for layer in (0, e.desc.n_layers - 1):
            for pos in (0, 17, 39):
                assert rel(e.get_key(layer, 1, pos), o.kv_get(0, layer, 1, pos)) <= TOL
                assert rel(e.get_value(layer, 0, pos), o.kv_get(1, layer, 0, pos)) <= TOL
        # Forward does not touch SeqLen (engine/forward.go:54-138)
        assert e.seq_len == 0


@pytest.mark.parametrize("name", ["tiny05", "tiny15", "tiny7", "tiny3"])
def test_generate_greedy_parity(models, name):
    path = models[name]
    with K.Engine(path, max_tokens=512) as e, O.OracleModel(path, max_tokens=512, nthreads=4) as o:
        rng = np.random.default_rng(3)
        prompt = rng.integers(0, e.desc.vocab - 3, 24).astype(np.int32)
        nx_g = e.ingest_from(0, prompt)
        nx_o = o.ingest_from(0, prompt)
        assert rel(nx_g, nx_o) <= TOL
        assert e.seq_len == len(prompt) == o.seq_len
        assert np.array_equal(e.token_ids(), prompt)
        got = e.generate(96, penalty=1.15, window=64, stop_on_special=True)
        want, margins, maxabs = o.generate(nx_o, 96, penalty=1.15, window=64, stop_on_special=True)
        k = assert_greedy_parity(got, want, margins, maxabs, min_steps=1)
        if k == len(want):
            assert e.seq_len == o.seq_len
            assert np.array_equal(e.token_ids(), o.token_ids(o.seq_len))


def test_chunked_ingestion_equals_one_shot(models):
    """c2slm_test.go:42-89: prefix then suffix gives the one-shot logits, the
    fingerprint is recorded, and a session turn grows the cache."""
    with K.Engine(models["tiny15"], max_tokens=256) as e:
        toks = np.arange(5, 37, dtype=np.int32) * 7 % e.desc.vocab
        e.reset()
        e.ingest_from(0, toks)
        ref = e.compute_logits()
        e.reset()
        split = len(toks) // 2
        e.ingest_from(0, toks[:split])
        e.ingest_from(split, toks[split:])
        assert e.seq_len == len(toks)
        assert np.array_equal(e.token_ids(), toks)
        got = e.compute_logits()
        assert np.abs(got - ref).max() <= 1e-5
        before = e.seq_len
        e.generate_stream_session(np.array([3, 4, 5], np.int32), 4)
        assert before < e.seq_len <= e.max_tokens


def test_rewind_and_clamp_semantics(models):
    """IngestFrom clamps pos into [0, SeqLen] and rewinds without copying
    (c2slm.go:92-115, engine/kvcache.go:101-117)."""
    with K.Engine(models["tiny05"], max_tokens=128) as e:
        toks = np.arange(1, 21, dtype=np.int32)
        e.ingest_from(0, toks)
        assert e.seq_len == 20
        e.rewind(5)
        assert e.seq_len == 15
        e.rewind(100)
        assert e.seq_len == 0
        e.ingest_from(0, toks)
        e.ingest_from(50, toks[:2])  # pos > SeqLen is clamped to SeqLen
        assert e.seq_len == 22
        e.ingest_from(-3, toks[:4])  # negative pos -> 0, rewinds to 0
        assert e.seq_len == 4
        # capacity: ingestion stops at MaxTokens
        e.reset()
        e.ingest_from(0, np.arange(140, dtype=np.int32) % 100)
        assert e.seq_len == 128
        assert len(e.generate(10)) == 0


def test_restricted_logits_match_full(models):
    """engine/forward_test.go:123-172 (Q8_0 output: both paths use f32 x)."""
    with K.Engine(models["tiny05"], max_tokens=64) as e:
        nx = e.forward(5, 0)
        full = e.compute_logits(normx=nx)
        targets = np.array([0, 1, 100, 200, 300, 1000, 2000, 2047, -1, 99999], np.int32)
        out = np.full(e.desc.vocab, np.nan, np.float32)
        e.compute_logits(normx=nx, targets=targets, out=out)
        for t in targets:
            if 0 <= t < e.desc.vocab:
                assert abs(out[t] - full[t]) <= 1e-5 * max(1.0, abs(full[t]))


def test_stop_on_special_forwards_the_stop_token(models):
    """c2slm.go:183-189: selecting im_end/eos forwards it, records it, stops."""
    path = models["tiny05"]
    with K.Engine(path, max_tokens=256) as e, O.OracleModel(path, max_tokens=256, nthreads=2) as o:
        for seed in range(3):
            prompt = np.random.default_rng(seed).integers(0, 2000, 8).astype(np.int32)
            e.reset(); o.reset()
            e.ingest_from(0, prompt)
            nx = o.ingest_from(0, prompt)
            got = e.generate(40, stop_on_special=True)
            want, m, mx = o.generate(nx, 40, stop_on_special=True)
            assert_greedy_parity(got, want, m, mx, 1)
            assert e.seq_len == o.seq_len


def test_decode_step_matches_generate(models):
    path = models["tiny15"]
    with K.Engine(path, max_tokens=256) as e:
        prompt = np.arange(10, 26, dtype=np.int32)
        e.ingest_from(0, prompt)
        ref = e.generate(12, stop_on_special=False)
        e.reset()
        e.ingest_from(0, prompt[:-1])
        tok = int(prompt[-1])
        got = []
        for _ in range(12):
            tok = e.decode_step(tok)
            got.append(tok)
        assert got == list(ref)


def test_engine_from_caller_mapped_tensors(models):
    """c2s_engine_create: the cgo path, tensors mapped by the caller's reader."""
    from c2slm_b200 import gguf
    path = models["tiny7"]
    with gguf.File(path) as f:
        e = K.Engine(gguf_file=f, max_tokens=64)
    with e, K.Engine(path, max_tokens=64) as e2:
        assert np.array_equal(e.forward(11, 0), e2.forward(11, 0))


@pytest.mark.slow
def test_qwen05b_config1_parity_within_reference_build_envelope(model_cache):
    """BASELINE config 1 (0.5B-shaped, Q5_0/Q4_K/Q6_K/Q8_0), 32-token prompt,
    64 greedy steps teacher-forced with the scalar reference's choices.

    The reference quantises SwiGLU outputs to Q8_K before ffn_down, so a
    last-bit f32 difference anywhere upstream can flip an int8 and move the
    residual stream: the reference's own AVX2 build (restated in the oracle)
    differs from its scalar build by up to ~2e-2 on single steps and their
    free-running greedy sequences part within 64 steps.  The GPU path must
    stay inside that envelope:
      * median per-step logits error <= 1e-3 (the north_star tolerance);
      * steps above 1e-3 are Q8_K rounding events, which both reference
        builds also show (at the same steps): no more of them than 1.5x the
        AVX2 build's count + 2, none larger than 3x its largest;
      * greedy disagreements with the scalar build only at steps where the
        scalar build's own top-2 margin is within that step's error, and no
        more of them than 3x the AVX2 build's + 2;
      * the vocabulary projection on identical NormX within 1e-5 at every
        step."""
    path = synth.cached_model("qwen05b", cache_dir=model_cache)
    e = K.Engine(path, max_tokens=512)
    o = O.OracleModel(path, max_tokens=512, nthreads=8)
    a = O.OracleModel(path, max_tokens=512, nthreads=8, simd_order=True)
    try:
        prompt = np.random.default_rng(0).integers(0, 151643, 32).astype(np.int32)
        ng, no, na = e.ingest_from(0, prompt), o.ingest_from(0, prompt), a.ingest_from(0, prompt)
        assert rel(ng, no) <= TOL
        pos, eg, ea, dis_g, dis_a = 32, [], [], 0, 0
        for _ in range(64):
            lg, lo, la = e.compute_logits(), o.compute_logits(no), a.compute_logits(na)
            assert rel(lg, o.compute_logits(ng)) <= 1e-5
            bo, po = o.select(lo, pos)
            bg, _ = o.select(lg, pos)
            ba, _ = o.select(la, pos)
            eg.append(rel(lg, lo))
            ea.append(rel(la, lo))
            if bg != bo:  # a near-tie of the reference, closed by this step's error
                top = np.sort(po)[::-1]
                assert (top[0] - top[1]) / np.max(np.abs(lo)) <= 2 * eg[-1]
            dis_g += bg != bo
            dis_a += ba != bo
            ng = e.forward(bo, pos); e.store_token_id(pos, bo); e.seq_len = pos + 1
            no = o.forward(bo, pos); o.store_token_id(pos, bo); o.seq_len = pos + 1
            na = a.forward(bo, pos); a.store_token_id(pos, bo); a.seq_len = pos + 1
            pos += 1
        print(f"gpu-vs-scalar median {np.median(eg):.2e} max {max(eg):.2e} argmax diff {dis_g}; "
              f"avx2-vs-scalar median {np.median(ea):.2e} max {max(ea):.2e} argmax diff {dis_a}")
        assert np.median(eg) <= TOL
        events_g, events_a = sum(x > TOL for x in eg), sum(x > TOL for x in ea)
        assert events_g <= 1.5 * events_a + 2
        assert max(eg) <= 3 * max(ea)
        assert dis_g <= 3 * dis_a + 2
    finally:
        e.close(); o.close(); a.close()


@pytest.mark.slow
@pytest.mark.parametrize("name", ["qwen15b", "qwen7b"])
def test_large_shapes_reduced_depth(model_cache, name):
    """BASELINE configs 2 and 3 at full width, 2 layers (oracle time bound)."""
    path = synth.cached_model(name, layers=2, cache_dir=model_cache)
    with K.Engine(path, max_tokens=128) as e, O.OracleModel(path, max_tokens=128, nthreads=8) as o:
        prompt = np.random.default_rng(1).integers(0, 151643, 12).astype(np.int32)
        nx_g = e.ingest_from(0, prompt)
        nx_o = o.ingest_from(0, prompt)
        assert rel(nx_g, nx_o) <= TOL
        assert rel(e.compute_logits(), o.compute_logits(nx_g)) <= 1e-5
        got = e.generate(8, stop_on_special=False)
        want, m, mx = o.generate(nx_o, 8, stop_on_special=False)
        assert_greedy_parity(got, want, m, mx, 8)


@pytest.mark.slow
def test_long_context_split_attention(model_cache, monkeypatch):
    """Contexts longer than one attention split (head_dim 128: 128 positions
    per split at this capacity): the splits' partial softmax sums are combined
    by the last split of each kv head.  Against the oracle after a 400-token
    prompt, and the persistent and per-phase decode paths against each other
    while the context grows past further split boundaries."""
    path = synth.cached_model("qwen15b", layers=2, cache_dir=model_cache)
    prompt = np.random.default_rng(5).integers(0, 151643, 400).astype(np.int32)
    with K.Engine(path, max_tokens=1024) as e, O.OracleModel(path, max_tokens=1024, nthreads=16) as o:
        nx_g = e.ingest_from(0, prompt)
        nx_o = o.ingest_from(0, prompt)
        assert rel(nx_g, nx_o) <= TOL
        assert rel(e.compute_logits(), o.compute_logits(nx_g)) <= 1e-5
    out = {}
    for mode in ("graph", "persistent"):
        monkeypatch.setenv("C2S_DECODE", mode)
        with K.Engine(path, max_tokens=1024) as e:
            e.ingest_from(0, prompt[:250])
            toks = e.generate(24, stop_on_special=False)  # positions 250..273: splits 1 -> 2 -> 3
            out[mode] = (toks, e.compute_logits())
    assert np.array_equal(out["graph"][0], out["persistent"][0])
    assert np.array_equal(out["graph"][1], out["persistent"][1])


@pytest.mark.parametrize("name", ["tiny05", "tiny15", "tiny7", "tiny3"])
def test_persistent_decode_equals_graph_decode(models, name, monkeypatch):
    """The persistent decode kernel and the per-phase CUDA-graph path run the
    same device arithmetic: identical ids, SeqLen and fingerprint."""
    path = models[name]
    prompt = np.arange(3, 40, dtype=np.int32) * 11 % 1000
    out = {}
    for mode in ("graph", "persistent"):
        monkeypatch.setenv("C2S_DECODE", mode)
        with K.Engine(path, max_tokens=256) as e:
            e.ingest_from(0, prompt)
            toks = e.generate(60, stop_on_special=False)
            out[mode] = (toks, e.seq_len, e.token_ids(), e.compute_logits())
    g, p = out["graph"], out["persistent"]
    assert np.array_equal(g[0], p[0]) and g[1] == p[1] and np.array_equal(g[2], p[2])
    assert np.array_equal(g[3], p[3])


def test_many_split_attention_paths_agree(model_cache, monkeypatch):
    """A 4096-token context of the 7B shape (head_dim 128, 7 query heads per
    kv head): 33 attention splits per kv head.  The per-phase kernel's combine
    (the last split combines every head, in several staged blocks) and the
    persistent kernel's distributed combine (each split combines a slice)
    give identical ids and logits."""
    path = synth.cached_model("qwen7b", layers=2, cache_dir=model_cache)
    prompt = np.random.default_rng(9).integers(0, 151643, 4096).astype(np.int32)
    out = {}
    for mode in ("graph", "persistent"):
        monkeypatch.setenv("C2S_DECODE", mode)
        with K.Engine(path, max_tokens=4160) as e:
            e.ingest_from(0, prompt)
            toks = e.generate(6, stop_on_special=False)
            out[mode] = (toks, e.compute_logits())
    assert np.array_equal(out["graph"][0], out["persistent"][0])
    assert np.array_equal(out["graph"][1], out["persistent"][1])


@pytest.mark.parametrize("n_prompt", [2, 65, 300, 1100])
def test_prefill_on_tensor_cores_matches_token_by_token(model_cache, monkeypatch, n_prompt):
    """IngestFrom of a prompt through the tcgen05 int8 GEMM prefill (chunks of
    up to 1024 tokens, 128-token tiles, a ragged last tile; 2 and 65 tokens:
    a nearly empty token tile and key tiles of 64 plus one) against the
    per-token forward path (itself pinned to the oracle by the tests above):
    the last NormX within the tolerance, the K/V cache rows, the same
    TokenIDs and SeqLen, and the same first greedy token after it."""
    path = synth.cached_model("qwen15b", layers=2, cache_dir=model_cache)
    prompt = np.random.default_rng(7).integers(0, 151643, n_prompt).astype(np.int32)
    out = {}
    for mode in ("1", "0"):
        monkeypatch.setenv("C2S_PREFILL", mode)
        with K.Engine(path, max_tokens=1536) as e:
            nx = e.ingest_from(0, prompt)
            kv = [np.concatenate([e.get_key(l, g, p), e.get_value(l, g, p)])
                  for l in (0, 1) for g in (0, 1) for p in (0, n_prompt // 2, n_prompt - 1)]
            out[mode] = (nx, kv, e.seq_len, e.token_ids()[:n_prompt].copy(), e.generate(8, stop_on_special=False))
    (nx1, kv1, sl1, ids1, g1), (nx0, kv0, sl0, ids0, g0) = out["1"], out["0"]
    print(f"prefill n={n_prompt}: normx rel {rel(nx1, nx0):.2e}, kv rel {[f'{rel(a, b):.1e}' for a, b in zip(kv1, kv0)]}"
          f" gen tc {g1.tolist()} token {g0.tolist()}")
    assert sl1 == sl0 == n_prompt and np.array_equal(ids1, ids0)
    assert rel(nx1, nx0) <= TOL
    # layer 0 sees identical Q8_K activations on both paths: its K/V rows
    # differ only by the float order of the K-quant sums; deeper rows can
    # also carry a Q8_K byte that a last-bit difference moved (one
    # quantisation step of one activation), so most, not all, stay that close
    r = np.array([rel(a, b) for a, b in zip(kv1, kv0)])
    assert np.all(r[:6] <= 1e-5)
    assert np.median(r) <= 1e-5 and np.max(r) <= 1e-2
    assert g1[0] == g0[0]


def test_prefill_suffix_and_rewind_match_token_by_token(model_cache, monkeypatch):
    """IngestFrom of a suffix after an earlier ingest (the chunk attends to the
    cached prefix) and after a rewind into the prefix: the tensor-core prefill
    against the per-token path on the same calls."""
    path = synth.cached_model("qwen15b", layers=2, cache_dir=model_cache)
    rng = np.random.default_rng(11)
    a = rng.integers(0, 151643, 200).astype(np.int32)
    b = rng.integers(0, 151643, 300).astype(np.int32)
    c = rng.integers(0, 151643, 150).astype(np.int32)
    out = {}
    for mode in ("1", "0"):
        monkeypatch.setenv("C2S_PREFILL", mode)
        with K.Engine(path, max_tokens=1024) as e:
            e.ingest_from(0, a)
            nx_b = e.ingest_from(200, b)          # suffix after the prefix
            sl_b = e.seq_len
            nx_c = e.ingest_from(120, c)          # rewinds to 120, then 150 tokens
            out[mode] = (nx_b, sl_b, nx_c, e.seq_len, e.token_ids()[:e.seq_len].copy(),
                         e.get_key(0, 1, 121), e.generate(4, stop_on_special=False))
    t, r = out["1"], out["0"]
    assert t[1] == r[1] == 500 and t[3] == r[3] == 270 and np.array_equal(t[4], r[4])
    print(f"suffix normx rel {rel(t[0], r[0]):.2e}, rewound normx rel {rel(t[2], r[2]):.2e}")
    assert rel(t[0], r[0]) <= TOL
    # After the rewind the last token's attention output differs from the
    # per-token path's by ~6e-6 of max|out| (the tensor-core kernel and the
    # per-token FP32 kernel round differently; both are as close to float64
    # attention, test_prefill_attention_tensor_cores_against_float64), which
    # moves 3 of its 1752 Q8_K bytes by one step before attn_output: the
    # NormX then differs by ~2e-3.  One quantisation step is the bound.
    assert rel(t[2], r[2]) <= 1e-2
    assert rel(t[5], r[5]) <= 1e-5  # a layer-0 row the rewound ingest rewrote
    assert t[6][0] == r[6][0]


def _attention_f64(q, kc, vc, p0, qpk, hd):
    """Causal attention in float64 of queries q [T][H*hd] at positions p0..
    over K/V rows kc, vc [G][N][hd] (the reference's scores x scale, softmax
    after the maximum, probabilities times V: engine/forward.go:143-155)."""
    T, H = q.shape[0], q.shape[1] // hd
    sc = np.float64(np.float32(1.0 / np.sqrt(np.float64(hd))))
    out = np.zeros((T, H * hd))
    mask = np.arange(kc.shape[1])[None, :] > (p0 + np.arange(T))[:, None]
    for h in range(H):
        g = h // qpk
        s = (q[:, h * hd:(h + 1) * hd].astype(np.float64) @ kc[g].T.astype(np.float64)) * sc
        s[mask] = -np.inf
        p = np.exp(s - s.max(axis=1, keepdims=True))
        out[:, h * hd:(h + 1) * hd] = (p / p.sum(axis=1, keepdims=True)) @ vc[g].astype(np.float64)
    return out


@pytest.mark.parametrize("name,n_prompt", [("qwen15b", 1100), ("qwen7b", 600), ("tiny64", 1100)])
def test_prefill_attention_tensor_cores_against_float64(model_cache, monkeypatch, name, n_prompt):
    """The prefill's causal attention on the tensor cores (k_pf_attn: TF32
    operands split hi + lo, three products per term) and on the CUDA cores in
    FP32 (k_pf_flash, selected by C2S_PF_ATTN=fp32), each against float64
    attention computed from the very q, k and v the kernel saw (one-layer
    models: both runs see the same inputs).  The seeded random-weight models
    give large, peaked scores, so that the f32 rounding of a score moves the
    result by up to ~1e-4 of max|out| in either kernel; the tensor-core
    kernel is held to the FP32 kernel's own error (x 2, + 1e-6).  1100
    tokens: the second chunk's 76 tokens attend to all 1100 keys in splits of
    512 (the split combine); the 7B shape: 7 query heads per kv head;
    tiny64: 64-wide heads."""
    cfg = synth.get_config(name)
    hd = cfg.embd // cfg.heads
    path = synth.cached_model(name, layers=1, cache_dir=model_cache)
    prompt = np.random.default_rng(5).integers(0, min(cfg.vocab, 151643), n_prompt).astype(np.int32)
    last = n_prompt - 1024 if n_prompt > 1024 else n_prompt
    err = {}
    for mode in ("tc", "fp32"):
        if mode == "fp32":
            monkeypatch.setenv("C2S_PF_ATTN", "fp32")
        else:
            monkeypatch.delenv("C2S_PF_ATTN", raising=False)
        with K.Engine(path, max_tokens=1536) as e:
            e.ingest_from(0, prompt)
            att = e.prefill_debug("attention", last, cfg.heads)
            q = e.prefill_debug("queries", last, cfg.heads)
            kc = np.stack([np.stack([e.get_key(0, g, p) for p in range(n_prompt)]) for g in range(cfg.kv_heads)])
            vc = np.stack([np.stack([e.get_value(0, g, p) for p in range(n_prompt)]) for g in range(cfg.kv_heads)])
        assert np.all(np.isfinite(att))
        err[mode] = rel(att, _attention_f64(q, kc, vc, n_prompt - last, cfg.heads // cfg.kv_heads, hd))
    print(f"{name} n={n_prompt}: max err / max|out| against float64: tensor cores {err['tc']:.2e}, "
          f"FP32 kernel {err['fp32']:.2e}")
    assert err["tc"] <= 2.0 * err["fp32"] + 1e-6


def _long_context_case(name):
    import json
    import os
    p = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "long_context.json")
    if not os.path.exists(p):
        pytest.skip("tests/golden/long_context.json not generated")
    return json.load(open(p))[name]


@pytest.mark.slow
def test_attention_over_4096_positions_against_the_oracle(model_cache):
    """The 7B shape (2 layers) after a 4096-token IngestFrom, against the CPU
    oracle's committed results (tests/golden/make_long_context_fixtures.py):
    the last NormX, then greedy decode at positions 4096.. whose attention
    covers 33 position splits per kv head, with the tolerance-tie rule."""
    c = _long_context_case("attn4096")
    path = synth.cached_model(c["model"], layers=c["layers"], cache_dir=model_cache)
    prompt = np.random.default_rng(c["seed"]).integers(0, 151643, c["n"]).astype(np.int32)
    with K.Engine(path, max_tokens=c["max_tokens"]) as e:
        nx = e.ingest_from(0, prompt)
        assert rel(nx, c["normx"]) <= TOL, rel(nx, c["normx"])
        got = e.generate(c["gen"], stop_on_special=False)
    ones = np.ones(len(c["ids"]))
    assert_greedy_parity(got, c["ids"], np.array(c["rel_margin"]), ones, len(c["ids"]))


@pytest.mark.slow
def test_prefill_2048_tokens_against_the_oracle(model_cache):
    """IngestFrom of a 2048-token prompt through the tensor-core prefill (two
    1024-token chunks, the second attending to the first) against the CPU
    oracle's token-by-token results: the last NormX, the K/V cache rows at
    positions 0, 1024 and 2047 of both layers, and the first greedy ids."""
    c = _long_context_case("prefill2048")
    path = synth.cached_model(c["model"], layers=c["layers"], cache_dir=model_cache)
    prompt = np.random.default_rng(c["seed"]).integers(0, 151643, c["n"]).astype(np.int32)
    with K.Engine(path, max_tokens=c["max_tokens"]) as e:
        nx = e.ingest_from(0, prompt)
        assert rel(nx, c["normx"]) <= TOL, rel(nx, c["normx"])
        errs = []
        for r in c["kv"]:
            ek = rel(e.get_key(r["layer"], r["kv_head"], r["pos"]), r["k"])
            ev = rel(e.get_value(r["layer"], r["kv_head"], r["pos"]), r["v"])
            errs.append(max(ek, ev))
            if r["layer"] == 0:  # identical Q8_K activations: only the f32 order of the K-quant sums differs
                assert max(ek, ev) <= 1e-5, (r["pos"], ek, ev)
        print(f"prefill 2048 vs oracle: normx {rel(nx, c['normx']):.2e}, kv rows {['%.1e' % x for x in errs]}")
        # layer 1 rows see layer 0's residual, which a Q8_K byte moved by a
        # last-bit difference can shift by one quantisation step
        assert np.median(errs) <= 1e-4 and max(errs) <= 1e-2
        got = e.generate(c["gen"], stop_on_special=False)
    ones = np.ones(len(c["ids"]))
    assert_greedy_parity(got, c["ids"], np.array(c["rel_margin"]), ones, len(c["ids"]))


@pytest.mark.parametrize("ggml_type,nbytes_per", [(1, 2.0), (2, 18 / 32)])
def test_f16_and_q4_0_projections_are_rejected(models, ggml_type, nbytes_per):
    """F16 (type 1) and Q4_0 (type 2) tensors are sized by both GGUF readers
    as gguf/reader.go:513-546 does, but the reference's DispatchGEMV
    (engine/model.go:250-270) yields zero rows for them: the engine refuses
    such a projection at creation (C2S_ERR_UNSUPPORTED) rather than build a
    model that computes nothing."""
    from c2slm_b200 import gguf
    import c2slm_b200.engine as KE
    with gguf.File(models["tiny05"]) as f:
        ti = f.tensor_map["blk.0.attn_q.weight"]
        cols, rows = int(ti.dimensions[0]), int(ti.dimensions[1])
        ti.type = ggml_type
        ti.data = memoryview(bytearray(int(rows * cols * nbytes_per)))
        with pytest.raises(KE.C2SError) as exc:
            K.Engine(gguf_file=f, max_tokens=64)
    assert exc.value.code == -4 and f"type {ggml_type}" in str(exc.value)

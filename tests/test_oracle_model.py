"""Model-level oracle semantics on small synthetic GGUFs (CPU only):
KVCache, IngestFrom, the generate loop and thread-count independence."""
import numpy as np
import pytest

from c2slm_b200 import gguf, synth
from oracle import oracle as O


@pytest.fixture(scope="module")
def tiny(model_cache):
    return {n: synth.cached_model(n, cache_dir=model_cache) for n in ("tiny05", "tiny15", "tiny3")}


def test_more_bits_layers():
    """Q4_K_M layer sets: {0,1,2,5,8,..,20,21,22,23} at 24 and {0..3,6,..,21,24..27} at 28."""
    assert [i for i in range(24) if synth.more_bits(i, 24)] == [0, 1, 2, 5, 8, 11, 14, 17, 20, 21, 22, 23]
    assert [i for i in range(28) if synth.more_bits(i, 28)] == [0, 1, 2, 3, 6, 9, 12, 15, 18, 21, 24, 25, 26, 27]


def test_gguf_reader_matches_writer(tiny):
    with gguf.File(tiny["tiny05"]) as f:
        assert f.get_uint32("qwen2.embedding_length") == (256, True)
        assert f.get_float32("qwen2.rope.freq_base")[0] == 1e6
        toks, ok = f.get_string_slice("tokenizer.ggml.tokens")
        assert ok and toks[-1] == "<|im_end|>"
        te = f.tensor_map["token_embd.weight"]
        assert te.type == gguf.Q8_0 and te.dimensions == [256, 2048]
        assert len(te.data) == 2048 * (256 // 32) * 34
        for i in range(3):
            t = gguf.Q6_K if synth.more_bits(i, 3) else gguf.Q4_K
            assert f.tensor_map[f"blk.{i}.ffn_down.weight"].type == t


def test_gguf_rejects_corrupt_files(tmp_path, tiny):
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUF" + b"\0" * 4)
    with pytest.raises(gguf.GGUFError):
        gguf.File(str(bad))
    data = open(tiny["tiny05"], "rb").read()
    trunc = tmp_path / "trunc.gguf"
    trunc.write_bytes(data[: len(data) // 2])
    with pytest.raises(gguf.GGUFError):
        gguf.File(str(trunc))
    with pytest.raises(RuntimeError):
        O.OracleModel(str(trunc), max_tokens=16)


def test_kv_store_get_roundtrip_and_rewind(tiny):
    """engine/kvcache_test.go round trip and Reset/Rewind semantics."""
    with O.OracleModel(tiny["tiny15"], max_tokens=64) as m:
        m.forward(3, 5)
        k = m.kv_get(0, 1, 1, 5)
        assert np.abs(k).sum() > 0
        m.seq_len = 10
        m.rewind(3)
        assert m.seq_len == 7
        m.rewind(100)
        assert m.seq_len == 0
        m.store_token_id(70, 9)  # out of range: ignored
        m.store_token_id(2, 9)
        assert m.token_ids(3)[2] == 9


def test_chunked_ingestion_equals_one_shot(tiny):
    """c2slm_test.go:42-89 on a synthetic model."""
    with O.OracleModel(tiny["tiny05"], max_tokens=128) as m:
        toks = (np.arange(20, dtype=np.int32) * 37) % 2000
        nx = m.ingest_from(0, toks)
        ref = m.compute_logits(nx)
        m.reset()
        m.ingest_from(0, toks[:9])
        nx2 = m.ingest_from(9, toks[9:])
        assert m.seq_len == 20 and np.array_equal(m.token_ids(20), toks)
        assert np.abs(m.compute_logits(nx2) - ref).max() <= 1e-5


def test_thread_count_does_not_change_results(tiny):
    outs = []
    for th in (1, 4):
        with O.OracleModel(tiny["tiny15"], max_tokens=300, nthreads=th) as m:
            toks = np.arange(1, 270, dtype=np.int32)  # pos >= 256 takes the parallel-heads path
            nx = m.ingest_from(0, toks)
            outs.append((nx, m.compute_logits(nx)))
    assert np.array_equal(outs[0][0], outs[1][0]) and np.array_equal(outs[0][1], outs[1][1])


def test_restricted_logits_equal_full_for_q8_0_output(tiny):
    """engine/forward_test.go:123-172 (tied Q8_0 output: both paths use f32 x)."""
    with O.OracleModel(tiny["tiny05"], max_tokens=16) as m:
        nx = m.forward(7, 0)
        full = m.compute_logits(nx)
        targets = [0, 1, 100, 2047, -1, 5000]
        part = m.compute_logits(nx, targets)
        for t in targets:
            if 0 <= t < 2048:
                assert abs(part[t] - full[t]) <= 1e-5


def test_penalty_and_argmax_rules(tiny):
    """c2slm.go:156-180: penalty per window occurrence, specials skipped,
    strict '>' so ties keep the lowest id."""
    with O.OracleModel(tiny["tiny05"], max_tokens=16) as m:
        v = m.info.vocab
        lg = np.zeros(v, np.float32)
        lg[5] = 2.0
        lg[6] = -2.0
        lg[7] = 1.9
        for p, t in enumerate([5, 5, 6, m.info.im_end, 7]):
            m.store_token_id(p, t)
        best, out = m.select(lg, 5, 1.15, 64)
        assert out[5] == np.float32(np.float32(2.0) / np.float32(1.15)) / np.float32(1.15)
        assert out[6] == np.float32(-2.0) * np.float32(1.15)
        assert best == 7 or out[best] >= out[7]
        lg2 = np.zeros(v, np.float32)
        b2, _ = m.select(lg2, 0, 1.15, 64)
        assert b2 == 0


def test_generate_stops_after_forwarding_special(tiny):
    with O.OracleModel(tiny["tiny05"], max_tokens=200) as m:
        nx = m.ingest_from(0, np.array([1, 2, 3], np.int32))
        toks, margins, mx = m.generate(nx, 150, stop_on_special=True)
        if len(toks) < 150:
            assert toks[-1] in (m.info.im_end, m.info.eos)
        assert m.seq_len == 3 + len(toks)
        assert np.array_equal(m.token_ids(m.seq_len)[3:], toks)


def test_greedy_fixture_is_reproduced_by_the_oracle(model_cache):
    """tests/golden/greedy_qwen05b.json (made by make_greedy_fixtures.py) is
    what the oracle computes: prompt 0's first 8 greedy ids and margins."""
    import json
    import os
    from c2slm_b200 import synth
    p = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "greedy_qwen05b.json")
    fx = json.load(open(p))
    path = synth.cached_model(fx["model"], cache_dir=model_cache)
    pr = fx["prompts"][0]
    prompt = np.random.default_rng(fx["seed_base"] + pr["seed"]).integers(0, 151643, fx["plen"]).astype(np.int32)
    with O.OracleModel(path, max_tokens=fx["plen"] + 16, nthreads=os.cpu_count() or 1) as o:
        nx = o.ingest_from(0, prompt)
        ids, m, mx = o.generate(nx, 8, penalty=fx["penalty"], window=fx["window"], stop_on_special=False)
    assert list(ids) == pr["ids"][:8]
    np.testing.assert_allclose(m / mx, pr["rel_margin"][:8], rtol=1e-3)

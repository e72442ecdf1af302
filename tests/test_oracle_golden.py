"""Pins the CPU oracle against the reference's own golden vectors and KATs.

Every case cites the reference test it restates.  The oracle is only trusted
as the parity checker for the CUDA path once these pass.
"""
import json
import math
import os
import struct

import numpy as np
import pytest

from oracle import oracle as O

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "ref_c_oracles.json")))


def bits(v):
    return struct.unpack("<I", struct.pack("<f", v))[0]


def f32(b):
    return struct.unpack("<f", struct.pack("<I", b))[0]


# ---- reference inline C oracles (tensor/oracle_q4_k_test.go, oracle_q6_k_test.go) ----
@pytest.mark.parametrize("kind,key", [(O.Q4_K, "q4_k"), (O.Q6_K, "q6_k")])
def test_kquant_f32_dot_bit_exact_vs_reference_c(kind, key):
    """tensor/oracle_q4_k_test.go:193-217 and :284-296; oracle_q6_k_test.go same
    structure: DotQ*_K(unit e_i) and the dense dot are bit-identical to the C."""
    for case in GOLD[key]:
        blk = bytes.fromhex(case["block"])
        for i in range(256):
            e = np.zeros(256, np.float32)
            e[i] = 1.0
            got = O.dot_f32x(kind, blk, e, 256)
            want = f32(case["dequant_bits"][i])
            assert not math.isnan(got)
            assert bits(got) == case["dequant_bits"][i] or (got == 0 and want == 0), (case["name"], i, got, want)
        if case["name"] == "fixture":
            got = O.dot_f32x(kind, blk, np.array(case["dense"], np.float32), 256)
            assert bits(got) == case["dot_bits"], (got, f32(case["dot_bits"]))


@pytest.mark.parametrize("kind,key", [(O.Q4_K, "q4_k"), (O.Q6_K, "q6_k")])
def test_kquant_dequant_row_matches_reference_c(kind, key):
    for case in GOLD[key]:
        got = O.dequant_row(kind, bytes.fromhex(case["block"]), 256)
        want = np.array(case["dequant_bits"], np.uint32).view(np.float32)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)) or np.array_equal(got, want)


def test_q5_0_vs_reference_c():
    """tensor/oracle_c_test.go:93-149 (unit vectors, tolerance 1e-6; we also get bit equality)."""
    case = GOLD["q5_0"][0]
    blk = bytes.fromhex(case["block"])
    deq = O.dequant_row(O.Q5_0, blk, 32)
    for i in range(32):
        e = np.zeros(32, np.float32)
        e[i] = 1
        got = O.dot_f32x(O.Q5_0, blk, e, 32)
        want = f32(case["dequant_bits"][i])
        assert abs(got - want) <= 1e-6
        assert bits(got) == case["dequant_bits"][i]
        assert bits(float(deq[i])) == case["dequant_bits"][i]


def test_q8_0_closed_form():
    """tensor/oracle_c_test.go:151-169."""
    blk = bytearray(34)
    struct.pack_into("<H", blk, 0, 0x3C00)
    for i in range(32):
        blk[2 + i] = (i * 2 - 31) & 0xFF
    for i in range(32):
        e = np.zeros(32, np.float32)
        e[i] = 1
        assert abs(O.dot_f32x(O.Q8_0, bytes(blk), e, 32) - float(i * 2 - 31)) <= 1e-6


# ---- Q8_K quantisation + K-quant x Q8_K --------------------------------------------
def q6k_gemv2_fixture():
    """internal/simd/c2_tensor_gemv2_q6_k_q8_k_test.go:9-47."""
    cols, nb = 512, 2
    w0 = bytearray(nb * 210)
    w1 = bytearray(nb * 210)
    for b in range(nb):
        o = b * 210
        w0[o + 208], w0[o + 209] = 0x00, 0x3C
        for i in range(128):
            w0[o + i] = (b * 37 + i * 19 + 17) & 0xFF
        for i in range(64):
            w0[o + 128 + i] = (b * 13 + i * 7 + 3) & 0xFF
        for i in range(16):
            w0[o + 192 + i] = (i * 3 - 8) & 0xFF
        w1[o + 208], w1[o + 209] = 0x00, 0x38
        for i in range(128):
            w1[o + i] = (b * 41 + i * 23 + 19) & 0xFF
        for i in range(64):
            w1[o + 128 + i] = (b * 17 + i * 11 + 5) & 0xFF
        for i in range(16):
            w1[o + 192 + i] = (i * 2 - 7) & 0xFF
    x = np.array([((i % 17) - 8) * 0.125 for i in range(cols)], np.float32)
    return bytes(w0), bytes(w1), x, cols


def test_q6k_gemv2_golden_values():
    """internal/simd/c2_tensor_gemv2_q6_k_q8_k_test.go:54-69: the reference pins
    want0 = -8705.69238281 and want1 = 3759.21655273 (tolerance 1e-2)."""
    w0, w1, x, cols = q6k_gemv2_fixture()
    q8 = O.quantize_row_q8_k(x)
    g0, g1 = O.gemv2(O.Q6_K, w0, w1, q8, cols)
    assert abs(g0 - (-8705.69238281)) <= 1e-2, g0
    assert abs(g1 - 3759.21655273) <= 1e-2, g1


def q4k_dot_fixture():
    """internal/simd/c2_tensor_dot_q4_k_q8_k_test.go:148-172."""
    cols, nb = 512, 2
    w = bytearray(nb * 144)
    for b in range(nb):
        o = b * 144
        w[o:o + 4] = bytes([0x00, 0x3C, 0x00, 0x38])
        for i in range(12):
            w[o + 4 + i] = (b * 37 + i * 19 + 17) & 0xFF
        for i in range(128):
            w[o + 16 + i] = (b * 13 + i * 7 + 3) & 0xFF
    x = np.array([((i % 17) - 8) * 0.125 for i in range(cols)], np.float32)
    return bytes(w), x, cols


def dequant_q8k(q8, cols):
    out = np.zeros(cols, np.float64)
    for b in range(cols // 256):
        d = struct.unpack_from("<f", q8, b * 292)[0]
        q = np.frombuffer(bytes(q8[b * 292 + 4:b * 292 + 260]), np.int8).astype(np.float64)
        out[b * 256:(b + 1) * 256] = d * q
    return out


def test_q4k_q8k_dot_cross_validated_by_dequant_route():
    """The Q4_K x Q8_K golden output lives in C sources absent from the reference
    tree (internal/simd/c2_tensor_dot_q4_k_q8_k_test.go:91-106); cross-validate
    the integer path on its fixture: dot == dequant(W) . dequant(Q8_K) up to f32
    rounding, and the single-row kernel equals the row-pair kernel."""
    w, x, cols = q4k_dot_fixture()
    q8 = O.quantize_row_q8_k(x)
    got = O.dot_q4_k_q8_k(w, q8, cols)
    wd = O.dequant_row(O.Q4_K, w, cols).astype(np.float64)
    ref = float(np.dot(wd, dequant_q8k(q8, cols)))
    assert abs(got - ref) <= 1e-4 * max(1.0, abs(ref)), (got, ref)
    g0, g1 = O.gemv2(O.Q4_K, w, w, q8, cols)
    assert bits(g0) == bits(got) and bits(g1) == bits(got)


def test_q6k_q8k_matches_dequant_route():
    w0, w1, x, cols = q6k_gemv2_fixture()
    q8 = O.quantize_row_q8_k(x)
    g0, _ = O.gemv2(O.Q6_K, w0, w1, q8, cols)
    wd = O.dequant_row(O.Q6_K, w0, cols).astype(np.float64)
    ref = float(np.dot(wd, dequant_q8k(q8, cols)))
    assert abs(g0 - ref) <= 1e-5 * abs(ref)


def test_quantize_q8k_block_invariants():
    """c2_quantize_q8_k_gen.go:11-91: d = amax/127, q = trunc(x*127/amax +- 0.5)
    clamped to +-127, bsums are sums of 16 quants; an all-zero block is all zero."""
    rng = np.random.default_rng(3)
    x = rng.normal(0, 1, 1024).astype(np.float32)
    x[256:512] = 0
    q8 = O.quantize_row_q8_k(x)
    for b in range(4):
        blk = q8[b * 292:(b + 1) * 292]
        xb = x[b * 256:(b + 1) * 256]
        d = np.frombuffer(blk[:4].tobytes(), np.float32)[0]
        q = blk[4:260].view(np.int8).astype(np.int32)
        bs = blk[260:292].view(np.int16).astype(np.int32)
        if b == 1:
            assert not blk.any()
            continue
        amax = np.float32(np.abs(xb).max())
        assert d == np.float32(amax / np.float32(127))
        iscale = np.float32(np.float32(127) / amax)
        v = (xb * iscale).astype(np.float32)
        r = np.where(v >= 0, v + np.float32(0.5), v - np.float32(0.5)).astype(np.float32)
        want = np.clip(np.trunc(r).astype(np.int32), -127, 127)
        assert np.array_equal(q, want)
        assert np.array_equal(bs, q.reshape(16, 16).sum(1))


def test_kquant_partials_reassemble_outputs():
    """The int32 partials (bit-exact contract) reproduce the f32 result with the
    reference's accumulation order."""
    rng = np.random.default_rng(11)
    from c2slm_b200 import synth
    rows, cols = 6, 1024
    w4 = synth.gen_blocks(rng, O.Q4_K, rows, cols)
    w6 = synth.gen_blocks(rng, O.Q6_K, rows, cols)
    x = rng.normal(0, 1, cols).astype(np.float32)
    q8 = O.quantize_row_q8_k(x)
    dots, pairs = O.q4k_q8k_partials(w4, q8, rows, cols)
    isum = O.q6k_q8k_partials(w6, q8, rows, cols)
    y4 = O.gemv(O.Q4_K, w4, x, rows, cols)
    y6 = O.gemv(O.Q6_K, w6, x, rows, cols)
    nsb = cols // 256
    d8 = np.frombuffer(q8.tobytes(), np.uint8).reshape(nsb, 292)[:, :4].copy().view(np.float32).reshape(-1)
    for r in range(rows):
        acc = np.float32(0)
        for b in range(nsb):
            d6 = np.frombuffer(w6[(r * nsb + b) * 210 + 208:(r * nsb + b) * 210 + 210].tobytes(), np.float16)[0]
            acc = np.float32(acc + np.float32(np.float32(isum[r, b]) * np.float32(np.float32(d6) * d8[b])))
        assert bits(float(acc)) == bits(float(y6[r]))
    assert dots.shape == (rows, nsb, 8) and pairs.shape == (nsb, 4)
    # bsum pairs are the sums of the two 16-element bsums of each 32-element half
    bs = np.frombuffer(q8.tobytes(), np.uint8).reshape(nsb, 292)[:, 260:292].copy().view(np.int16).astype(np.int32)
    for j in range(4):
        assert np.array_equal(pairs[:, j], bs[:, 2 * j] + bs[:, 2 * j + 1])


# ---- small ops: tensor/ops_test.go, rope_test.go, swiglu_test.go ---------------------
def test_fp16_cases():
    """tensor/ops_test.go:10-28."""
    for h, want in [(0x0000, 0.0), (0x3C00, 1.0), (0xBC00, -1.0), (0x4000, 2.0), (0x3555, 0.33325195)]:
        assert abs(O.fp16_to_f32(h) - want) <= 1e-4
    # exhaustive: equals IEEE half for every finite pattern
    hs = np.arange(65536, dtype=np.uint16)
    finite = np.isfinite(hs.view(np.float16))
    for h in hs[finite][::97]:
        assert O.fp16_to_f32(int(h)) == float(np.uint16(h).view(np.float16))


def test_rmsnorm_closed_form():
    """tensor/ops_test.go:30-43."""
    out = O.rmsnorm([1, 2, 3, 4], [1, 1, 1, 1], 1e-6)
    assert abs(out[0] - 1.0 / math.sqrt(7.5)) <= 1e-5


def test_rope():
    """tensor/rope_test.go:10-66 and ops_test.go:45-61."""
    c, s = O.rope_table(16384, 128, 1e6)
    assert c.size == 16384 * 64 and s.size == 16384 * 64
    tbl = O.rope_table(16, 8, 1e6)
    vec = np.arange(1, 9, dtype=np.float32)
    for pos in (16, 16 + 1000, -1):
        assert np.array_equal(O.rope_apply(tbl, 16, 8, vec, 1, pos), vec)
    assert np.array_equal(O.rope_apply(tbl, 16, 8, vec, 2, 1), vec)
    tbl4 = O.rope_table(4, 8, 1e6)
    v = O.rope_apply(tbl4, 4, 8, np.array([1, 0, 0, 0, 0, 0, 0, 0], np.float32), 1, 1)
    assert 0 < v[0] < 1 and abs(v[4]) > 1e-9
    ones = np.ones(64, np.float32)
    assert np.allclose(O.rope_neox(ones, 1, 64, 0, 1e6), 1.0, atol=1e-6)


def test_softmax():
    """tensor/ops_test.go:63-79."""
    x = O.softmax([1, 2, 3])
    assert abs(x.sum() - 1.0) <= 1e-6 and x[0] < x[1] < x[2]


def test_swiglu_vs_float64():
    """internal/simd/c2_tensor_swiglu_test.go:8-36 (max diff 1e-4)."""
    n = 6144
    g = np.array([(i - 3072) / 256.0 for i in range(n)], np.float32)
    u = np.array([(i % 100) / 100.0 for i in range(n)], np.float32)
    ref = (g.astype(np.float64) / (1 + np.exp(-g.astype(np.float64)))).astype(np.float32) * u
    assert np.abs(O.swiglu(g, u) - ref).max() <= 1e-4


def attn_fixture(hd, pos, seed):
    """internal/simd/c2_tensor_attn_test.go:28-68 (LCG fixture)."""
    state = [seed]

    def nxt():
        state[0] = (state[0] * 1664525 + 1013904223) & 0xFFFFFFFF
        return np.float32(((state[0] >> 8) & 0xFFFFFF) / float(0x1000000))

    nk = (pos + 1) * hd
    q = np.array([nxt() * 2 - 1 for _ in range(hd)], np.float32)
    k = np.array([nxt() * 2 - 1 for _ in range(nk)], np.float32)
    v = np.array([0.25 + 0.5 * nxt() for _ in range(nk)], np.float32)
    sc = np.array([0.25 + 0.5 * nxt() for _ in range(pos + 1)], np.float32)
    return q, k, v, sc


@pytest.mark.parametrize("hd,pos,seed", [(64, 0, 7), (64, 1, 7), (64, 63, 11), (64, 255, 13),
                                         (64, 256, 17), (128, 512, 23), (128, 128, 29)])
def test_attn_qk_av_rel_1e5(hd, pos, seed):
    """internal/simd/c2_tensor_attn_test.go:132-177: QK and AV within rel 1e-5
    (float64 stands in for the absent C oracle)."""
    q, k, v, sc = attn_fixture(hd, pos, seed)
    qk = O.attn_qk(q, k, pos, hd, 0.125, hd)
    ref = (k.reshape(pos + 1, hd).astype(np.float64) @ q.astype(np.float64)) * 0.125
    rel = np.abs(qk - ref) / np.maximum(np.abs(ref), 1)
    assert rel.max() <= 1e-5
    av = O.attn_av(sc, v, pos, hd, hd)
    ref = sc.astype(np.float64) @ v.reshape(pos + 1, hd).astype(np.float64)
    rel = np.abs(av - ref) / np.maximum(np.abs(ref), 1)
    assert rel.max() <= 1e-5

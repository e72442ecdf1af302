"""Tensor-parallel shard plan (host side, no GPU): the 7B-shaped config's
split of query heads into pairs of head_dim-128 heads (one 256-column
superblock of attn_output's input each), FFN rows into superblocks, the
vocabulary into an even padded split; every head, FFN row and vocabulary
row held by exactly one rank."""
import pytest

import c2slm_b200.engine as KE

SHAPES = {  # embd, layers, heads, kv heads, ffn, vocab
    "qwen7b": (3584, 28, 28, 4, 18944, 152064),
    "qwen15b": (1536, 28, 12, 2, 8960, 151936),
}


def desc(name):
    d = KE.ModelDesc()
    d.embd, d.n_layers, d.n_heads, d.n_kv_heads, d.ffn, d.vocab = SHAPES[name]
    d.head_dim = 0  # derived: embd / heads
    return d


def plans(name, world):
    return [KE.tp_plan(desc(name), r, world) for r in range(world)]


@pytest.mark.parametrize("world,heads,ffn_sb", [
    (2, [14, 14], [37, 37]),
    (4, [8, 8, 6, 6], [19, 19, 18, 18]),
    (8, [4, 4, 4, 4, 4, 4, 2, 2], [10, 10, 9, 9, 9, 9, 9, 9]),
])
def test_7b_split_follows_head_pairs_and_superblocks(world, heads, ffn_sb):
    ps = plans("qwen7b", world)
    assert [p["h1"] - p["h0"] for p in ps] == heads
    assert [p["f1"] - p["f0"] for p in ps] == ffn_sb
    assert all(p["vpad"] == 152064 // world for p in ps)


@pytest.mark.parametrize("name", list(SHAPES))
@pytest.mark.parametrize("world", [2, 4, 8])
def test_shards_partition_the_model(name, world):
    embd, _, nh, nkv, ffn, vocab = SHAPES[name]
    if (nh // 2) < world:
        pytest.skip("fewer head pairs than ranks")
    ps = plans(name, world)
    qpk = nh // nkv
    assert ps[0]["h0"] == 0 and ps[-1]["h1"] == nh
    assert ps[0]["f0"] == 0 and ps[-1]["f1"] == ffn // 256
    assert ps[0]["v0"] == 0 and ps[-1]["v1"] == vocab
    for a, b in zip(ps, ps[1:]):
        assert a["h1"] == b["h0"] and a["f1"] == b["f0"] and a["v1"] == b["v0"]
    for p in ps:
        assert p["h1"] > p["h0"] and (p["h1"] - p["h0"]) % 2 == 0  # whole superblocks at head_dim 128
        # the kv heads a rank holds are exactly those its query heads use
        assert p["g0"] == p["h0"] // qpk and p["g1"] == -(-p["h1"] // qpk)
        assert p["v1"] - p["v0"] <= p["vpad"]


def test_plan_rejects_shapes_that_do_not_split():
    d = KE.ModelDesc()
    d.embd, d.n_layers, d.n_heads, d.n_kv_heads, d.ffn, d.vocab = 896, 24, 14, 2, 4864, 151936
    d.head_dim = 0
    with pytest.raises(KE.C2SError):  # 14 heads of 64 do not group into 256-column superblocks
        KE.tp_plan(d, 0, 2)
    assert KE.tp_plan(d, 0, 1)["h1"] == 14  # one GPU: the whole model

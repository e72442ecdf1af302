"""c2s_gemv_noalloc: the matvec whose operands live in the library's static
device array (no device allocation or free per call), for callers that
cannot allocate device memory when they need a matvec.  Checked against the
CPU oracle at the tolerance of the other matvec tests, and bit for bit
against c2s_gemv, the allocating entry point (both run the same kernel), on
the same seeded inputs.

Collected last (file name) so that it also runs after every other test has
used the device; it passes alone as well."""
import numpy as np
import pytest

import c2slm_b200.engine as KE
from c2slm_b200 import synth
from oracle import oracle as O

CASES = [
    (KE.Q4_K, 512, 4864),   # ffn_down-shaped rows (config 0 columns)
    (KE.Q6_K, 256, 4864),
    (KE.Q5_0, 896, 896),    # config 1 attention / FFN-up shapes
    (KE.Q8_0, 1000, 896),   # vocabulary-projection rows
]


@pytest.mark.gpu
@pytest.mark.parametrize("kind,rows,cols", CASES)
def test_gemv_noalloc_matches_gemv_on_two_calls_in_a_row(kind, rows, cols):
    rng = np.random.default_rng(kind * 1000 + rows)
    w = synth.gen_blocks(rng, kind, rows, cols)
    for _ in range(2):  # two inputs, each through both entry points
        x = rng.standard_normal(cols).astype(np.float32)
        ref = KE.gemv(kind, w, x, rows, cols)
        want = O.gemv(kind, w, x, rows, cols)
        for _ in range(2):  # two calls in a row on the same static array
            got = KE.gemv_noalloc(kind, w, x, rows, cols)
            assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
            err = np.abs(got.astype(np.float64) - want).max() / max(np.abs(want).max(), 1e-30)
            assert err <= 1e-5, err


def test_gemv_noalloc_rejects_a_call_beyond_its_static_array():
    """Weights + x + y must fit in the 4 MiB array; the size check comes
    before any device work (so this also holds without a GPU)."""
    rows, cols = 4096, 4864  # 11.2 MB of Q4_K
    w = np.zeros(rows * (cols // 256) * 144, np.uint8)
    x = np.zeros(cols, np.float32)
    with pytest.raises(KE.C2SError) as exc:
        KE.gemv_noalloc(KE.Q4_K, w, x, rows, cols)
    assert exc.value.code == -1 and "static scratch" in str(exc.value)

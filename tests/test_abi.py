"""The C-ABI library builds, loads and exports every symbol the header
declares (no compute calls: this runs without a GPU)."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "c2slm_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(c2s_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from c2slm_b200 import build
    build.build()
    return ctypes.CDLL(build.LIB)


def test_header_declares_the_boundary():
    names = declared_functions()
    for must in ("c2s_engine_open", "c2s_forward", "c2s_compute_logits", "c2s_generate",
                 "c2s_ingest_from", "c2s_quantize_row_q8_k", "c2s_gemv", "c2s_kv_rewind"):
        assert must in names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_every_symbol():
    from c2slm_b200 import engine
    assert sorted(engine.SIGNATURES) == declared_functions()


def test_library_is_sm100a_only():
    from c2slm_b200 import build
    cmd = build.nvcc_cmd()
    assert "arch=compute_100a,code=sm_100a" in cmd


def test_version_and_error_paths_without_gpu(lib):
    from c2slm_b200 import engine as E
    E.load_library()
    assert b"sm_100a" in E.load_library().c2s_version()
    h = ctypes.c_void_p()
    rc = E.load_library().c2s_engine_open(b"/nonexistent.gguf", 0, 64, ctypes.byref(h))
    assert rc < 0 and not h.value
    assert E.load_library().c2s_last_error()


def test_host_rejects_bad_arguments_before_any_launch(lib):
    from c2slm_b200 import engine as E
    L = E.load_library()
    assert L.c2s_forward(None, 1, 0, None) == -1
    assert L.c2s_kv_rewind(None, 1) == -1
    assert L.c2s_generate(None, 4, 1.15, 64, 1, None, None) == -1


def test_ring_warp_groups_own_whole_slots(lib):
    """The persistent kernel's many-row phases split the compute warps into
    2^lng groups; group g consumes ring chunks g, g + ng, ... and chunk k uses
    slot k % nslot.  For every ring the engine can build (2..8 slots) and
    every group count it can ask for, the count it uses must give each slot
    to one group only: chunks k and k + nslot belong to the same group."""
    from c2slm_b200 import engine as E
    L = E.load_library()
    for nslot in range(2, 9):
        for want in range(0, 4):
            lng = L.c2s_ring_groups(nslot, want)
            ng = 1 << lng
            assert 0 <= lng <= want and ng <= nslot
            for k in range(4 * nslot * ng):
                assert k % ng == (k + nslot) % ng, (nslot, want, lng, k)
            # the largest count that keeps the property is the one used
            best = max(l for l in range(want + 1) if nslot % (1 << l) == 0)
            assert lng == best


def test_failed_create_releases_the_callers_mapping(lib, model_cache):
    """c2s_engine_create over tensors the caller keeps mapped (the cgo path):
    when creation fails (here: no device, or a rejected tensor on a GPU box)
    the binding keeps no view of the mapping, so the caller can close it."""
    import c2slm_b200 as K
    from c2slm_b200 import gguf, synth
    path = synth.cached_model("tiny05", cache_dir=model_cache)
    with gguf.File(path) as f:
        ti = f.tensor_map["blk.0.attn_q.weight"]
        ti.type = 1  # F16: sized by the reader, rejected by the engine
        ti.data = memoryview(bytearray(int(ti.dimensions[0]) * int(ti.dimensions[1]) * 2))
        with pytest.raises(K.C2SError) as exc:
            K.Engine(gguf_file=f, max_tokens=64)
    assert exc.value.code in (-2, -4)  # no CUDA device here; UNSUPPORTED on a GPU box

"""Generates tests/golden/ref_c_oracles.json from the reference's OWN C oracles.

The reference keeps C dequantisation oracles as Go raw-string constants in its
test files (tensor/oracle_q4_k_test.go:15-124, tensor/oracle_q6_k_test.go:15-130,
tensor/oracle_c_test.go:16-91).  oracle/build_ref.sh compiles them where they
lie into oracle/_ref/; this script feeds them the fixtures the reference tests
build and records the outputs (float32 bit patterns) so the GPU box, which has
no reference tree, can pin the oracle and the CUDA kernels against them.

Fixtures restated from the reference tests:
  Q4_K  tensor/oracle_q4_k_test.go:140-155 (block + dense x) and :234-265 (hostile)
  Q6_K  tensor/oracle_q6_k_test.go:146-162 and :243-273 (hostile)
  Q5_0  tensor/oracle_c_test.go:106-115

Run:  python tests/golden/make_golden.py   (needs the reference tree + gcc)
"""
from __future__ import annotations

import json
import os
import struct
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
REF_BIN = os.path.join(ROOT, "oracle", "_ref")


def run_ref(binary: str, block: bytes, dense: np.ndarray | None, nout: int):
    with tempfile.TemporaryDirectory() as td:
        fin = os.path.join(td, "in.bin")
        fout = os.path.join(td, "out.bin")
        with open(fin, "wb") as f:
            f.write(block)
        args = [os.path.join(REF_BIN, binary), fin]
        if dense is not None:
            fd = os.path.join(td, "dense.bin")
            dense.astype("<f4").tofile(fd)
            args.append(fd)
        args.append(fout)
        subprocess.run(args, check=True)
        raw = open(fout, "rb").read()
    assert len(raw) == nout * 4, (binary, len(raw))
    return list(struct.unpack("<%dI" % nout, raw))


def q4k_fixture() -> bytes:
    b = bytearray(144)
    struct.pack_into("<HH", b, 0, 0x3C00, 0x3800)
    for i in range(12):
        b[4 + i] = (i * 37 + 193) & 0xFF
    for i in range(128):
        b[16 + i] = (i * 13 + 7) & 0xFF
    return bytes(b)


def q6k_fixture() -> bytes:
    b = bytearray(210)
    for i in range(128):
        b[i] = (i * 19 + 5) & 0xFF
    for i in range(64):
        b[128 + i] = (i * 29 + 17) & 0xFF
    for i in range(16):
        b[192 + i] = (i * 7 - 31) & 0xFF
    struct.pack_into("<H", b, 208, 0x3C00)
    return bytes(b)


def hostile(n: int, val: int, d_off: int, d_vals) -> bytes:
    b = bytearray([val] * n)
    struct.pack_into("<" + "H" * len(d_vals), b, d_off, *d_vals)
    return bytes(b)


def q5_0_fixture() -> bytes:
    b = bytearray(22)
    struct.pack_into("<HI", b, 0, 0x3C00, 0xAAAAAAAA)
    for i in range(16):
        b[6 + i] = (i * 17) & 0xFF
    return bytes(b)


def main() -> None:
    subprocess.run([os.path.join(ROOT, "oracle", "build_ref.sh")], check=True)
    if not os.path.exists(os.path.join(REF_BIN, "q4_k_dequant")):
        sys.exit("reference C oracles not built (no reference tree?)")
    out = {"source": "reference inline C oracles (tensor/oracle_*_test.go), outputs as float32 bits",
           "q4_k": [], "q6_k": [], "q5_0": []}
    dense_q4 = np.array([(i % 17) - 8 for i in range(256)], np.float32)
    dense_q6 = np.array([(i % 13) - 6 for i in range(256)], np.float32)
    ones = np.ones(256, np.float32)
    cases_q4 = [("fixture", q4k_fixture(), dense_q4)]
    cases_q6 = [("fixture", q6k_fixture(), dense_q6)]
    for name, val in (("AllZero", 0x00), ("AllOne", 0xFF), ("AlternatingAA", 0xAA), ("Alternating55", 0x55)):
        cases_q4.append((name, hostile(144, val, 0, (0x3C00, 0x3800)), ones))
        cases_q6.append((name, hostile(210, val, 208, (0x3C00,)), ones))
    for name, blk, dense in cases_q4:
        bits = run_ref("q4_k_dequant", blk, dense, 257)
        out["q4_k"].append({"name": name, "block": blk.hex(), "dense": [float(v) for v in dense],
                            "dequant_bits": bits[:256], "dot_bits": bits[256]})
    for name, blk, dense in cases_q6:
        bits = run_ref("q6_k_dequant", blk, dense, 257)
        out["q6_k"].append({"name": name, "block": blk.hex(), "dense": [float(v) for v in dense],
                            "dequant_bits": bits[:256], "dot_bits": bits[256]})
    blk = q5_0_fixture()
    bits = run_ref("q5_0_dequant", blk, None, 32)
    out["q5_0"].append({"name": "fixture", "block": blk.hex(), "dequant_bits": bits})
    path = os.path.join(HERE, "ref_c_oracles.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=0)
    print("wrote", path)


if __name__ == "__main__":
    main()

"""Generates the golden fixtures of this directory (run in a container that has the reference).

    python tests/golden/make_golden.py [--ref /path/to/reference]

1. kat_matmulnbits.json -- the reference's known-answer tests for MatMulNBits,
   transcribed case by case from tests/ModelSharp.Tests/MatMulNBitsTests.cs (hand-packed
   weights and hand-computed Y; the file's tolerance is 1e-4 absolute, line 23).
2. ref_native.npz -- outputs of the reference's own native kernel ms_qgemm_nbits
   (native/src/qgemm.cpp:77-118, built from the reference sources by oracle/Makefile) on the
   seeded cases of tests/golden/cases.py that it accepts (fp32, packed or absent zero
   points), plus input checksums so a change in the generator is caught.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import oracle  # noqa: E402
from tests.golden import cases  # noqa: E402

HERE = Path(__file__).resolve().parent


def pack4(lo: int, hi: int) -> int:
    return (lo & 0xF) | ((hi & 0xF) << 4)


# MatMulNBitsTests.cs -- each entry cites the [Fact] it transcribes.
KATS = [
    dict(name="Bits4_DefaultZeroPoint_SingleBlock", cite="MatMulNBitsTests.cs:57-82",
         a_shape=[1, 4], a=[1, 2, 3, 4], b_shape=[2, 1, 2],
         b=[pack4(8, 9), pack4(7, 10), pack4(0, 15), pack4(8, 4)], scales=[2.0, 0.5],
         zp_kind="none", zp=None, N=2, K=4, bits=4, block_size=4, y_shape=[1, 2], expected=[14, -5]),
    dict(name="Bits4_DefaultZeroPoint_TwoBlocks_PerBlockScale", cite="MatMulNBitsTests.cs:86-115",
         a_shape=[1, 8], a=[1, 2, 3, 4, 5, 6, 7, 8], b_shape=[2, 2, 2],
         b=[pack4(8, 10), pack4(8, 8), pack4(8, 8), pack4(12, 8),
            pack4(9, 8), pack4(8, 7), pack4(8, 8), pack4(8, 15)],
         scales=[1, 2, 0.5, 1], zp_kind="none", zp=None, N=2, K=8, bits=4, block_size=4,
         y_shape=[1, 2], expected=[60, 54.5]),
    dict(name="Bits4_PackedZeroPoints", cite="MatMulNBitsTests.cs:119-144",
         a_shape=[1, 4], a=[1, 2, 3, 4], b_shape=[2, 1, 2],
         b=[pack4(8, 9), pack4(7, 10), pack4(0, 15), pack4(8, 4)], scales=[2.0, 0.5],
         zp_kind="packed", zp=[pack4(6, 0), pack4(10, 0)], zp_shape=[2],
         N=2, K=4, bits=4, block_size=4, y_shape=[1, 2], expected=[54, -15]),
    dict(name="Bits4_FloatZeroPoints", cite="MatMulNBitsTests.cs:148-165",
         a_shape=[1, 4], a=[1, 2, 3, 4], b_shape=[2, 1, 2],
         b=[pack4(8, 9), pack4(7, 10), pack4(0, 15), pack4(8, 4)], scales=[2.0, 0.5],
         zp_kind="float", zp=[6.0, 10.0], zp_shape=[2],
         N=2, K=4, bits=4, block_size=4, y_shape=[1, 2], expected=[54, -15]),
    dict(name="Bits4_BatchedA", cite="MatMulNBitsTests.cs:169-191",
         a_shape=[2, 4], a=[1, 2, 3, 4, 2, 0, 1, 0], b_shape=[2, 1, 2],
         b=[pack4(8, 9), pack4(7, 10), pack4(0, 15), pack4(8, 4)], scales=[2.0, 0.5],
         zp_kind="none", zp=None, N=2, K=4, bits=4, block_size=4, y_shape=[2, 2], expected=[14, -5, -2, -8]),
    dict(name="Bits4_ThreeDimA_PreservesLeadingDims", cite="MatMulNBitsTests.cs:195-213",
         a_shape=[2, 1, 4], a=[1, 2, 3, 4, 2, 0, 1, 0], b_shape=[2, 1, 2],
         b=[pack4(8, 9), pack4(7, 10), pack4(0, 15), pack4(8, 4)], scales=[2.0, 0.5],
         zp_kind="none", zp=None, N=2, K=4, bits=4, block_size=4, y_shape=[2, 1, 2],
         expected=[14, -5, -2, -8]),
    dict(name="Bits4_KNotMultipleOfBlockSize", cite="MatMulNBitsTests.cs:217-241",
         a_shape=[1, 6], a=[1, 2, 3, 4, 5, 6], b_shape=[1, 2, 2],
         b=[pack4(8, 9), pack4(8, 7), pack4(10, 8), pack4(6, 6)], scales=[1, 2],
         zp_kind="none", zp=None, N=1, K=6, bits=4, block_size=4, y_shape=[1, 1], expected=[18]),
    dict(name="Bits8_DefaultZeroPoint", cite="MatMulNBitsTests.cs:245-267",
         a_shape=[1, 4], a=[1, 2, 3, 4], b_shape=[2, 1, 4],
         b=[128, 130, 126, 132, 120, 128, 140, 128], scales=[2.0, 0.5],
         zp_kind="none", zp=None, N=2, K=4, bits=8, block_size=4, y_shape=[1, 2], expected=[28, 14]),
]


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        if a is not None:
            h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()[:16]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=None,
                    help="reference checkout (default: $MODELSHARP_REFERENCE, else ../reference beside the repo)")
    args = ap.parse_args()
    oracle.build(args.ref or oracle.reference_root())
    if not oracle.reference_available():
        raise SystemExit("reference kernel not built; is the reference tree present?")

    (HERE / "kat_matmulnbits.json").write_text(json.dumps(
        {"source": "tests/ModelSharp.Tests/MatMulNBitsTests.cs", "tolerance_abs": 1e-4, "cases": KATS}, indent=1))

    arrays, meta = {}, []
    groups = [("qgemm", len(cases.QGEMM_GRID), cases.qgemm_case),
              ("gpu", len(cases.GPU_PARITY_GRID), cases.gpu_parity_case),
              ("base", len(cases.BASELINE_GEMV), cases.baseline_case)]
    for tag, n, make in groups:
        for i in range(n):
            c = make(i)
            key = f"{tag}{i}"
            entry = dict(key=key, M=c["M"], N=c["N"], K=c["K"], bits=c["bits"], block_size=c["block_size"],
                         zp_kind=c["zp_kind"], inputs=digest(c["a"], c["b"], c["scales"], c["zp"]))
            if c["zp_kind"] != "float":
                arrays[key] = oracle.reference_native(c)
                entry["y"] = "reference ms_qgemm_nbits"
            else:
                arrays[key] = oracle.f64(c)
                entry["y"] = "dequant + double dot (qgemm_test.cpp:60-89); ms_qgemm_nbits has no float zp"
            meta.append(entry)
    np.savez_compressed(HERE / "ref_native.npz", **arrays)
    # the reference's approximate int8-activation kernel on the 4-bit cases of the qgemm grid
    w4 = {}
    for i in cases.W4A8_CASES:
        c = cases.qgemm_case(i)
        w4[f"qgemm{i}"] = oracle.reference_w4a8(c)
    np.savez_compressed(HERE / "ref_w4a8.npz", **w4)
    (HERE / "ref_native.json").write_text(json.dumps(
        {"generator": "tests/golden/make_golden.py", "reference_build": oracle._ref_lib().ms_build_info().decode(),
         "cases": meta}, indent=1))
    print(f"wrote {len(KATS)} KATs, {len(meta)} reference outputs and {len(w4)} ms_qgemm_w4a8 outputs")


if __name__ == "__main__":
    main()

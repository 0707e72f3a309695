"""The parity checker itself, pinned against the reference before anything trusts it.

* the reference's known-answer tests (MatMulNBitsTests.cs, transcribed into
  tests/golden/kat_matmulnbits.json) within the file's own 1e-4 absolute tolerance;
* the reference's native ms_qgemm_nbits outputs on seeded cases (tests/golden/ref_native.npz,
  written by tests/golden/make_golden.py) at rel-L2 <= 1e-6;
* the generator still produces the inputs those outputs were computed from;
* the restatement of the reference's int8-activation ms_qgemm_w4a8 against that kernel's own
  outputs (tests/golden/ref_w4a8.npz) at rel-L2 <= 1e-6 (the integer parts are exact; only the
  fp32 order of the per-block sum differs from the reference's vectorised loop).
"""
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle
from tests.golden import cases
from tests.golden.make_golden import digest

GOLD = Path(__file__).resolve().parent / "golden"
KATS = json.loads((GOLD / "kat_matmulnbits.json").read_text())
META = json.loads((GOLD / "ref_native.json").read_text())
MAKERS = {"qgemm": cases.qgemm_case, "gpu": cases.gpu_parity_case, "base": cases.baseline_case}


def kat_case(k: dict) -> dict:
    zp = None
    if k["zp"] is not None:
        zp = np.array(k["zp"], np.float32 if k["zp_kind"] == "float" else np.uint8)
    return dict(a=np.array(k["a"], np.float32).reshape(k["a_shape"]), b=np.array(k["b"], np.uint8),
                scales=np.array(k["scales"], np.float32), zp=zp, zp_kind=k["zp_kind"], N=k["N"], K=k["K"],
                bits=k["bits"], block_size=k["block_size"])


def golden_case(key: str) -> dict:
    tag = key.rstrip("0123456789")
    return MAKERS[tag](int(key[len(tag):]))


@pytest.mark.parametrize("k", KATS["cases"], ids=[k["name"] for k in KATS["cases"]])
def test_oracle_known_answers(k):
    c = kat_case(k)
    for fn in (oracle.managed, oracle.f64):
        y = fn(c).reshape(-1)
        np.testing.assert_allclose(y, np.array(k["expected"], np.float32), rtol=0, atol=KATS["tolerance_abs"])


@pytest.mark.parametrize("e", META["cases"], ids=[e["key"] for e in META["cases"]])
def test_oracle_matches_reference_native(e):
    c = golden_case(e["key"])
    assert digest(c["a"], c["b"], c["scales"], c["zp"]) == e["inputs"], "input generator drifted"
    ref = np.load(GOLD / "ref_native.npz")[e["key"]]
    assert oracle.rel_l2(oracle.managed(c), ref) <= 1e-6
    assert oracle.rel_l2(oracle.f64(c), ref) <= 1e-6


@pytest.mark.skipif(not oracle.reference_available(), reason="reference kernel not built here")
def test_reference_native_live():
    """When oracle/_ref is built, re-run the reference kernel live on one case per group."""
    for key in ("qgemm5", "gpu3", "base0"):
        c = golden_case(key)
        ref = np.load(GOLD / "ref_native.npz")[key]
        assert oracle.rel_l2(oracle.reference_native(c), ref) == 0.0


def test_oracle_ignores_codes_past_k():
    """Codes of a ragged last block past K, and the unused high zp nibble, must not matter."""
    c = cases.gpu_parity_case(9)  # K=20, bs=16: last block half used
    y0 = oracle.managed(c)
    c2 = dict(c)
    b = c["b"].copy()
    b[:, -1, 2:] ^= 0xFF  # in-block indices 4..15 of the last block lie past K
    c2["b"] = b
    np.testing.assert_array_equal(oracle.managed(c2), y0)
    c3 = cases.gpu_parity_case(3)  # packed zp, nb = 3 -> high nibble of byte 1 unused
    y3 = oracle.managed(c3)
    z = c3["zp"].copy()
    z[:, -1] ^= 0xF0
    c4 = dict(c3)
    c4["zp"] = z
    np.testing.assert_array_equal(oracle.managed(c4), y3)


W4A8 = np.load(GOLD / "ref_w4a8.npz")


@pytest.mark.parametrize("i", cases.W4A8_CASES)
def test_w4a8_restatement_matches_reference_outputs(i):
    c = cases.qgemm_case(i)
    ref = W4A8[f"qgemm{i}"]
    got = oracle.w4a8(c)
    assert oracle.rel_l2(got, ref) <= 1e-6
    assert oracle.rel_l2(got, oracle.managed(c)) > 1e-4  # approximate: activations quantised to int8


@pytest.mark.skipif(not oracle.reference_available(), reason="reference kernel not built here")
def test_w4a8_reference_live():
    for i in cases.W4A8_CASES[::5]:
        c = cases.qgemm_case(i)
        np.testing.assert_array_equal(oracle.reference_w4a8(c), W4A8[f"qgemm{i}"])

"""Pins the CPU oracle (oracle/nnc_oracle.c) before anything is compared
against it:

* against every committed golden fixture — the reference's own runtime KATs
  and seeded cases whose expected outputs came from the compiled reference
  (tests/golden/make_golden.py) — bit for bit;
* against the compiled reference itself (oracle/_ref/libref_ops.so) on
  freshly seeded, larger inputs, when that library is present.
"""

import numpy as np
import pytest

import golden_cases as G
import opcases as C
from oracle import oracle as O


@pytest.fixture(scope="module")
def orc():
    return O.load_oracle()


@pytest.mark.parametrize("name", G.names())
def test_oracle_matches_golden(orc, name):
    case = G.by_name(name)
    got = C.run_host(orc, case, G.inputs(case))
    want = G.outputs(case)
    assert set(got) == set(want)
    for k in want:
        C.assert_close(got[k], want[k], "exact", f"{name}:{k}")


def _bigger_cases():
    r = np.random.default_rng(1234)
    x = r.standard_normal((3, 16, 20, 20)).astype(np.float32)
    w = (r.standard_normal((24, 16, 3, 3)) / 12).astype(np.float32)
    b = r.uniform(-0.1, 0.1, 24).astype(np.float32)
    yield ({"name": "conv_s2", "op": "nnc_conv_relu", "args": [C._t("x"), C._t("w"), C._t("b"), C._o("out", (3, 24, 10, 10)),
            C._i(3), C._i(3), C._i(2), C._i(2), C._i(1), C._i(1)]}, {"x": x, "w": w, "b": b})
    yield ({"name": "conv3x3", "op": "nnc_conv3x3_s1", "args": [C._t("x"), C._t("w"), C._t("b"), C._o("out", (3, 24, 20, 20))]},
           {"x": x, "w": w, "b": b})
    a = r.standard_normal((2, 4, 32, 16)).astype(np.float32)
    bb = r.standard_normal((2, 4, 16, 24)).astype(np.float32)
    yield ({"name": "bmm", "op": "nnc_matmul", "args": [C._t("a"), C._t("b"), C._o("out", (2, 4, 32, 24))]}, {"a": a, "b": bb})
    g = r.standard_normal((64, 200)).astype(np.float32)
    yield ({"name": "softmax", "op": "nnc_softmax", "args": [C._t("x"), C._o("out", (64, 200)), C._i(-1)]}, {"x": g})
    yield ({"name": "ln", "op": "nnc_layernorm", "args": [C._t("x"), C.NULL, C.NULL, C._o("out", (64, 200)), C._i(1), C._f(1e-5)]},
           {"x": g})
    yield ({"name": "rsum", "op": "nnc_reducesum", "args": [C._t("x"), C._o("out", (64,)), C._i(1), C._i(0)]}, {"x": g})
    p = r.standard_normal((2, 8, 17, 15)).astype(np.float32)
    yield ({"name": "maxpool", "op": "nnc_maxpool2d", "args": [C._t("x"), C._o("out", (2, 8, 9, 8)), C._i(3), C._i(3),
            C._i(2), C._i(2), C._i(1), C._i(1)]}, {"x": p})


@pytest.mark.skipif(not O.reference_available(), reason="compiled reference (oracle/_ref) not built here")
@pytest.mark.parametrize("case_arrays", list(_bigger_cases()), ids=lambda ca: ca[0]["name"])
def test_oracle_matches_compiled_reference(orc, case_arrays):
    case, arrays = case_arrays
    ref = O.load_reference()
    got = C.run_host(orc, case, arrays)
    want = C.run_host(ref, case, arrays)
    for k in want:
        C.assert_close(got[k], want[k], "exact", f"{case['name']}:{k}")


def test_reference_batched_matmul_offsets_restated(orc):
    """The reference offsets batch i of a batched matmul by i * (number of
    matrices) elements (ops.c:1686-1708); the oracle restates that rule, so
    batch 1 of a [2, 3, 4] x [2, 4, 5] product is NOT a[1] @ b[1]."""
    r = np.random.default_rng(7)
    a = r.standard_normal((2, 3, 4)).astype(np.float32)
    b = r.standard_normal((2, 4, 5)).astype(np.float32)
    case = {"name": "q", "op": "nnc_matmul", "args": [C._t("a"), C._t("b"), C._o("out", (2, 3, 5))]}
    got = C.run_host(orc, case, {"a": a, "b": b})["out"]
    flat_a, flat_b = a.reshape(-1), b.reshape(-1)
    expect1 = flat_a[2:2 + 12].reshape(3, 4).astype(np.float64) @ flat_b[2:2 + 20].reshape(4, 5)
    np.testing.assert_allclose(got[1], expect1, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(got[0], a[0].astype(np.float64) @ b[0], rtol=1e-5, atol=1e-5)

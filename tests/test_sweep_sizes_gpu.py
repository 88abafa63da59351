"""Parity at the sizes the single-op and model sweeps measure (the BASELINE
configurations that bench.py does not run), against the CPU oracle.

Where the oracle would take minutes on the whole problem, it checks a
subset whose values do not depend on the rest: rows of a GEMM (every output
row is its own dot products), images of a convolution, slices of an
element-wise op, the first samples of a CNN batch (their samples are
independent in every operator). The transformer's are not (the reference's
batched MatMul offsets), so its batch-256 build is checked against the
reference's own batch-256 build. Row reductions, softmax and LayerNorm are
checked whole.
"""

from __future__ import annotations

import pathlib

import numpy as np
import pytest

import opcases as C
from nnc_cuda import lib as L
from nnc_cuda import workloads as W

pytestmark = pytest.mark.gpu


def _oracle():
    from oracle import oracle as O

    return O.load_oracle()


def _normal(seed, shape):
    return np.random.default_rng(seed).standard_normal(shape, dtype=np.float32)


# ------------------------------------------------------------------ GEMM --
@pytest.mark.parametrize("prec", [L.PRECISION_TF32, L.PRECISION_3XTF32])
@pytest.mark.parametrize("op", ["nnc_gemm", "nnc_gemm_nt"])
@pytest.mark.parametrize("n", [2048, 8192])
def test_gemm_sweep_sizes_rows_vs_oracle(cuda_lib, n, op, prec):
    """M = N = K = n on the GPU; the oracle recomputes 32 rows from the top
    and 32 from the bottom of the output (different M tiles and, at 8192,
    different CTA-pair tiles)."""
    a = _normal(n, (n, n))
    b = _normal(n + 1, (n, n))
    tail = [C._f(1.0), C._f(0.0)] + ([C._i(0), C._i(0)] if op == "nnc_gemm" else [])
    case = {"name": op, "op": op, "args": [C._t("a"), C._t("b"), C.NULL, C._o("out", (n, n))] + tail}
    cuda_lib.nnc_cuda_set_precision(prec)
    got = C.run_cuda(cuda_lib, case, {"a": a, "b": b})["out"]
    rows = np.r_[0:32, n - 32:n]
    sub = {"name": op, "op": op, "args": [C._t("a"), C._t("b"), C.NULL, C._o("out", (len(rows), n))] + tail}
    want = C.run_host(_oracle(), sub, {"a": np.ascontiguousarray(a[rows]), "b": b})["out"]
    C.assert_close(got[rows], want, C.TC_RTOL[prec], f"{op} {n}^3 prec{prec}")
    absdot = C.run_host(_oracle(), sub, {"a": np.abs(a[rows]), "b": np.abs(b)})["out"]
    C.assert_dot_close(got[rows], want, absdot, C.DOT_RTOL[prec], f"{op} {n}^3 prec{prec} per element")


# ------------------------------------------------------------------ conv --
@pytest.mark.parametrize("prec", [L.PRECISION_TF32, L.PRECISION_3XTF32])
@pytest.mark.parametrize("ch", [(64, 56), (128, 28), (256, 14), (512, 7)])
def test_conv_sweep_sizes_images_vs_oracle(cuda_lib, ch, prec):
    """3x3 pad 1 stride 1 at batch 64, NCHW (the reference's API) and
    channels-last; the oracle recomputes images 0, 31 and 63."""
    c, h = ch
    n = 64
    x = _normal(c, (n, c, h, h))
    w = (_normal(c + 1, (c, c, 3, 3)) * np.float32(0.05)).astype(np.float32)
    b = (_normal(c + 2, (c,)) * np.float32(0.01)).astype(np.float32)

    def case(batch):
        return {"name": "conv", "op": "nnc_conv",
                "args": [C._t("x"), C._t("w"), C._t("b"), C._o("out", (batch, c, h, h))] + [C._i(v) for v in (3, 3, 1, 1, 1, 1)]}

    cuda_lib.nnc_cuda_set_precision(prec)
    got = C.run_cuda(cuda_lib, case(n), {"x": x, "w": w, "b": b})["out"]
    got_cl = C.run_cuda(cuda_lib, case(n), {"x": x, "w": w, "b": b}, nhwc={"x", "out"})["out"]
    imgs = [0, 31, 63]
    want = C.run_host(_oracle(), case(len(imgs)), {"x": np.ascontiguousarray(x[imgs]), "w": w, "b": b})["out"]
    C.assert_close(got[imgs], want, C.TC_RTOL[prec], f"conv {ch} NCHW prec{prec}")
    C.assert_close(got_cl[imgs], want, C.TC_RTOL[prec], f"conv {ch} channels-last prec{prec}")
    # Per element against sum |x| |w| (the bias, below 0.03, is left out of
    # the bound's sum but is exact in both).
    absdot = C.run_host(_oracle(), case(len(imgs)), {"x": np.abs(x[imgs]), "w": np.abs(w),
                                                       "b": np.zeros_like(b)})["out"]
    absdot = absdot + np.abs(b)[None, :, None, None]
    C.assert_dot_close(got[imgs], want, absdot, C.DOT_RTOL[prec], f"conv {ch} NCHW prec{prec} per element")
    C.assert_dot_close(got_cl[imgs], want, absdot, C.DOT_RTOL[prec], f"conv {ch} channels-last prec{prec} per element")


# ------------------------------------------------------------- row ops --
def test_softmax_4096x4096_vs_oracle(cuda_lib):
    x = _normal(41, (4096, 4096))
    case = {"name": "sm", "op": "nnc_softmax", "args": [C._t("x"), C._o("out", x.shape), C._i(-1)]}
    got = C.run_cuda(cuda_lib, case, {"x": x})["out"]
    want = C.run_host(_oracle(), case, {"x": x})["out"]
    C.assert_close(got, want, 2e-6, "softmax [4096,4096]")


def test_layernorm_32768x1024_vs_oracle(cuda_lib):
    r = np.random.default_rng(42)
    x = r.standard_normal((32768, 1024), dtype=np.float32)
    g = r.uniform(0.5, 1.5, 1024).astype(np.float32)
    b = r.uniform(-0.1, 0.1, 1024).astype(np.float32)
    case = {"name": "ln", "op": "nnc_layernorm",
            "args": [C._t("x"), C._t("g"), C._t("b"), C._o("out", x.shape), C._i(-1), C._f(1e-5)]}
    got = C.run_cuda(cuda_lib, case, {"x": x, "g": g, "b": b})["out"]
    want = C.run_host(_oracle(), case, {"x": x, "g": g, "b": b})["out"]
    C.assert_close(got, want, 1e-5, "layernorm [32768,1024]")


@pytest.mark.parametrize("op", ["nnc_reducesum", "nnc_reducemean"])
def test_reduce_16384x4096_vs_oracle(cuda_lib, op):
    x = _normal(43, (16384, 4096))
    case = {"name": op, "op": op, "args": [C._t("x"), C._o("out", (16384, 1)), C._i(-1), C._i(1)]}
    got = C.run_cuda(cuda_lib, case, {"x": x})["out"]
    want = C.run_host(_oracle(), case, {"x": x})["out"]
    C.assert_close(got, want, 1e-6, f"{op} [16384,4096]")


# ---------------------------------------------------------- element-wise --
@pytest.mark.parametrize("op,tol", [("nnc_add", "exact"), ("nnc_sigmoid", 2e-6)])
def test_eltwise_2pow28_slices_vs_oracle(cuda_lib, op, tol):
    """2^28 elements (1 GiB per tensor) on the GPU; the oracle recomputes
    the first and the last 2^20 elements."""
    n = 1 << 28
    binary = op == "nnc_add"
    arrays = {"a": _normal(44, (n,))}
    if binary:
        arrays["b"] = _normal(45, (n,))
    ins = [C._t("a"), C._t("b")] if binary else [C._t("a")]
    case = {"name": op, "op": op, "args": ins + [C._o("out", (n,))]}
    got = C.run_cuda(cuda_lib, case, arrays)["out"]
    s = 1 << 20
    for lo in (0, n - s):
        sub_arrays = {k: np.ascontiguousarray(v[lo:lo + s]) for k, v in arrays.items()}
        sub = {"name": op, "op": op, "args": ins + [C._o("out", (s,))]}
        want = C.run_host(_oracle(), sub, sub_arrays)["out"]
        C.assert_close(got[lo:lo + s], want, tol, f"{op} 2^28 [{lo}:+{s}]")


# ---------------------------------------------------------------- models --
GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "models.npz"
MODEL_RTOL = C.MODEL_RTOL


@pytest.fixture(scope="module")
def golden():
    z = np.load(GOLDEN)
    return {k: z[k] for k in z.files}


@pytest.mark.parametrize("prec", [L.PRECISION_TF32, L.PRECISION_3XTF32])
@pytest.mark.parametrize("tag,model,batch,key,k", [
    ("lenet5_o1_b8192", "lenet5", 8192, "lenet5_b16", 16),
    ("lenet5_o3_b8192", "lenet5", 8192, "lenet5_b16", 16),
    ("resnet18_o1_b64", "resnet18", 64, "resnet18_b2", 2),
    ("resnet18_o1_b256", "resnet18", 256, "resnet18_b2", 2),
])
def test_sweep_models_first_samples_vs_reference(cuda_lib, golden, tag, model, batch, key, k, prec):
    """The sweep's model builds at their measured batch: the first k samples
    of the seeded batch against the reference's x86 build of the same graph
    (the seeded input's first samples are the golden's samples)."""
    from nnc_cuda.model import CudaModel

    m = CudaModel(tag)
    m.init(0)
    try:
        m.load_constants(W.BUILDERS[model](batch))
        cuda_lib.nnc_cuda_set_precision(prec)
        got = m.run_host(W.BUILDERS[model](batch).input_array(batch))
    finally:
        m.free()
    assert np.array_equal(golden[f"{key}/input"], W.BUILDERS[model](k).input_array(k))
    C.assert_close(got[:k], golden[f"{key}/output"], MODEL_RTOL[prec], f"{tag}[:{k}] prec{prec}")


@pytest.mark.parametrize("prec", [L.PRECISION_TF32, L.PRECISION_3XTF32])
@pytest.mark.parametrize("tag", ["transformer_o1_b256", "transformer_o3_b256"])
def test_transformer_b256_vs_reference(cuda_lib, golden, tag, prec):
    """The transformer at batch 256. Its samples are not independent in the
    reference: batched MatMul offsets batch b by b times the batch count
    (ops.c:1680-1700), so the attention products of one sample read other
    samples' rows and the batch-256 result differs from a batch-1 run. The
    golden is the reference's own batch-256 x86 build (samples 0, 101, 255
    kept), which the cuda build must reproduce quirk and all."""
    from nnc_cuda.model import CudaModel

    m = CudaModel(tag)
    m.init(0)
    try:
        model = W.transformer(256)
        m.load_constants(model)
        cuda_lib.nnc_cuda_set_precision(prec)
        got = m.run_host(model.input_array(256))
    finally:
        m.free()
    keep = golden["transformer_b256/samples"]
    C.assert_close(got[keep], golden["transformer_b256/output"], MODEL_RTOL[prec], f"{tag} prec{prec}")

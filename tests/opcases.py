"""Operator cases shared by the oracle pin tests, the golden-fixture
generator and the GPU parity tests.

A case is a JSON-able dict::

    {"name": ..., "op": "nnc_conv", "tol": "exact" | "tc" | <rtol float>,
     "args": [arg, ...]}

with arguments
    {"k": "t", "n": <array name>}            input tensor
    {"k": "o", "n": <name>, "shape": [...]}  output tensor (pre-filled 7.0)
    {"k": "null"}                            NULL tensor
    {"k": "i", "v": int} / {"k": "f", "v": float}
    {"k": "perm", "v": [..] | None}          int64_t* (NULL when None)
    {"k": "tl", "n": [names]}                Tensor** of inputs
    {"k": "ol", "n": [names], "shape": [[..], ..]}  Tensor** of outputs

and the input arrays in a dict {name: np.ndarray}. The same case runs on
any library exporting the reference's nnc_* symbols over host memory
(oracle, compiled reference) via :func:`run_host`, or on the CUDA library
via :func:`run_cuda`.
"""

from __future__ import annotations

import ctypes
import zlib

import numpy as np

from nnc_cuda import lib as L
from nnc_cuda import tensor as T

SENTINEL = 7.0


# ----------------------------------------------------------------- running --
def _outputs(case):
    outs = []
    for a in case["args"]:
        if a["k"] == "o":
            outs.append((a["n"], a["shape"], a.get("dtype", "float32")))
        elif a["k"] == "ol":
            for n, s in zip(a["n"], a["shape"]):
                outs.append((n, s, a.get("dtype", "float32")))
    return outs


def _scalar(a):
    if a["k"] == "i":
        return ctypes.c_int(int(a["v"]))
    if a["k"] == "f":
        return ctypes.c_float(float(a["v"]))
    raise KeyError(a["k"])


def run_host(so, case, arrays):
    """Runs `case` on a host-memory library; returns {output name: array}."""
    keep = []
    bufs = {n: np.ascontiguousarray(v).copy() for n, v in arrays.items()}
    for n, s, dt in _outputs(case):
        bufs[n] = np.full(s, SENTINEL, dtype=dt)
    cargs = []
    for a in case["args"]:
        k = a["k"]
        if k in ("t", "o"):
            r = T.from_numpy(bufs[a["n"]])
            keep.append(r)
            cargs.append(r.ptr)
        elif k == "null":
            cargs.append(None)
        elif k in ("i", "f"):
            cargs.append(_scalar(a))
        elif k == "perm":
            if a["v"] is None:
                cargs.append(None)
            else:
                arr = (ctypes.c_int64 * len(a["v"]))(*a["v"])
                keep.append(arr)
                cargs.append(ctypes.cast(arr, ctypes.POINTER(ctypes.c_int64)))
        elif k in ("tl", "ol"):
            refs = [T.from_numpy(bufs[n]) for n in a["n"]]
            keep.extend(refs)
            arr = T.tensor_array(refs)
            keep.append(arr)
            cargs.append(arr)
        else:
            raise KeyError(k)
    getattr(so, case["op"])(*cargs)
    return {n: bufs[n] for n, _, _ in _outputs(case)}


def run_cuda(so, case, arrays, nhwc=()):
    """Runs `case` on libnnc_cuda.so with device buffers.

    Names in `nhwc` are 4-D tensors passed channels-last with the
    NNC_CUDA_TAG_NHWC tag (logical NCHW shape kept); their results are
    converted back to NCHW.
    """
    import torch

    keep = []
    dev = {}

    def to_dev(name, a):
        t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
        if name in nhwc:
            t = t.permute(0, 2, 3, 1).contiguous()
        return t

    for n, v in arrays.items():
        dev[n] = to_dev(n, v)
    for n, s, dt in _outputs(case):
        dev[n] = to_dev(n, np.full(s, SENTINEL, dtype=dt))

    def ref(name):
        t = dev[name]
        if name in nhwc:
            shape = (t.shape[0], t.shape[3], t.shape[1], t.shape[2])
            return T.from_torch(t, tag=L.TAG_NHWC, shape=shape)
        return T.from_torch(t)

    cargs = []
    for a in case["args"]:
        k = a["k"]
        if k in ("t", "o"):
            r = ref(a["n"])
            keep.append(r)
            cargs.append(r.ptr)
        elif k == "null":
            cargs.append(None)
        elif k in ("i", "f"):
            cargs.append(_scalar(a))
        elif k == "perm":
            if a["v"] is None:
                cargs.append(None)
            else:
                arr = (ctypes.c_int64 * len(a["v"]))(*a["v"])
                keep.append(arr)
                cargs.append(ctypes.cast(arr, ctypes.POINTER(ctypes.c_int64)))
        elif k in ("tl", "ol"):
            refs = [ref(n) for n in a["n"]]
            keep.extend(refs)
            arr = T.tensor_array(refs)
            keep.append(arr)
            cargs.append(arr)
        else:
            raise KeyError(k)
    so.nnc_cuda_set_stream(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    getattr(so, case["op"])(*cargs)
    torch.cuda.synchronize()
    status = so.nnc_cuda_get_last_error()
    assert status == 0, so.nnc_cuda_get_last_error_string().decode()
    out = {}
    for n, _, _ in _outputs(case):
        t = dev[n]
        if n in nhwc:
            t = t.permute(0, 3, 1, 2).contiguous()
        out[n] = t.cpu().numpy()
    return out


# ------------------------------------------------------------- comparing --
def assert_close(got, want, tol, what=""):
    """tol: "exact" — every non-NaN value bit-identical (signed zeros
    included) and NaNs in the same places (NaN payload bits are not compared:
    the GPU produces canonical NaNs where x86 propagates an operand's payload)
    — or a float rtol applied normwise: |got - want| <= rtol * (|want| +
    max|want|), NaNs in the same places."""
    assert got.shape == want.shape, f"{what}: shape {got.shape} vs {want.shape}"
    if tol == "exact" and got.dtype.kind != "f":
        assert got.dtype == want.dtype, f"{what}: dtype {got.dtype} vs {want.dtype}"
        bad = np.flatnonzero(got.reshape(-1) != want.reshape(-1))
        assert bad.size == 0, (f"{what}: {bad.size} of {got.size} differ; first at {bad[0]}: "
                               f"got {got.flat[bad[0]]!r} want {want.flat[bad[0]]!r}")
        return
    if tol == "exact":
        g = got.view(np.uint32 if got.dtype == np.float32 else np.uint64)
        w = want.view(np.uint32 if want.dtype == np.float32 else np.uint64)
        differ = g != w
        if got.dtype.kind == "f":
            gn, wn = np.isnan(got), np.isnan(want)
            differ = np.where(gn & wn, False, differ)
        bad = np.flatnonzero(differ)
        assert bad.size == 0, (
            f"{what}: {bad.size} of {g.size} differ; first at {bad[0]}: "
            f"got {got.flat[bad[0]]!r} want {want.flat[bad[0]]!r}"
        )
        return
    gn, wn = np.isnan(got), np.isnan(want)
    assert np.array_equal(gn, wn), f"{what}: NaN positions differ"
    g = np.where(gn, 0, got).astype(np.float64)
    w = np.where(wn, 0, want).astype(np.float64)
    scale = float(np.max(np.abs(w))) if w.size else 0.0
    err = np.abs(g - w)
    lim = tol * (np.abs(w) + scale)
    bad = np.flatnonzero(err > lim)
    assert bad.size == 0, (
        f"{what}: {bad.size} of {g.size} exceed rtol {tol} (normwise); worst rel "
        f"{float(np.max(err) / max(scale, 1e-30)):.3g}; first at {bad[0]}: "
        f"got {got.flat[bad[0]]!r} want {want.flat[bad[0]]!r}"
    )


# Tolerances of the tensor-core contractions (normwise rtol, see assert_close).
TC_RTOL = {0: 2e-3, 1: 1e-5}  # NNC_CUDA_PRECISION_TF32, _3XTF32
# Whole models against the reference's x86 build (normwise). Measured on
# B200: TF32 1.7e-3 (ResNet-18) to 2.6e-3 (transformer); 3xTF32 (chunked
# accumulation) 3.5e-6 (ResNet-18), 3.9e-6 (the batch-1024 bench images),
# 2.8e-6 (transformer), 3.7e-7 (LeNet-5).
MODEL_RTOL = {0: 5e-3, 1: 1e-5}
# Per-element bound of a contraction's error relative to the sum of the
# magnitudes of its products, |d_ij| <= rtol * sum_k |a_ik| |b_kj| (the
# standard dot-product error bound; holds even where the result cancels).
DOT_RTOL = {0: 1e-3, 1: 1e-6}


def assert_dot_close(got, want, absdot, tol, what=""):
    """Per-element check of a contraction: |got - want| <= tol * absdot, with
    absdot the same contraction of |a| and |b| (computed by the oracle)."""
    assert got.shape == want.shape == absdot.shape, what
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    lim = tol * absdot.astype(np.float64) + 1e-30
    bad = np.flatnonzero(err > lim)
    assert bad.size == 0, (f"{what}: {bad.size} of {err.size} exceed {tol} x sum|a||b|; worst "
                           f"{float(np.max(err / lim)) * tol:.3g}")


# --------------------------------------------------------- seeded cases --
def rng_for(name: str) -> np.random.Generator:
    return np.random.default_rng(zlib.crc32(name.encode()))


def _t(n):
    return {"k": "t", "n": n}


def _o(n, shape, dtype="float32"):
    return {"k": "o", "n": n, "shape": list(shape), "dtype": dtype}


NULL = {"k": "null"}


def _i(v):
    return {"k": "i", "v": int(v)}


def _f(v):
    return {"k": "f", "v": float(v)}


EDGE = np.array(
    [0.0, -0.0, 1.0, -1.0, np.nan, -np.nan, np.inf, -np.inf, 3.4e38, -3.4e38, 1e-40, -1e-40,
     0.5, -2.5, 88.7, -88.7, 1e-8, 7.0, -7.0, 20.0],
    dtype=np.float32,
)


def conv_out(h, k, s, p):
    return (h + 2 * p - k) // s + 1


def seeded_cases():
    """(case, arrays) pairs: small seeded cases per hot-path op."""
    out = []

    def add(case, arrays):
        out.append((case, {k: np.asarray(v, dtype=v.dtype) for k, v in arrays.items()}))

    # --- binary element-wise, incl. every broadcast branch of ops.c:82-118
    for op in ("nnc_add", "nnc_sub", "nnc_mul", "nnc_div", "nnc_add_relu", "nnc_add_sigmoid"):
        tol = 2e-6 if op == "nnc_add_sigmoid" else "exact"
        for tag, sa, sb, so in (
            ("same", (3, 5, 7), (3, 5, 7), (3, 5, 7)),
            ("bscalar", (4, 33), (1,), (4, 33)),
            ("ascalar", (1,), (4, 33), (4, 33)),
            ("bsuffix", (6, 8, 12), (12,), (6, 8, 12)),
            ("asuffix", (10,), (7, 10), (7, 10)),
            ("bodd", (5, 7), (7,), (5, 7)),
            ("partial", (6,), (4,), (10,)),
        ):
            name = f"{op}_{tag}"
            r = rng_for(name)
            a = r.standard_normal(sa).astype(np.float32)
            b = r.standard_normal(sb).astype(np.float32)
            if op == "nnc_div":
                b = np.where(np.abs(b) < 0.05, 0.5, b).astype(np.float32)
            add({"name": name, "op": op, "tol": tol, "args": [_t("a"), _t("b"), _o("out", so)]},
                {"a": a, "b": b})
        name = f"{op}_edge"
        a = np.tile(EDGE, 4)
        b = np.repeat(EDGE, 4)
        add({"name": name, "op": op, "tol": "exact" if tol == "exact" else tol,
             "args": [_t("a"), _t("b"), _o("out", a.shape)]}, {"a": a, "b": b})

    # --- unary
    for op, tol in (("nnc_relu", "exact"), ("nnc_sigmoid", 2e-6), ("nnc_tanh", 2e-6),
                    ("nnc_sqrt", "exact"), ("nnc_pow", "exact"), ("nnc_exp", 2e-6),
                    ("nnc_log", 2e-6), ("nnc_abs", "exact"), ("nnc_neg", "exact")):
        for tag, shape in (("vec", (1027,)), ("mat", (17, 19))):
            name = f"{op}_{tag}"
            r = rng_for(name)
            x = (r.standard_normal(shape) * 3).astype(np.float32)
            add({"name": name, "op": op, "tol": tol, "args": [_t("x"), _o("out", shape)]}, {"x": x})
        add({"name": f"{op}_edge", "op": op, "tol": tol, "args": [_t("x"), _o("out", EDGE.shape)]},
            {"x": EDGE.copy()})
    for lo, hi in ((-1.0, 1.0), (0.0, 6.0), (-3.402823e38, 3.402823e38)):
        name = f"nnc_clip_{lo:g}_{hi:g}"
        r = rng_for(name)
        x = np.concatenate([r.standard_normal(500).astype(np.float32) * 4, EDGE])
        add({"name": name, "op": "nnc_clip", "tol": "exact",
             "args": [_t("x"), _o("out", x.shape), _f(lo), _f(hi)]}, {"x": x})

    # --- softmax / layernorm / reduce
    for tag, shape, axis in (("last", (37, 129), -1), ("axis0", (5, 6, 7), 0),
                             ("mid", (4, 9, 6), 1), ("wide", (3, 9000), 1), ("ten", (2, 10), 1),
                             ("block4096", (9, 4096), -1), ("block2052", (5, 2052), -1),
                             ("block8192", (3, 8192), -1)):
        name = f"nnc_softmax_{tag}"
        r = rng_for(name)
        x = (r.standard_normal(shape) * 2).astype(np.float32)
        add({"name": name, "op": "nnc_softmax", "tol": 2e-6,
             "args": [_t("x"), _o("out", shape), _i(axis)]}, {"x": x})
    for tag, shape, axis, with_params in (("last", (33, 300), -1, True), ("slab", (4, 6, 5), 1, True),
                                          ("noparams", (8, 64), -1, False), ("wide", (3, 10000), -1, True),
                                          ("grp768", (37, 768), -1, True), ("grp1024", (11, 1024), -1, False),
                                          ("grp_inner", (5, 3, 256), 1, True)):
        name = f"nnc_layernorm_{tag}"
        r = rng_for(name)
        x = r.standard_normal(shape).astype(np.float32)
        norm = shape[axis]
        arrays = {"x": x}
        args = [_t("x")]
        if with_params:
            arrays["g"] = r.uniform(0.5, 1.5, norm).astype(np.float32)
            arrays["b"] = r.uniform(-0.1, 0.1, norm).astype(np.float32)
            args += [_t("g"), _t("b")]
        else:
            args += [NULL, NULL]
        args += [_o("out", shape), _i(axis), _f(1e-5)]
        add({"name": name, "op": "nnc_layernorm", "tol": 1e-5, "args": args}, arrays)
    for op in ("nnc_reducesum", "nnc_reducemean"):
        for tag, shape, axis, keep, tol in (("last", (17, 301), -1, 1, 1e-6), ("lastnk", (9, 64), 1, 0, 1e-6),
                                            ("axis0", (9, 8, 7), 0, 1, "exact"), ("mid", (3, 50, 4), 1, 0, "exact")):
            name = f"{op}_{tag}"
            r = rng_for(name)
            x = r.standard_normal(shape).astype(np.float32)
            oshape = list(shape)
            if keep:
                oshape[axis] = 1
            else:
                oshape.pop(axis)
            add({"name": name, "op": op, "tol": tol,
                 "args": [_t("x"), _o("out", oshape), _i(axis), _i(keep)]}, {"x": x})

    # --- pooling
    for op in ("nnc_maxpool2d", "nnc_avgpool2d"):
        for tag, shape, k, s, p in (("k3s2p1", (2, 3, 11, 13), 3, 2, 1), ("k2s2", (2, 6, 28, 28), 2, 2, 0),
                                    ("global7", (2, 8, 7, 7), 7, 7, 0), ("empty", (1, 1, 2, 2), 1, 1, 4),
                                    ("k3s1p1", (1, 4, 6, 5), 3, 1, 1), ("k2s2odd", (2, 3, 11, 10), 2, 2, 0),
                                    ("k2s2oddw", (1, 2, 6, 9), 2, 2, 0)):
            name = f"{op}_{tag}"
            r = rng_for(name)
            x = r.standard_normal(shape).astype(np.float32)
            if tag in ("k3s2p1", "k2s2odd"):
                x.flat[::17] = np.nan
            oh, ow = conv_out(shape[2], k, s, p), conv_out(shape[3], k, s, p)
            add({"name": name, "op": op, "tol": "exact",
                 "args": [_t("x"), _o("out", (shape[0], shape[1], oh, ow)), _i(k), _i(k), _i(s), _i(s), _i(p), _i(p)]},
                {"x": x})

    # --- convolution (tensor-core tolerance)
    for tag, n, c, h, w, co, k, s, p, bias in (
        ("k3s1p1", 2, 5, 9, 11, 7, 3, 1, 1, True),
        ("k3s2p1", 2, 8, 12, 10, 16, 3, 2, 1, True),
        ("k1s2", 2, 32, 8, 8, 40, 1, 2, 0, True),
        ("k5p0", 3, 1, 32, 32, 6, 5, 1, 0, True),
        ("k7s2p3", 1, 3, 23, 23, 8, 7, 2, 3, True),
        ("c64", 2, 64, 8, 8, 64, 3, 1, 1, False),
        ("c130", 1, 32, 6, 6, 130, 3, 1, 1, True),
    ):
        for op in ("nnc_conv", "nnc_conv_relu"):
            name = f"{op}_{tag}"
            r = rng_for(name)
            x = r.standard_normal((n, c, h, w)).astype(np.float32)
            wt = (r.standard_normal((co, c, k, k)) / np.sqrt(c * k * k)).astype(np.float32)
            arrays = {"x": x, "w": wt}
            if bias:
                arrays["b"] = r.uniform(-0.1, 0.1, co).astype(np.float32)
            oh, ow = conv_out(h, k, s, p), conv_out(w, k, s, p)
            add({"name": name, "op": op, "tol": "tc",
                 "args": [_t("x"), _t("w"), _t("b") if bias else NULL, _o("out", (n, co, oh, ow)),
                          _i(k), _i(k), _i(s), _i(s), _i(p), _i(p)]}, arrays)
    for op, k, s, p, extra in (("nnc_conv3x3_s1", 3, 1, 1, []), ("nnc_conv_relu3x3_s1", 3, 1, 1, []),
                               ("nnc_conv7x7_s2", 7, 2, 3, []), ("nnc_conv_relu7x7_s2", 7, 2, 3, []),
                               ("nnc_conv1x1", 1, 2, 0, [2, 2, 0, 0]), ("nnc_conv_relu1x1", 1, 1, 0, [1, 1, 0, 0])):
        name = f"{op}_seeded"
        r = rng_for(name)
        c, h, co = (3, 30, 16) if k == 7 else (24, 10, 20)
        x = r.standard_normal((2, c, h, h)).astype(np.float32)
        wt = (r.standard_normal((co, c, k, k)) / np.sqrt(c * k * k)).astype(np.float32)
        b = r.uniform(-0.1, 0.1, co).astype(np.float32)
        oh = conv_out(h, k, s, p)
        add({"name": name, "op": op, "tol": "tc",
             "args": [_t("x"), _t("w"), _t("b"), _o("out", (2, co, oh, oh))] + [_i(v) for v in extra]},
            {"x": x, "w": wt, "b": b})
    name = "nnc_conv_sigmoid_seeded"
    r = rng_for(name)
    x = r.standard_normal((2, 6, 9, 9)).astype(np.float32)
    wt = (r.standard_normal((10, 6, 3, 3)) / 7).astype(np.float32)
    add({"name": name, "op": "nnc_conv_sigmoid", "tol": "tc",
         "args": [_t("x"), _t("w"), NULL, _o("out", (2, 10, 9, 9)), _i(3), _i(3), _i(1), _i(1), _i(1), _i(1)]},
        {"x": x, "w": wt})

    # --- gemm / gemm_nt / matmul
    for ta in (0, 1):
        for tb in (0, 1):
            for cmode in ("none", "row", "full"):
                name = f"nnc_gemm_t{ta}{tb}_{cmode}"
                r = rng_for(name)
                M, N, K = 70, 50, 36
                a = r.standard_normal((K, M) if ta else (M, K)).astype(np.float32)
                b = r.standard_normal((N, K) if tb else (K, N)).astype(np.float32)
                arrays = {"a": a, "b": b}
                cargs = NULL
                if cmode != "none":
                    arrays["c"] = r.standard_normal((N,) if cmode == "row" else (M, N)).astype(np.float32)
                    cargs = _t("c")
                add({"name": name, "op": "nnc_gemm", "tol": "tc",
                     "args": [_t("a"), _t("b"), cargs, _o("out", (M, N)), _f(0.75), _f(-1.25), _i(ta), _i(tb)]},
                    arrays)
    for tag, M, N, K in (("tc", 200, 160, 96), ("oddk", 130, 70, 57), ("small", 5, 3, 4)):
        name = f"nnc_gemm_nt_{tag}"
        r = rng_for(name)
        a = r.standard_normal((M, K)).astype(np.float32)
        b = r.standard_normal((N, K)).astype(np.float32)
        c = r.standard_normal((N,)).astype(np.float32)
        add({"name": name, "op": "nnc_gemm_nt", "tol": "tc",
             "args": [_t("a"), _t("b"), _t("c"), _o("out", (M, N)), _f(1.0), _f(1.0)]}, {"a": a, "b": b, "c": c})
    for tag, sa, sb, so in (("2d", (96, 64), (64, 80), (96, 80)), ("vecmat", (40,), (40, 24), (24,)),
                            ("matvec", (24, 40), (40,), (24,)), ("batched", (2, 3, 4, 5), (2, 3, 5, 6), (2, 3, 4, 6)),
                            ("bcast", (3, 64, 32), (32, 48), (3, 64, 48)), ("b1", (1, 128, 64), (64, 72), (1, 128, 72))):
        name = f"nnc_matmul_{tag}"
        r = rng_for(name)
        a = r.standard_normal(sa).astype(np.float32)
        b = r.standard_normal(sb).astype(np.float32)
        add({"name": name, "op": "nnc_matmul", "tol": "tc", "args": [_t("a"), _t("b"), _o("out", so)]},
            {"a": a, "b": b})

    # --- data movement
    for tag, shape, perm in (("2d", (5, 7), (1, 0)), ("3d", (2, 3, 4), (1, 0, 2)), ("3dlast", (4, 5, 6), (0, 2, 1)),
                             ("null", (3, 4, 5), None), ("heads", (2, 8, 4, 16), (0, 2, 1, 3)),
                             ("4dgen", (2, 3, 5, 7), (3, 1, 0, 2)), ("keys", (2, 8, 4, 16), (0, 2, 3, 1)),
                             ("unit", (3, 1, 4, 1, 5), (4, 1, 2, 0, 3)), ("merge5", (2, 3, 4, 5, 6), (2, 3, 0, 1, 4)),
                             ("oddinner", (3, 5, 7), (1, 0, 2)), ("ident", (2, 3, 4), (0, 1, 2))):
        name = f"nnc_transpose_{tag}"
        r = rng_for(name)
        x = r.standard_normal(shape).astype(np.float32)
        p = perm if perm is not None else tuple(reversed(range(len(shape))))
        oshape = tuple(shape[i] for i in p)
        add({"name": name, "op": "nnc_transpose", "tol": "exact",
             "args": [_t("x"), _o("out", oshape), {"k": "perm", "v": list(perm) if perm else None}, _i(len(shape))]},
            {"x": x})
    for op in ("nnc_reshape", "nnc_flatten", "nnc_squeeze", "nnc_unsqueeze", "nnc_identity"):
        name = f"{op}_seeded"
        r = rng_for(name)
        x = r.standard_normal((4, 6, 5)).astype(np.float32)
        extra = {"nnc_reshape": [{"k": "perm", "v": [24, 5]}, _i(2)], "nnc_identity": []}.get(op, [_i(1)])
        add({"name": name, "op": op, "tol": "exact", "args": [_t("x"), _o("out", (24, 5))] + extra}, {"x": x})
    for tag, shapes, axis, dt in (("axis0", [(2, 3), (4, 3)], 0, np.float32), ("axis1", [(2, 3, 4), (2, 5, 4), (2, 1, 4)], 1, np.float32),
                                  ("last", [(3, 2), (3, 7)], -1, np.float32), ("i64", [(2, 3), (2, 2)], 1, np.int64)):
        name = f"nnc_concat_{tag}"
        r = rng_for(name)
        arrays = {}
        for j, s in enumerate(shapes):
            arrays[f"x{j}"] = (r.standard_normal(s) * 100).astype(dt)
        ax = axis % len(shapes[0])
        oshape = list(shapes[0])
        oshape[ax] = sum(s[ax] for s in shapes)
        dts = "int64" if dt == np.int64 else "float32"
        add({"name": name, "op": "nnc_concat", "tol": "exact",
             "args": [{"k": "tl", "n": list(arrays)}, _o("out", oshape, dts), _i(len(shapes)), _i(axis)]}, arrays)
    for tag, shape, parts, axis in (("axis1", (2, 6, 3), 3, 1), ("axis0", (4, 5), 2, 0), ("last", (3, 8), 4, -1)):
        name = f"nnc_split_{tag}"
        r = rng_for(name)
        x = r.standard_normal(shape).astype(np.float32)
        ax = axis % len(shape)
        os_ = list(shape)
        os_[ax] //= parts
        names = [f"out{j}" for j in range(parts)]
        add({"name": name, "op": "nnc_split", "tol": "exact",
             "args": [_t("x"), {"k": "ol", "n": names, "shape": [os_] * parts}, _i(parts), _i(axis)]}, {"x": x})
    out.extend(library_cases())
    return out


def library_cases():
    """The operators off the BASELINE models' path (cast, comparisons and
    logic, shape / expand / tile, gather, batchnorm, LSTM), including the
    reference's broadcast, clamping and fallback branches."""
    out = []

    def add(case, arrays):
        out.append((case, arrays))

    cast_in = np.concatenate([EDGE, np.array([3e9, -3e9, 2.1e9, -2.1e9, 0.7, -0.7, 1e19, -1e19, 9.9e18],
                                             dtype=np.float32), rng_for("cast").standard_normal(40).astype(np.float32) * 50])
    bools = (rng_for("bools").random(37) > 0.5).astype(np.uint8)
    for to, odt, tag in ((0, "float32", "f32"), (2, "int32", "i32"), (6, "int64", "i64"), (5, "uint8", "bool"),
                         (1, "float32", "f16copy"), (9, "float32", "unknown")):
        add({"name": f"nnc_cast_float_to_{tag}", "op": "nnc_cast", "tol": "exact",
             "args": [_t("x"), _o("out", cast_in.shape, odt), _i(to)]}, {"x": cast_in.copy()})
    for to, odt, tag in ((0, "float32", "f32"), (2, "int32", "i32"), (6, "int64", "i64"), (5, "uint8", "bool")):
        add({"name": f"nnc_cast_bool_to_{tag}", "op": "nnc_cast", "tol": "exact",
             "args": [_t("x"), _o("out", bools.shape, odt), _i(to)]}, {"x": bools.copy()})
    for op in ("nnc_equal", "nnc_and", "nnc_greater"):
        odt = "uint8" if op == "nnc_greater" else "float32"
        for tag, sa, sb, so in (("same", (5, 7), (5, 7), (5, 7)), ("bscalar", (4, 9), (1,), (4, 9)),
                                ("ascalar", (1,), (4, 9), (4, 9)), ("bsuffix", (3, 8), (8,), (3, 8)),
                                ("asuffix", (6,), (5, 6), (5, 6)), ("partial", (6,), (4,), (10,))):
            if op == "nnc_greater" and tag == "partial":
                continue  # the reference reads both operands modulo their sizes over the whole output
            name = f"{op}_{tag}"
            r = rng_for(name)
            a = r.integers(-2, 3, sa).astype(np.float32)
            b = r.integers(-2, 3, sb).astype(np.float32)
            add({"name": name, "op": op, "tol": "exact", "args": [_t("a"), _t("b"), _o("out", so, odt)]},
                {"a": a, "b": b})
    r = rng_for("logic")
    a = (r.random(50) > 0.5).astype(np.uint8)
    b = (r.random(50) > 0.5).astype(np.uint8)
    add({"name": "nnc_or_seeded", "op": "nnc_or", "tol": "exact",
         "args": [_t("a"), _t("b"), _o("out", (50,), "uint8")]}, {"a": a, "b": b})
    add({"name": "nnc_not_seeded", "op": "nnc_not", "tol": "exact",
         "args": [_t("a"), _o("out", (50,), "uint8")]}, {"a": a})
    x = rng_for("shape").standard_normal((2, 3, 5)).astype(np.float32)
    add({"name": "nnc_shape_runtime", "op": "nnc_shape", "tol": "exact",
         "args": [_t("x"), _o("out", (3,), "int64"), {"k": "perm", "v": None}, _i(3)]}, {"x": x})
    add({"name": "nnc_shape_given", "op": "nnc_shape", "tol": "exact",
         "args": [_t("x"), _o("out", (4,), "int64"), {"k": "perm", "v": [7, 1, 9, 4]}, _i(4)]}, {"x": x})
    add({"name": "nnc_constantofshape_seeded", "op": "nnc_constantofshape", "tol": "exact",
         "args": [_o("out", (3, 4, 5)), _f(-2.5), _i(3)]}, {})
    for tag, si, so in (("rows", (7,), (4, 7)), ("same", (3, 4), (3, 4)), ("odd", (5,), (2, 6))):
        name = f"nnc_expand_{tag}"
        add({"name": name, "op": "nnc_expand", "tol": "exact",
             "args": [_t("x"), _o("out", so), {"k": "perm", "v": list(so)}, _i(len(so))]},
            {"x": rng_for(name).standard_normal(si).astype(np.float32)})
    for tag, si, rep, so in (("2d", (2, 3), [2, 3], (4, 9)), ("3d", (2, 1, 3), [1, 4, 2], (2, 4, 6)),
                             ("null", (3, 4), None, (3, 4)), ("longrep", (3, 2), [2, 2, 1], (6, 2))):
        name = f"nnc_tile_{tag}"
        add({"name": name, "op": "nnc_tile", "tol": "exact",
             "args": [_t("x"), _o("out", so), {"k": "perm", "v": rep}, _i(len(rep) if rep else len(si))]},
            {"x": rng_for(name).standard_normal(si).astype(np.float32)})
    # gather: (tag, data shape, data dtype, indices, axis, output shape)
    for tag, ds, ddt, idx, axis, os_ in (
            ("f1_scalar", (9,), 0, np.array(4), 0, (3,)),
            ("f1_neg", (9,), 0, np.array([-2]), 0, (1,)),
            ("f2_scalar_ax0", (5, 6), 0, np.array([3]), 0, (1, 6)),
            ("f2_scalar_ax1", (5, 6), 0, np.array(7), 1, (5, 1)),
            ("f3_ax0_out2", (3, 4, 5), 0, np.array(1), 0, (4, 5)),
            ("f3_ax0_out3", (3, 4, 5), 0, np.array([2]), 0, (1, 4, 5)),
            ("f3_ax1", (3, 4, 5), 0, np.array(-1), 1, (3, 5)),
            ("f3_ax2", (3, 4, 5), 0, np.array(9), -1, (3, 4)),
            ("i1_scalar", (6,), 1, np.array(2), 0, (1,)),
            ("i2_rows", (4, 3), 1, np.array([1]), 0, (3,)),
            ("i1_list", (6,), 1, np.array([5, 0, -1, 9, -9]), 0, (5,)),
            ("f2_list_ax0", (5, 4), 0, np.array([4, 0, -1, 2]), 0, (4, 4)),
            ("f2_list_ax1", (5, 4), 0, np.array([3, -4, 8]), 1, (5, 3)),
            ("f3_list_fallback", (2, 3, 4), 0, np.array([1, 0]), 1, (2, 2, 4)),
            ("i3_list_fallback", (2, 3, 4), 1, np.array([1, 0]), 0, (2, 3, 4))):
        name = f"nnc_gather_{tag}"
        r = rng_for(name)
        data = (r.integers(-50, 50, ds).astype(np.int64) if ddt else r.standard_normal(ds).astype(np.float32))
        add({"name": name, "op": "nnc_gather", "tol": "exact",
             "args": [_t("data"), _t("idx"), _o("out", os_, "int64" if ddt else "float32"), _i(axis), _i(ddt)]},
            {"data": data, "idx": np.asarray(idx, dtype=np.int64)})
    x = rng_for("bn").standard_normal((2, 3, 4, 4)).astype(np.float32)
    prm = {k: rng_for("bn" + k).standard_normal(3).astype(np.float32) for k in ("s", "b", "m")}
    prm["v"] = np.abs(prm["m"]) + 0.5
    add({"name": "nnc_batchnorm_untouched", "op": "nnc_batchnorm", "tol": "exact",
         "args": [_t("x"), _t("s"), _t("b"), _t("m"), _t("v"), _o("out", x.shape), _f(1e-5), _i(0)]},
        dict(x=x, **prm))
    for tag, T, B, I, H, direction, bias in (("fwd", 3, 2, 5, 4, 0, True), ("bidir", 4, 2, 3, 6, 2, True),
                                             ("nobias", 2, 3, 4, 5, 0, False), ("wide", 3, 1, 16, 40, 0, True)):
        name = f"nnc_lstm_{tag}"
        r = rng_for(name)
        D = 2 if direction == 2 else 1
        arrays = {"X": r.standard_normal((T, B, I)).astype(np.float32),
                  "W": (r.standard_normal((D, 4 * H, I)) * 0.4).astype(np.float32),
                  "R": (r.standard_normal((D, 4 * H, H)) * 0.4).astype(np.float32)}
        if bias:
            arrays["Bv"] = (r.standard_normal((D, 8 * H)) * 0.1).astype(np.float32)
        add({"name": name, "op": "nnc_lstm", "tol": 2e-6,
             "args": [_t("X"), _t("W"), _t("R"), _t("Bv") if bias else NULL, _o("Y", (T, D, B, H)),
                      _o("Yh", (D, B, H)), _o("Yc", (D, B, H)), _i(direction), _i(H)]}, arrays)
    return out


def fused_cases():
    """Cases for the entry points without a reference counterpart; their
    expected values come from the oracle's restatement of the reference
    composition."""
    out = []
    for op, k, s, p, extra in (("nnc_conv_add_relu", 3, 2, 1, [3, 3, 2, 2, 1, 1]),
                               ("nnc_conv_add_relu1x1", 1, 2, 0, [2, 2, 0, 0]),
                               ("nnc_conv_add_relu3x3_s1", 3, 1, 1, [])):
        name = f"{op}_seeded"
        r = rng_for(name)
        x = r.standard_normal((2, 16, 10, 10)).astype(np.float32)
        wt = (r.standard_normal((24, 16, k, k)) / np.sqrt(16 * k * k)).astype(np.float32)
        b = r.uniform(-0.1, 0.1, 24).astype(np.float32)
        oh = conv_out(10, k, s, p)
        res = r.standard_normal((2, 24, oh, oh)).astype(np.float32)
        out.append(({"name": name, "op": op, "tol": "tc",
                     "args": [_t("x"), _t("w"), _t("b"), _t("res"), _o("out", (2, 24, oh, oh))] + [_i(v) for v in extra]},
                    {"x": x, "w": wt, "b": b, "res": res}))
    for op in ("nnc_gemm_relu", "nnc_gemm_nt_relu"):
        name = f"{op}_seeded"
        r = rng_for(name)
        a = r.standard_normal((150, 64)).astype(np.float32)
        b = r.standard_normal((90, 64)).astype(np.float32)
        c = r.standard_normal((90,)).astype(np.float32)
        tail = [_f(1.0), _f(1.0)] + ([_i(0), _i(1)] if op == "nnc_gemm_relu" else [])
        out.append(({"name": name, "op": op, "tol": "tc",
                     "args": [_t("a"), _t("b"), _t("c"), _o("out", (150, 90))] + tail}, {"a": a, "b": b, "c": c}))
    for tag, sa, sb in (("2d", (300, 96), (96, 264)), ("batched", (3, 128, 256), (256, 72)),
                        ("small", (5, 12), (12, 7))):
        name = f"nnc_matmul_bias_{tag}"
        r = rng_for(name)
        a = r.standard_normal(sa).astype(np.float32)
        b = r.standard_normal(sb).astype(np.float32)
        bias = r.standard_normal((sb[-1],)).astype(np.float32)
        out.append(({"name": name, "op": "nnc_matmul_bias", "tol": "tc",
                     "args": [_t("a"), _t("b"), _t("bias"), _o("out", sa[:-1] + sb[-1:])]},
                    {"a": a, "b": b, "bias": bias}))
    # Scaled attention scores with a row softmax: rows of 128 (fused into the
    # GEMM epilogue), of 72 (a partial tile), of 200 (longer than a tile: the
    # contraction, then the softmax kernel) and a tiny case (SIMT contraction).
    for tag, sa, sb, alpha in (("heads", (2, 4, 128, 64), (2, 4, 64, 128), 0.125),
                               ("ragged", (3, 100, 40), (3, 40, 72), 0.5),
                               ("long", (2, 130, 64), (2, 64, 200), 0.25),
                               ("small", (6, 8), (8, 5), 2.0)):
        name = f"nnc_matmul_scale_softmax_{tag}"
        r = rng_for(name)
        a = r.standard_normal(sa).astype(np.float32)
        b = r.standard_normal(sb).astype(np.float32)
        out.append(({"name": name, "op": "nnc_matmul_scale_softmax", "tol": "tc",
                     "args": [_t("a"), _t("b"), _o("out", sa[:-1] + sb[-1:]), _f(alpha)]}, {"a": a, "b": b}))
    name = "nnc_matmul_relu_seeded"
    r = rng_for(name)
    a = r.standard_normal((128, 48)).astype(np.float32)
    b = r.standard_normal((48, 40)).astype(np.float32)
    bias = r.standard_normal((40,)).astype(np.float32)
    out.append(({"name": name, "op": "nnc_matmul_relu", "tol": "tc",
                 "args": [_t("a"), _t("b"), _t("bias"), _o("out", (128, 40))]}, {"a": a, "b": b, "bias": bias}))
    return out

"""GPU parity: every golden case through libnnc_cuda.so (device buffers,
C-ABI), against the committed fixtures; tensor-core cases in both precision
modes; the NHWC-tagged and prepacked-weight paths; host-side validation."""

import ctypes

import numpy as np
import pytest

import golden_cases as G
import opcases as C
from nnc_cuda import lib as L

pytestmark = pytest.mark.gpu

CONV_OPS = {"nnc_conv", "nnc_conv_relu", "nnc_conv_sigmoid", "nnc_conv1x1", "nnc_conv_relu1x1", "nnc_conv3x3_s1",
            "nnc_conv_relu3x3_s1", "nnc_conv7x7_s2", "nnc_conv_relu7x7_s2", "nnc_conv_add_relu",
            "nnc_conv_add_relu1x1", "nnc_conv_add_relu3x3_s1"}
POOL_OPS = {"nnc_maxpool2d", "nnc_avgpool2d"}


def _tol(case, precision):
    return C.TC_RTOL[precision] if case["tol"] == "tc" else case["tol"]


def _check(case, got, precision, what=""):
    want = G.outputs(case)
    assert set(got) == set(want)
    for k in want:
        C.assert_close(got[k], want[k], _tol(case, precision), f"{case['name']}{what}:{k}")


@pytest.mark.parametrize("name", G.names())
def test_golden_case(cuda_lib, name):
    case = G.by_name(name)
    precisions = (0, 1) if case["tol"] == "tc" else (0,)
    for p in precisions:
        cuda_lib.nnc_cuda_set_precision(p)
        got = C.run_cuda(cuda_lib, case, G.inputs(case))
        _check(case, got, p, f"[prec{p}]")


def _nhwc_names(case):
    names = set()
    for a in case["args"]:
        if a["k"] in ("t", "o") and a["n"] in ("x", "out", "res", "input_data"):
            names.add(a["n"])
    return names


@pytest.mark.parametrize("name", [c["name"] for c in G.cases() if c["op"] in CONV_OPS | POOL_OPS])
def test_golden_case_nhwc_tagged(cuda_lib, name):
    """Activations passed channels-last with NNC_CUDA_TAG_NHWC (the layout the
    cuda codegen target keeps in its arena) give the same results."""
    case = G.by_name(name)
    ins = G.inputs(case)
    nhwc = {n for n in _nhwc_names(case) if n == "out" or (n in ins and ins[n].ndim == 4)}
    for p in ((0, 1) if case["tol"] == "tc" else (0,)):
        cuda_lib.nnc_cuda_set_precision(p)
        got = C.run_cuda(cuda_lib, case, ins, nhwc=nhwc)
        _check(case, got, p, f"[nhwc,prec{p}]")


@pytest.mark.parametrize("name", [c["name"] for c in G.cases() if c["op"] in CONV_OPS])
def test_conv_prepacked_weight(cuda_lib, name):
    """A weight re-laid out once by nnc_cuda_prepack_conv_weight (as the cuda
    target's constant loader does) gives the same results as raw OIHW."""
    import torch

    from nnc_cuda import tensor as T

    case = G.by_name(name)
    ins = G.inputs(case)
    wname = next(a["n"] for a in case["args"][1:2])
    w = torch.from_numpy(ins[wname]).cuda()
    wref = T.from_torch(w)
    nbytes = cuda_lib.nnc_cuda_prepacked_conv_weight_bytes(wref.ptr)
    packed = torch.empty(nbytes // 4, dtype=torch.float32, device="cuda")
    assert cuda_lib.nnc_cuda_prepack_conv_weight(wref.ptr, ctypes.c_void_p(packed.data_ptr()), nbytes) == 0
    assert wref.struct.dtype & L.TAG_PACKED_CONV
    for p in (0, 1):
        cuda_lib.nnc_cuda_set_precision(p)
        got = _run_with_weight(cuda_lib, case, ins, wname, wref)
        _check(case, got, p, f"[packed,prec{p}]")


def _run_with_weight(so, case, ins, wname, wref):
    """run_cuda with the weight argument replaced by a prepared descriptor."""
    import torch

    from nnc_cuda import tensor as T

    keep, cargs, outs = [], [], {}
    for a in case["args"]:
        if a["k"] == "t" and a["n"] == wname:
            cargs.append(wref.ptr)
        elif a["k"] == "t":
            t = torch.from_numpy(ins[a["n"]]).cuda()
            r = T.from_torch(t)
            keep.append(r)
            cargs.append(r.ptr)
        elif a["k"] == "o":
            t = torch.full(a["shape"], C.SENTINEL, dtype=torch.float32, device="cuda")
            outs[a["n"]] = t
            r = T.from_torch(t)
            keep.append(r)
            cargs.append(r.ptr)
        elif a["k"] == "null":
            cargs.append(None)
        elif a["k"] == "i":
            cargs.append(ctypes.c_int(a["v"]))
        elif a["k"] == "f":
            cargs.append(ctypes.c_float(a["v"]))
    so.nnc_cuda_set_stream(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    getattr(so, case["op"])(*cargs)
    torch.cuda.synchronize()
    assert so.nnc_cuda_get_last_error() == 0, so.nnc_cuda_get_last_error_string()
    return {k: v.cpu().numpy() for k, v in outs.items()}


# ---------------------------------------------------------------- bigger --
def _oracle():
    from oracle import oracle as O

    return O.load_oracle()


@pytest.mark.parametrize("prec", [0, 1])
@pytest.mark.parametrize("shape", [(512, 512, 512), (1000, 384, 256), (256, 1000, 512), (300, 700, 124)])
def test_gemm_nt_sizes_vs_oracle(cuda_lib, prec, shape):
    M, N, K = shape
    r = np.random.default_rng(M * 7 + N)
    arrays = {"a": r.standard_normal((M, K)).astype(np.float32), "b": r.standard_normal((N, K)).astype(np.float32),
              "c": r.standard_normal((N,)).astype(np.float32)}
    case = {"name": "g", "op": "nnc_gemm_nt", "args": [C._t("a"), C._t("b"), C._t("c"), C._o("out", (M, N)),
                                                       C._f(1.0), C._f(1.0)]}
    cuda_lib.nnc_cuda_set_precision(prec)
    got = C.run_cuda(cuda_lib, case, arrays)["out"]
    want = C.run_host(_oracle(), case, arrays)["out"]
    C.assert_close(got, want, C.TC_RTOL[prec], f"gemm_nt{shape}")


# [K, N] B operands read MN-major by the tensor-core kernel (N % 4 == 0), the
# transposed fallback (N % 4 != 0), ragged M/N/K tile edges, the reference's
# overlapping batch offsets, and the TMA-store epilogue with bias / C / alpha.
MATMUL_CASES = [
    ("mm", (300, 200), (200, 132)), ("mm", (257, 36), (36, 260)), ("mm", (128, 256), (256, 1024)),
    ("mm", (130, 1000), (1000, 36)), ("mm", (200, 64), (64, 130)), ("mm", (96, 40), (40, 4096)),
    ("mm", (4, 2, 128, 64), (4, 2, 64, 128)), ("mm", (4, 2, 128, 128), (4, 2, 128, 64)),
    ("mm", (8, 128, 256), (256, 256)), ("mm", (3, 100, 48), (3, 48, 72)),
    ("gemm00", (300, 100), (100, 200)), ("gemm10", (64, 200), (64, 132)), ("gemm01", (150, 96), (260, 96)),
]


@pytest.mark.parametrize("prec", [0, 1])
@pytest.mark.parametrize("cfg", MATMUL_CASES)
def test_matmul_layouts_vs_oracle(cuda_lib, prec, cfg):
    kind, sa, sb = cfg
    r = np.random.default_rng(sum(sa) * 31 + sum(sb))
    arrays = {"a": r.standard_normal(sa).astype(np.float32), "b": r.standard_normal(sb).astype(np.float32)}
    if kind == "mm":
        nd = max(len(sa), len(sb))
        lead = (sa if len(sa) == nd else sb)[:-2]
        so = tuple(lead) + (sa[-2], sb[-1])
        case = {"name": "m", "op": "nnc_matmul", "args": [C._t("a"), C._t("b"), C._o("out", so)]}
    else:
        ta, tb = int(kind[4]), int(kind[5])
        M = sa[1] if ta else sa[0]
        N = sb[0] if tb else sb[1]
        arrays["c"] = r.standard_normal((M, N)).astype(np.float32)
        case = {"name": "g", "op": "nnc_gemm", "args": [C._t("a"), C._t("b"), C._t("c"), C._o("out", (M, N)),
                                                        C._f(0.75), C._f(-1.25), C._i(ta), C._i(tb)]}
    cuda_lib.nnc_cuda_set_precision(prec)
    got = C.run_cuda(cuda_lib, case, arrays)["out"]
    want = C.run_host(_oracle(), case, arrays)["out"]
    C.assert_close(got, want, C.TC_RTOL[prec], f"{kind}{sa}x{sb}")


# Large TF32 problems: the CTA-pair GEMM kernel (N > 128, M >= 256, at least
# ~64 tiles of 256 x 256) with [K, N] B read MN-major and [N, K] B K-major,
# the reference's batch offsets, ragged M / N / K, C matrix with alpha /
# beta, relu; then many-tile short-K problems.
PAIR_GEMM_CASES = [
    ("mm", (2048, 128), (128, 2048)), ("mm", (64, 256, 96), (64, 96, 264)),
    ("gemm01", (4100, 36), (1032, 36)), ("gemm00_relu", (1300, 64), (64, 3000)),
    # Short K against one B over many tiles (single-CTA kernel): batched A
    # with a shared [K, N] B, and a K-major B with a ragged k-block and a row
    # bias.
    ("mm", (300, 128, 64), (64, 136)), ("gemmnt_bias", (19000, 100), (260, 100)),
    # Batches of at most 128 rows against one B on CTA pairs, one batch per
    # CTA (the reference's overlapping batch offsets; ragged M and N).
    ("mm", (132, 100, 64), (64, 264)), ("mm", (128, 128, 32), (32, 384)),
    # An odd batch count on that route: the last pair's second CTA has no
    # batch (its A tile reads as zeros through the tensor map's bounds and
    # its store is skipped); also with a row bias and relu in the epilogue.
    ("mm", (131, 100, 64), (64, 264)), ("mmrelu_bias", (129, 128, 32), (32, 384)),
]


@pytest.mark.parametrize("cfg", PAIR_GEMM_CASES, ids=lambda c: c[0] + "x".join(map(str, c[1] + c[2])))
def test_gemm_cta_pairs_vs_oracle(cuda_lib, cfg):
    kind, sa, sb = cfg
    r = np.random.default_rng(sum(sa) * 7 + sum(sb))
    arrays = {"a": r.standard_normal(sa).astype(np.float32), "b": r.standard_normal(sb).astype(np.float32)}
    if kind == "mm":
        so = sa[:-1] + sb[-1:]
        case = {"name": "m", "op": "nnc_matmul", "args": [C._t("a"), C._t("b"), C._o("out", so)]}
    elif kind == "mmrelu_bias":
        so = sa[:-1] + sb[-1:]
        arrays["bias"] = r.standard_normal((sb[-1],)).astype(np.float32)
        case = {"name": "m", "op": "nnc_matmul_relu", "args": [C._t("a"), C._t("b"), C._t("bias"), C._o("out", so)]}
    elif kind == "gemmnt_bias":
        M, N = sa[0], sb[0]
        arrays["c"] = r.standard_normal((N,)).astype(np.float32)
        case = {"name": "g", "op": "nnc_gemm_nt", "args": [C._t("a"), C._t("b"), C._t("c"), C._o("out", (M, N)),
                                                           C._f(1.0), C._f(1.0)]}
    else:
        tb = int(kind[5])
        M, N = sa[0], (sb[0] if tb else sb[1])
        arrays["c"] = r.standard_normal((M, N)).astype(np.float32)
        op = "nnc_gemm_relu" if kind.endswith("relu") else "nnc_gemm"
        case = {"name": "g", "op": op, "args": [C._t("a"), C._t("b"), C._t("c"), C._o("out", (M, N)),
                                                C._f(0.75), C._f(-1.25), C._i(0), C._i(tb)]}
    cuda_lib.nnc_cuda_set_precision(0)
    got = C.run_cuda(cuda_lib, case, arrays)["out"]
    want = C.run_host(_oracle(), case, arrays)["out"]
    C.assert_close(got, want, C.TC_RTOL[0], f"{kind}{sa}x{sb}")


@pytest.mark.parametrize("prec", [0, 1])
@pytest.mark.parametrize("cfg", [(4, 64, 28, 64, 3, 1, 1), (2, 128, 14, 256, 3, 2, 1), (2, 256, 7, 512, 3, 1, 1),
                                 (2, 3, 56, 64, 7, 2, 3), (2, 64, 28, 128, 1, 2, 0)])
def test_conv_resnet_layers_vs_oracle(cuda_lib, prec, cfg):
    n, c, h, co, k, s, p = cfg
    r = np.random.default_rng(sum(cfg))
    oh = C.conv_out(h, k, s, p)
    arrays = {"x": r.standard_normal((n, c, h, h)).astype(np.float32),
              "w": (r.standard_normal((co, c, k, k)) * np.sqrt(2.0 / (c * k * k))).astype(np.float32),
              "b": r.uniform(-0.01, 0.01, co).astype(np.float32),
              "res": r.standard_normal((n, co, oh, oh)).astype(np.float32)}
    case = {"name": "c", "op": "nnc_conv_add_relu", "args": [C._t("x"), C._t("w"), C._t("b"), C._t("res"),
            C._o("out", (n, co, oh, oh)), C._i(k), C._i(k), C._i(s), C._i(s), C._i(p), C._i(p)]}
    cuda_lib.nnc_cuda_set_precision(prec)
    want = C.run_host(_oracle(), case, arrays)["out"]
    got = C.run_cuda(cuda_lib, case, arrays)["out"]
    C.assert_close(got, want, C.TC_RTOL[prec], f"conv{cfg}")
    got_nhwc = C.run_cuda(cuda_lib, case, arrays, nhwc={"x", "res", "out"})["out"]
    C.assert_close(got_nhwc, want, C.TC_RTOL[prec], f"conv{cfg}[nhwc]")


# Stride-1 windows (and 1 x 1 windows with stride 2) over 32-channel blocks
# take the halo-tile kernel in TF32 mode (the im2col kernel in 3xTF32 mode):
# ragged output blocks, partial C_out tiles (48, 200), C_out not a multiple of
# 4 (scalar epilogue), three channel blocks, a 4 x 4 window, 1 x 1 windows.
# Tiles run on CTA pairs, neighbouring tiles side by side; an odd tile count
# (5 tiles of 24 x 40, 49 x 3 of the stride-2 case) leaves the last pair's
# second CTA a stand-in tile that is computed and not stored.
HALO_CASES = [
    # n, c, h, w, co, k, p, op
    (2, 32, 30, 30, 48, 3, 1, "nnc_conv_add_relu"),
    (1, 96, 24, 40, 64, 3, 1, "nnc_conv_add_relu"),
    (2, 64, 32, 32, 200, 3, 1, "nnc_conv_add_relu"),
    (1, 32, 30, 30, 64, 4, 2, "nnc_conv_add_relu"),
    (2, 96, 28, 28, 128, 1, 0, "nnc_conv_relu"),
    (2, 32, 30, 30, 30, 3, 1, "nnc_conv"),
    (2, 64, 56, 56, 128, 1, 0, "nnc_conv"),  # the ResNet stage-2 projection, stride 2
    (1, 128, 56, 56, 256, 1, 0, "nnc_conv_add_relu"),  # stride 2, two 128-channel tiles
    (2, 32, 20, 20, 64, 1, 0, "nnc_conv_relu"),  # 1 x 1 over 32 channels (chunk order)
    (3, 64, 56, 56, 64, 1, 0, "nnc_conv_add_relu"),  # stride 2, 64 channels: strided windows
]


@pytest.mark.parametrize("prec", [0, 1])
@pytest.mark.parametrize("cfg", HALO_CASES, ids=lambda c: "x".join(str(v) for v in c[:7]))
def test_conv_stride1_blocks_vs_oracle(cuda_lib, prec, cfg):
    n, c, h, w, co, k, p, op = cfg
    st = 2 if (k == 1 and h == 56) else 1
    r = np.random.default_rng(7 + sum(cfg[:7]))
    oh, ow = C.conv_out(h, k, st, p), C.conv_out(w, k, st, p)
    arrays = {"x": r.standard_normal((n, c, h, w)).astype(np.float32),
              "w": (r.standard_normal((co, c, k, k)) * np.sqrt(2.0 / (c * k * k))).astype(np.float32),
              "b": r.uniform(-0.01, 0.01, co).astype(np.float32),
              "res": r.standard_normal((n, co, oh, ow)).astype(np.float32)}
    args = [C._t("x"), C._t("w"), C._t("b")]
    nhwc = {"x", "out"}
    if op == "nnc_conv_add_relu":
        args.append(C._t("res"))
        nhwc.add("res")
    args += [C._o("out", (n, co, oh, ow)), C._i(k), C._i(k), C._i(sh), C._i(sw), C._i(p), C._i(p)]
    case = {"name": "c", "op": op, "args": args}
    cuda_lib.nnc_cuda_set_precision(prec)
    want = C.run_host(_oracle(), case, arrays)["out"]
    got = C.run_cuda(cuda_lib, case, arrays)["out"]
    C.assert_close(got, want, C.TC_RTOL[prec], f"conv{cfg}")
    got_nhwc = C.run_cuda(cuda_lib, case, arrays, nhwc=nhwc)["out"]
    C.assert_close(got_nhwc, want, C.TC_RTOL[prec], f"conv{cfg}[nhwc]")


# C_out above 64 over 32-channel NHWC inputs runs on CTA pairs in TF32 mode
# (one 256-pixel x 256- or 128-channel tile per pair, the odd CTA holding the
# upper 128 pixels and half of the weight rows): tiles whose upper half is partly or wholly past
# the last pixel (196, 49 and 784 pixels), partial channel tiles (384, 200 —
# the latter not a multiple of 32), stride 2, and 98 tiles for fewer pairs,
# so pairs run several tiles through both accumulators.
PAIR_CASES = [
    # n, c, h, w, co, k, s, p, op
    (4, 256, 14, 14, 256, 3, 1, 1, "nnc_conv_add_relu"),
    (1, 128, 14, 14, 256, 3, 1, 1, "nnc_conv_relu"),
    (1, 256, 7, 7, 512, 3, 1, 1, "nnc_conv"),
    (3, 128, 28, 28, 256, 3, 2, 1, "nnc_conv_relu"),
    (2, 64, 16, 16, 384, 3, 1, 1, "nnc_conv_add_relu"),
    (2, 160, 10, 12, 200, 3, 1, 1, "nnc_conv"),
    (64, 32, 14, 14, 512, 3, 1, 1, "nnc_conv_add_relu"),
    # C_out in (64, 128]: 128-channel pair tiles (the ResNet stage-2
    # stride-2 conv; a 100-channel tile past a 20-row image's halo limit).
    (2, 64, 56, 56, 128, 3, 2, 1, "nnc_conv_relu"),
    (1, 96, 20, 20, 100, 3, 1, 1, "nnc_conv_add_relu"),
]



# Stream-K on CTA pairs (TF32, stride 1): whole tiles would fill the last
# wave of the 74 resident pairs under 90%, so tiles are split along K between
# pairs and the pair that ends a tile adds the others' partial sums. For 74
# pairs: 8 tiles of 144 k-blocks (15-16 per pair, each tile over ~10 pairs;
# the last tile's upper half past the last pixel; residual and relu); 49
# tiles of 36 (128-channel tiles); 8 tiles with C_out 200 (the staged
# epilogue); 150 tiles of 16, the first 74 whole and the other 76 split.
STREAMK_CASES = [
    # n, c, h, w, co, k, s, p, op
    (16, 512, 7, 7, 512, 3, 1, 1, "nnc_conv_add_relu"),
    (64, 128, 14, 14, 128, 3, 1, 1, "nnc_conv_relu"),
    (16, 512, 10, 12, 200, 3, 1, 1, "nnc_conv"),
    (1200, 512, 4, 4, 512, 1, 1, 0, "nnc_conv_add_relu"),
]


# Reshape -> Transpose and Transpose -> Reshape as one call (the
# transformer's head split and merge at -O3): bit-exact against the oracle's
# composition of the reference's reshape and transpose; NULL in_shape, a
# reversed (NULL) perm, float4 and scalar paths.
SHAPED_TRANSPOSE_CASES = [
    # input shape, in_shape (None: own), perm (None: reverse)
    ((2, 128, 256), (2, 128, 4, 64), (0, 2, 1, 3)),
    ((2, 128, 256), (2, 128, 4, 64), (0, 2, 3, 1)),
    ((2, 4, 128, 64), None, (0, 2, 1, 3)),
    ((3, 5, 7), (5, 3, 7), None),
    ((6, 10), (2, 3, 10), (2, 0, 1)),
]


@pytest.mark.parametrize("cfg", SHAPED_TRANSPOSE_CASES, ids=lambda c: str(c).replace(" ", ""))
def test_transpose_shaped_vs_oracle(cuda_lib, cfg):
    shape, in_shape, perm = cfg
    r = np.random.default_rng(41 + sum(shape))
    arrays = {"x": r.standard_normal(shape).astype(np.float32)}
    ish = in_shape or shape
    nd = len(ish)
    pm = perm or tuple(reversed(range(nd)))
    n = int(np.prod(shape))
    args = [C._t("x"), C._o("out", (n,)), {"k": "perm", "v": list(ish) if in_shape else None},
            {"k": "perm", "v": list(pm) if perm else None}, C._i(nd)]
    case = {"name": "t", "op": "nnc_transpose_shaped", "args": args, "tol": "exact"}
    want = C.run_host(_oracle(), case, arrays)["out"]
    got = C.run_cuda(cuda_lib, case, arrays)["out"]
    C.assert_close(got, want, "exact", f"transpose_shaped{cfg}")
    np.testing.assert_array_equal(got.reshape(-1), np.transpose(arrays["x"].reshape(ish), pm).reshape(-1))


# Add -> LayerNorm as one call (the transformer's post-LN residual joins):
# the warp kernel (256 and 100 values per slab), the four-warps-per-slab
# kernel (768), and a long slab (4096: the sum into the output, then the
# normalisation in place), against the oracle's composition of the
# reference's add and layernorm.
ADD_LN_CASES = [
    # shape, axis
    ((64, 128, 256), -1),
    ((37, 100), -1),
    ((50, 768), -1),
    ((9, 4096), -1),
    ((4, 6, 8, 8), 1),
]


@pytest.mark.parametrize("cfg", ADD_LN_CASES, ids=lambda c: "x".join(map(str, c[0])) + f"a{c[1]}")
def test_add_layernorm_vs_oracle(cuda_lib, cfg):
    shape, axis = cfg
    r = np.random.default_rng(53 + sum(shape))
    ax = axis % len(shape)
    norm = int(np.prod(shape[ax:]))
    arrays = {"a": r.standard_normal(shape).astype(np.float32), "b": r.standard_normal(shape).astype(np.float32),
              "g": r.uniform(0.5, 1.5, norm).astype(np.float32), "bt": r.uniform(-0.1, 0.1, norm).astype(np.float32)}
    args = [C._t("a"), C._t("b"), C._t("g"), C._t("bt"), C._o("out", shape), C._i(axis), C._f(1e-5)]
    case = {"name": "aln", "op": "nnc_add_layernorm", "args": args}
    want = C.run_host(_oracle(), case, arrays)["out"]
    got = C.run_cuda(cuda_lib, case, arrays)["out"]
    C.assert_close(got, want, 1e-5, f"add_layernorm{cfg}")
    # The same as the library's own add then layernorm.
    s = {"name": "s", "op": "nnc_add", "args": [C._t("a"), C._t("b"), C._o("out", shape)]}
    arrays["s"] = C.run_cuda(cuda_lib, s, arrays)["out"]
    ln = {"name": "ln", "op": "nnc_layernorm",
          "args": [C._t("s"), C._t("g"), C._t("bt"), C._o("out", shape), C._i(axis), C._f(1e-5)]}
    np.testing.assert_array_equal(got, C.run_cuda(cuda_lib, ln, arrays)["out"])


# The GlobalAveragePool -> Flatten -> Gemm head as one call (the ResNet
# classifier; odd extents, no bias, a [N, O] bias with alpha/beta), both
# precisions, NCHW and channels-last inputs, against the oracle's composition
# of the reference's avgpool, flatten and gemm_nt.
GAP_GEMM_CASES = [
    # n, c, h, w, o, bias
    (8, 512, 7, 7, 1000, "row"),
    (3, 96, 5, 3, 33, None),
    (130, 64, 2, 2, 257, "full"),
]


@pytest.mark.parametrize("prec", [0, 1])
@pytest.mark.parametrize("cfg", GAP_GEMM_CASES, ids=lambda c: "x".join(str(v) for v in c))
def test_gap_gemm_nt_vs_oracle(cuda_lib, prec, cfg):
    n, c, h, w, o, bias = cfg
    r = np.random.default_rng(29 + n + c + o)
    arrays = {"x": r.standard_normal((n, c, h, w)).astype(np.float32),
              "b": (r.standard_normal((o, c)) * 0.05).astype(np.float32)}
    args = [C._t("x"), C._t("b")]
    if bias == "row":
        arrays["c"] = r.uniform(-0.01, 0.01, o).astype(np.float32)
        args.append(C._t("c"))
    elif bias == "full":
        arrays["c"] = r.standard_normal((n, o)).astype(np.float32)
        args.append(C._t("c"))
    else:
        args.append({"k": "null"})
    alpha, beta = (1.0, 1.0) if bias != "full" else (0.5, -2.0)
    args += [C._o("out", (n, o)), C._f(alpha), C._f(beta)]
    case = {"name": "g", "op": "nnc_gap_gemm_nt", "args": args}
    cuda_lib.nnc_cuda_set_precision(prec)
    want = C.run_host(_oracle(), case, arrays)["out"]
    for nhwc in (set(), {"x"}):
        got = C.run_cuda(cuda_lib, case, arrays, nhwc=nhwc)["out"]
        C.assert_close(got, want, C.TC_RTOL[prec], f"gap_gemm_nt{cfg}{sorted(nhwc)}")


# Stride-2 3 x 3 windows over 32-channel blocks (the CTA-pair im2col route in
# TF32 mode): the ResNet stage-2 shape, pad 1 and pad 0, a ragged 25 x 31
# output with three channel blocks and C_out 100 (staged epilogue), two
# 128-channel tiles.
S2_CASES_3X3 = [
    # n, c, h, w, co, k, s, p, op
    (2, 64, 56, 56, 128, 3, 2, 1, "nnc_conv_relu"),
    (2, 64, 57, 57, 64, 3, 2, 0, "nnc_conv"),
    (1, 96, 50, 62, 100, 3, 2, 1, "nnc_conv_add_relu"),
    (1, 64, 64, 64, 256, 3, 2, 1, "nnc_conv_add_relu"),
]


@pytest.mark.parametrize("prec", [0, 1])
@pytest.mark.parametrize("cfg", S2_CASES_3X3, ids=lambda c: "x".join(str(v) for v in c[:8]))
def test_conv_stride2_3x3_vs_oracle(cuda_lib, prec, cfg):
    test_conv_cta_pairs_vs_oracle(cuda_lib, prec, cfg)


@pytest.mark.parametrize("cfg", STREAMK_CASES, ids=lambda c: "x".join(str(v) for v in c[:8]))
def test_conv_stream_k_vs_oracle(cuda_lib, cfg):
    test_conv_cta_pairs_vs_oracle(cuda_lib, 0, cfg, repeat=3)
    assert cuda_lib.nnc_cuda_check_device_status() == 0  # no bounded wait expired


@pytest.mark.parametrize("prec", [0, 1])
@pytest.mark.parametrize("cfg", PAIR_CASES, ids=lambda c: "x".join(str(v) for v in c[:8]))
def test_conv_cta_pairs_vs_oracle(cuda_lib, prec, cfg, repeat=1):
    n, c, h, w, co, k, st, p, op = cfg
    r = np.random.default_rng(13 + sum(cfg[:8]))
    oh, ow = C.conv_out(h, k, st, p), C.conv_out(w, k, st, p)
    arrays = {"x": r.standard_normal((n, c, h, w)).astype(np.float32),
              "w": (r.standard_normal((co, c, k, k)) * np.sqrt(2.0 / (c * k * k))).astype(np.float32),
              "b": r.uniform(-0.01, 0.01, co).astype(np.float32),
              "res": r.standard_normal((n, co, oh, ow)).astype(np.float32)}
    args = [C._t("x"), C._t("w"), C._t("b")]
    nhwc = {"x", "out"}
    if op == "nnc_conv_add_relu":
        args.append(C._t("res"))
        nhwc.add("res")
    args += [C._o("out", (n, co, oh, ow)), C._i(k), C._i(k), C._i(st), C._i(st), C._i(p), C._i(p)]
    case = {"name": "c", "op": op, "args": args}
    cuda_lib.nnc_cuda_set_precision(prec)
    want = C.run_host(_oracle(), case, arrays)["out"]
    got_nhwc = C.run_cuda(cuda_lib, case, arrays, nhwc=nhwc)["out"]
    C.assert_close(got_nhwc, want, C.TC_RTOL[prec], f"conv{cfg}[nhwc]")
    # Later calls reuse whatever earlier calls left behind (stream-K's
    # counters return to zero after every launch): same result each time.
    for _ in range(repeat - 1):
        again = C.run_cuda(cuda_lib, case, arrays, nhwc=nhwc)["out"]
        np.testing.assert_array_equal(again, got_nhwc)
    got = C.run_cuda(cuda_lib, case, arrays)["out"]
    C.assert_close(got, want, C.TC_RTOL[prec], f"conv{cfg}")


# Stride-2 windows over at most 8 channels run as stride-1 windows over a
# space-to-depth copy of the input (TF32 mode): 7x7 p3 (the ResNet stem), odd
# extents, one channel, a 3x3 window whose prepacked weight is in element
# order, 8 channels, a 1x1 window; raw and prepacked weights, NCHW and NHWC.
S2D_CASES = [
    # n, c, h, w, co, k, p, op
    (2, 3, 64, 64, 64, 7, 3, "nnc_conv_relu"),
    (1, 3, 61, 63, 48, 7, 3, "nnc_conv_add_relu"),
    (2, 1, 64, 64, 32, 5, 2, "nnc_conv"),
    (2, 3, 64, 63, 64, 3, 1, "nnc_conv_add_relu"),
    (1, 8, 64, 64, 96, 3, 1, "nnc_conv_relu"),
    (2, 4, 64, 64, 64, 1, 0, "nnc_conv"),
    (1, 3, 30, 30, 64, 7, 3, "nnc_conv_relu"),  # 15 x 15 output: the general path
]


@pytest.mark.parametrize("prec", [0, 1])
@pytest.mark.parametrize("cfg", S2D_CASES, ids=lambda c: "x".join(str(v) for v in c[:7]))
def test_conv_stride2_few_channels_vs_oracle(cuda_lib, prec, cfg):
    import torch

    from nnc_cuda import tensor as T

    n, c, h, w, co, k, p, op = cfg
    r = np.random.default_rng(11 + sum(cfg[:7]))
    oh, ow = C.conv_out(h, k, 2, p), C.conv_out(w, k, 2, p)
    arrays = {"x": r.standard_normal((n, c, h, w)).astype(np.float32),
              "w": (r.standard_normal((co, c, k, k)) * np.sqrt(2.0 / (c * k * k))).astype(np.float32),
              "b": r.uniform(-0.01, 0.01, co).astype(np.float32),
              "res": r.standard_normal((n, co, oh, ow)).astype(np.float32)}
    args = [C._t("x"), C._t("w"), C._t("b")]
    nhwc = {"x", "out"}
    if op == "nnc_conv_add_relu":
        args.append(C._t("res"))
        nhwc.add("res")
    args += [C._o("out", (n, co, oh, ow)), C._i(k), C._i(k), C._i(2), C._i(2), C._i(p), C._i(p)]
    case = {"name": "c", "op": op, "args": args}
    cuda_lib.nnc_cuda_set_precision(prec)
    want = C.run_host(_oracle(), case, arrays)["out"]
    got = C.run_cuda(cuda_lib, case, arrays)["out"]
    C.assert_close(got, want, C.TC_RTOL[prec], f"conv{cfg}")
    got_nhwc = C.run_cuda(cuda_lib, case, arrays, nhwc=nhwc)["out"]
    C.assert_close(got_nhwc, want, C.TC_RTOL[prec], f"conv{cfg}[nhwc]")
    # Prepacked weight (the cuda target's constants), NCHW tensors.
    wt = torch.from_numpy(arrays["w"]).cuda()
    wref = T.from_torch(wt)
    nbytes = cuda_lib.nnc_cuda_prepacked_conv_weight_bytes(wref.ptr)
    packed = torch.empty(nbytes // 4, dtype=torch.float32, device="cuda")
    assert cuda_lib.nnc_cuda_prepack_conv_weight(wref.ptr, ctypes.c_void_p(packed.data_ptr()), nbytes) == 0
    got_p = _run_with_weight(cuda_lib, case, arrays, "w", wref)["out"]
    C.assert_close(got_p, want, C.TC_RTOL[prec], f"conv{cfg}[prepacked]")


# relu(conv) then max pooling in one call: the fused space-to-depth halo
# kernel with a pooled epilogue for stem-like shapes and a channels-last
# output (ragged extents, a 2x2 pool, C_out 48), and the conv + pool
# composition otherwise (NCHW output, 3xTF32, 8 input channels, stride 1).
POOL_CASES = [
    # n, c, h, w, co, k, s, p, (pool k, stride, pad)
    (2, 3, 224, 224, 64, 7, 2, 3, (3, 2, 1)),
    (1, 3, 62, 58, 64, 7, 2, 3, (3, 2, 1)),
    (2, 3, 64, 64, 48, 7, 2, 3, (2, 2, 0)),
    (2, 8, 40, 40, 64, 3, 2, 1, (3, 2, 1)),
    (2, 16, 20, 20, 32, 3, 1, 1, (3, 2, 1)),
    # 2x2 windows with a top/left pad: centres inside (fused), and a last
    # centre past the conv result (the conv + pool composition).
    (1, 3, 62, 62, 64, 7, 2, 3, (2, 2, 1)),
    (1, 3, 64, 64, 64, 7, 2, 3, (2, 2, 1)),
    # More images than SMs: CTAs walk several images (carries reset at each).
    (150, 3, 56, 56, 64, 7, 2, 3, (3, 2, 1)),
    # An odd image count (the pooled epilogue runs on single CTAs).
    (3, 3, 64, 64, 64, 7, 2, 3, (3, 2, 1)),
]


@pytest.mark.parametrize("prec", [0, 1])
@pytest.mark.parametrize("cfg", POOL_CASES, ids=lambda c: "x".join(str(v) for v in c[:8]))
def test_conv_relu_maxpool_vs_oracle(cuda_lib, prec, cfg):
    n, c, h, w, co, k, st, p, (pk, ps, pp) = cfg
    r = np.random.default_rng(5 + sum(cfg[:8]))
    oh, ow = C.conv_out(h, k, st, p), C.conv_out(w, k, st, p)
    ph, pw = C.conv_out(oh, pk, ps, pp), C.conv_out(ow, pk, ps, pp)
    arrays = {"x": r.standard_normal((n, c, h, w)).astype(np.float32),
              "w": (r.standard_normal((co, c, k, k)) * np.sqrt(2.0 / (c * k * k))).astype(np.float32),
              "b": r.uniform(-0.01, 0.01, co).astype(np.float32)}
    args = [C._t("x"), C._t("w"), C._t("b"), C._o("out", (n, co, ph, pw))] + [
        C._i(v) for v in (k, k, st, st, p, p, oh, ow, pk, pk, ps, ps, pp, pp)]
    case = {"name": "c", "op": "nnc_conv_relu_maxpool", "args": args}
    cuda_lib.nnc_cuda_set_precision(prec)
    want = C.run_host(_oracle(), case, arrays)["out"]
    for layout in ((), ("out",), ("x", "out")):
        got = C.run_cuda(cuda_lib, case, arrays, nhwc=set(layout))["out"]
        C.assert_close(got, want, C.TC_RTOL[prec], f"conv_relu_maxpool{cfg}[{layout}]")


# Few output channels over a short reduction (C_out <= 16, C KH KW <= 256)
# run on the direct CUDA-core kernel up to 37,887 output pixels (and at any
# size in 3xTF32 mode): LeNet's two layers, stride 2 with
# padding and a residual, sigmoid, NCHW and channels-last tensors, raw and
# prepacked (element and chunk order) weights, both precision modes. Stride-1
# 3- and 5-wide windows take the row-blocked kernel (4 pixels per thread,
# ragged row ends included), the others the per-pixel one.
DIRECT_CASES = [
    # n, c, h, w, co, k, s, p, op
    (4, 1, 32, 32, 6, 5, 1, 0, "nnc_conv_relu"),
    (4, 6, 14, 14, 16, 5, 1, 0, "nnc_conv"),
    (2, 3, 17, 19, 8, 3, 2, 1, "nnc_conv_add_relu"),
    (2, 12, 11, 9, 13, 3, 1, 2, "nnc_conv_sigmoid"),
    (3, 2, 9, 13, 4, 3, 1, 1, "nnc_conv_add_relu"),
    (2, 4, 12, 7, 10, 5, 1, 2, "nnc_conv_relu"),
    (2, 3, 17, 19, 8, 3, (2, 1), 1, "nnc_conv_relu"),  # row stride 2, column stride 1
]


def _check_direct_conv(cuda_lib, prec, cfg, tol):
    """Runs one few-channel conv case NCHW, channels-last and with prepacked
    weights against the oracle; returns the NCHW result and the oracle's."""
    import torch

    from nnc_cuda import tensor as T

    n, c, h, w, co, k, st, p, op = cfg
    sh, sw = st if isinstance(st, tuple) else (st, st)  # one stride, or (rows, columns)
    r = np.random.default_rng(17 + sum(sum(v) if isinstance(v, tuple) else v for v in cfg[:8]))
    oh, ow = C.conv_out(h, k, sh, p), C.conv_out(w, k, sw, p)
    arrays = {"x": r.standard_normal((n, c, h, w)).astype(np.float32),
              "w": (r.standard_normal((co, c, k, k)) * np.sqrt(2.0 / (c * k * k))).astype(np.float32),
              "b": r.uniform(-0.01, 0.01, co).astype(np.float32),
              "res": r.standard_normal((n, co, oh, ow)).astype(np.float32)}
    args = [C._t("x"), C._t("w"), C._t("b")]
    nhwc = {"x", "out"}
    if op == "nnc_conv_add_relu":
        args.append(C._t("res"))
        nhwc.add("res")
    args += [C._o("out", (n, co, oh, ow)), C._i(k), C._i(k), C._i(sh), C._i(sw), C._i(p), C._i(p)]
    case = {"name": "c", "op": op, "args": args}
    cuda_lib.nnc_cuda_set_precision(prec)
    want = C.run_host(_oracle(), case, arrays)["out"]
    got = C.run_cuda(cuda_lib, case, arrays)["out"]
    C.assert_close(got, want, tol, f"conv{cfg}")
    C.assert_close(C.run_cuda(cuda_lib, case, arrays, nhwc=nhwc)["out"], want, tol, f"conv{cfg}[nhwc]")
    C.assert_close(C.run_cuda(cuda_lib, case, arrays, nhwc={"x"})["out"], want, tol, f"conv{cfg}[nhwc in]")
    # Prepacked weight (element order for K <= 64, chunk order above).
    wt = torch.from_numpy(arrays["w"]).cuda()
    wref = T.from_torch(wt)
    nbytes = cuda_lib.nnc_cuda_prepacked_conv_weight_bytes(wref.ptr)
    packed = torch.empty(nbytes // 4, dtype=torch.float32, device="cuda")
    assert cuda_lib.nnc_cuda_prepack_conv_weight(wref.ptr, ctypes.c_void_p(packed.data_ptr()), nbytes) == 0
    C.assert_close(_run_with_weight(cuda_lib, case, arrays, "w", wref)["out"], want, tol,
                   f"conv{cfg}[prepacked]")
    return got, want


@pytest.mark.parametrize("prec", [0, 1])
@pytest.mark.parametrize("cfg", DIRECT_CASES, ids=lambda c: "x".join(str(v) for v in c[:8]))
def test_conv_direct_small_vs_oracle(cuda_lib, prec, cfg):
    _check_direct_conv(cuda_lib, prec, cfg, 1e-5)  # fp32 FMA accumulation in either precision mode


# The same few-channel convs with at least 37,888 output pixels (two 128-pixel
# tiles per SM) run in TF32 mode on tensor cores (3xTF32 keeps them on the fp32
# CUDA-core kernels), each case NCHW, channels-last, channels-last in with
# NCHW out, and with prepacked weights:
# * the row-banded kernel where the input rows are contiguous (one channel or
#   channels-last) and an output row fits one MMA (OW C_out <= 256): whole
#   images per tile with a partial last tile, vertical padding read as zeros
#   by the tensor map, horizontal padding in the banded weight, input rows of
#   one to six k-blocks, float4 and scalar staging of channels-last outputs,
#   NCHW outputs, a residual;
# * the im2col tile kernel otherwise (reduction <= 160 over <= 32 taps): one,
#   two and five 32-float k-blocks, channel pairs loaded as float2, stride 2,
#   sigmoid.
SMALL_TC_CASES = [
    # n, c, h, w, co, k, s, p, op
    (66, 1, 32, 32, 6, 5, 1, 0, "nnc_conv_relu"),      # LeNet conv1: banded (C = 1), 16.5 tiles of 4 images
    (512, 6, 14, 14, 16, 5, 1, 0, "nnc_conv"),         # LeNet conv2: banded channels-last, im2col NCHW
    (100, 2, 20, 20, 8, 5, 1, 2, "nnc_conv_relu"),     # banded with padding, M = 40,000
    (80, 7, 24, 24, 9, 3, 1, 0, "nnc_conv_add_relu"),  # banded, 6 k-blocks, OW C_out = 198 (scalar staging)
    (160, 3, 33, 31, 8, 3, 2, 1, "nnc_conv_add_relu"),  # im2col, M = 43,520, K = 27
    (48, 5, 30, 30, 13, 5, 1, 2, "nnc_conv_sigmoid"),  # im2col, M = 43,200, K = 125
    (64, 2, 30, 30, 10, 5, 1, 2, "nnc_conv_relu"),     # im2col, M = 57,600, K = 50
    (80, 2, 28, 28, 12, 3, 1, 1, "nnc_conv"),          # im2col, M = 62,720, K = 18
    (66, 1, 32, 64, 6, 5, (1, 2), 0, "nnc_conv_relu"),  # banded, column stride 2, OW C_out = 180
    (160, 3, 31, 33, 8, 3, (2, 1), 1, "nnc_conv_add_relu"),  # im2col, row stride 2, M = 84,480
]


@pytest.mark.parametrize("prec", [0, 1])
@pytest.mark.parametrize("cfg", SMALL_TC_CASES, ids=lambda c: "x".join(str(v) for v in c[:8]))
def test_conv_small_tensor_core_vs_oracle(cuda_lib, prec, cfg):
    got, want = _check_direct_conv(cuda_lib, prec, cfg, C.TC_RTOL[prec])
    if prec == 0:
        # TF32 operands: the result is not the fp32 one, so the tensor-core
        # kernel (not a CUDA-core one) produced it.
        assert not np.allclose(got, want, rtol=0, atol=1e-7)


# Row-op dispatch: one warp per row up to 1024 elements, a block per row with
# the row in shared memory up to 32768, a block re-reading the row beyond;
# LayerNorm slabs over several axes (scale/bias indexed by i / inner) on the
# warp and shared-memory paths. Tolerances as in the seeded cases.
ROW_CASES = [
    ("nnc_softmax", (300, 10), 1), ("nnc_softmax", (64, 1024), 1), ("nnc_softmax", (4, 4096), 1),
    ("nnc_softmax", (2, 40000), 1), ("nnc_layernorm", (8, 1024), -1), ("nnc_layernorm", (5, 2000), -1),
    ("nnc_layernorm", (2, 40000), -1), ("nnc_layernorm", (3, 4, 200), 1), ("nnc_layernorm", (2, 40, 50), 1),
    # 16-byte rows (ragged float4 runs per lane) and scalar rows of the warp kernels
    ("nnc_softmax", (37, 100), 1), ("nnc_softmax", (33, 128), 1), ("nnc_softmax", (16, 260), 1),
    ("nnc_softmax", (9, 250), 1), ("nnc_layernorm", (33, 100), -1), ("nnc_layernorm", (64, 256), -1),
    ("nnc_layernorm", (8, 6, 20), 1), ("nnc_layernorm", (7, 98), -1), ("nnc_layernorm", (5, 1000), -1),
]


@pytest.mark.parametrize("case", ROW_CASES, ids=lambda c: f"{c[0]}_{'x'.join(map(str, c[1]))}")
def test_row_ops_dispatch_vs_oracle(cuda_lib, case):
    op, shape, axis = case
    r = np.random.default_rng(sum(shape) + len(op))
    x = (r.standard_normal(shape) * 2).astype(np.float32)
    arrays = {"x": x}
    if op == "nnc_softmax":
        args, tol = [C._t("x"), C._o("out", shape), C._i(axis)], 2e-6
    else:
        norm = int(np.prod(shape[axis:])) // int(np.prod(shape[axis + 1:])) if axis >= 0 else shape[-1]
        arrays["g"] = r.uniform(0.5, 1.5, norm).astype(np.float32)
        arrays["b"] = r.uniform(-0.1, 0.1, norm).astype(np.float32)
        args, tol = [C._t("x"), C._t("g"), C._t("b"), C._o("out", shape), C._i(axis), C._f(1e-5)], 1e-5
    c = {"name": "row", "op": op, "args": args}
    want = C.run_host(_oracle(), c, arrays)["out"]
    got = C.run_cuda(cuda_lib, c, arrays)["out"]
    C.assert_close(got, want, tol, f"{op}{shape}")


# ------------------------------------------------------------ validation --
def test_invalid_shapes_set_status_without_launch(cuda_lib):
    import torch

    from nnc_cuda import tensor as T

    x = torch.zeros((1, 3, 8, 8), device="cuda")
    w = torch.zeros((4, 5, 3, 3), device="cuda")  # C_in mismatch
    o = torch.zeros((1, 4, 8, 8), device="cuda")
    rx, rw, ro = T.from_torch(x), T.from_torch(w), T.from_torch(o)
    cuda_lib.nnc_conv(rx.ptr, rw.ptr, None, ro.ptr, 3, 3, 1, 1, 1, 1)
    assert cuda_lib.nnc_cuda_get_last_error() == L.ERR_INVALID
    cuda_lib.nnc_cuda_clear_error()
    cuda_lib.nnc_conv3x3_s1(rx.ptr, rw.ptr, None, T.from_torch(torch.zeros((1, 4, 7, 7), device="cuda")).ptr)
    assert cuda_lib.nnc_cuda_get_last_error() == L.ERR_INVALID
    cuda_lib.nnc_cuda_clear_error()
    assert cuda_lib.nnc_cuda_check_device_status() == 0

"""Regenerates tests/golden/{cases.json,golden.npz}.

Run where the reference checkout and its compiled operator library exist
(``make -C oracle ref``):

    python tests/golden/make_golden.py [--ref <nnc-py checkout>]

Three groups of fixtures:

* ``kat_*``  — the known-answer tests of the reference's own runtime suite
  (tests/test_x86_runtime.py): the input arrays are read out of that file's
  test bodies (their literal ``np.*`` assignments, evaluated with numpy) and
  the expected outputs are what the reference's compiled ops.c returns;
* seeded cases from tests/opcases.py, expected = the compiled reference;
* the fused entry points without a reference counterpart (conv+add+relu,
  gemm+relu, matmul+relu), expected = the oracle's restatement of the
  reference composition (marked ``"expect": "oracle"``).

The fixtures are small (well under 1 MB) and are what the CPU and GPU tests
load; nothing at test time reads the reference checkout.
"""

from __future__ import annotations

import argparse
import os
import ast
import json
import pathlib
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path[:0] = [str(ROOT), str(ROOT / "nnc-py_b200"), str(ROOT / "tests")]

import opcases as C  # noqa: E402
from oracle import oracle as O  # noqa: E402

REF_TESTS = "tests/test_x86_runtime.py"


def conv_out(h, k, s, p):
    return (h + 2 * p - k) // s + 1


# test function -> (op, args). Arg strings: "t:<var>" input array,
# "o:<python expr>" output shape, "tl:<v1>,<v2>" / "ol:<expr>;<expr>" lists,
# "i:<int>", "f:<float>", "p:<var>" int64 pointer (None -> NULL).
KATS = {
    "test_add": ("nnc_add", ["t:a", "t:b", "o:a.shape"]),
    "test_mul": ("nnc_mul", ["t:a", "t:b", "o:a.shape"]),
    "test_sub": ("nnc_sub", ["t:a", "t:b", "o:a.shape"]),
    "test_div": ("nnc_div", ["t:a", "t:b", "o:a.shape"]),
    "test_relu": ("nnc_relu", ["t:a", "o:a.shape"]),
    "test_sigmoid": ("nnc_sigmoid", ["t:a", "o:a.shape"]),
    "test_tanh": ("nnc_tanh", ["t:a", "o:a.shape"]),
    "test_softmax": ("nnc_softmax", ["t:a", "o:a.shape", "i:1"]),
    "test_maxpool2d_matches_reference": (
        "nnc_maxpool2d",
        ["t:input_data", "o:(1, 2, conv_out(4, 3, 2, 1), conv_out(4, 3, 2, 1))", "i:3", "i:3", "i:2", "i:2", "i:1", "i:1"],
    ),
    "test_conv_no_padding_matches_reference": ("nnc_conv", ["t:input_data", "t:weight_data", "t:bias_data", "o:CONV(3,3,1,1,0,0)", "i:3", "i:3", "i:1", "i:1", "i:0", "i:0"]),
    "test_conv_same_padding_matches_reference": ("nnc_conv", ["t:input_data", "t:weight_data", "t:bias_data", "o:CONV(3,3,1,1,1,1)", "i:3", "i:3", "i:1", "i:1", "i:1", "i:1"]),
    "test_conv_same_padding_wide_matches_reference": ("nnc_conv", ["t:input_data", "t:weight_data", "t:bias_data", "o:CONV(3,3,1,1,1,1)", "i:3", "i:3", "i:1", "i:1", "i:1", "i:1"]),
    "test_conv_same_padding_stride2_matches_reference": ("nnc_conv", ["t:input_data", "t:weight_data", "t:bias_data", "o:CONV(3,3,2,2,1,1)", "i:3", "i:3", "i:2", "i:2", "i:1", "i:1"]),
    "test_conv_same_padding_stride2_wide_matches_reference": ("nnc_conv", ["t:input_data", "t:weight_data", "t:bias_data", "o:CONV(3,3,2,2,1,1)", "i:3", "i:3", "i:2", "i:2", "i:1", "i:1"]),
    "test_conv_1x1_matches_reference": ("nnc_conv", ["t:input_data", "t:weight_data", "t:bias_data", "o:CONV(1,1,1,1,0,0)", "i:1", "i:1", "i:1", "i:1", "i:0", "i:0"]),
    "test_conv1x1_matches_reference": ("nnc_conv1x1", ["t:input_data", "t:weight_data", "t:bias_data", "o:CONV(1,1,1,1,0,0)", "i:1", "i:1", "i:0", "i:0"]),
    "test_conv_relu1x1_matches_reference": ("nnc_conv_relu1x1", ["t:input_data", "t:weight_data", "t:bias_data", "o:CONV(1,1,1,1,0,0)", "i:1", "i:1", "i:0", "i:0"]),
    "test_conv3x3_s1_matches_reference": ("nnc_conv3x3_s1", ["t:input_data", "t:weight_data", "t:bias_data", "o:CONV(3,3,1,1,1,1)"]),
    "test_conv_relu3x3_s1_matches_reference": ("nnc_conv_relu3x3_s1", ["t:input_data", "t:weight_data", "t:bias_data", "o:CONV(3,3,1,1,1,1)"]),
    "test_conv7x7_s2_matches_reference": ("nnc_conv7x7_s2", ["t:input_data", "t:weight_data", "t:bias_data", "o:CONV(7,7,2,2,3,3)"]),
    "test_conv_relu7x7_s2_matches_reference": ("nnc_conv_relu7x7_s2", ["t:input_data", "t:weight_data", "t:bias_data", "o:CONV(7,7,2,2,3,3)"]),
    "test_matmul_2d": ("nnc_matmul", ["t:a", "t:b", "o:(a.shape[0], b.shape[1])"]),
    "test_gemm_transposed_weight_with_bias": ("nnc_gemm", ["t:a", "t:b", "t:c", "o:(a.shape[0], b.shape[0])", "f:1.0", "f:1.0", "i:0", "i:1"]),
    "test_gemm_nt_matches_reference": ("nnc_gemm_nt", ["t:a", "t:b", "t:c", "o:(a.shape[0], b.shape[0])", "f:1.0", "f:1.0"]),
    "test_matmul_vector_matrix": ("nnc_matmul", ["t:a", "t:b", "o:(b.shape[1],)"]),
    "test_matmul_matrix_vector": ("nnc_matmul", ["t:a", "t:b", "o:(a.shape[0],)"]),
    "test_transpose": ("nnc_transpose", ["t:a", "o:a.T.shape", "p:perm", "i:2"]),
    "test_transpose_3d": ("nnc_transpose", ["t:a", "o:tuple(a.shape[i] for i in perm)", "p:perm", "i:3"]),
    "test_reshape": ("nnc_reshape", ["t:a", "o:tuple(new_shape)", "p:new_shape", "i:2"]),
    "test_concat": ("nnc_concat", ["tl:a,b", "o:np.concatenate([a, b], 0).shape", "i:2", "i:0"]),
    "test_concat_axis1": ("nnc_concat", ["tl:a,b", "o:np.concatenate([a, b], 1).shape", "i:2", "i:1"]),
    "test_split": ("nnc_split", ["t:a", "ol:(a.shape[0], a.shape[1] // 2);(a.shape[0], a.shape[1] // 2)", "i:2", "i:1"]),
    "test_reducemean": ("nnc_reducemean", ["t:a", "o:(a.shape[0], 1)", "i:1", "i:1"]),
    "test_reducemean_no_keepdims": ("nnc_reducemean", ["t:a", "o:(a.shape[0],)", "i:1", "i:0"]),
    "test_reducesum": ("nnc_reducesum", ["t:a", "o:(1, a.shape[1])", "i:0", "i:1"]),
    "test_reducesum_no_keepdims": ("nnc_reducesum", ["t:a", "o:(a.shape[1],)", "i:0", "i:0"]),
    "test_sqrt": ("nnc_sqrt", ["t:a", "o:a.shape"]),
    "test_exp": ("nnc_exp", ["t:a", "o:a.shape"]),
    "test_log": ("nnc_log", ["t:a", "o:a.shape"]),
    "test_abs": ("nnc_abs", ["t:a", "o:a.shape"]),
    "test_neg": ("nnc_neg", ["t:a", "o:a.shape"]),
}
TC_OPS = {"nnc_conv", "nnc_conv1x1", "nnc_conv_relu1x1", "nnc_conv3x3_s1", "nnc_conv_relu3x3_s1",
          "nnc_conv7x7_s2", "nnc_conv_relu7x7_s2", "nnc_matmul", "nnc_gemm", "nnc_gemm_nt"}
APPROX = {"nnc_sigmoid": 2e-6, "nnc_tanh": 2e-6, "nnc_softmax": 2e-6, "nnc_exp": 2e-6, "nnc_log": 2e-6}


def test_inputs(src: str):
    """{test name: (line, {var: value})} for the data assignments of each test."""
    out = {}
    tree = ast.parse(src)
    for fn in ast.walk(tree):
        if not (isinstance(fn, ast.FunctionDef) and fn.name in KATS):
            continue
        env = {"np": np}
        for st in fn.body:
            if not isinstance(st, ast.Assign) or len(st.targets) != 1 or not isinstance(st.targets[0], ast.Name):
                continue
            text = ast.unparse(st.value)
            if any(w in text for w in ("self", "ctypes", "_reference", "tensor_", "expected")):
                continue
            try:
                env[st.targets[0].id] = eval(compile(ast.Expression(st.value), "<kat>", "eval"), env)
            except Exception:
                continue
        out[fn.name] = (fn.lineno, {k: v for k, v in env.items() if k != "np"})
    return out


def kat_case(test, line, env):
    op, spec = KATS[test]
    arrays, args = {}, []
    ns = dict(env, np=np, conv_out=conv_out)
    if "input_data" in env and "weight_data" in env:
        x, w = env["input_data"], env["weight_data"]
        ns["CONV"] = lambda kh, kw, sh, sw, ph, pw: (x.shape[0], w.shape[0], conv_out(x.shape[2], kh, sh, ph), conv_out(x.shape[3], kw, sw, pw))
    for s in spec:
        k, v = s.split(":", 1)
        if k == "t":
            arrays[v] = np.asarray(env[v], dtype=np.float32)
            args.append({"k": "t", "n": v})
        elif k == "o":
            args.append({"k": "o", "n": "out", "shape": [int(d) for d in eval(v, ns)]})
        elif k == "tl":
            names = v.split(",")
            for n in names:
                arrays[n] = np.asarray(env[n], dtype=np.float32)
            args.append({"k": "tl", "n": names})
        elif k == "ol":
            shapes = [[int(d) for d in eval(e, ns)] for e in v.split(";")]
            args.append({"k": "ol", "n": [f"out{j}" for j in range(len(shapes))], "shape": shapes})
        elif k == "i":
            args.append({"k": "i", "v": int(v)})
        elif k == "f":
            args.append({"k": "f", "v": float(v)})
        elif k == "p":
            val = env.get(v)
            args.append({"k": "perm", "v": None if val is None else [int(d) for d in val]})
    tol = "tc" if op in TC_OPS else APPROX.get(op, "exact")
    return {"name": f"kat_{test[5:]}", "op": op, "tol": tol, "source": f"{REF_TESTS}:{line}", "args": args}, arrays


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("NNC_REFERENCE"), required="NNC_REFERENCE" not in os.environ,
                    help="nnc-py checkout (default: $NNC_REFERENCE)")
    opt = ap.parse_args()
    ref = O.load_reference()
    orc = O.load_oracle()
    src = (pathlib.Path(opt.ref) / REF_TESTS).read_text()
    inputs = test_inputs(src)
    missing = sorted(set(KATS) - set(inputs))
    assert not missing, f"KATs not found in {REF_TESTS}: {missing}"

    cases, blobs = [], {}

    def record(case, arrays, expect_lib, expect):
        outs = C.run_host(expect_lib, case, arrays)
        case = dict(case, expect=expect)
        cases.append(case)
        for n, a in arrays.items():
            blobs[f"{case['name']}/in/{n}"] = a
        for n, a in outs.items():
            blobs[f"{case['name']}/out/{n}"] = a

    for test, (line, env) in sorted(inputs.items(), key=lambda kv: kv[1][0]):
        case, arrays = kat_case(test, line, env)
        record(case, arrays, ref, "reference")
    for case, arrays in C.seeded_cases():
        record(case, arrays, ref, "reference")
    for case, arrays in C.fused_cases():
        record(case, arrays, orc, "oracle")

    (HERE / "cases.json").write_text(json.dumps(cases, indent=1) + "\n")
    np.savez_compressed(HERE / "golden.npz", **blobs)
    size = (HERE / "golden.npz").stat().st_size
    print(f"{len(cases)} cases, golden.npz {size / 1e3:.0f} kB")


if __name__ == "__main__":
    main()

"""Builds the reference's own x86 code for the workload graphs —
TEST INFRASTRUCTURE ONLY (model-level checker and CPU baseline).

For each (model, batch, opt level) it runs nnc-py's compiler pipeline on the
seeded graph (nnc_cuda.workloads, converted to nnc-py IR), lets nnc-py's
X86Backend emit model.c / tensors.c / constants_loader.c / constants.bin,
and compiles them with the reference's runtime/x86/ops.c and
oracle/ref_model_main.c using the flags of nnc-py's benchmark harness
(gcc -O3 -std=c11, benchmarks/harness.py:253) into oracle/_ref/<tag>/model_x86.

Needs the reference checkout (nnc-py importable); run by
__graft_entry__.build() where it exists. Outputs stay in oracle/_ref/
(git-ignored; they travel to the GPU box with the rest of the tree).

    python oracle/ref_models.py [--ref <nnc-py checkout>]
"""

from __future__ import annotations

import argparse
import os
import json
import pathlib
import shutil
import subprocess
import sys

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parent
sys.path[:0] = [str(ROOT / "nnc-py_b200")]

# (tag, model, batch, opt): opt 1 = nnc-py's O1 list; 3 = its legacy O3 list
# (passes/base.py:113-124; the default O3 needs the absent joint solver).
BUILDS = [
    ("resnet18_o1_b1", "resnet18", 1, 1),
    ("resnet18_o3_b1", "resnet18", 1, 3),
    ("resnet18_o1_b2", "resnet18", 2, 1),
    ("lenet5_o0_b1", "lenet5", 1, 0),
    ("lenet5_o1_b16", "lenet5", 16, 1),
    ("transformer_o1_b1", "transformer", 1, 1),
    # The reference's batched MatMul offsets batches by the batch count
    # (ops.c:1680-1700), not by the matrix size, so a sample's result depends
    # on the batch it runs in: batch 256 needs its own build.
    ("transformer_o1_b256", "transformer", 256, 1),
    # Debug builds: every intermediate tensor printed (nnc-py's debug dump).
    ("resnet18_o1_b1_debug", "resnet18", 1, 1),
    ("lenet5_o1_b1_debug", "lenet5", 1, 1),
]


def build_one(ref: pathlib.Path, tag: str, model_name: str, batch: int, opt: int) -> pathlib.Path:
    sys.path.insert(0, str(ref / "src"))
    from nnc_py.codegen.x86_backend import X86Backend
    from nnc_py.ir.context import CompileContext
    from nnc_py.passes.base import PassManager

    from nnc_cuda import workloads as W
    from nnc_cuda.codegen import to_nnc_graph

    model = W.BUILDERS[model_name](batch)
    ctx = CompileContext(to_nnc_graph(model), "x86", opt)
    ctx.metadata["entry_point"] = "nnc_run"
    pm = PassManager()
    for p in PassManager.get_default_passes(opt):
        pm.register(p)
    pm.run(ctx)
    debug = tag.endswith("_debug")
    res = X86Backend(debug_mode=debug).generate(ctx)
    out = HERE / "_ref" / tag
    shutil.rmtree(out, ignore_errors=True)
    out.mkdir(parents=True)
    for a in res.files:
        p = out / a.filename
        p.write_bytes(a.content) if isinstance(a.content, bytes) else p.write_text(a.content)
    sym_in = ctx.tensor_symbols[model.inputs[0]]
    sym_out = ctx.tensor_symbols[model.outputs[0]]
    srcs = [str(out / f) for f in ("model.c", "tensors.c", "constants_loader.c")]
    cmd = ["gcc", "-O3", "-std=c11", "-D_GNU_SOURCE", f"-I{ref / 'runtime' / 'include'}", f"-I{out}",
           f"-DMODEL_INPUT={sym_in}", f"-DMODEL_OUTPUT={sym_out}", *srcs, str(ref / "runtime" / "x86" / "ops.c"),
           str(HERE / "ref_model_main.c"), "-lm", "-lpthread", "-o", str(out / "model_x86")]
    if debug:
        cmd.insert(1, "-DNNC_DEBUG_DUMP")
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    consts = [[n, ctx.tensor_symbols[n]] for n in ctx.graph.constants]
    (out / "build.json").write_text(json.dumps({"model": model_name, "batch": batch, "opt_level": opt,
                                                "input": sym_in, "output": sym_out, "cflags": "-O3 -std=c11",
                                                "constants": consts}) + "\n")
    # The constants container is regenerated from the seeded Model at run
    # time (byte-identical NNCB), so the large file need not travel.
    (out / "constants.bin").unlink()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("NNC_REFERENCE"), required="NNC_REFERENCE" not in os.environ,
                    help="nnc-py checkout (default: $NNC_REFERENCE)")
    ap.add_argument("--only", default=None)
    opt = ap.parse_args()
    ref = pathlib.Path(opt.ref)
    for tag, m, b, o in BUILDS:
        if opt.only and opt.only != tag:
            continue
        out = build_one(ref, tag, m, b, o)
        print(f"built {out / 'model_x86'}")


if __name__ == "__main__":
    main()

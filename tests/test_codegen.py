"""The cuda codegen target (CPU-only; needs nnc-py importable, i.e. where the
reference checkout exists — skipped elsewhere)."""

import os
import pathlib
import re
import sys

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parent.parent
REF_SRC = pathlib.Path(os.environ.get("NNC_REFERENCE", "-")) / "src"
if REF_SRC.exists() and str(REF_SRC) not in sys.path:
    sys.path.insert(0, str(REF_SRC))
nnc_py = pytest.importorskip("nnc_py")

from nnc_cuda import codegen as CG  # noqa: E402
from nnc_cuda import workloads as W  # noqa: E402

GEN = ROOT / "nnc-py_b200" / "models_gen"


def test_committed_sources_are_up_to_date(tmp_path):
    sys.path.insert(0, str(GEN))
    import generate

    for d, model, batch, opt in generate.CONFIGS:
        out = tmp_path / d
        CG.compile_model(W.BUILDERS[model](batch), out, opt_level=opt, debug=generate.is_debug(d))
        for f in sorted(p.name for p in out.iterdir()):
            assert (GEN / d / f).read_text() == (out / f).read_text(), f"{d}/{f} is stale: rerun generate.py"


def _x86_calls(model, opt):
    from nnc_py.codegen.x86_backend import X86Backend
    from nnc_py.ir.context import CompileContext
    from nnc_py.passes.base import PassManager

    ctx = CompileContext(CG.to_nnc_graph(model), "x86", opt)
    ctx.metadata["entry_point"] = "nnc_run"
    pm = PassManager()
    for p in PassManager.get_default_passes(opt):
        pm.register(p)
    pm.run(ctx)
    src = next(a.content for a in X86Backend().generate(ctx).files if a.filename == "model.c")
    return re.findall(r"^\s*(nnc_\w+\(.*\));", src, re.M)


@pytest.mark.parametrize("name,batch", [("resnet18", 2), ("lenet5", 4), ("transformer", 1)])
def test_o1_call_lines_equal_the_x86_backend(tmp_path, name, batch):
    """At O1 the cuda target emits exactly the operator calls nnc-py's x86
    backend emits (the library is a drop-in for ops.c)."""
    model = W.BUILDERS[name](batch)
    CG.compile_model(model, tmp_path, opt_level=1)
    ours = re.findall(r"^\s*(nnc_\w+\(.*\));", (tmp_path / "model.c").read_text(), re.M)
    assert ours == _x86_calls(model, 1)


def test_o3_fuses_every_residual_join(tmp_path):
    man = CG.compile_model(W.resnet18(2), tmp_path, opt_level=3)
    calls = man["calls"]
    assert calls.count("nnc_conv_add_relu3x3_s1") == 8
    assert "nnc_add" not in calls and "nnc_relu" not in calls and "nnc_add_relu" not in calls
    assert calls.count("nnc_conv_relu3x3_s1") + calls.count("nnc_conv_relu") == 8
    assert calls[0] == "nnc_conv_relu_maxpool" and calls[-1] == "nnc_gap_gemm_nt"


def test_o3_conv_relu_maxpool_group(tmp_path):
    """The stem's Conv+ReLU -> MaxPool is one call carrying the conv extent
    and the pool geometry (its conv result never exists in the arena); with
    the group disabled the two calls come back."""
    man = CG.compile_model(W.resnet18(2), tmp_path, opt_level=3)
    calls = man["calls"]
    assert calls[0] == "nnc_conv_relu_maxpool" and "nnc_maxpool2d" not in calls
    line = next(l for l in (tmp_path / "model.c").read_text().splitlines() if "nnc_conv_relu_maxpool(" in l)
    assert line.strip().endswith("7, 7, 2, 2, 3, 3, 112, 112, 3, 3, 2, 2, 1, 1);")
    off = CG.compile_model(W.resnet18(2), tmp_path / "off", opt_level=3, fuse_conv_relu_maxpool=False)
    assert off["calls"][:2] == ["nnc_conv_relu7x7_s2", "nnc_maxpool2d"]


def test_o3_gemm_relu_group(tmp_path):
    """LeNet's Gemm -> Relu pairs become nnc_gemm_nt_relu calls (ReLU in the
    GEMM epilogue, PrepackLowering's gemm_nt form kept); the last Gemm feeds
    the softmax and stays a plain gemm_nt."""
    man = CG.compile_model(W.lenet5(4), tmp_path, opt_level=3)
    calls = man["calls"]
    assert calls.count("nnc_gemm_nt_relu") == 2 and calls.count("nnc_gemm_nt") == 1
    assert "nnc_relu" not in calls[calls.index("nnc_flatten"):]
    # LeNet's stride-1 convs keep their pool separate (no pooled epilogue).
    assert calls.count("nnc_maxpool2d") == 2 and "nnc_conv_relu_maxpool" not in calls


def test_o3_gap_gemm_head(tmp_path):
    """ResNet's GlobalAveragePool -> Flatten -> Gemm head becomes one
    nnc_gap_gemm_nt call reading the channels-last stage-4 output; the pooled
    and flattened tensors leave the graph (no arena slots)."""
    man = CG.compile_model(W.resnet18(2), tmp_path, opt_level=3)
    calls = man["calls"]
    assert calls[-1] == "nnc_gap_gemm_nt" and calls.count("nnc_gap_gemm_nt") == 1
    assert "nnc_avgpool2d" not in calls and "nnc_flatten" not in calls and "nnc_gemm_nt" not in calls
    src = (tmp_path / "model.c").read_text()
    assert "nnc_gap_gemm_nt(&tensor_layer4_1_out_relu, &tensor_fc_w, &tensor_fc_b, &tensor_logits, 1.0f, 1.0f);" in src
    tensors = (tmp_path / "tensors.c").read_text()
    assert "Tensor tensor_gap " not in tensors and "Tensor tensor_flat " not in tensors
    assert "tensor_layer4_1_out_relu = {.data = NULL, .dtype = (nnc_dtype_t)(NNC_DTYPE_FLOAT32 | NNC_CUDA_TAG_NHWC)" in tensors


def test_o3_matmul_epilogue_groups(tmp_path):
    """The transformer's MatMul -> Add(bias) [-> Relu] and MatMul -> Div(8) ->
    Softmax chains each become one call, as do the residual Add ->
    LayerNorm joins and the reshapes around the head transposes; the
    probs . V MatMul stays."""
    man = CG.compile_model(W.transformer(1), tmp_path, opt_level=3)
    calls = man["calls"]
    layers = 4
    assert calls.count("nnc_matmul_bias") == 5 * layers  # q, k, v, output projection, FFN2
    assert calls.count("nnc_matmul_relu") == layers       # FFN1
    assert calls.count("nnc_matmul_scale_softmax") == layers
    assert calls.count("nnc_matmul") == layers            # probs . V
    assert "nnc_softmax" not in calls and "nnc_div" not in calls and "nnc_add_relu" not in calls
    # Residual joins: Add -> LayerNorm as one call each.
    assert calls.count("nnc_add_layernorm") == 2 * layers
    assert "nnc_add" not in calls and "nnc_layernorm" not in calls
    src = (tmp_path / "model.c").read_text()
    line = next(l for l in src.splitlines() if "nnc_matmul_scale_softmax(" in l)
    assert line.strip().endswith("0.125f);")  # 1 / sqrt(64)
    # Head split (Reshape -> Transpose of q, k, v) and merge (Transpose ->
    # Reshape of the context): the reshapes fold into the transpose calls.
    assert "nnc_reshape" not in calls and "nnc_transpose" not in calls
    assert calls.count("nnc_transpose_shaped") == 4 * layers
    assert "nnc_transpose_shaped(&tensor_l0_q_out, &tensor_l0_q_heads, in_shape, perm, 4);" in src
    assert "static int64_t in_shape[4] = {1, 128, 4, 64};" in src
    assert "nnc_transpose_shaped(&tensor_l0_ctx_heads, &tensor_l0_ctx, in_shape, perm, 4);" in src


def test_channels_last_assignment(tmp_path):
    man = CG.compile_model(W.resnet18(2), tmp_path, opt_level=3)
    cl = set(man["channels_last"])
    assert "tensor_input" not in cl          # user-facing NCHW input
    # The pooled classifier head (one call) reads the stage-4 output
    # channels-last; its pooled and flattened tensors are gone.
    assert "tensor_pool1" in cl and "tensor_layer4_1_out_relu" in cl and "tensor_gap" not in cl
    assert "tensor_logits" not in cl and "tensor_flat" not in cl  # 2-D
    man_t = CG.compile_model(W.transformer(1), tmp_path / "t", opt_level=1)
    assert man_t["channels_last"] == []  # 4-D tensors meet transpose/softmax


def test_arena_offsets_follow_the_cost_aware_plan(tmp_path):
    man = CG.compile_model(W.resnet18(8), tmp_path, opt_level=3)
    src = (tmp_path / "tensors.c").read_text()
    offs = [int(v) for v in re.findall(r"\{&tensor_\w+, (\d+)u\}", src)]
    assert offs and all(o % 16 == 0 for o in offs)
    assert max(offs) < man["arena_bytes"]
    # reuse: the arena is far smaller than all activations back to back
    total = sum(int(np.prod(s)) * 4 for n, s in W.resnet18(8).shapes.items() if not n.endswith(("_w", "_b")))
    assert man["arena_bytes"] < total / 3


def test_compiler_and_cli_gain_the_cuda_target():
    CG.install()
    from nnc_py import cli as nnc_cli
    from nnc_py.compiler import Compiler

    c = Compiler(target="cuda", opt_level=3)
    assert isinstance(c.backend, CG.CudaBackend)
    names = [p.name for p in c._get_passes()]
    assert "CudaConvAddReluFusion" in names
    target = next(p for p in nnc_cli.compile.params if p.name == "target")
    assert "cuda" in target.type.choices


def test_constants_blob_matches_reference_container():
    """The NNCB bytes the runtime uploads equal what nnc-py's x86 backend
    writes for the same graph."""
    from nnc_py.codegen.x86_emitters.constants_loader import generate_constants_binary
    from nnc_py.ir.context import CompileContext

    model = W.lenet5(1)
    ctx = CompileContext(CG.to_nnc_graph(model), "x86", 1)
    CG.CudaBackend()._assign_symbols(ctx)
    ref_bytes, _ = generate_constants_binary(ctx)
    ours = W.nncb_bytes([(ctx.tensor_symbols[n], a) for n, a in model.constants.items()])
    assert ours == ref_bytes

"""The ``cuda`` target for nnc-py's compiler (needs nnc-py importable).

Plugs in where nnc-py adds targets — ``Compiler._create_backend``
(compiler.py:266-285) and the CLI's ``-t`` choice (cli.py:33-37) — and emits
the same artifact set as the x86 backend (codegen/x86_backend.py:89-147):

* ``model.c``    nnc-py's own CEmitter (codegen/c_emitter.py) with one
                 addition: nodes fused by :class:`ConvAddReluFusionPass`
                 call ``nnc_conv_add_relu*``; every other call line is the
                 one the reference emits;
* ``model.h``    entry points (nnc_run + device/arena/constant management);
* ``tensors.c``  the Tensor globals; activations are bound at run time into
                 ONE device arena sized by the cost_aware liveness plan
                 (passes/memory_planning.py:72-111), constants into one slab;
                 4-D activations that only meet conv / pool / element-wise
                 ops carry NNC_CUDA_TAG_NHWC (channels-last);
* ``constants_loader.c``  reads the NNCB v1 container
                 (codegen/x86_emitters/constants_loader.py:40-144), uploads
                 once per device and prepacks conv weights on the device;
* ``model_runtime.c``     arena/slab allocation and per-device binding;
* ``test_runner.c``       shards the batch over the GPUs of one node, gathers
                 the outputs to GPU 0 over NVLink and writes them;
* ``Makefile``   nvcc, -arch=sm_100a, links libnnc_cuda.so;
* ``manifest.json``  shapes, constant order/symbols, arena size.
"""

from __future__ import annotations

import json
import os
import pathlib
import re
import sys
from typing import Any

import numpy as np

from .workloads import Model

def _import_nnc_py():
    """Imports nnc-py: from the environment, else from the checkout that the
    NNC_REFERENCE variable names (its ``src`` directory)."""
    try:
        import nnc_py  # noqa: F401
    except ImportError:
        ref = os.environ.get("NNC_REFERENCE")
        if ref and (pathlib.Path(ref) / "src" / "nnc_py").exists():
            sys.path.insert(0, str(pathlib.Path(ref) / "src"))
        import nnc_py  # noqa: F401


_import_nnc_py()

from nnc_py.codegen.base import BackendBase, CodeGenResult  # noqa: E402
from nnc_py.codegen.c_emitter import CEmitter  # noqa: E402
from nnc_py.ir.context import CompileContext  # noqa: E402
from nnc_py.ir.graph import Graph  # noqa: E402
from nnc_py.ir.node import Node, OpType  # noqa: E402
from nnc_py.ir.tensor import TensorShape, TensorType  # noqa: E402
from nnc_py.ir.types import DataType  # noqa: E402
from nnc_py.passes.base import PassBase, PassManager  # noqa: E402
from nnc_py.utils.name_manager import NameManager  # noqa: E402

TAG_NHWC = 0x100
ARENA_ALIGN = 256


# --------------------------------------------------------------- graph ----
def to_nnc_graph(model: Model) -> Graph:
    """Builds nnc-py IR (ir/graph.py) from a workload Model."""
    g = Graph(model.name)
    for name, shape in model.shapes.items():
        g.add_tensor(TensorType(DataType.FLOAT32, TensorShape(list(shape)), name))
    for name, arr in model.constants.items():
        g.constants[name] = arr
    for n in model.nodes:
        g.add_node(Node(OpType(n.op), n.name, list(n.inputs), list(n.outputs), dict(n.attrs)))
    g.inputs = list(model.inputs)
    g.outputs = list(model.outputs)
    return g


# -------------------------------------------------------------- passes ----
class ConvAddReluFusionPass(PassBase):
    """Collapses Conv -> Add(+ReLU) into one conv whose epilogue adds the
    residual and applies ReLU (the Conv+Add+Relu group the cuda target adds
    next to nnc-py's built-in patterns, pattern/fusion_patterns.py:104-152).

    Runs after PatternFusion, so the Add+ReLU is already a FUSED_ADD_RELU
    node. The conv must feed only that node. The fused node keeps op type
    CONV2D (so liveness, memory planning and PrepackLowering treat it as a
    conv, never in-place) with inputs [x, w, b, residual] and
    metadata ``cuda_fused = "conv_add_relu"``.
    """

    @property
    def name(self) -> str:
        return "CudaConvAddReluFusion"

    def _execute(self, ctx: CompileContext) -> None:
        g = ctx.graph
        for node in list(g.topological_sort()):
            if node.op_type != OpType.FUSED_ADD_RELU or len(node.inputs) != 2:
                continue
            for pos in (0, 1):
                src = node.inputs[pos]
                prods = g.get_producers(src)
                if len(prods) != 1:
                    continue
                conv = prods[0]
                if conv.op_type != OpType.CONV2D or conv.metadata.get("cuda_fused"):
                    continue
                if len(g.get_consumers(src)) != 1 or src in g.outputs:
                    continue
                residual = node.inputs[1 - pos]
                if list(g.tensors[residual].shape.dims) != list(g.tensors[node.outputs[0]].shape.dims):
                    continue
                inputs = list(conv.inputs)
                if len(inputs) == 2:
                    inputs.append("")  # no bias
                fused = Node(OpType.CONV2D, f"{conv.name}_add_relu", inputs[:3] + [residual],
                             list(node.outputs), dict(conv.attrs),
                             metadata={"cuda_fused": "conv_add_relu", "fused_from": [conv.name, node.name]})
                g.nodes.pop(conv.name)
                g.nodes.pop(node.name)
                g.tensors.pop(src, None)
                g.add_node(fused)  # also drops nnc-py's cached dependency graph
                break


class ConvReluMaxPoolFusionPass(PassBase):
    """Collapses Conv+ReLU -> MaxPool into one call, nnc_conv_relu_maxpool
    (the ResNet stem), so the conv result
    (1024 x 64 x 112 x 112 floats for the bench batch) is never written.

    Runs after PatternFusion (the Conv+ReLU is then a FUSED_CONV_RELU node)
    and requires that node to feed only the pool. The fused node keeps op
    type FUSED_CONV_RELU with the conv's inputs and attributes, the pool's
    output, and metadata ``cuda_fused = "conv_relu_maxpool"`` carrying the
    conv result's extent and the pool's kernel, strides and pads.
    """

    @property
    def name(self) -> str:
        return "CudaConvReluMaxPoolFusion"

    def _execute(self, ctx: CompileContext) -> None:
        g = ctx.graph
        for node in list(g.topological_sort()):
            if node.op_type != OpType.MAXPOOL or not node.inputs:
                continue
            src = node.inputs[0]
            prods = g.get_producers(src)
            if len(prods) != 1:
                continue
            conv = prods[0]
            if conv.op_type != OpType.FUSED_CONV_RELU or conv.metadata.get("cuda_fused"):
                continue
            if len(g.get_consumers(src)) != 1 or src in g.outputs:
                continue
            dims = [int(d) for d in g.tensors[src].shape.dims]
            if len(dims) != 4:
                continue
            # Only where the pooled epilogue runs (the space-to-depth route:
            # a stride-2 conv over at most 8 channels into at most 64, pooled
            # by a stride-2 window of at most 3 with pad <= 1); elsewhere the
            # entry point would only compose the two kernels through a
            # temporary allocation.
            cin = int(g.tensors[conv.inputs[0]].shape.dims[1])
            pk = list(node.attrs.get("kernel_shape", [2, 2]))
            ps = list(node.attrs.get("strides", [2, 2]))
            pp = list(node.attrs.get("pads", [0, 0, 0, 0]))
            if (list(conv.attrs.get("strides", [1, 1])) != [2, 2] or cin > 8 or dims[1] > 64 or ps != [2, 2]
                    or max(pk) > 3 or max(pp) > 1):
                continue
            meta = {"cuda_fused": "conv_relu_maxpool", "conv_out_hw": dims[2:4],
                    "pool_kernel": list(node.attrs.get("kernel_shape", [2, 2])),
                    "pool_strides": list(node.attrs.get("strides", [2, 2])),
                    "pool_pads": list(node.attrs.get("pads", [0, 0, 0, 0])),
                    "fused_from": [conv.name, node.name]}
            fused = Node(OpType.FUSED_CONV_RELU, f"{conv.name}_maxpool", list(conv.inputs), list(node.outputs),
                         dict(conv.attrs), metadata=meta)
            g.nodes.pop(conv.name)
            g.nodes.pop(node.name)
            g.tensors.pop(src, None)
            g.add_node(fused)


def _single_consumer(g, tensor):
    """The only consumer of `tensor`, or None (several, none, or a graph output)."""
    cons = g.get_consumers(tensor)
    if len(cons) != 1 or tensor in g.outputs:
        return None
    return cons[0]


def _replace(g, old_nodes, new_node, dropped_tensors):
    for n in old_nodes:
        g.nodes.pop(n.name)
    for t in dropped_tensors:
        g.tensors.pop(t, None)
    g.add_node(new_node)  # also drops nnc-py's cached dependency graph


class GemmReluFusionPass(PassBase):
    """Collapses Gemm -> ReLU into one GEMM node whose call is
    nnc_gemm_relu / nnc_gemm_nt_relu (ReLU in the GEMM epilogue): the
    Gemm+Relu group of the cuda target's O3 list (LeNet's fully connected
    layers). nnc-py's own registry fuses MatMul+Relu
    (pattern/fusion_patterns.py:147-155) but not Gemm+Relu. The node keeps op
    type GEMM (PrepackLowering still picks the gemm_nt form) with metadata
    ``cuda_fused = "gemm_relu"``."""

    @property
    def name(self) -> str:
        return "CudaGemmReluFusion"

    def _execute(self, ctx: CompileContext) -> None:
        g = ctx.graph
        for node in list(g.topological_sort()):
            if node.op_type != OpType.GEMM or node.metadata.get("cuda_fused"):
                continue
            relu = _single_consumer(g, node.outputs[0])
            if relu is None or relu.op_type != OpType.RELU:
                continue
            fused = Node(OpType.GEMM, f"{node.name}_relu", list(node.inputs), list(relu.outputs),
                         dict(node.attrs), metadata={"cuda_fused": "gemm_relu", "fused_from": [node.name, relu.name]})
            _replace(g, [node, relu], fused, [node.outputs[0]])


class MatMulEpilogueFusionPass(PassBase):
    """Collapses the transformer's MatMul epilogues into the MatMul call:

    * MatMul -> Add(bias) with a constant bias of the MatMul's last extent
      (N values, broadcast per row as the reference's modular add does) ->
      ``nnc_matmul_bias``; after PatternFusion's add_relu, MatMul ->
      FusedAddRelu(bias) -> FUSED_MATMUL_RELU [a, b, bias], which nnc-py's
      CEmitter emits as ``nnc_matmul_relu(a, b, bias, out)``
      (codegen/c_emitter.py:1143-1171);
    * MatMul -> Div(s) (or Mul(1 / s)) by a constant power-of-two scalar ->
      Softmax over the last axis -> ``nnc_matmul_scale_softmax(a, b, out,
      1 / s)`` (scaled attention scores; x / s == x * (1 / s) exactly for a
      power of two, so the fused scale is the reference's division).

    Each intermediate must feed only the next node of its group.
    """

    @property
    def name(self) -> str:
        return "CudaMatMulEpilogueFusion"

    @staticmethod
    def _const_scalar(g, t):
        if t in g.constants:
            arr = np.asarray(g.constants[t])
            if arr.size == 1:
                return float(arr.reshape(-1)[0])
        return None

    def _execute(self, ctx: CompileContext) -> None:
        g = ctx.graph
        for node in list(g.topological_sort()):
            if node.name not in g.nodes or node.op_type != OpType.MATMUL or node.metadata.get("cuda_fused"):
                continue
            if len(node.inputs) != 2:
                continue
            mm = node.outputs[0]
            nxt = _single_consumer(g, mm)
            if nxt is None:
                continue
            dims = [int(d) for d in g.tensors[mm].shape.dims]
            if nxt.op_type in (OpType.ADD, OpType.FUSED_ADD_RELU) and len(nxt.inputs) == 2:
                bias = nxt.inputs[1] if nxt.inputs[0] == mm else nxt.inputs[0]
                if bias == mm or bias not in g.constants:
                    continue
                if list(np.asarray(g.constants[bias]).shape) != dims[-1:]:
                    continue
                if list(g.tensors[nxt.outputs[0]].shape.dims) != dims:
                    continue
                relu = nxt.op_type == OpType.FUSED_ADD_RELU
                fused = Node(OpType.FUSED_MATMUL_RELU if relu else OpType.MATMUL,
                             f"{node.name}_bias{'_relu' if relu else ''}", list(node.inputs) + [bias],
                             list(nxt.outputs), dict(node.attrs),
                             metadata={"fused_from": [node.name, nxt.name]} if relu else
                             {"cuda_fused": "matmul_bias", "fused_from": [node.name, nxt.name]})
                _replace(g, [node, nxt], fused, [mm])
                continue
            if nxt.op_type in (OpType.DIV, OpType.MUL) and len(nxt.inputs) == 2 and nxt.inputs[0] == mm:
                s = self._const_scalar(g, nxt.inputs[1])
                if s is None or s == 0.0 or not np.isfinite(s):
                    continue
                alpha = 1.0 / s if nxt.op_type == OpType.DIV else s
                mant, _ = np.frexp(abs(alpha))
                if alpha <= 0.0 or mant != 0.5:  # a positive power of two
                    continue
                scaled = nxt.outputs[0]
                sm = _single_consumer(g, scaled)
                if sm is None or sm.op_type != OpType.SOFTMAX:
                    continue
                axis = int(sm.attrs.get("axis", -1))
                if axis not in (-1, len(dims) - 1):
                    continue
                fused = Node(OpType.MATMUL, f"{node.name}_scale_softmax", list(node.inputs), list(sm.outputs),
                             dict(node.attrs), metadata={"cuda_fused": "matmul_scale_softmax", "alpha": alpha,
                                                         "fused_from": [node.name, nxt.name, sm.name]})
                _replace(g, [node, nxt, sm], fused, [mm, scaled])


class GapGemmFusionPass(PassBase):
    """Collapses the classifier head GlobalAveragePool -> Flatten(axis 1) ->
    Gemm into one GEMM node called as nnc_gap_gemm_nt (the pooled features
    stay in the library's scratch; no flatten copy). The Gemm must not
    transpose A and its B must be a constant or already transposed, so that
    PrepackLowering leaves it in the gemm_nt form (passes/prepack_lowering.py:
    80-117). The node keeps op type GEMM with metadata ``cuda_fused =
    "gap_gemm"`` and inputs [pool input, B, C]."""

    @property
    def name(self) -> str:
        return "CudaGapGemmFusion"

    def _execute(self, ctx: CompileContext) -> None:
        g = ctx.graph
        for node in list(g.topological_sort()):
            if node.name not in g.nodes or node.op_type != OpType.GLOBAL_AVGPOOL or len(node.inputs) != 1:
                continue
            flat = _single_consumer(g, node.outputs[0])
            if flat is None or flat.op_type != OpType.FLATTEN or int(flat.attrs.get("axis", 1)) != 1:
                continue
            gemm = _single_consumer(g, flat.outputs[0])
            if gemm is None or gemm.op_type != OpType.GEMM or gemm.metadata.get("cuda_fused"):
                continue
            if gemm.inputs[0] != flat.outputs[0] or int(gemm.attrs.get("transA", 0)) != 0:
                continue
            if len(gemm.inputs) < 2 or not (int(gemm.attrs.get("transB", 0)) == 1 or gemm.inputs[1] in g.constants):
                continue
            fused = Node(OpType.GEMM, f"{gemm.name}_gap", [node.inputs[0]] + list(gemm.inputs[1:]),
                         list(gemm.outputs), dict(gemm.attrs),
                         metadata={"cuda_fused": "gap_gemm", "fused_from": [node.name, flat.name, gemm.name]})
            _replace(g, [node, flat, gemm], fused, [node.outputs[0], flat.outputs[0]])


class AddLayerNormFusionPass(PassBase):
    """Collapses Add -> LayerNormalization (a post-LN transformer's residual
    joins) into one LAYER_NORM node called as nnc_add_layernorm: the sum is
    formed as the rows are loaded and never stored. Both addends must be
    activations of the LayerNorm input's extents (no broadcast) and the sum
    must feed only the LayerNorm. Metadata ``cuda_fused = "add_layernorm"``;
    inputs [a, b, scale, bias]."""

    @property
    def name(self) -> str:
        return "CudaAddLayerNormFusion"

    def _execute(self, ctx: CompileContext) -> None:
        g = ctx.graph
        for node in list(g.topological_sort()):
            if node.name not in g.nodes or node.op_type != OpType.LAYER_NORM or not node.inputs:
                continue
            x = node.inputs[0]
            add = next((n for n in g.nodes.values() if x in n.outputs), None)
            if add is None or add.op_type != OpType.ADD or len(add.inputs) != 2:
                continue
            if _single_consumer(g, x) is not node:
                continue
            dims = list(g.tensors[x].shape.dims)
            if any(t in g.constants or list(g.tensors[t].shape.dims) != dims for t in add.inputs):
                continue
            fused = Node(OpType.LAYER_NORM, f"{node.name}_add", list(add.inputs) + list(node.inputs[1:]),
                         list(node.outputs), dict(node.attrs),
                         metadata={"cuda_fused": "add_layernorm", "fused_from": [add.name, node.name]})
            _replace(g, [add, node], fused, [x])


class ReshapeTransposeFusionPass(PassBase):
    """Folds the reshapes around transposes into the transpose call
    (nnc_transpose_shaped): Reshape -> Transpose reads the reshape's input
    with the reshaped extents, Transpose -> Reshape writes the reshape's
    output as the permuted extents, so neither reshape copies (the
    transformer's head split and merge). The node keeps op type TRANSPOSE
    with metadata ``cuda_fused = "transpose_shaped"`` and ``in_shape`` (the
    extents its input is read with)."""

    @property
    def name(self) -> str:
        return "CudaReshapeTransposeFusion"

    def _execute(self, ctx: CompileContext) -> None:
        g = ctx.graph
        for node in list(g.topological_sort()):
            if node.name not in g.nodes or node.op_type != OpType.TRANSPOSE or not node.inputs:
                continue
            perm = node.attrs.get("perm")
            if perm is None:
                continue
            cur = node
            in_shape = list(node.metadata.get("in_shape") or [int(d) for d in g.tensors[node.inputs[0]].shape.dims])
            inputs, outputs, dropped, old = list(node.inputs), list(node.outputs), [], [node]
            src = next((n for n in g.nodes.values() if inputs[0] in n.outputs), None)
            if (src is not None and src.op_type == OpType.RESHAPE and src.inputs and
                    _single_consumer(g, inputs[0]) is node and src.inputs[0] not in g.constants):
                dropped.append(inputs[0])
                old.append(src)
                inputs = [src.inputs[0]]
            dst = _single_consumer(g, outputs[0])
            if dst is not None and dst.op_type == OpType.RESHAPE and dst.inputs and dst.inputs[0] == outputs[0]:
                dropped.append(outputs[0])
                old.append(dst)
                outputs = list(dst.outputs)
            if len(old) == 1:
                continue
            fused = Node(OpType.TRANSPOSE, f"{cur.name}_shaped", inputs, outputs, dict(node.attrs),
                         metadata={"cuda_fused": "transpose_shaped", "in_shape": in_shape,
                                   "fused_from": [n.name for n in old]})
            _replace(g, old, fused, dropped)


# Whether O3 fuses Conv+ReLU -> MaxPool into nnc_conv_relu_maxpool. On: on
# the ResNet stem at batch 1024 the fused call (pooled epilogue in the conv
# kernel, 1.83 ms) beats the conv and pool kernels it replaces (2.42 ms) and
# never writes the 3.3 GB un-pooled activation.
FUSE_CONV_RELU_MAXPOOL = True


def cuda_passes(opt_level: int, fuse_conv_relu_maxpool: bool | None = None) -> list[PassBase]:
    """Pass lists of the cuda target.

    O0-O2: nnc-py's own lists (passes/base.py:88-106). O3: cleanup, nnc-py's
    PatternFusion (conv_relu, add_relu, ...), the Conv+Add+Relu group (and
    the Conv+Relu+MaxPool group when enabled), the Gemm+Relu group, the
    GlobalAveragePool+Flatten+Gemm head, the MatMul epilogue groups (bias,
    bias+relu, scale+softmax), the reshapes folded into their transposes,
    Add+LayerNorm, PrepackLowering
    (entry-point selection, Gemm weight prepack), liveness and the
    cost_aware arena plan. nnc-py's NPU tiling passes are not used:
    the GPU kernels tile internally.
    """
    from nnc_py.passes.dead_code_elimination import DeadCodeEliminationPass
    from nnc_py.passes.identity_elimination import IdentityEliminationPass
    from nnc_py.passes.liveness import LivenessAnalysisPass
    from nnc_py.passes.memory_planning import MemoryPlanningPassV2
    from nnc_py.passes.pattern_fusion import PatternFusionPass
    from nnc_py.passes.prepack_lowering import PrepackLoweringPass

    if opt_level < 3:
        return PassManager.get_default_passes(opt_level)
    fuse_pool = FUSE_CONV_RELU_MAXPOOL if fuse_conv_relu_maxpool is None else fuse_conv_relu_maxpool
    return [IdentityEliminationPass(), DeadCodeEliminationPass(), PatternFusionPass(), ConvAddReluFusionPass()] + (
        [ConvReluMaxPoolFusionPass()] if fuse_pool else []) + [
        GemmReluFusionPass(), GapGemmFusionPass(), MatMulEpilogueFusionPass(), ReshapeTransposeFusionPass(),
        AddLayerNormFusionPass(),
        PrepackLoweringPass(), LivenessAnalysisPass(), MemoryPlanningPassV2()]


# -------------------------------------------------------------- layout ----
_NHWC_OPS = {OpType.CONV2D, OpType.FUSED_CONV_RELU, OpType.FUSED_CONV_SIGMOID, OpType.FUSED_CONV_BIAS_RELU,
             OpType.MAXPOOL, OpType.AVGPOOL, OpType.GLOBAL_AVGPOOL}
_ELTWISE = {OpType.RELU, OpType.SIGMOID, OpType.TANH, OpType.CLIP, OpType.ADD, OpType.SUB, OpType.MUL,
            OpType.DIV, OpType.FUSED_ADD_RELU, OpType.FUSED_ADD_SIGMOID}


def channels_last_tensors(ctx: CompileContext) -> set[str]:
    """4-D activations that can live channels-last: every producer/consumer
    is a conv/pool (which take either layout) or an element-wise op whose 4-D
    operands all share one layout. Graph inputs/outputs stay NCHW unless
    their spatial extent is 1 x 1 (then both layouts have the same bytes)."""
    g = ctx.graph
    four_d = {n for n, t in g.tensors.items() if n not in g.constants and len(t.shape.dims) == 4}
    parent = {n: n for n in four_d}

    def find(a):
        while parent[a] != a:
            parent[a] = parent[parent[a]]
            a = parent[a]
        return a

    bad = set()
    for node in g.nodes.values():
        acts = [t for t in list(node.inputs) + list(node.outputs) if t in four_d]
        if node.op_type in _ELTWISE:
            full = [t for t in acts if list(g.tensors[t].shape.dims) == list(g.tensors[node.outputs[0]].shape.dims)]
            for t in full[1:]:
                parent[find(t)] = find(full[0])
            for t in acts:
                if t not in full:
                    bad.add(t)  # broadcast operand: keep logical order
        elif node.metadata.get("cuda_fused") == "gap_gemm":
            continue  # its 4-D input may be channels-last (the pooling reads either)
        elif node.op_type in _NHWC_OPS:
            if node.op_type in (OpType.MAXPOOL, OpType.AVGPOOL, OpType.GLOBAL_AVGPOOL):
                if node.inputs[0] in four_d and node.outputs[0] in four_d:
                    parent[find(node.outputs[0])] = find(node.inputs[0])
            if node.metadata.get("cuda_fused") == "conv_add_relu":
                res, out = node.inputs[3], node.outputs[0]
                if res in four_d and out in four_d:
                    parent[find(res)] = find(out)
        else:
            for t in acts:
                dims = g.tensors[t].shape.dims
                if int(dims[2]) * int(dims[3]) != 1:
                    bad.add(t)
    for t in list(g.inputs) + list(g.outputs):
        if t in four_d:
            dims = g.tensors[t].shape.dims
            if int(dims[2]) * int(dims[3]) != 1:
                bad.add(t)
    bad_roots = {find(t) for t in bad}
    return {t for t in four_d if find(t) not in bad_roots}


# ------------------------------------------------------------- emitter ----
class CudaEmitter(CEmitter):
    """nnc-py's CEmitter with the cuda target's fused calls: conv+add+relu,
    conv+relu+maxpool, gemm+relu, the pooled classifier head (gap+gemm),
    matmul+bias and matmul+scale+softmax."""

    def _emit_includes(self, ctx: CompileContext) -> None:
        super()._emit_includes(ctx)
        self.write_line('#include "nnc_cuda.h"')
        self.write_line()

    def _emit_operator_call(self, ctx: CompileContext, node: Node) -> None:
        if node.metadata.get("cuda_fused") == "conv_relu_maxpool":
            sym = ctx.tensor_symbols
            x, w = node.inputs[:2]
            b = node.inputs[2] if len(node.inputs) > 2 else ""
            bias = f"&{sym[b]}" if b else "NULL"
            m = node.metadata
            ks = node.attrs.get("kernel_shape", [1, 1])
            st = node.attrs.get("strides", [1, 1])
            pd = node.attrs.get("pads", [0, 0, 0, 0])
            vals = [ks[0], ks[1], st[0], st[1], pd[0], pd[1], *m["conv_out_hw"], *m["pool_kernel"][:2],
                    *m["pool_strides"][:2], m["pool_pads"][0], m["pool_pads"][1]]
            args = [f"&{sym[x]}", f"&{sym[w]}", bias, f"&{sym[node.outputs[0]]}"] + [str(int(v)) for v in vals]
            self.write_line(f"nnc_conv_relu_maxpool({', '.join(args)});")
            return
        fused = node.metadata.get("cuda_fused")
        if fused == "gemm_relu":
            # nnc-py's own Gemm call line (gemm or gemm_nt form), ReLU variant.
            lines = []
            write = self.write_line
            self.write_line = lambda text="": lines.append(text)
            try:
                self._emit_gemm_call(ctx, node)
            finally:
                self.write_line = write
            for text in lines:
                text = text.replace("nnc_gemm_nt(", "nnc_gemm_nt_relu(").replace("nnc_gemm(", "nnc_gemm_relu(")
                self.write_line(text)
            return
        if fused == "add_layernorm":
            sym = ctx.tensor_symbols
            a, b = node.inputs[:2]
            scale = f"&{sym[node.inputs[2]]}" if len(node.inputs) > 2 and node.inputs[2] else "NULL"
            bias = f"&{sym[node.inputs[3]]}" if len(node.inputs) > 3 and node.inputs[3] else "NULL"
            axis = node.attrs.get("axis", -1)
            eps = node.attrs.get("epsilon", 1e-5)
            self.write_line(f"nnc_add_layernorm(&{sym[a]}, &{sym[b]}, {scale}, {bias}, &{sym[node.outputs[0]]}, "
                            f"{axis}, {eps}f);")
            return
        if fused == "transpose_shaped":
            sym = ctx.tensor_symbols
            perm = [int(v) for v in node.attrs["perm"]]
            shape = [int(v) for v in node.metadata["in_shape"]]
            self.write_line("{")
            self.write_line(f"    static int64_t in_shape[{len(shape)}] = {{{', '.join(map(str, shape))}}};")
            self.write_line(f"    static int64_t perm[{len(perm)}] = {{{', '.join(map(str, perm))}}};")
            self.write_line(f"    nnc_transpose_shaped(&{sym[node.inputs[0]]}, &{sym[node.outputs[0]]}, in_shape, perm, "
                            f"{len(perm)});")
            self.write_line("}")
            return
        if fused == "gap_gemm":
            sym = ctx.tensor_symbols
            x, w = node.inputs[:2]
            c = node.inputs[2] if len(node.inputs) > 2 and node.inputs[2] else ""
            alpha = float(node.attrs.get("alpha", 1.0))
            beta = float(node.attrs.get("beta", 1.0))
            args = [f"&{sym[x]}", f"&{sym[w]}", f"&{sym[c]}" if c else "NULL", f"&{sym[node.outputs[0]]}",
                    f"{alpha!r}f", f"{beta!r}f"]
            self.write_line(f"nnc_gap_gemm_nt({', '.join(args)});")
            return
        if fused in ("matmul_bias", "matmul_scale_softmax"):
            sym = ctx.tensor_symbols
            args = [f"&{sym[t]}" for t in node.inputs] + [f"&{sym[node.outputs[0]]}"]
            if fused == "matmul_scale_softmax":
                args.append(f"{float(node.metadata['alpha'])!r}f")
            self.write_line(f"nnc_{fused}({', '.join(args)});")
            return
        if node.metadata.get("cuda_fused") == "conv_add_relu":
            sym = ctx.tensor_symbols
            x, w, b, r = node.inputs[:4]
            out = node.outputs[0]
            bias = f"&{sym[b]}" if b else "NULL"
            args = [f"&{sym[x]}", f"&{sym[w]}", bias, f"&{sym[r]}", f"&{sym[out]}"]
            kind = node.metadata.get("lowering", {}).get("kernel_kind")
            ks = node.attrs.get("kernel_shape", [1, 1])
            st = node.attrs.get("strides", [1, 1])
            pd = node.attrs.get("pads", [0, 0, 0, 0])
            if kind == "spatial_3x3":
                self.write_line(f"nnc_conv_add_relu3x3_s1({', '.join(args)});")
            elif kind == "pointwise_1x1":
                self.write_line(f"nnc_conv_add_relu1x1({', '.join(args + [str(st[0]), str(st[1]), str(pd[0]), str(pd[1])])});")
            else:
                extra = [str(ks[0]), str(ks[1]), str(st[0]), str(st[1]), str(pd[0]), str(pd[1])]
                self.write_line(f"nnc_conv_add_relu({', '.join(args + extra)});")
            return
        super()._emit_operator_call(ctx, node)


# ------------------------------------------------------------- backend ----
def _c_array(vals) -> str:
    return "{" + ", ".join(str(int(v)) for v in vals) + "}"


def _align(x: int, a: int = ARENA_ALIGN) -> int:
    return (x + a - 1) // a * a


def _packed_conv_bytes(shape) -> int:
    """Size of nnc_cuda_prepack_conv_weight's output (conv.cu weight_layout):
    hi + lo planes of [C_out][K_pad]; K_pad = C_in*KH*KW rounded up to 32 when
    that is <= 64 (element order; a 1 x 1 window over a multiple of 4
    channels takes the chunk order, which has the same K_pad), else
    KH*KW*C4 rounded up to 32 with C4 = C_in rounded up to 4 (chunk order)."""
    cout, cin, kh, kw = (int(s) for s in shape)
    ke = (cin * kh * kw + 31) // 32 * 32
    kpad = ke if ke <= 64 else (kh * kw * ((cin + 3) // 4 * 4) + 31) // 32 * 32
    return 2 * cout * kpad * 4


class CudaBackend(BackendBase):
    """Backend for ``Compiler(target="cuda")`` (see module docstring)."""

    def __init__(self, debug_mode: bool = False, channels_last: bool = True):
        self.debug_mode = debug_mode
        self.channels_last = channels_last

    def generate(self, ctx: CompileContext) -> CodeGenResult:
        self._assign_symbols(ctx)
        res = CodeGenResult()
        plan = ctx.metadata.get("memory_allocation_plan")
        if plan is None:
            raise ValueError("cuda target needs a memory plan (run liveness + memory planning)")
        layout = channels_last_tensors(ctx) if self.channels_last else set()
        arena, arena_bytes = self._arena_offsets(ctx, plan)
        consts, const_bytes = self._const_layout(ctx)
        entry = ctx.metadata.get("entry_point", "nnc_run")
        model_c = CudaEmitter().emit(ctx)
        if self.debug_mode:
            model_c = inject_debug_dumps(model_c, ctx)
        res.add_file("model.c", model_c, "source")
        res.add_file("model.h", self._model_h(ctx, entry), "header")
        res.add_file("tensors.c", self._tensors_c(ctx, arena, arena_bytes, consts, const_bytes, layout), "source")
        res.add_file("constants_loader.c", _CONSTANTS_LOADER, "source")
        res.add_file("model_runtime.c", _MODEL_RUNTIME + (_DEBUG_RUNTIME if self.debug_mode else ""), "source")
        runner = self._runner_c(ctx)
        if self.debug_mode:
            runner = runner.replace("    int avail = 0;\n", "    int avail = 0;\n"
                                    "    if (nnc_model_set_debug_file(\"nnc_debug_output.txt\") != 0) return 1;\n", 1)
        res.add_file("test_runner.c", runner, "source")
        res.add_file("Makefile", _MAKEFILE, "build")
        manifest = {
            "graph": ctx.graph.name,
            "inputs": [{"name": n, "symbol": ctx.tensor_symbols[n], "shape": list(map(int, ctx.graph.tensors[n].shape.dims))} for n in ctx.graph.inputs],
            "outputs": [{"name": n, "symbol": ctx.tensor_symbols[n], "shape": list(map(int, ctx.graph.tensors[n].shape.dims))} for n in ctx.graph.outputs],
            "constants": [{"name": c["name"], "symbol": c["symbol"], "shape": c["shape"]} for c in consts],
            "arena_bytes": arena_bytes,
            "const_bytes": const_bytes,
            "channels_last": sorted(ctx.tensor_symbols[t] for t in layout),
            "calls": re.findall(r"\b(nnc_[a-z0-9_]+)\(&", res.files[0].content),
        }
        res.add_file("manifest.json", json.dumps(manifest, indent=1) + "\n", "build")
        res.metadata["manifest"] = manifest
        return res

    # symbols as nnc-py's x86 backend names them (x86_backend.py:3563-3576)
    def _assign_symbols(self, ctx: CompileContext) -> None:
        nm = NameManager()
        for t in ctx.graph.tensors:
            ctx.tensor_symbols[t] = nm.get_symbol(t, prefix="tensor_")
        for n in ctx.graph.nodes:
            ctx.node_symbols[n] = nm.get_symbol(n, prefix="node_")

    def _arena_offsets(self, ctx, plan):
        """Byte offsets of every activation in the single device arena: the
        cost_aware plan's offsets as they are (aliases and reuse included;
        the plan aligns to 16 bytes, which is what the kernels' vector and
        TMA paths need). Tensors the plan leaves out are appended."""
        offsets = {name: int(a.offset) for name, a in plan.tensor_allocations.items()}
        end = max([int(plan.total_fast_memory)] +
                  [int(a.offset) + int(a.size) for a in plan.tensor_allocations.values()])
        for t in list(ctx.graph.inputs) + list(ctx.graph.outputs):
            if t not in offsets:
                offsets[t] = _align(end)
                end = offsets[t] + _align(int(np.prod(ctx.graph.tensors[t].shape.dims)) * 4)
        for t, tt in ctx.graph.tensors.items():
            if t in ctx.graph.constants or t in offsets:
                continue
            used = any(t in n.inputs or t in n.outputs for n in ctx.graph.nodes.values())
            if used:
                offsets[t] = _align(end)
                end = offsets[t] + _align(int(np.prod(tt.shape.dims)) * 4)
        return offsets, _align(end)

    def _const_layout(self, ctx):
        conv_weights = set()
        for n in ctx.graph.nodes.values():
            if n.op_type in (OpType.CONV2D, OpType.FUSED_CONV_RELU, OpType.FUSED_CONV_SIGMOID,
                             OpType.FUSED_CONV_BIAS_RELU) and len(n.inputs) > 1 and n.inputs[1] in ctx.graph.constants:
                conv_weights.add(n.inputs[1])
        consts, off = [], 0
        for name, arr in ctx.graph.constants.items():
            arr = np.asarray(arr)
            entry = {"name": name, "symbol": ctx.tensor_symbols[name], "shape": [int(s) for s in arr.shape],
                     "nbytes": int(arr.nbytes), "offset": off, "packed_offset": -1, "packed_bytes": 0}
            off = _align(off + int(arr.nbytes))
            consts.append(entry)
        for e in consts:
            if e["name"] in conv_weights and len(e["shape"]) == 4:
                e["packed_offset"] = off
                e["packed_bytes"] = _packed_conv_bytes(e["shape"])
                off = _align(off + e["packed_bytes"])
        return consts, _align(max(off, ARENA_ALIGN))

    def _model_h(self, ctx, entry):
        ins = ", ".join(ctx.tensor_symbols[n] for n in ctx.graph.inputs)
        outs = ", ".join(ctx.tensor_symbols[n] for n in ctx.graph.outputs)
        debug_decls = ("/* Debug build: every intermediate tensor is dumped after its node, in\n"
                       " * nnc-py's x86 debug-dump text format, to this file (NULL: stdout). */\n"
                       "int nnc_model_set_debug_file(const char* path);\n"
                       "void nnc_model_debug_dump(const char* name, int node_idx, const Tensor* t);\n"
                       ) if self.debug_mode else ""
        return f"""/* Auto-generated by nnc_cuda (cuda target) - DO NOT EDIT */
#ifndef NNC_MODEL_H
#define NNC_MODEL_H

#include <stddef.h>
#include "nnc_types.h"

#ifdef __cplusplus
extern "C" {{
#endif

/* Inputs: {ins}; outputs: {outs}. Tensor data are device pointers. */

/* Enqueues the forward pass on the calling thread's current stream
 * (nnc_cuda_set_stream); returns without synchronising. */
void {entry}(void);

/* Selects `device`, allocates its activation arena and constant slab
 * (one cudaMalloc each) and binds the tensors to them. */
int nnc_model_init(int device);
/* Rebinds the tensors to an initialised device's arena / constants. */
int nnc_model_select(int device);
void nnc_model_free(int device);
/* Reads an NNCB v1 constants file, uploads it to the selected device and
 * prepacks the conv weights there. Call once per device. */
int nnc_load_constants(const char* path);
int nnc_load_constants_from_memory(const void* data, size_t size);
size_t nnc_model_arena_bytes(void);
size_t nnc_model_const_bytes(void);
int nnc_model_num_inputs(void);
int nnc_model_num_outputs(void);
Tensor* nnc_model_input(int i);
Tensor* nnc_model_output(int i);
/* Synchronous host-buffer forward on the selected device: input host ->
 * device, forward, output device -> host (pinned buffers recommended). */
int nnc_model_run_host(const void* input, void* output);
{debug_decls}
#ifdef __cplusplus
}}
#endif

#endif
"""

    def _tensors_c(self, ctx, arena, arena_bytes, consts, const_bytes, layout):
        g = ctx.graph
        L = ["/* Auto-generated by nnc_cuda (cuda target) - DO NOT EDIT */",
             "#include <stddef.h>", "#include <stdint.h>", '#include "nnc_types.h"', '#include "nnc_cuda.h"',
             '#include "nnc_model_tables.h"', "",
             f"const size_t nnc_arena_bytes = {arena_bytes}u;",
             f"const size_t nnc_const_bytes = {const_bytes}u;", ""]
        act_entries, const_entries = [], []
        for name, tt in g.tensors.items():
            sym = ctx.tensor_symbols[name]
            dims = [int(d) for d in tt.shape.dims]
            n = int(np.prod(dims)) if dims else 1
            is_const = name in g.constants
            if not is_const and name not in arena:
                continue
            tag = " | NNC_CUDA_TAG_NHWC" if name in layout else ""
            L.append(f"static int64_t {sym}_dims[] = {_c_array(dims or [1])};")
            L.append(f"Tensor {sym} = {{.data = NULL, .dtype = (nnc_dtype_t)(NNC_DTYPE_FLOAT32{tag}), "
                     f".shape = {sym}_dims, .ndim = {len(dims)}, .nbytes = {n * 4}}};")
            if not is_const:
                act_entries.append(f"    {{&{sym}, {arena[name]}u}},")
        L.append("")
        for c in consts:
            const_entries.append(f'    {{"{c["symbol"]}", &{c["symbol"]}, {c["offset"]}u, {c["packed_offset"]}, '
                                 f'{c["packed_bytes"]}u, {c["nbytes"]}u}},')
        L.append("const nnc_arena_entry nnc_arena_table[] = {")
        L += act_entries or ["    {NULL, 0u},"]
        L.append("};")
        L.append(f"const int nnc_arena_count = {len(act_entries)};")
        L.append("const nnc_const_entry nnc_const_table[] = {")
        L += const_entries or ['    {"", NULL, 0u, -1, 0u, 0u},']
        L.append("};")
        L.append(f"const int nnc_const_count = {len(const_entries)};")
        L.append("Tensor* const nnc_input_table[] = {" + ", ".join(f"&{ctx.tensor_symbols[n]}" for n in g.inputs) + "};")
        L.append(f"const int nnc_input_count = {len(g.inputs)};")
        L.append("Tensor* const nnc_output_table[] = {" + ", ".join(f"&{ctx.tensor_symbols[n]}" for n in g.outputs) + "};")
        L.append(f"const int nnc_output_count = {len(g.outputs)};")
        return "\n".join(L) + "\n"

    def _runner_c(self, ctx):
        return _TEST_RUNNER


_TABLES_H = """/* Shared declarations of the generated tables (cuda target). */
#ifndef NNC_MODEL_TABLES_H
#define NNC_MODEL_TABLES_H
#include <stddef.h>
#include "nnc_types.h"
typedef struct { Tensor* tensor; size_t offset; } nnc_arena_entry;
typedef struct {
    const char* symbol; Tensor* tensor; size_t offset; long long packed_offset;
    size_t packed_bytes; size_t nbytes;
} nnc_const_entry;
extern const size_t nnc_arena_bytes, nnc_const_bytes;
extern const nnc_arena_entry nnc_arena_table[];
extern const int nnc_arena_count;
extern const nnc_const_entry nnc_const_table[];
extern const int nnc_const_count;
extern Tensor* const nnc_input_table[];
extern const int nnc_input_count;
extern Tensor* const nnc_output_table[];
extern const int nnc_output_count;
#endif
"""

_MODEL_RUNTIME = r"""/* Auto-generated by nnc_cuda (cuda target) - DO NOT EDIT
 * Device arena / constant slab management: one cudaMalloc each per device;
 * the Tensor globals are rebound when another device is selected. */
#include <cuda_runtime.h>
#include <stdio.h>
#include "model.h"
#include "nnc_cuda.h"
#include "nnc_model_tables.h"

#define NNC_MAX_DEVICES 16
typedef struct { char* arena; char* slab; int ready; int packed; } nnc_device_state;
static nnc_device_state g_dev[NNC_MAX_DEVICES];
static int g_cur = -1;

static int report(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return 0;
    fprintf(stderr, "nnc_model: %s: %s\n", what, cudaGetErrorString(e));
    return 1;
}

size_t nnc_model_arena_bytes(void) { return nnc_arena_bytes; }
size_t nnc_model_const_bytes(void) { return nnc_const_bytes; }
int nnc_model_num_inputs(void) { return nnc_input_count; }
int nnc_model_num_outputs(void) { return nnc_output_count; }
Tensor* nnc_model_input(int i) { return (i >= 0 && i < nnc_input_count) ? nnc_input_table[i] : NULL; }
Tensor* nnc_model_output(int i) { return (i >= 0 && i < nnc_output_count) ? nnc_output_table[i] : NULL; }

int nnc_model_select(int device) {
    if (device < 0 || device >= NNC_MAX_DEVICES || !g_dev[device].ready) return 1;
    if (report(cudaSetDevice(device), "cudaSetDevice")) return 1;
    nnc_cuda_init(device);
    for (int i = 0; i < nnc_arena_count; ++i)
        nnc_arena_table[i].tensor->data = g_dev[device].arena + nnc_arena_table[i].offset;
    for (int i = 0; i < nnc_const_count; ++i) {
        const nnc_const_entry* c = &nnc_const_table[i];
        const int packed = g_dev[device].packed && c->packed_offset >= 0;
        c->tensor->data = g_dev[device].slab + (packed ? (size_t)c->packed_offset : c->offset);
    }
    g_cur = device;
    return 0;
}

int nnc_model_init(int device) {
    if (device < 0 || device >= NNC_MAX_DEVICES) return 1;
    if (g_dev[device].ready) return nnc_model_select(device);
    if (report(cudaSetDevice(device), "cudaSetDevice")) return 1;
    if (nnc_cuda_init(device) != 0) return 1;
    if (report(cudaMalloc((void**)&g_dev[device].arena, nnc_arena_bytes), "arena cudaMalloc")) return 1;
    if (report(cudaMalloc((void**)&g_dev[device].slab, nnc_const_bytes), "constant slab cudaMalloc")) return 1;
    g_dev[device].ready = 1;
    g_dev[device].packed = 0;
    return nnc_model_select(device);
}

void nnc_model_free(int device) {
    if (device < 0 || device >= NNC_MAX_DEVICES || !g_dev[device].ready) return;
    cudaSetDevice(device);
    cudaFree(g_dev[device].arena);
    cudaFree(g_dev[device].slab);
    g_dev[device].ready = 0;
    if (g_cur == device) g_cur = -1;
}

/* Used by the constants loader. */
char* nnc_model_slab(void) { return g_cur >= 0 ? g_dev[g_cur].slab : NULL; }
void nnc_model_mark_packed(void) { if (g_cur >= 0) g_dev[g_cur].packed = 1; }
int nnc_model_is_packed(void) { return g_cur >= 0 ? g_dev[g_cur].packed : 0; }

int nnc_model_run_host(const void* input, void* output) {
    if (g_cur < 0) return 1;
    cudaStream_t s = (cudaStream_t)nnc_cuda_get_stream();
    Tensor* in = nnc_input_table[0];
    Tensor* out = nnc_output_table[0];
    if (report(cudaMemcpyAsync(in->data, input, (size_t)in->nbytes, cudaMemcpyHostToDevice, s), "input copy")) return 1;
    nnc_run();
    if (report(cudaMemcpyAsync(output, out->data, (size_t)out->nbytes, cudaMemcpyDeviceToHost, s), "output copy")) return 1;
    if (report(cudaStreamSynchronize(s), "sync")) return 1;
    return nnc_cuda_get_last_error();
}
"""

# Debug builds (CudaBackend(debug_mode=True)): every intermediate tensor is
# written after its node in the text format of nnc-py's x86 debug builds
# (codegen/x86_emitters/model_source.py, debug dumps), which nnc-py's
# DebugOutputParser (tools/debug_compare.py) reads: DEBUG_TENSOR_START
# <name> <node index>, SHAPE <ndim>, DIM <i> <extent> lines, DATA_START, one
# "%f" line per element in logical (NCHW, row-major) order, DATA_END,
# DEBUG_TENSOR_END <name>. Channels-last tensors are reordered to NCHW.
_DEBUG_RUNTIME = r"""
/* ---- debug dumps (debug builds only) ---- */
#include <stdlib.h>
static FILE* g_debug_file = NULL;

/* Where the dumps go (NULL: stdout, as in nnc-py's x86 debug builds). */
int nnc_model_set_debug_file(const char* path) {
    if (g_debug_file) fclose(g_debug_file);
    g_debug_file = NULL;
    if (!path) return 0;
    g_debug_file = fopen(path, "w");
    return g_debug_file ? 0 : 1;
}

/* Waits for the current stream, copies the tensor to the host and writes it. */
void nnc_model_debug_dump(const char* name, int node_idx, const Tensor* t) {
    FILE* f = g_debug_file ? g_debug_file : stdout;
    if (report(cudaStreamSynchronize((cudaStream_t)nnc_cuda_get_stream()), "debug dump sync")) return;
    size_t n = 1;
    for (int i = 0; i < t->ndim; ++i) n *= (size_t)t->shape[i];
    float* h = (float*)malloc(n * sizeof(float) + 1);
    float* o = (float*)malloc(n * sizeof(float) + 1);
    if (!h || !o) { free(h); free(o); return; }
    if (n && report(cudaMemcpy(h, t->data, n * sizeof(float), cudaMemcpyDeviceToHost), "debug dump copy")) {
        free(h); free(o); return;
    }
    const float* v = h;
    if ((t->dtype & NNC_CUDA_TAG_NHWC) && t->ndim == 4) {
        const size_t N = (size_t)t->shape[0], C = (size_t)t->shape[1], H = (size_t)t->shape[2], W = (size_t)t->shape[3];
        for (size_t b = 0; b < N; ++b)
            for (size_t y = 0; y < H; ++y)
                for (size_t x = 0; x < W; ++x)
                    for (size_t c = 0; c < C; ++c)
                        o[((b * C + c) * H + y) * W + x] = h[((b * H + y) * W + x) * C + c];
        v = o;
    }
    fprintf(f, "DEBUG_TENSOR_START %s %d\n", name, node_idx);
    fprintf(f, "SHAPE %d\n", t->ndim);
    for (int i = 0; i < t->ndim; ++i) fprintf(f, "DIM %d %d\n", i, (int)t->shape[i]);
    fprintf(f, "DATA_START\n");
    for (size_t i = 0; i < n; ++i) fprintf(f, "%f\n", v[i]);
    fprintf(f, "DATA_END\n");
    fprintf(f, "DEBUG_TENSOR_END %s\n\n", name);
    fflush(f);
    free(h);
    free(o);
}
"""


def inject_debug_dumps(model_c: str, ctx: CompileContext) -> str:
    """Adds, after each node call in nnc_run, a dump of the node's
    non-constant outputs (node index = position among the non-constant nodes
    in topological order, as nnc-py's x86 debug builds number them)."""
    g = ctx.graph
    after: dict[str, list[str]] = {}
    idx = 0
    for node in g.topological_sort():
        if node.op_type == OpType.CONSTANT:
            continue
        sym = ctx.node_symbols.get(node.name, node.name)
        after[f"{sym}();"] = [
            f'    nnc_model_debug_dump("{t}", {idx}, &{ctx.tensor_symbols[t]});'
            for t in node.outputs if t in g.tensors and t not in g.constants]
        idx += 1
    out, in_run = [], False
    for line in model_c.split("\n"):
        out.append(line)
        if line.startswith("void nnc_run(void)"):
            in_run = True
            continue
        if in_run:
            if line.startswith("}"):
                in_run = False
            else:
                out.extend(after.get(line.strip(), []))
    src = "\n".join(out)
    decl = "void nnc_model_debug_dump(const char* name, int node_idx, const Tensor* t);\n"
    first_fn = src.index("void node_") if "void node_" in src else src.index("void nnc_run")
    return src[:first_fn] + decl + "\n" + src[first_fn:]


_CONSTANTS_LOADER = r"""/* Auto-generated by nnc_cuda (cuda target) - DO NOT EDIT
 * Loads nnc-py's NNCB v1 constants container: 'NNCB', u32 version (1),
 * u32 count, then per constant u32 name_len, name (NUL-terminated), u32
 * dtype, u32 ndim, i64 shape[ndim], u64 nbytes, data. Entries must appear in
 * the order and with the names/sizes of the generated table (as nnc-py's x86
 * loader requires). Data go to the selected device's constant slab; conv
 * weights are then prepacked on the device (nnc_cuda_prepack_conv_weight). */
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include "model.h"
#include "nnc_cuda.h"
#include "nnc_model_tables.h"

char* nnc_model_slab(void);
void nnc_model_mark_packed(void);
int nnc_model_is_packed(void);

static int rd(const unsigned char** p, const unsigned char* end, void* dst, size_t n) {
    if ((size_t)(end - *p) < n) return 1;
    memcpy(dst, *p, n);
    *p += n;
    return 0;
}

int nnc_load_constants_from_memory(const void* data, size_t size) {
    const unsigned char* p = (const unsigned char*)data;
    const unsigned char* end = p + size;
    char* slab = nnc_model_slab();
    uint32_t version = 0, count = 0;
    if (!slab) { fprintf(stderr, "nnc_load_constants: no device selected\n"); return 1; }
    if (size < 12 || memcmp(p, "NNCB", 4) != 0) { fprintf(stderr, "nnc_load_constants: bad magic\n"); return 1; }
    p += 4;
    if (rd(&p, end, &version, 4) || version != 1) { fprintf(stderr, "nnc_load_constants: unsupported version %u\n", version); return 1; }
    if (rd(&p, end, &count, 4) || (int)count != nnc_const_count) {
        fprintf(stderr, "nnc_load_constants: %u constants in file, model has %d\n", count, nnc_const_count);
        return 1;
    }
    for (int i = 0; i < nnc_const_count; ++i) {
        const nnc_const_entry* c = &nnc_const_table[i];
        uint32_t name_len = 0, dtype = 0, ndim = 0;
        uint64_t nbytes = 0;
        if (rd(&p, end, &name_len, 4) || name_len == 0 || (size_t)(end - p) < name_len) return 1;
        if (strncmp((const char*)p, c->symbol, name_len) != 0) {
            fprintf(stderr, "nnc_load_constants: entry %d is '%.*s', expected '%s'\n", i, (int)name_len, (const char*)p, c->symbol);
            return 1;
        }
        p += name_len;
        if (rd(&p, end, &dtype, 4) || rd(&p, end, &ndim, 4) || ndim > 8) return 1;
        if ((size_t)(end - p) < 8u * ndim) return 1;
        p += 8u * ndim;
        if (rd(&p, end, &nbytes, 8) || nbytes != c->nbytes || (uint64_t)(end - p) < nbytes) {
            fprintf(stderr, "nnc_load_constants: '%s' has %llu bytes, expected %zu\n", c->symbol, (unsigned long long)nbytes, c->nbytes);
            return 1;
        }
        if (cudaMemcpy(slab + c->offset, p, nbytes, cudaMemcpyHostToDevice) != cudaSuccess) return 1;
        p += nbytes;
    }
    if (!nnc_model_is_packed()) {
        for (int i = 0; i < nnc_const_count; ++i) {
            const nnc_const_entry* c = &nnc_const_table[i];
            if (c->packed_offset < 0) continue;
            c->tensor->data = slab + c->offset;
            c->tensor->dtype = (nnc_dtype_t)((int)c->tensor->dtype & NNC_CUDA_DTYPE_MASK);
            if (nnc_cuda_prepack_conv_weight(c->tensor, slab + c->packed_offset, c->packed_bytes) != 0) return 1;
        }
        nnc_model_mark_packed();
    } else {
        /* Re-upload on an already packed device: repack from the fresh raw data. */
        for (int i = 0; i < nnc_const_count; ++i) {
            const nnc_const_entry* c = &nnc_const_table[i];
            if (c->packed_offset < 0) continue;
            int tagged = (int)c->tensor->dtype;
            c->tensor->data = slab + c->offset;
            c->tensor->dtype = (nnc_dtype_t)(tagged & NNC_CUDA_DTYPE_MASK);
            if (nnc_cuda_prepack_conv_weight(c->tensor, slab + c->packed_offset, c->packed_bytes) != 0) return 1;
        }
    }
    if (cudaStreamSynchronize((cudaStream_t)nnc_cuda_get_stream()) != cudaSuccess) return 1;
    return nnc_cuda_get_last_error();
}

int nnc_load_constants(const char* path) {
    FILE* f = fopen(path, "rb");
    if (!f) { fprintf(stderr, "nnc_load_constants: cannot open %s\n", path); return 1; }
    fseek(f, 0, SEEK_END);
    long n = ftell(f);
    fseek(f, 0, SEEK_SET);
    void* buf = malloc((size_t)n);
    int rc = (buf && fread(buf, 1, (size_t)n, f) == (size_t)n) ? nnc_load_constants_from_memory(buf, (size_t)n) : 1;
    free(buf);
    fclose(f);
    return rc;
}
"""

_TEST_RUNNER = r"""/* Auto-generated by nnc_cuda (cuda target) - DO NOT EDIT
 * Usage: ./model constants.bin input.bin output.bin [num_gpus] [iters]
 * input.bin holds num_gpus x (compiled batch) samples; GPU g runs samples
 * [g*B, (g+1)*B) with its own arena and constants; the outputs are gathered
 * to GPU 0 (peer copies over NVLink) and written to output.bin. With
 * iters > 0 the forward is timed with CUDA events (max over GPUs). */
#include <cuda_runtime.h>
#include <stdio.h>
#include <stdlib.h>
#include "model.h"
#include "nnc_cuda.h"

#define CHECK(x) do { cudaError_t e_ = (x); if (e_ != cudaSuccess) { fprintf(stderr, "%s: %s\n", #x, cudaGetErrorString(e_)); return 1; } } while (0)

int main(int argc, char** argv) {
    if (argc < 4) { fprintf(stderr, "usage: %s constants.bin input.bin output.bin [num_gpus] [iters]\n", argv[0]); return 2; }
    int gpus = argc > 4 ? atoi(argv[4]) : 1;
    int iters = argc > 5 ? atoi(argv[5]) : 0;
    int avail = 0;
    CHECK(cudaGetDeviceCount(&avail));
    if (gpus < 1 || gpus > avail || gpus > 16) { fprintf(stderr, "need %d GPUs, have %d\n", gpus, avail); return 2; }
    Tensor* in = nnc_model_input(0);
    Tensor* out = nnc_model_output(0);
    size_t in_b = (size_t)in->nbytes, out_b = (size_t)out->nbytes;
    FILE* f = fopen(argv[2], "rb");
    if (!f) { fprintf(stderr, "cannot open %s\n", argv[2]); return 1; }
    char* host_in = NULL;
    char* host_out = NULL;
    CHECK(cudaMallocHost((void**)&host_in, in_b * gpus));
    CHECK(cudaMallocHost((void**)&host_out, out_b * gpus));
    if (fread(host_in, 1, in_b * gpus, f) != in_b * gpus) { fprintf(stderr, "input.bin must hold %zu bytes\n", in_b * gpus); return 1; }
    fclose(f);
    cudaStream_t streams[16];
    cudaEvent_t t0[16], t1[16];
    void* out_dev[16];
    for (int g = 0; g < gpus; ++g) {
        if (nnc_model_init(g) != 0) return 1;
        CHECK(cudaStreamCreateWithFlags(&streams[g], cudaStreamNonBlocking));
        nnc_cuda_set_stream(streams[g]);
        if (nnc_load_constants(argv[1]) != 0) { fprintf(stderr, "constants failed on GPU %d\n", g); return 1; }
        CHECK(cudaEventCreate(&t0[g]));
        CHECK(cudaEventCreate(&t1[g]));
        out_dev[g] = out->data;
        if (g > 0) { int ok = 0; cudaDeviceCanAccessPeer(&ok, 0, g); if (ok) { cudaSetDevice(0); cudaDeviceEnablePeerAccess(g, 0); cudaSetDevice(g); } }
    }
    void* gather = NULL;
    nnc_model_select(0);
    CHECK(cudaMalloc(&gather, out_b * gpus));
    int reps = iters > 0 ? iters : 1;
    float worst = 0.f;
    for (int it = 0; it < reps + (iters > 0 ? 1 : 0); ++it) {
        for (int g = 0; g < gpus; ++g) {
            nnc_model_select(g);
            nnc_cuda_set_stream(streams[g]);
            CHECK(cudaMemcpyAsync(in->data, host_in + (size_t)g * in_b, in_b, cudaMemcpyHostToDevice, streams[g]));
            CHECK(cudaEventRecord(t0[g], streams[g]));
            nnc_run();
            CHECK(cudaEventRecord(t1[g], streams[g]));
        }
        for (int g = 0; g < gpus; ++g) {
            CHECK(cudaSetDevice(g));
            CHECK(cudaStreamSynchronize(streams[g]));
            float ms = 0.f;
            CHECK(cudaEventElapsedTime(&ms, t0[g], t1[g]));
            if (it > 0 || iters == 0) worst = ms > worst ? ms : worst;
        }
    }
    CHECK(cudaSetDevice(0));
    for (int g = 0; g < gpus; ++g)
        CHECK(cudaMemcpyPeerAsync((char*)gather + (size_t)g * out_b, 0, out_dev[g], g, out_b, streams[0]));
    CHECK(cudaMemcpyAsync(host_out, gather, out_b * gpus, cudaMemcpyDeviceToHost, streams[0]));
    CHECK(cudaStreamSynchronize(streams[0]));
    if (nnc_cuda_get_last_error() != 0) { fprintf(stderr, "runtime error: %s\n", nnc_cuda_get_last_error_string()); return 1; }
    f = fopen(argv[3], "wb");
    if (!f || fwrite(host_out, 1, out_b * gpus, f) != out_b * gpus) return 1;
    fclose(f);
    printf("forward over %d GPU(s): %.3f ms (max over GPUs)\n", gpus, worst);
    return 0;
}
"""

_MAKEFILE = """# Auto-generated by nnc_cuda (cuda target) - DO NOT EDIT
# NNC_CUDA_ROOT: repository root holding include/ and nnc-py_b200/nnc_cuda/libnnc_cuda.so
NNC_CUDA_ROOT ?= ../../..
NVCC ?= nvcc
CFLAGS = -O2 -arch=sm_100a -Xcompiler -fPIC -I. -I$(NNC_CUDA_ROOT)/include
LIBDIR = $(NNC_CUDA_ROOT)/nnc-py_b200/nnc_cuda
LDFLAGS = -L$(LIBDIR) -lnnc_cuda -Xlinker -rpath,$(abspath $(LIBDIR))
SRCS = model.c tensors.c constants_loader.c model_runtime.c

all: libmodel.so model

libmodel.so: $(SRCS) model.h nnc_model_tables.h
\t$(NVCC) $(CFLAGS) -x cu -shared -o $@ $(SRCS) $(LDFLAGS)

model: test_runner.c libmodel.so
\t$(NVCC) $(CFLAGS) -x cu -o $@ test_runner.c -L. -lmodel -Xlinker -rpath,'$$ORIGIN' $(LDFLAGS)

clean:
\trm -f libmodel.so model

.PHONY: all clean
"""


def compile_model(model: Model, out_dir: str | pathlib.Path, opt_level: int = 3,
                  channels_last: bool = True, fuse_conv_relu_maxpool: bool | None = None,
                  debug: bool = False) -> dict[str, Any]:
    """Runs the cuda target on a workload Model and writes the artifacts."""
    ctx = CompileContext(to_nnc_graph(model), "cuda", opt_level)
    ctx.metadata["entry_point"] = "nnc_run"
    pm = PassManager()
    for p in cuda_passes(opt_level, fuse_conv_relu_maxpool):
        pm.register(p)
    pm.run(ctx)
    res = CudaBackend(debug_mode=debug, channels_last=channels_last).generate(ctx)
    out = pathlib.Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    for a in res.files:
        (out / a.filename).write_text(a.content) if isinstance(a.content, str) else (out / a.filename).write_bytes(a.content)
    (out / "nnc_model_tables.h").write_text(_TABLES_H)
    return res.metadata["manifest"]


def install() -> None:
    """Adds the ``cuda`` target to nnc-py's Compiler and CLI in-process."""
    from nnc_py import cli as nnc_cli
    from nnc_py import compiler as nnc_compiler

    orig_create = nnc_compiler.Compiler._create_backend
    orig_passes = nnc_compiler.Compiler._get_passes

    def _create_backend(self, target):
        if target == "cuda":
            return CudaBackend(debug_mode=self.debug_mode)
        return orig_create(self, target)

    def _get_passes(self):
        if self.target == "cuda":
            return cuda_passes(self.opt_level)
        return orig_passes(self)

    nnc_compiler.Compiler._create_backend = _create_backend
    nnc_compiler.Compiler._get_passes = _get_passes
    for p in nnc_cli.compile.params:
        if p.name == "target" and "cuda" not in p.type.choices:
            p.type.choices = list(p.type.choices) + ["cuda"]

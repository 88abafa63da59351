"""The BASELINE configurations as seeded operator graphs (pure numpy).

Each builder returns a :class:`Model`: tensors with shapes, constants, and
nodes in topological order, using nnc-py's operator names (ir/node.py
OpType values) and ONNX attributes. The codegen turns a Model into an
nnc-py ``Graph``; the bench and the model-level tests use the same Model to
produce identical weights and inputs on machines without nnc-py.

Seeds: weights come from ``numpy.random.default_rng(0)`` drawn in node order
(weight, then bias); inputs from ``default_rng(1)``, so the first k images
of any batch are the same images. Initialisers:
  * conv / FC weights: Kaiming-uniform U(+-sqrt(6 / fan_in));
  * transformer projections: Xavier-uniform U(+-sqrt(6 / (fan_in + fan_out)));
  * biases: U(-0.01, 0.01); LayerNorm gamma = 1, beta = 0.
BatchNorm is folded into the conv weights/bias (the model has none).
"""

from __future__ import annotations

import dataclasses
import io
import struct
from typing import Callable

import numpy as np


@dataclasses.dataclass
class Node:
    op: str
    name: str
    inputs: list[str]
    outputs: list[str]
    attrs: dict = dataclasses.field(default_factory=dict)


@dataclasses.dataclass
class Model:
    name: str
    batch: int
    inputs: list[str]
    outputs: list[str]
    shapes: dict[str, tuple[int, ...]]
    constants: dict[str, np.ndarray]
    nodes: list[Node]
    flops_per_sample: float = 0.0

    def input_array(self, batch: int | None = None, offset: int = 0) -> np.ndarray:
        """Seeded input batch (images offset .. offset + batch of the stream)."""
        n = self.batch if batch is None else batch
        shape = self.shapes[self.inputs[0]]
        per = int(np.prod(shape[1:]))
        rng = np.random.default_rng(1)
        flat = rng.standard_normal((offset + n) * per, dtype=np.float32)[offset * per:]
        return flat.reshape((n,) + tuple(shape[1:]))


class _Builder:
    def __init__(self, name: str, batch: int):
        self.m = Model(name, batch, [], [], {}, {}, [])
        self.rng = np.random.default_rng(0)
        self.count = 0

    def tensor(self, name, shape):
        self.m.shapes[name] = tuple(int(s) for s in shape)
        return name

    def const(self, name, arr):
        self.m.constants[name] = np.ascontiguousarray(arr, dtype=np.float32)
        self.m.shapes[name] = tuple(arr.shape)
        return name

    def node(self, op, inputs, outputs, **attrs):
        self.count += 1
        self.m.nodes.append(Node(op, f"{op.lower()}_{self.count}", list(inputs), list(outputs), attrs))

    def kaiming(self, shape, fan_in):
        b = np.sqrt(6.0 / fan_in)
        return self.rng.uniform(-b, b, shape).astype(np.float32)

    def bias(self, n):
        return self.rng.uniform(-0.01, 0.01, n).astype(np.float32)


def _conv_out(h, k, s, p):
    return (h + 2 * p - k) // s + 1


def resnet18(batch: int) -> Model:
    """ResNet-18, 224x224, BN folded (configs 3 and 5 of BASELINE.json)."""
    B = _Builder("resnet18", batch)
    N = batch
    x = B.tensor("input", (N, 3, 224, 224))
    B.m.inputs = [x]
    flops = 0.0

    def conv(inp, cin, cout, k, s, p, tag):
        nonlocal flops
        _, _, h, w = B.m.shapes[inp]
        oh, ow = _conv_out(h, k, s, p), _conv_out(w, k, s, p)
        wn = B.const(f"{tag}_w", B.kaiming((cout, cin, k, k), cin * k * k))
        bn = B.const(f"{tag}_b", B.bias(cout))
        out = B.tensor(f"{tag}_out", (N, cout, oh, ow))
        B.node("Conv", [inp, wn, bn], [out], kernel_shape=[k, k], strides=[s, s], pads=[p, p, p, p])
        flops += 2.0 * cout * oh * ow * cin * k * k
        return out

    def relu(inp, tag):
        out = B.tensor(f"{tag}_relu", B.m.shapes[inp])
        B.node("Relu", [inp], [out])
        return out

    c1 = relu(conv(x, 3, 64, 7, 2, 3, "conv1"), "conv1")
    p1 = B.tensor("pool1", (N, 64, 56, 56))
    B.node("MaxPool", [c1], [p1], kernel_shape=[3, 3], strides=[2, 2], pads=[1, 1, 1, 1])
    cur, cin = p1, 64
    for stage, cout in enumerate((64, 128, 256, 512), start=1):
        for blk in range(2):
            s = 2 if (stage > 1 and blk == 0) else 1
            tag = f"layer{stage}_{blk}"
            a = relu(conv(cur, cin, cout, 3, s, 1, f"{tag}_conv1"), f"{tag}_conv1")
            bb = conv(a, cout, cout, 3, 1, 1, f"{tag}_conv2")
            sc = conv(cur, cin, cout, 1, s, 0, f"{tag}_down") if (s != 1 or cin != cout) else cur
            summed = B.tensor(f"{tag}_sum", B.m.shapes[bb])
            B.node("Add", [bb, sc], [summed])
            cur, cin = relu(summed, f"{tag}_out"), cout
    gap = B.tensor("gap", (N, 512, 1, 1))
    B.node("GlobalAveragePool", [cur], [gap])
    flat = B.tensor("flat", (N, 512))
    B.node("Flatten", [gap], [flat], axis=1)
    fw = B.const("fc_w", B.kaiming((1000, 512), 512))
    fb = B.const("fc_b", B.bias(1000))
    logits = B.tensor("logits", (N, 1000))
    B.node("Gemm", [flat, fw, fb], [logits], alpha=1.0, beta=1.0, transA=0, transB=1)
    flops += 2.0 * 512 * 1000
    B.m.outputs = [logits]
    B.m.flops_per_sample = flops
    return B.m


def lenet5(batch: int) -> Model:
    """LeNet-5 on 32x32 (config 1)."""
    B = _Builder("lenet5", batch)
    N = batch
    x = B.tensor("input", (N, 1, 32, 32))
    B.m.inputs = [x]
    w1 = B.const("conv1_w", B.kaiming((6, 1, 5, 5), 25))
    b1 = B.const("conv1_b", B.bias(6))
    B.node("Conv", [x, w1, b1], [B.tensor("c1", (N, 6, 28, 28))], kernel_shape=[5, 5], strides=[1, 1], pads=[0, 0, 0, 0])
    B.node("Relu", ["c1"], [B.tensor("r1", (N, 6, 28, 28))])
    B.node("MaxPool", ["r1"], [B.tensor("p1", (N, 6, 14, 14))], kernel_shape=[2, 2], strides=[2, 2], pads=[0, 0, 0, 0])
    w2 = B.const("conv2_w", B.kaiming((16, 6, 5, 5), 150))
    b2 = B.const("conv2_b", B.bias(16))
    B.node("Conv", ["p1", w2, b2], [B.tensor("c2", (N, 16, 10, 10))], kernel_shape=[5, 5], strides=[1, 1], pads=[0, 0, 0, 0])
    B.node("Relu", ["c2"], [B.tensor("r2", (N, 16, 10, 10))])
    B.node("MaxPool", ["r2"], [B.tensor("p2", (N, 16, 5, 5))], kernel_shape=[2, 2], strides=[2, 2], pads=[0, 0, 0, 0])
    B.node("Flatten", ["p2"], [B.tensor("flat", (N, 400))], axis=1)
    prev = "flat"
    for i, (fi, fo) in enumerate(((400, 120), (120, 84), (84, 10)), start=1):
        w = B.const(f"fc{i}_w", B.kaiming((fo, fi), fi))
        b = B.const(f"fc{i}_b", B.bias(fo))
        g = B.tensor(f"fc{i}", (N, fo))
        B.node("Gemm", [prev, w, b], [g], alpha=1.0, beta=1.0, transA=0, transB=1)
        prev = g
        if i < 3:
            prev_r = B.tensor(f"fc{i}_relu", (N, fo))
            B.node("Relu", [g], [prev_r])
            prev = prev_r
    B.node("Softmax", [prev], [B.tensor("prob", (N, 10))], axis=1)
    B.m.outputs = ["prob"]
    B.m.flops_per_sample = 2.0 * (6 * 28 * 28 * 25 + 16 * 10 * 10 * 150 + 400 * 120 + 120 * 84 + 84 * 10)
    return B.m


def transformer(batch: int, layers: int = 4, d: int = 256, heads: int = 4, ffn: int = 1024, seq: int = 128) -> Model:
    """Post-LN transformer encoder from MatMul/Add/Div/Softmax/LayerNorm/
    Transpose/Reshape/Relu only (config 4)."""
    B = _Builder("transformer", batch)
    N, S, hd = batch, seq, d // heads
    x = B.tensor("input", (N, S, d))
    B.m.inputs = [x]
    scale = B.const("attn_scale", np.array([np.sqrt(hd)], dtype=np.float32))

    def xavier(fi, fo):
        b = np.sqrt(6.0 / (fi + fo))
        return B.rng.uniform(-b, b, (fi, fo)).astype(np.float32)

    def linear(inp, fi, fo, tag, shape):
        w = B.const(f"{tag}_w", xavier(fi, fo))
        bias = B.const(f"{tag}_b", B.bias(fo))
        mm = B.tensor(f"{tag}_mm", shape)
        B.node("MatMul", [inp, w], [mm])
        out = B.tensor(f"{tag}_out", shape)
        B.node("Add", [mm, bias], [out])
        return out

    cur = x
    for l in range(layers):
        t = f"l{l}"
        q = linear(cur, d, d, f"{t}_q", (N, S, d))
        k = linear(cur, d, d, f"{t}_k", (N, S, d))
        v = linear(cur, d, d, f"{t}_v", (N, S, d))
        heads_in = {}
        for nm, src, perm, shp in (("q", q, [0, 2, 1, 3], (N, heads, S, hd)), ("k", k, [0, 2, 3, 1], (N, heads, hd, S)),
                                   ("v", v, [0, 2, 1, 3], (N, heads, S, hd))):
            r = B.tensor(f"{t}_{nm}_split", (N, S, heads, hd))
            B.node("Reshape", [src], [r], shape=[N, S, heads, hd])
            tr = B.tensor(f"{t}_{nm}_heads", shp)
            B.node("Transpose", [r], [tr], perm=perm)
            heads_in[nm] = tr
        sc = B.tensor(f"{t}_scores", (N, heads, S, S))
        B.node("MatMul", [heads_in["q"], heads_in["k"]], [sc])
        scd = B.tensor(f"{t}_scaled", (N, heads, S, S))
        B.node("Div", [sc, scale], [scd])
        pr = B.tensor(f"{t}_probs", (N, heads, S, S))
        B.node("Softmax", [scd], [pr], axis=-1)
        ctxh = B.tensor(f"{t}_ctx_heads", (N, heads, S, hd))
        B.node("MatMul", [pr, heads_in["v"]], [ctxh])
        ctxt = B.tensor(f"{t}_ctx_t", (N, S, heads, hd))
        B.node("Transpose", [ctxh], [ctxt], perm=[0, 2, 1, 3])
        ctx = B.tensor(f"{t}_ctx", (N, S, d))
        B.node("Reshape", [ctxt], [ctx], shape=[N, S, d])
        o = linear(ctx, d, d, f"{t}_o", (N, S, d))
        res1 = B.tensor(f"{t}_res1", (N, S, d))
        B.node("Add", [o, cur], [res1])
        g1 = B.const(f"{t}_ln1_g", np.ones(d, np.float32))
        b1 = B.const(f"{t}_ln1_b", np.zeros(d, np.float32))
        y = B.tensor(f"{t}_ln1", (N, S, d))
        B.node("LayerNormalization", [res1, g1, b1], [y], axis=-1, epsilon=1e-5)
        h = linear(y, d, ffn, f"{t}_ffn1", (N, S, ffn))
        hr = B.tensor(f"{t}_ffn1_relu", (N, S, ffn))
        B.node("Relu", [h], [hr])
        f = linear(hr, ffn, d, f"{t}_ffn2", (N, S, d))
        res2 = B.tensor(f"{t}_res2", (N, S, d))
        B.node("Add", [f, y], [res2])
        g2 = B.const(f"{t}_ln2_g", np.ones(d, np.float32))
        b2 = B.const(f"{t}_ln2_b", np.zeros(d, np.float32))
        out = B.tensor(f"{t}_ln2", (N, S, d))
        B.node("LayerNormalization", [res2, g2, b2], [out], axis=-1, epsilon=1e-5)
        cur = out
    B.m.outputs = [cur]
    B.m.flops_per_sample = layers * (2.0 * S * d * d * 4 + 2.0 * 2 * S * S * d + 2.0 * 2 * S * d * ffn)
    return B.m


BUILDERS: dict[str, Callable[[int], Model]] = {"resnet18": resnet18, "lenet5": lenet5, "transformer": transformer}


def nncb_bytes(entries: list[tuple[str, np.ndarray]]) -> bytes:
    """Serialises constants in nnc-py's NNCB v1 container
    (codegen/x86_emitters/constants_loader.py:40-144): 'NNCB', u32 version 1,
    u32 count, then per constant u32 name_len (with NUL), name, u32 dtype
    (0 = float32), u32 ndim, i64 shape[ndim], u64 nbytes, raw data."""
    buf = io.BytesIO()
    buf.write(b"NNCB")
    buf.write(struct.pack("<II", 1, len(entries)))
    for name, arr in entries:
        arr = np.ascontiguousarray(arr, dtype=np.float32)
        nb = name.encode() + b"\x00"
        buf.write(struct.pack("<I", len(nb)))
        buf.write(nb)
        buf.write(struct.pack("<II", 0, arr.ndim))
        buf.write(struct.pack(f"<{arr.ndim}q", *arr.shape))
        buf.write(struct.pack("<Q", arr.nbytes))
        buf.write(arr.tobytes())
    return buf.getvalue()

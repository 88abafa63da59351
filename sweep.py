"""Measures the BASELINE configurations that bench.py does not, on one GPU:
the single-op sweep against the measured peaks (tensor pipe for conv/GEMM,
HBM for every other op) and the model throughput of LeNet-5 (N = 8192),
ResNet-18 -O1 (N = 64, 256) and the small transformer (B = 256).

    python sweep.py [--reps 10] [--json sweep.json] [--only ops|models]
    python sweep.py --case <name>        (one op three times, for ncu captures)

Every number is a median over `reps` calls timed with CUDA events on the
launching stream. Each op call is captured once into a CUDA graph and replayed
per rep (the events bracket its kernels, not the host-side setup of a direct
call); before each rep the runner reads a 512 MB buffer (larger than the
126 MB L2), so inputs come from HBM. A model step replays one captured CUDA
graph of the whole forward. Denominators: MEASURED_PEAKS.json at the repository root
(HBM copy GB/s; dense TF32 = bf16 / 2), else the pool's fallback figures
(6650 GB/s, 1590 TFLOP/s bf16), read by bench.peaks(); each op is timed
alone in short bursts, so the burst figure applies (bench.tf32_peak's rule
with the clocks at their maximum). Inputs are seeded
N(0, 1), the shapes are BASELINE.json's.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import pathlib
import statistics
import sys

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT), str(ROOT / "nnc-py_b200")]

import bench  # noqa: E402
from nnc_cuda import lib as L  # noqa: E402
from nnc_cuda import tensor as T  # noqa: E402


def peaks() -> dict:
    pk = bench.peaks()
    tf32, note = bench.tf32_peak(pk, None)
    return {"hbm_gbs": pk["hbm_gbs"], "tf32_tflops": tf32, "tf32_note": note, "source": pk["source"]}


class Timer:
    def __init__(self, so, torch, stream, reps: int):
        self.so, self.torch, self.stream, self.reps = so, torch, stream, reps
        self.flush_buf = torch.empty(512 << 18, dtype=torch.float32, device="cuda")  # 512 MB

    def time_op(self, fn, warmup: int = 2) -> float:
        """Median device time in ms of fn() (library calls on the stream).

        The call is captured once into a CUDA graph (nnc_cuda_graph_*) and
        each timed rep replays it between two events, so the interval holds
        the op's kernels and not the host work (argument checks, tensor-map
        encoding) that a direct call would put between the events."""
        torch, so = self.torch, self.so
        with torch.cuda.stream(self.stream):
            for _ in range(warmup):
                fn()
        self.stream.synchronize()
        if so.nnc_cuda_graph_begin() != 0:
            raise RuntimeError("nnc_cuda_graph_begin failed")
        fn()
        graph = so.nnc_cuda_graph_end()
        if not graph:
            raise RuntimeError(so.nnc_cuda_get_last_error_string().decode())
        times = []
        try:
            for _ in range(self.reps):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                with torch.cuda.stream(self.stream):
                    # Read (not write) the buffer: L2 then holds clean lines, so
                    # the timed call pays no write-back of the flush.
                    self.flush_sink = self.flush_buf.sum()
                    e0.record(self.stream)
                    if so.nnc_cuda_graph_launch(ctypes.c_void_p(graph)) != 0:
                        raise RuntimeError(so.nnc_cuda_get_last_error_string().decode())
                    e1.record(self.stream)
                e1.synchronize()
                times.append(e0.elapsed_time(e1))
        finally:
            so.nnc_cuda_graph_destroy(ctypes.c_void_p(graph))
        if so.nnc_cuda_get_last_error() != 0:
            raise RuntimeError(so.nnc_cuda_get_last_error_string().decode())
        return statistics.median(times)


def op_sweep(so, torch, timer: Timer, pk: dict) -> list[dict]:
    g = torch.Generator(device="cuda").manual_seed(1)
    rows = []

    def rnd(*shape):
        return torch.randn(*shape, generator=g, device="cuda")

    def hbm(name, shape, fn, nbytes):
        ms = timer.time_op(fn)
        gbs = nbytes / (ms * 1e-3) / 1e9
        rows.append({"op": name, "shape": list(shape), "ms": round(ms, 4), "bound": "hbm",
                     "algorithmic_bytes": int(nbytes), "achieved": round(gbs, 1), "unit": "GB/s",
                     "frac": round(gbs / pk["hbm_gbs"], 3)})

    def tensor(name, shape, fn, flops, note=""):
        ms = timer.time_op(fn)
        tfs = flops / (ms * 1e-3) / 1e12
        row = {"op": name, "shape": list(shape), "ms": round(ms, 4), "bound": "tensor",
               "flops": int(flops), "achieved": round(tfs, 1), "unit": "TFLOP/s",
               "frac": round(tfs / pk["tf32_tflops"], 3)}
        if note:
            row["note"] = note
        rows.append(row)

    # GEMM M = N = K (NN and NT).
    for n in (512, 2048, 8192):
        a, b, o = rnd(n, n), rnd(n, n), torch.empty(n, n, device="cuda")
        ra, rb, ro = T.from_torch(a), T.from_torch(b), T.from_torch(o)
        tensor("nnc_gemm", (n, n, n), lambda: so.nnc_gemm(ra.ptr, rb.ptr, None, ro.ptr, 1.0, 0.0, 0, 0), 2.0 * n ** 3)
        tensor("nnc_gemm_nt", (n, n, n), lambda: so.nnc_gemm_nt(ra.ptr, rb.ptr, None, ro.ptr, 1.0, 0.0), 2.0 * n ** 3)
        del a, b, o
    # Conv 3x3 p1 s1 at batch 64: the reference API (NCHW tensors, converted
    # inside the call) and channels-last tensors (what generated models pass).
    for c, h in ((64, 56), (128, 28), (256, 14), (512, 7)):
        n = 64
        x, w, bias = rnd(n, c, h, h), rnd(c, c, 3, 3) * 0.05, rnd(c) * 0.01
        o = torch.empty(n, c, h, h, device="cuda")
        rx, rw, rbias, ro = T.from_torch(x), T.from_torch(w), T.from_torch(bias), T.from_torch(o)
        fl = 2.0 * n * c * c * h * h * 9
        tensor("nnc_conv 3x3 (NCHW)", (n, c, h, h),
               lambda: so.nnc_conv(rx.ptr, rw.ptr, rbias.ptr, ro.ptr, 3, 3, 1, 1, 1, 1), fl,
               "includes the NCHW -> channels-last copy of the input")
        xl = x.permute(0, 2, 3, 1).contiguous()
        ol = torch.empty(n, h, h, c, device="cuda")
        wp = torch.empty(so.nnc_cuda_prepacked_conv_weight_bytes(rw.ptr) // 4, device="cuda")
        rwp = T.from_torch(w.clone())
        assert so.nnc_cuda_prepack_conv_weight(rwp.ptr, ctypes.c_void_p(wp.data_ptr()), wp.numel() * 4) == 0
        rxl = T.from_torch(xl, tag=L.TAG_NHWC, shape=(n, c, h, h))
        rol = T.from_torch(ol, tag=L.TAG_NHWC, shape=(n, c, h, h))
        tensor("nnc_conv 3x3 (channels-last, prepacked)", (n, c, h, h),
               lambda: so.nnc_conv(rxl.ptr, rwp.ptr, rbias.ptr, rol.ptr, 3, 3, 1, 1, 1, 1), fl)
        del x, w, o, xl, ol, wp
    # Element-wise on 2^28 elements.
    n = 1 << 28
    a, b, o = rnd(n), rnd(n), torch.empty(n, device="cuda")
    ra, rb, ro = T.from_torch(a), T.from_torch(b), T.from_torch(o)
    hbm("nnc_add", (n,), lambda: so.nnc_add(ra.ptr, rb.ptr, ro.ptr), 12 * n)
    hbm("nnc_mul", (n,), lambda: so.nnc_mul(ra.ptr, rb.ptr, ro.ptr), 12 * n)
    hbm("nnc_relu", (n,), lambda: so.nnc_relu(ra.ptr, ro.ptr), 8 * n)
    hbm("nnc_sigmoid", (n,), lambda: so.nnc_sigmoid(ra.ptr, ro.ptr), 8 * n)
    hbm("nnc_tanh", (n,), lambda: so.nnc_tanh(ra.ptr, ro.ptr), 8 * n)
    hbm("nnc_clip [-1, 1]", (n,), lambda: so.nnc_clip(ra.ptr, ro.ptr, -1.0, 1.0), 8 * n)
    del a, b, o
    # Row ops.
    x, o = rnd(4096, 4096), torch.empty(4096, 4096, device="cuda")
    rx, ro = T.from_torch(x), T.from_torch(o)
    hbm("nnc_softmax", (4096, 4096), lambda: so.nnc_softmax(rx.ptr, ro.ptr, 1), 8 * 4096 * 4096)
    del x, o
    x, o = rnd(32768, 1024), torch.empty(32768, 1024, device="cuda")
    gam = torch.rand(1024, generator=g, device="cuda") + 0.5
    bet = (torch.rand(1024, generator=g, device="cuda") - 0.5) * 0.2
    rx, ro, rg, rbt = T.from_torch(x), T.from_torch(o), T.from_torch(gam), T.from_torch(bet)
    hbm("nnc_layernorm", (32768, 1024), lambda: so.nnc_layernorm(rx.ptr, rg.ptr, rbt.ptr, ro.ptr, -1, 1e-5),
        8 * 32768 * 1024 + 8 * 1024)
    del x, o
    x, o = rnd(16384, 4096), torch.empty(16384, 1, device="cuda")
    rx, ro = T.from_torch(x), T.from_torch(o)
    hbm("nnc_reducemean", (16384, 4096), lambda: so.nnc_reducemean(rx.ptr, ro.ptr, 1, 1), 4 * 16384 * 4096 + 4 * 16384)
    hbm("nnc_reducesum", (16384, 4096), lambda: so.nnc_reducesum(rx.ptr, ro.ptr, 1, 1), 4 * 16384 * 4096 + 4 * 16384)
    del x, o
    # The transformer's (batch 256, S 128, d 256, 4 heads) per-layer shapes,
    # with the reference's batched-matmul offsets.
    for name, sa, sb in (("linear", (256, 128, 256), (256, 256)), ("ffn1", (256, 128, 256), (256, 1024)),
                         ("ffn2", (256, 128, 1024), (1024, 256)), ("scores", (256, 4, 128, 64), (256, 4, 64, 128)),
                         ("probs@v", (256, 4, 128, 128), (256, 4, 128, 64))):
        so_ = sa[:-1] + sb[-1:]
        a, b, o = rnd(*sa), rnd(*sb), torch.empty(*so_, device="cuda")
        ra, rb, ro = T.from_torch(a), T.from_torch(b), T.from_torch(o)
        fl = 2.0 * o.numel() * sa[-1]
        tensor(f"nnc_matmul {name}", sa + sb, lambda: so.nnc_matmul(ra.ptr, rb.ptr, ro.ptr), fl,
               "B read MN-major; output-bound (small K)")
        del a, b, o
    x = rnd(256, 128, 4, 64)
    o = torch.empty(256, 4, 64, 128, device="cuda")
    rx, ro = T.from_torch(x), T.from_torch(o)
    perm = (ctypes.c_int64 * 4)(0, 2, 3, 1)
    hbm("nnc_transpose [0,2,3,1]", (256, 128, 4, 64), lambda: so.nnc_transpose(rx.ptr, ro.ptr, perm, 4),
        8 * x.numel())
    o2 = torch.empty(256, 4, 128, 64, device="cuda")
    ro2 = T.from_torch(o2)
    perm2 = (ctypes.c_int64 * 4)(0, 2, 1, 3)
    hbm("nnc_transpose [0,2,1,3]", (256, 128, 4, 64), lambda: so.nnc_transpose(rx.ptr, ro2.ptr, perm2, 4),
        8 * x.numel())
    del x, o, o2
    x, o = rnd(256, 4, 128, 128), torch.empty(256, 4, 128, 128, device="cuda")
    rx, ro = T.from_torch(x), T.from_torch(o)
    hbm("nnc_softmax", (256, 4, 128, 128), lambda: so.nnc_softmax(rx.ptr, ro.ptr, -1), 8 * x.numel())
    del x, o
    x, o = rnd(256, 128, 256), torch.empty(256, 128, 256, device="cuda")
    gam, bet = rnd(256), rnd(256)
    rx, ro, rg, rbt = T.from_torch(x), T.from_torch(o), T.from_torch(gam), T.from_torch(bet)
    hbm("nnc_layernorm", (256, 128, 256), lambda: so.nnc_layernorm(rx.ptr, rg.ptr, rbt.ptr, ro.ptr, -1, 1e-5),
        8 * x.numel())
    del x, o
    # LeNet-5 at batch 8192 (channels-last activations, as the model keeps them).
    for name, C, H, Co, cl in (("conv1 1->6 5x5", 1, 32, 6, False), ("conv2 6->16 5x5", 6, 14, 16, True)):
        n, OH = 8192, H - 4
        x = rnd(n, H, H, C) if cl else rnd(n, C, H, H)
        rx = T.from_torch(x, tag=L.TAG_NHWC if cl else 0, shape=(n, C, H, H))
        o = torch.empty(n, OH, OH, Co, device="cuda")
        ro = T.from_torch(o, tag=L.TAG_NHWC, shape=(n, Co, OH, OH))
        w, bias = rnd(Co, C, 5, 5) * 0.1, rnd(Co)
        rw, rbias = T.from_torch(w), T.from_torch(bias)
        hbm(f"nnc_conv LeNet {name}", (n, C, H, H),
            lambda: so.nnc_conv(rx.ptr, rw.ptr, rbias.ptr, ro.ptr, 5, 5, 1, 1, 0, 0), 4 * (x.numel() + o.numel()))
        del x, o
    x = rnd(8192, 28, 28, 6)
    o = torch.empty(8192, 14, 14, 6, device="cuda")
    rx = T.from_torch(x, tag=L.TAG_NHWC, shape=(8192, 6, 28, 28))
    ro = T.from_torch(o, tag=L.TAG_NHWC, shape=(8192, 6, 14, 14))
    hbm("nnc_maxpool2d 2x2/2 (C 6, channels-last)", (8192, 6, 28, 28),
        lambda: so.nnc_maxpool2d(rx.ptr, ro.ptr, 2, 2, 2, 2, 0, 0), 4 * (x.numel() + o.numel()))
    del x, o
    return rows


# Algorithmic FLOPs per sample of the BASELINE models (conv + GEMM/matmul).
MODEL_FLOPS = {"lenet5": 0.833e6, "resnet18": 3.628e9, "transformer": 0.872e9}


MODELS = (("lenet5_o1_b8192", "lenet5", 8192), ("lenet5_o3_b8192", "lenet5", 8192),
          ("resnet18_o1_b64", "resnet18", 64), ("resnet18_o1_b256", "resnet18", 256),
          ("transformer_o1_b256", "transformer", 256), ("transformer_o3_b256", "transformer", 256),
          ("transformer_o1_b2048", "transformer", 2048), ("transformer_o3_b2048", "transformer", 2048))


def model_runs(so, torch, pk: dict, reps: int, only_model: str | None = None) -> list[dict]:
    from nnc_cuda.model import CudaModel
    from nnc_cuda.workloads import BUILDERS

    rows = []
    for tag, name, batch in MODELS:
        if only_model and tag != only_model:
            continue
        m = CudaModel(tag)
        m.init(0)
        wl = BUILDERS[name](batch)
        m.load_constants(wl)
        stream = torch.cuda.Stream()
        m.set_stream(stream.cuda_stream)
        x = torch.from_numpy(wl.input_array(batch)).cuda()
        so.nnc_cuda_memcpy_async(ctypes.c_void_p(m.input_ptr()), ctypes.c_void_p(x.data_ptr()),
                                 x.numel() * 4, 3)
        with torch.cuda.stream(stream):
            for _ in range(3):
                m.run()
        stream.synchronize()
        m.capture()
        with torch.cuda.stream(stream):
            m.replay()
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(reps):
                m.replay()
            e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / reps
        m.release_graph()
        so.nnc_cuda_set_stream(None)
        if so.nnc_cuda_get_last_error() != 0:
            raise RuntimeError(so.nnc_cuda_get_last_error_string().decode())
        tf = MODEL_FLOPS[name] * batch / (ms * 1e-3) / 1e12
        rows.append({"model": tag, "batch": batch, "ms_per_forward": round(ms, 4),
                     "samples_per_s": round(batch / (ms * 1e-3), 1), "tflops": round(tf, 1),
                     "frac_tf32": round(tf / pk["tf32_tflops"], 3)})
    return rows


# Single-op cases for kernel captures (ncu): each is run three times (the
# first launch warms up, a capture takes the second with -s 1 -c 1). Inputs
# are larger than L2 so that DRAM counters mean something, but a few hundred
# MB at most.
PROFILE_CASES = ("layernorm", "layernorm256", "softmax", "softmax128", "transpose", "transpose_k", "add",
                 "stem", "stage1", "stage2s2", "lenet_conv1", "lenet_conv2")


def profile_case(so, torch, case: str) -> None:
    g = torch.Generator(device="cuda").manual_seed(0)
    keep = []

    def rnd(*shape):
        return torch.randn(*shape, generator=g, device="cuda")

    def R(t, tag=0, shape=None):
        r = T.from_torch(t, tag=tag, shape=shape)
        keep.append(r)
        return r.ptr

    if case in ("layernorm", "layernorm256"):
        rows, d = (32768, 1024) if case == "layernorm" else (131072, 256)
        x, gam, bet = rnd(rows, d), rnd(d) * 0.1 + 1, rnd(d) * 0.1
        o = torch.empty_like(x)
        fn = lambda: so.nnc_layernorm(R(x), R(gam), R(bet), R(o), -1, ctypes.c_float(1e-5))
    elif case in ("softmax", "softmax128"):
        x = rnd(8192, 4096) if case == "softmax" else rnd(1024, 4, 128, 128)
        o = torch.empty_like(x)
        fn = lambda: so.nnc_softmax(R(x), R(o), -1)
    elif case in ("transpose", "transpose_k"):
        x = rnd(1024, 128, 4, 64)
        perm = (ctypes.c_int64 * 4)(*((0, 2, 1, 3) if case == "transpose" else (0, 2, 3, 1)))
        o = torch.empty(1024, 4, 128, 64, device="cuda") if case == "transpose" else \
            torch.empty(1024, 4, 64, 128, device="cuda")
        fn = lambda: so.nnc_transpose(R(x), R(o), perm, 4)
    elif case == "add":
        a, b = rnd(1 << 26), rnd(1 << 26)
        o = torch.empty_like(a)
        fn = lambda: so.nnc_add(R(a), R(b), R(o))
    elif case == "stem":  # the ResNet stem at batch 192: space-to-depth + conv 7x7/2 + relu + max pool
        n = 192
        x, w, bias = rnd(n, 3, 224, 224), rnd(64, 3, 7, 7) * 0.1, rnd(64) * 0.01
        o = torch.empty(n, 56, 56, 64, device="cuda")
        fn = lambda: so.nnc_conv_relu_maxpool(R(x), R(w), R(bias), R(o, L.TAG_NHWC, (n, 64, 56, 56)),
                                              7, 7, 2, 2, 3, 3, 112, 112, 3, 3, 2, 2, 1, 1)
    elif case == "stage1":  # a stage-1 conv+add+relu at batch 128, channels-last, prepacked weights
        n = 128
        x, w, bias, res = rnd(n, 56, 56, 64), rnd(64, 64, 3, 3) * 0.05, rnd(64) * 0.01, rnd(n, 56, 56, 64)
        wp = torch.empty(so.nnc_cuda_prepacked_conv_weight_bytes(R(w)) // 4, device="cuda")
        rw = T.from_torch(w.clone())
        keep.append(rw)
        assert so.nnc_cuda_prepack_conv_weight(rw.ptr, ctypes.c_void_p(wp.data_ptr()), wp.numel() * 4) == 0
        o = torch.empty(n, 56, 56, 64, device="cuda")
        shp = (n, 64, 56, 56)
        fn = lambda: so.nnc_conv_add_relu3x3_s1(R(x, L.TAG_NHWC, shp), rw.ptr, R(bias), R(res, L.TAG_NHWC, shp),
                                                R(o, L.TAG_NHWC, shp))
    elif case == "stage2s2":  # the stage-2 3x3/2 conv+relu at batch 256, channels-last, prepacked
        n = 256
        x, w, bias = rnd(n, 56, 56, 64), rnd(128, 64, 3, 3) * 0.05, rnd(128) * 0.01
        wp = torch.empty(so.nnc_cuda_prepacked_conv_weight_bytes(R(w)) // 4, device="cuda")
        rw = T.from_torch(w.clone())
        keep.append(rw)
        assert so.nnc_cuda_prepack_conv_weight(rw.ptr, ctypes.c_void_p(wp.data_ptr()), wp.numel() * 4) == 0
        o = torch.empty(n, 28, 28, 128, device="cuda")
        fn = lambda: so.nnc_conv_relu(R(x, L.TAG_NHWC, (n, 64, 56, 56)), rw.ptr, R(bias),
                                      R(o, L.TAG_NHWC, (n, 128, 28, 28)), 3, 3, 2, 2, 1, 1)
    elif case in ("lenet_conv1", "lenet_conv2"):  # LeNet-5's convs at batch 8192 in the model's layouts
        n = 8192
        if case == "lenet_conv1":  # [n, 1, 32, 32] -> channels-last [n, 6, 28, 28]
            x, w, bias = rnd(n, 1, 32, 32), rnd(6, 1, 5, 5) * 0.2, rnd(6) * 0.01
            o = torch.empty(n, 28, 28, 6, device="cuda")
            xi, oi = R(x), R(o, L.TAG_NHWC, (n, 6, 28, 28))
        else:  # channels-last [n, 6, 14, 14] -> NCHW [n, 16, 10, 10]
            x, w, bias = rnd(n, 14, 14, 6), rnd(16, 6, 5, 5) * 0.1, rnd(16) * 0.01
            o = torch.empty(n, 16, 10, 10, device="cuda")
            xi, oi = R(x, L.TAG_NHWC, (n, 6, 14, 14)), R(o)
        wi, bi = R(w), R(bias)
        fn = lambda: so.nnc_conv_relu(xi, wi, bi, oi, 5, 5, 1, 1, 0, 0)
    else:
        raise SystemExit(f"unknown case {case}")
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    if so.nnc_cuda_get_last_error() != 0:
        raise RuntimeError(so.nnc_cuda_get_last_error_string().decode())
    print("ok", case)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", choices=PROFILE_CASES, default=None,
                    help="run one op case three times and exit (for kernel captures)")
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--json", type=str, default=None)
    ap.add_argument("--only", choices=["ops", "models"], default=None)
    ap.add_argument("--model", choices=[m[0] for m in MODELS], default=None,
                    help="run this model only (with --only models)")
    opt = ap.parse_args()
    import torch

    so = L.load()
    torch.cuda.set_device(0)
    if so.nnc_cuda_init(0) != 0:
        raise RuntimeError("nnc_cuda_init failed")
    so.nnc_cuda_set_precision(L.PRECISION_TF32)
    if opt.case:
        so.nnc_cuda_set_stream(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        profile_case(so, torch, opt.case)
        return 0
    pk = peaks()
    stream = torch.cuda.Stream()
    so.nnc_cuda_set_stream(ctypes.c_void_p(stream.cuda_stream))
    out = {"peaks": pk, "precision": "tf32"}
    if opt.only in (None, "ops"):
        out["ops"] = op_sweep(so, torch, Timer(so, torch, stream, opt.reps), pk)
        for r in out["ops"]:
            print(f"{r['op']:42s} {str(r['shape']):22s} {r['ms']:9.4f} ms {r['achieved']:9.1f} {r['unit']:8s} "
                  f"{r['frac']:.3f}", flush=True)
    if opt.only in (None, "models"):
        so.nnc_cuda_set_stream(None)
        out["models"] = model_runs(so, torch, pk, max(opt.reps, 20), opt.model)
        for r in out["models"]:
            print(f"{r['model']:22s} {r['ms_per_forward']:9.4f} ms {r['samples_per_s']:12.1f} /s "
                  f"{r['tflops']:7.1f} TF/s {r['frac_tf32']:.3f}", flush=True)
    if opt.json:
        pathlib.Path(opt.json).write_text(json.dumps(out, indent=1))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())

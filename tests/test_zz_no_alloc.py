"""nnc_conv_static_scratch, the conv entry point that allocates nothing.

It must give nnc_conv's results for the same arguments (within the
tensor-core tolerance the other conv tests use) while taking its scratch
from the library's fixed 16 MiB device array: consecutive calls of different
shapes reuse that array, so each call has to write what it reads. The file
name sorts last so the module also runs after every other GPU test in the
same process (a grown workspace, earlier calls' scratch contents); it also
passes alone in a fresh process.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import opcases as C
from nnc_cuda import lib as L
from nnc_cuda import tensor as T

pytestmark = pytest.mark.gpu

# (N, C_in, H, W, C_out, KH, KW, sh, sw, ph, pw): one per kernel feeding mode,
# each with an NCHW input so the scratch holds its NHWC copy (or, in element
# mode, its 3xTF32 hi/lo planes) and the packed weights. C_out > 16 keeps
# every case on the tensor-core kernels (smaller ones take a CUDA-core kernel
# that reads the weights in place and needs no scratch).
CASES = {
    "im2col128": (2, 64, 28, 28, 128, 3, 3, 1, 1, 1, 1),
    "im2col16_stem": (2, 3, 30, 30, 16, 7, 7, 2, 2, 3, 3),
    "chunk_gather": (1, 5, 17, 13, 24, 3, 5, 2, 1, 1, 2),
    "element": (4, 1, 12, 12, 24, 5, 5, 1, 1, 0, 0),
}
SCRATCH_LIMIT = 16 << 20


def _out_hw(h, k, s, p):
    return (h + 2 * p - k) // s + 1


def _inputs(name):
    n, c, h, w, co, kh, kw, sh, sw, ph, pw = CASES[name]
    rng = C.rng_for("no_alloc_" + name)
    x = rng.standard_normal((n, c, h, w), dtype=np.float32)
    wt = (rng.standard_normal((co, c, kh, kw), dtype=np.float32) / np.sqrt(c * kh * kw)).astype(np.float32)
    b = rng.standard_normal(co, dtype=np.float32)
    shape = (n, co, _out_hw(h, kh, sh, ph), _out_hw(w, kw, sw, pw))
    return x, wt, b, shape, (kh, kw, sh, sw, ph, pw)


def _run(so, entry, name):
    """Runs `entry` (a library function name) on case `name`; returns the
    output as numpy, after checking the call left the status clean."""
    import torch

    x, wt, b, oshape, geo = _inputs(name)
    dx, dw, db = (torch.from_numpy(a).cuda() for a in (x, wt, b))
    do = torch.full(oshape, float("nan"), dtype=torch.float32, device="cuda")
    refs = [T.from_torch(t) for t in (dx, dw, db, do)]
    so.nnc_cuda_set_stream(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    getattr(so, entry)(*(r.ptr for r in refs), *geo)
    torch.cuda.synchronize()
    assert so.nnc_cuda_get_last_error() == 0, so.nnc_cuda_get_last_error_string().decode()
    return do.cpu().numpy()


@pytest.mark.parametrize("precision", [L.PRECISION_TF32, L.PRECISION_3XTF32])
def test_matches_nnc_conv_on_consecutive_calls(cuda_lib, precision):
    so = cuda_lib
    so.nnc_cuda_set_precision(precision)
    want = {name: _run(so, "nnc_conv", name) for name in CASES}
    ws_before = so.nnc_cuda_get_workspace_capacity()
    launches_before = so.nnc_cuda_launch_count()
    # Every case twice in a row, then the first again after the others have
    # left their contents in the shared scratch.
    order = [name for name in CASES for _ in range(2)] + [next(iter(CASES))]
    for name in order:
        got = _run(so, "nnc_conv_static_scratch", name)
        C.assert_close(got, want[name], C.TC_RTOL[precision], f"{name} precision={precision}")
    # The calls ran on the GPU and never touched the growable workspace.
    assert so.nnc_cuda_launch_count() > launches_before
    assert so.nnc_cuda_get_workspace_capacity() == ws_before


@pytest.mark.parametrize("precision", [L.PRECISION_TF32, L.PRECISION_3XTF32])
def test_matches_cpu_oracle(cuda_lib, precision):
    """Beside the comparison with nnc_conv: every case against the CPU
    restatement of the reference's nnc_conv (double accumulation, one
    rounding), after the other cases have used the shared scratch."""
    from oracle import oracle as O

    so = cuda_lib
    so.nnc_cuda_set_precision(precision)
    orc = O.load_oracle()
    for name in reversed(list(CASES)):
        x, wt, b, oshape, geo = _inputs(name)
        case = {"name": name, "op": "nnc_conv",
                "args": [C._t("x"), C._t("w"), C._t("b"), C._o("out", oshape)] + [C._i(v) for v in geo]}
        want = C.run_host(orc, case, {"x": x, "w": wt, "b": b})["out"]
        got = _run(so, "nnc_conv_static_scratch", name)
        C.assert_close(got, want, C.TC_RTOL[precision], f"{name} vs oracle precision={precision}")


def test_rejects_scratch_beyond_limit(cuda_lib):
    """An NCHW input whose NHWC copy alone exceeds 16 MiB is refused before
    any work is queued: the output keeps its contents."""
    import torch

    so = cuda_lib
    n, c, h, w = 8, 64, 112, 112  # NHWC copy: 25.7 MB
    assert n * c * h * w * 4 > SCRATCH_LIMIT
    dx = torch.zeros((n, c, h, w), dtype=torch.float32, device="cuda")
    dw = torch.zeros((64, c, 3, 3), dtype=torch.float32, device="cuda")
    do = torch.full((n, 64, h, w), 7.0, dtype=torch.float32, device="cuda")
    refs = [T.from_torch(t) for t in (dx, dw, do)]
    launches_before = so.nnc_cuda_launch_count()
    so.nnc_cuda_set_stream(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    so.nnc_conv_static_scratch(refs[0].ptr, refs[1].ptr, None, refs[2].ptr, 3, 3, 1, 1, 1, 1)
    torch.cuda.synchronize()
    assert so.nnc_cuda_get_last_error() == L.ERR_INVALID
    assert b"static scratch" in so.nnc_cuda_get_last_error_string()
    assert so.nnc_cuda_launch_count() == launches_before
    assert bool(torch.all(do == 7.0))
    so.nnc_cuda_clear_error()

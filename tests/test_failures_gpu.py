"""Failure detection without a GPU fault: every failure here is made on the
host (a corrupted constants container, an injected allocation failure, a
device index out of range) or by a bounded in-kernel wait that is allowed to
run out on a barrier nothing completes. Each must fail cleanly — an error
status, no launch of the failing op, a context that keeps working."""

from __future__ import annotations

import ctypes
import struct
import threading

import numpy as np
import pytest

import opcases as C
from nnc_cuda import lib as L
from nnc_cuda import tensor as T
from nnc_cuda import workloads as W

pytestmark = pytest.mark.gpu

TAG = "lenet5_o1_b16"


def _entries(blob: bytes):
    """(offset of name_len, name, offset of nbytes, nbytes) of each NNCB
    entry (magic, version u32, count u32, then name_len u32, name, dtype
    u32, ndim u32, shape i64[ndim], nbytes u64, data)."""
    out = []
    p = 12
    count = struct.unpack_from("<I", blob, 8)[0]
    for _ in range(count):
        start = p
        (name_len,) = struct.unpack_from("<I", blob, p)
        p += 4
        name = blob[p:p + name_len]
        p += name_len
        _, ndim = struct.unpack_from("<II", blob, p)
        p += 8 + 8 * ndim
        nb_off = p
        (nbytes,) = struct.unpack_from("<Q", blob, p)
        p += 8 + nbytes
        out.append((start, name, nb_off, nbytes))
    return out


def _corruptions(blob: bytes):
    e = _entries(blob)
    first_name = e[0][0] + 4
    yield "bad magic", b"NNCX" + blob[4:]
    yield "bad version", blob[:4] + struct.pack("<I", 2) + blob[8:]
    yield "wrong count", blob[:8] + struct.pack("<I", len(e) + 1) + blob[12:]
    renamed = bytearray(blob)
    renamed[first_name] = ord("Z") if renamed[first_name] != ord("Z") else ord("Y")
    yield "renamed entry", bytes(renamed)
    nb = bytearray(blob)
    struct.pack_into("<Q", nb, e[1][2], e[1][3] + 4)
    yield "wrong size", bytes(nb)
    yield "truncated header", blob[:10]
    yield "truncated data", blob[: e[-1][2] + 8 + e[-1][3] // 2]


def test_constants_loader_rejects_corrupt_containers(cuda_lib):
    """The generated loader checks the NNCB container as the reference's
    does (magic, version, entry names in order, sizes; the reference's
    constants_loader.py:204-271) and also the entry count and every length
    against the bytes present: each corruption is refused with a nonzero
    return, and the intact container still loads and runs correctly."""
    from nnc_cuda.model import CudaModel

    m = CudaModel(TAG)
    m.init(0)
    model = W.lenet5(16)
    blob = m.constants_blob(model)
    for what, bad in _corruptions(blob):
        buf = ctypes.create_string_buffer(bad, len(bad))
        rc = m.lib.nnc_load_constants_from_memory(ctypes.cast(buf, ctypes.c_void_p), len(bad))
        assert rc != 0, f"{what}: accepted"
        cuda_lib.nnc_cuda_clear_error()
    m.load_constants(model)
    x = model.input_array(16)
    got = m.run_host(x)
    assert got.shape == (16, 10)
    assert np.allclose(got.sum(1), 1.0, atol=1e-5)  # softmax rows
    m.free()


def test_bounded_wait_expires_reports_and_context_stays_usable(cuda_lib):
    """A kernel waits (bounded, 20 ms) on an mbarrier that nothing
    completes: it records NNC_CUDA_ERR_DEVICE_TIMEOUT in the device error
    word and returns; the host reads the status, which then clears, and the
    next op runs normally."""
    import torch

    so = cuda_lib
    so.nnc_cuda_set_stream(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert so.nnc_cuda_check_device_status() == L.OK
    assert so.nnc_cuda_selftest_bounded_wait(20000) == L.OK
    torch.cuda.synchronize()
    assert so.nnc_cuda_check_device_status() == L.ERR_DEVICE_TIMEOUT
    assert b"bounded wait" in so.nnc_cuda_get_last_error_string()
    so.nnc_cuda_clear_error()
    assert so.nnc_cuda_check_device_status() == L.OK  # read and cleared
    # Out-of-range bounds are refused on the host.
    assert so.nnc_cuda_selftest_bounded_wait(0) == L.ERR_INVALID
    so.nnc_cuda_clear_error()
    # The context still works.
    case, arrays = next((c, a) for c, a in C.seeded_cases() if c["name"] == "nnc_add_same")
    got = C.run_cuda(so, case, arrays)["out"]
    assert np.array_equal(got, arrays["a"] + arrays["b"])


def test_injected_allocation_failure_fails_cleanly(cuda_lib):
    """An NCHW conv needs workspace for its channels-last copy; on a thread
    whose workspace is still empty, an injected allocation failure makes the
    call report NNC_CUDA_ERR_NOMEM and queue nothing, leaving the output as
    it was. The next call on that thread allocates and succeeds."""
    import torch

    so = cuda_lib
    x = torch.randn(2, 40, 12, 12, device="cuda")
    w = torch.randn(48, 40, 3, 3, device="cuda") * 0.05
    out = torch.full((2, 48, 12, 12), 7.0, device="cuda")
    refs = [T.from_torch(t) for t in (x, w, out)]
    stream = torch.cuda.current_stream().cuda_stream
    seen = {}

    def worker():
        so.nnc_cuda_init(0)
        so.nnc_cuda_set_stream(ctypes.c_void_p(stream))
        assert so.nnc_cuda_get_workspace_capacity() == 0  # a fresh thread
        so.nnc_cuda_inject_alloc_failures(1)
        before = so.nnc_cuda_launch_count()
        so.nnc_conv(refs[0].ptr, refs[1].ptr, None, refs[2].ptr, 3, 3, 1, 1, 1, 1)
        seen["status"] = so.nnc_cuda_get_last_error()
        seen["msg"] = so.nnc_cuda_get_last_error_string()
        seen["launched"] = so.nnc_cuda_launch_count() - before
        torch.cuda.synchronize()
        seen["untouched"] = bool(torch.all(out == 7.0))
        so.nnc_cuda_clear_error()
        so.nnc_conv(refs[0].ptr, refs[1].ptr, None, refs[2].ptr, 3, 3, 1, 1, 1, 1)
        torch.cuda.synchronize()
        seen["retry_status"] = so.nnc_cuda_get_last_error()

    t = threading.Thread(target=worker)
    t.start()
    t.join()
    so.nnc_cuda_inject_alloc_failures(0)
    assert seen["status"] == L.ERR_NOMEM, seen
    assert b"injected" in seen["msg"]
    assert seen["launched"] == 0
    assert seen["untouched"]
    assert seen["retry_status"] == L.OK
    assert not bool(torch.all(out == 7.0))


def test_device_index_out_of_range_is_refused(cuda_lib):
    import torch

    count = torch.cuda.device_count()
    assert cuda_lib.nnc_cuda_init(count) == L.ERR_INVALID
    assert cuda_lib.nnc_cuda_init(-1) == L.ERR_INVALID
    assert b"out of range" in cuda_lib.nnc_cuda_get_last_error_string()
    cuda_lib.nnc_cuda_clear_error()
    assert cuda_lib.nnc_cuda_init(0) == L.OK

"""The per-op trace in the costmodel runtime's format: the same two-stage
graph as nnc-py's own costmodel test (Relu, then Add; its
tests/test_costmodel_runtime.py:55-87) and the same checks on the printed
lines, plus the byte counts and the device times' ordering."""

from __future__ import annotations

import re

import numpy as np
import pytest

import opcases as C

pytestmark = pytest.mark.gpu

LINE = re.compile(r"^\[costmodel\] #(\d+) op=(\w+) cu=(\d+) start=(\d+) end=(\d+) read=0 compute=(\d+) "
                  r"write=0 in=(\d+)B out=(\d+)B$")


def test_trace_dump_prints_costmodel_lines(cuda_lib, capfd):
    so = cuda_lib
    x = np.array([[-1.0, 2.0, -3.0, 4.0]], dtype=np.float32)
    one = np.ones((1, 4), dtype=np.float32)
    relu = {"name": "relu0", "op": "nnc_relu", "args": [C._t("x"), C._o("out", (1, 4))]}
    so.nnc_cuda_trace_clear()
    so.nnc_cuda_trace_enable(1)
    try:
        r = C.run_cuda(so, relu, {"x": x})["out"]
        add = {"name": "add0", "op": "nnc_add", "args": [C._t("r"), C._t("c"), C._o("out", (1, 4))]}
        y = C.run_cuda(so, add, {"r": r, "c": one})["out"]
        capfd.readouterr()
        assert so.nnc_cuda_trace_dump() == 2
    finally:
        so.nnc_cuda_trace_enable(0)
    out = capfd.readouterr().out
    assert np.array_equal(y, np.maximum(x, 0) + 1)
    assert "[costmodel] #1 op=nnc_relu" in out
    assert "[costmodel] #2 op=nnc_add" in out
    assert "[costmodel] summary ops=2" in out
    assert "total_cycles=" in out
    recs = [LINE.match(l) for l in out.splitlines() if l.startswith("[costmodel] #")]
    assert all(recs) and len(recs) == 2
    (_, _, cu1, s1, e1, c1, in1, out1), (_, _, cu2, s2, e2, c2, in2, out2) = (m.groups() for m in recs)
    assert int(s1) == 0 and int(e1) >= int(s1) and int(s2) >= int(e1) and int(e2) >= int(s2)
    assert int(c1) == int(e1) - int(s1)
    assert (int(in1), int(out1)) == (16, 16) and (int(in2), int(out2)) == (32, 16)
    assert cu1 == cu2 == "0"
    assert f"[costmodel] summary cu=0 ready={e2}" in out
    assert so.nnc_cuda_trace_count() == 0  # dumped logs are cleared

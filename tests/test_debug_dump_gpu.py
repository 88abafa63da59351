"""Layer-by-layer parity: the cuda target's debug builds dump every
intermediate tensor in nnc-py's x86 debug-dump format; each tensor is
compared with the reference's own x86 debug build of the same graph on the
same image (tests/golden/debug_dumps.npz, made by
tests/golden/make_debug_golden.py), so a model-level difference can be
traced to the layer where it starts. Both dumps print "%f" (six decimals),
which bounds the comparison's resolution at 1e-6 absolute.

With NNC_DEBUG_TABLE=<path> the per-layer errors are also written there as
JSON (the table in the design notes comes from such a run)."""

from __future__ import annotations

import ctypes
import json
import os
import pathlib

import numpy as np
import pytest

import debugdump as D
import opcases as C
from nnc_cuda import lib as L
from nnc_cuda import workloads as W

pytestmark = pytest.mark.gpu

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "debug_dumps.npz"
PRINT_ABS = 2e-6  # two "%f" roundings


def _x86(key):
    z = np.load(GOLDEN)
    meta = json.loads(bytes(z[f"{key}/meta"]).decode())
    return meta, {m["name"]: (z[f"{key}/{m['name']}/idx"], z[f"{key}/{m['name']}/val"]) for m in meta}


@pytest.mark.parametrize("prec", [L.PRECISION_TF32, L.PRECISION_3XTF32])
@pytest.mark.parametrize("key,model", [("resnet18_o1_b1", "resnet18"), ("lenet5_o1_b1", "lenet5")])
def test_debug_dump_matches_x86_layer_by_layer(cuda_lib, tmp_path, key, model, prec):
    from nnc_cuda.model import CudaModel

    meta, want = _x86(key)
    m = CudaModel(f"{key}_debug")
    m.lib.nnc_model_set_debug_file.restype = ctypes.c_int
    m.lib.nnc_model_set_debug_file.argtypes = [ctypes.c_char_p]
    m.init(0)
    path = tmp_path / "nnc_debug_output.txt"
    try:
        m.load_constants(W.BUILDERS[model](1))
        cuda_lib.nnc_cuda_set_precision(prec)
        assert m.lib.nnc_model_set_debug_file(str(path).encode()) == 0
        m.run_host(W.BUILDERS[model](1).input_array(1))
    finally:
        m.lib.nnc_model_set_debug_file(None)
        m.free()
    got = D.parse(path.read_text())
    assert [n["name"] for n in meta] == sorted(got, key=lambda n: got[n]["node"])
    rows = []
    for mt in meta:
        g = got[mt["name"]]
        assert g["node"] == mt["node"] and g["shape"] == mt["shape"], mt["name"]
        idx, ref = want[mt["name"]]
        val = g["data"].reshape(-1)[idx].astype(np.float64)
        ref = ref.astype(np.float64)
        scale = float(np.max(np.abs(ref))) if ref.size else 0.0
        err = np.abs(val - ref)
        normwise = float(np.max(err / (np.abs(ref) + scale + 1e-30))) if ref.size else 0.0
        rows.append({"tensor": mt["name"], "node": mt["node"], "shape": mt["shape"], "max_abs": float(err.max()),
                     "normwise": normwise})
        lim = C.MODEL_RTOL[prec] * (np.abs(ref) + scale) + PRINT_ABS
        bad = np.flatnonzero(err > lim)
        assert bad.size == 0, f"{key} prec{prec}: layer {mt['name']} (node {mt['node']}) off: {rows[-1]}"
    table = os.environ.get("NNC_DEBUG_TABLE")
    if table:
        p = pathlib.Path(table)
        data = json.loads(p.read_text()) if p.exists() else {}
        data[f"{key}/prec{prec}"] = rows
        p.write_text(json.dumps(data, indent=1))
    print(f"\n{key} prec{prec}: " + ", ".join(f"{r['tensor']} {r['normwise']:.2g}" for r in rows))

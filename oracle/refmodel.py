"""Runs the reference's x86 model builds in oracle/_ref/ (TEST
INFRASTRUCTURE ONLY: model-level checker and CPU baseline)."""

from __future__ import annotations

import json
import os
import pathlib
import subprocess
import sys
import tempfile

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent / "nnc-py_b200"))
from nnc_cuda import workloads as W  # noqa: E402


def available(tag: str) -> bool:
    return (HERE / "_ref" / tag / "model_x86").exists()


def info(tag: str) -> dict:
    return json.loads((HERE / "_ref" / tag / "build.json").read_text())


def write_constants(tag: str, path: pathlib.Path) -> None:
    meta = info(tag)
    model = W.BUILDERS[meta["model"]](meta["batch"])
    path.write_bytes(W.nncb_bytes([(sym, model.constants[name]) for name, sym in meta["constants"]]))


def run(tag: str, x: np.ndarray, reps: int = 1, workdir: str | None = None) -> tuple[np.ndarray, float]:
    """Runs samples of x (a multiple of the compiled batch) through the x86
    build; returns (outputs, best seconds per compiled batch)."""
    meta = info(tag)
    tmp = pathlib.Path(workdir or tempfile.mkdtemp(prefix="nnc_ref_"))
    consts = tmp / "constants.bin"
    if not consts.exists():
        write_constants(tag, consts)
    (tmp / "input.bin").write_bytes(np.ascontiguousarray(x, np.float32).tobytes())
    exe = HERE / "_ref" / tag / "model_x86"
    r = subprocess.run([str(exe), str(consts), str(tmp / "input.bin"), str(tmp / "output.bin"), str(reps)],
                       capture_output=True, text=True, check=True)
    secs = float(r.stdout.strip().split("seconds_per_run=")[1])
    out = np.fromfile(tmp / "output.bin", dtype=np.float32)
    per = x.shape[0] // meta["batch"]
    model = W.BUILDERS[meta["model"]](meta["batch"])
    oshape = model.shapes[model.outputs[0]]
    return out.reshape((per * oshape[0],) + tuple(oshape[1:])), secs

"""The generated standalone runner (test_runner.c, built as `model` beside
each model library): reads constants.bin and input.bin, shards the batch
over the GPUs it is given, gathers the outputs to GPU 0 and writes
output.bin — the cuda target's counterpart of nnc-py's x86 test_runner.c
(codegen/x86_emitters/build_files.py:136-325). Its output is compared with
the reference's x86 build on the same seeded samples."""

from __future__ import annotations

import pathlib
import subprocess

import numpy as np
import pytest

import opcases as C
from nnc_cuda import lib as L
from nnc_cuda import workloads as W
from nnc_cuda.model import GEN_DIR, CudaModel

pytestmark = pytest.mark.gpu

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "models.npz"


def _run_runner(tmp_path, tag, model, x, gpus):
    exe = GEN_DIR / tag / "model"
    assert exe.exists(), f"{exe} missing: build with make -C nnc-py_b200/models_gen"
    consts = tmp_path / "constants.bin"
    consts.write_bytes(CudaModel(tag).constants_blob(model))
    (tmp_path / "input.bin").write_bytes(np.ascontiguousarray(x, np.float32).tobytes())
    r = subprocess.run([str(exe), str(consts), str(tmp_path / "input.bin"), str(tmp_path / "output.bin"), str(gpus)],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr + r.stdout
    assert "forward over" in r.stdout
    return np.fromfile(tmp_path / "output.bin", dtype=np.float32)


@pytest.mark.parametrize("tag,model_name,key,batch", [("lenet5_o1_b16", "lenet5", "lenet5_b16", 16),
                                                       ("resnet18_o3_b2", "resnet18", "resnet18_b2", 2)])
def test_runner_one_gpu_matches_reference(cuda_lib, tmp_path, tag, model_name, key, batch):
    g = np.load(GOLDEN)
    out = _run_runner(tmp_path, tag, W.BUILDERS[model_name](batch), g[f"{key}/input"], 1)
    want = g[f"{key}/output"]
    C.assert_close(out.reshape(want.shape), want, C.MODEL_RTOL[L.PRECISION_TF32], f"{tag} runner")


def test_runner_shards_over_all_gpus(cuda_lib, tmp_path):
    """Every GPU of the box runs one shard; each shard here holds the same
    16 samples, so every gathered shard must equal the reference's output."""
    import torch

    gpus = torch.cuda.device_count()
    g = np.load(GOLDEN)
    x = np.concatenate([g["lenet5_b16/input"]] * gpus)
    out = _run_runner(tmp_path, "lenet5_o1_b16", W.lenet5(16), x, gpus).reshape(gpus, 16, 10)
    for s in range(gpus):
        C.assert_close(out[s], g["lenet5_b16/output"], C.MODEL_RTOL[L.PRECISION_TF32], f"shard {s} of {gpus}")

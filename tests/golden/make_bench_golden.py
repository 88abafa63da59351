"""Regenerates tests/golden/bench_resnet18_o3.npz: the reference's own -O3 x86
build of ResNet-18 (nnc-py X86Backend with its legacy O3 pass list,
runtime/x86/ops.c, gcc -O3; built by oracle/ref_models.py as
oracle/_ref/resnet18_o3_b1) run on selected images of the benchmark's seeded
batch-1024 input.

The indices are the first and last image of every 128-image shard (the
per-GPU shards at 1, 2, 4 and 8 GPUs all start and end on these) plus 16
seeded interior images. The fixture stores the indices and the reference's
logits; the inputs are regenerated from the seed (nnc_cuda.workloads), so
the file stays small. Run where oracle/_ref is built:

    python tests/golden/make_bench_golden.py
"""

import pathlib
import subprocess
import sys
import tempfile

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path[:0] = [str(ROOT), str(ROOT / "nnc-py_b200")]

from nnc_cuda import workloads as W  # noqa: E402
from oracle import refmodel as R  # noqa: E402

TAG = "resnet18_o3_b1"
GLOBAL_BATCH = 1024
SHARD = 128


def indices() -> np.ndarray:
    edges = [i for s in range(0, GLOBAL_BATCH, SHARD) for i in (s, s + SHARD - 1)]
    rng = np.random.default_rng(2024)
    interior = [i for i in rng.permutation(GLOBAL_BATCH) if i not in edges][:16]
    return np.array(sorted(edges + interior), dtype=np.int64)


def main():
    idx = indices()
    x = W.resnet18(1).input_array(GLOBAL_BATCH)[idx]
    work = pathlib.Path(tempfile.mkdtemp(prefix="nnc_bench_golden_"))
    consts = work / "constants.bin"
    R.write_constants(TAG, consts)
    (work / "input.bin").write_bytes(np.ascontiguousarray(x).tobytes())
    exe = ROOT / "oracle" / "_ref" / TAG / "model_x86"
    procs = 8
    chunks = np.array_split(np.arange(len(idx)), procs)
    ps = [subprocess.Popen([str(exe), str(consts), str(work / "input.bin"), str(work / f"out{j}.bin"), "1",
                            str(int(c[0])), str(len(c))], stdout=subprocess.DEVNULL)
          for j, c in enumerate(chunks) if len(c)]
    if any(p.wait() for p in ps):
        raise RuntimeError("reference build failed")
    logits = np.concatenate([np.fromfile(work / f"out{j}.bin", dtype=np.float32).reshape(-1, 1000)
                             for j, c in enumerate(chunks) if len(c)])
    assert logits.shape == (len(idx), 1000)
    np.savez_compressed(HERE / "bench_resnet18_o3.npz", indices=idx, logits=logits)
    print(f"{len(idx)} images, logits {logits.shape}")


if __name__ == "__main__":
    main()

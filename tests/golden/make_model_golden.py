"""Regenerates tests/golden/models.npz: outputs of the reference's own x86
build (nnc-py X86Backend + runtime/x86/ops.c, built by oracle/ref_models.py)
for the seeded workload inputs. Run where oracle/_ref is built:

    python tests/golden/make_model_golden.py
"""

import pathlib
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path[:0] = [str(ROOT), str(ROOT / "nnc-py_b200")]

from nnc_cuda import workloads as W  # noqa: E402
from oracle import refmodel as R  # noqa: E402

# (fixture key, reference build, model, number of samples)
CASES = [("resnet18_b2", "resnet18_o1_b2", "resnet18", 2),
         ("lenet5_b16", "lenet5_o1_b16", "lenet5", 16),
         ("transformer_b1", "transformer_o1_b1", "transformer", 1)]


def main():
    blobs = {}
    for key, tag, model, n in CASES:
        x = W.BUILDERS[model](n).input_array(n)
        y, _ = R.run(tag, x)
        blobs[f"{key}/input"] = x
        blobs[f"{key}/output"] = y
        print(key, y.shape)
    np.savez_compressed(HERE / "models.npz", **blobs)


if __name__ == "__main__":
    main()

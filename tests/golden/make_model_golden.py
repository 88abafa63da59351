"""Regenerates tests/golden/models.npz: outputs of the reference's own x86
build (nnc-py X86Backend + runtime/x86/ops.c, built by oracle/ref_models.py)
for the seeded workload inputs. Run where oracle/_ref is built:

    python tests/golden/make_model_golden.py [fixture key ...]   (only these; the rest kept)
"""

import pathlib
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path[:0] = [str(ROOT), str(ROOT / "nnc-py_b200")]

from nnc_cuda import workloads as W  # noqa: E402
from oracle import refmodel as R  # noqa: E402

# (fixture key, reference build, model, number of samples, samples kept or
# None for all). Inputs are stored only when every sample is kept (the others
# are regenerated from the seed by nnc_cuda.workloads).
CASES = [("resnet18_b2", "resnet18_o1_b2", "resnet18", 2, None),
         ("lenet5_b16", "lenet5_o1_b16", "lenet5", 16, None),
         ("transformer_b1", "transformer_o1_b1", "transformer", 1, None),
         # Batch 256 runs ~5 minutes on one core; its first, a middle and the
         # last sample are kept.
         ("transformer_b256", "transformer_o1_b256", "transformer", 256, [0, 101, 255])]


def main():
    only = sys.argv[1:]
    path = HERE / "models.npz"
    blobs = dict(np.load(path)) if (only and path.exists()) else {}
    for key, tag, model, n, keep in CASES:
        if only and key not in only:
            continue
        x = W.BUILDERS[model](n).input_array(n)
        y, _ = R.run(tag, x)
        if keep is None:
            blobs[f"{key}/input"] = x
            blobs[f"{key}/output"] = y
        else:
            blobs[f"{key}/samples"] = np.array(keep, dtype=np.int64)
            blobs[f"{key}/output"] = y[keep]
        print(key, y.shape)
    np.savez_compressed(path, **blobs)


if __name__ == "__main__":
    main()

"""Regenerates tests/golden/debug_dumps.npz: the per-tensor debug dumps of
the reference's own x86 debug builds (nnc-py X86Backend(debug_mode=True) +
runtime/x86/ops.c, built by oracle/ref_models.py as oracle/_ref/<tag>_debug)
on the first seeded image, for the layer-by-layer comparison with the cuda
target's debug builds. Each tensor keeps its node index, shape and up to
4096 values spread evenly over it (tests/debugdump.sample_index), in the
dump's "%f" text precision. Run where oracle/_ref is built:

    python tests/golden/make_debug_golden.py
"""

import json
import pathlib
import subprocess
import sys
import tempfile

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path[:0] = [str(ROOT), str(ROOT / "nnc-py_b200"), str(ROOT / "tests")]

import debugdump as D  # noqa: E402
from nnc_cuda import workloads as W  # noqa: E402
from oracle import refmodel as R  # noqa: E402

BUILDS = [("resnet18_o1_b1", "resnet18"), ("lenet5_o1_b1", "lenet5")]


def main():
    blobs = {}
    for key, model in BUILDS:
        tag = f"{key}_debug"
        work = pathlib.Path(tempfile.mkdtemp(prefix="nnc_dbg_"))
        R.write_constants(tag, work / "constants.bin")
        (work / "input.bin").write_bytes(W.BUILDERS[model](1).input_array(1).tobytes())
        exe = ROOT / "oracle" / "_ref" / tag / "model_x86"
        r = subprocess.run([str(exe), str(work / "constants.bin"), str(work / "input.bin"), str(work / "out.bin")],
                           capture_output=True, text=True, check=True)
        dumps = D.parse(r.stdout)
        order = sorted(dumps, key=lambda n: dumps[n]["node"])
        meta = []
        for name in order:
            d = dumps[name]
            flat = d["data"].reshape(-1)
            idx = D.sample_index(flat.size)
            blobs[f"{key}/{name}/idx"] = idx
            blobs[f"{key}/{name}/val"] = flat[idx]
            meta.append({"name": name, "node": d["node"], "shape": d["shape"]})
        blobs[f"{key}/meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
        print(key, len(order), "tensors")
    np.savez_compressed(HERE / "debug_dumps.npz", **blobs)
    print(f"debug_dumps.npz {(HERE / 'debug_dumps.npz').stat().st_size / 1e3:.0f} kB")


if __name__ == "__main__":
    main()

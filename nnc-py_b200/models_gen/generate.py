"""Regenerates the committed cuda-target sources in this directory.

Each subdirectory is the output of ``nnc_cuda.codegen.compile_model`` (the
cuda target of nnc-py's compiler) for one BASELINE configuration; the
sources are committed so machines without nnc-py (the GPU box) can build and
run them. tests/test_codegen.py checks that they are up to date.

    python nnc-py_b200/models_gen/generate.py        # needs nnc-py importable
"""

from __future__ import annotations

import pathlib
import sys

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))

# (directory, model, batch, opt level)
CONFIGS = [
    # config 5: ResNet-18 -O3, batch 1024 split over 1/2/4/8 GPUs
    ("resnet18_o3_b1024", "resnet18", 1024, 3),
    ("resnet18_o3_b512", "resnet18", 512, 3),
    ("resnet18_o3_b256", "resnet18", 256, 3),
    ("resnet18_o3_b128", "resnet18", 128, 3),
    ("resnet18_o3_b2", "resnet18", 2, 3),
    # config 3: ResNet-18 -O1
    ("resnet18_o1_b256", "resnet18", 256, 1),
    ("resnet18_o1_b64", "resnet18", 64, 1),
    ("resnet18_o1_b2", "resnet18", 2, 1),
    # config 1: LeNet-5
    ("lenet5_o1_b8192", "lenet5", 8192, 1),
    ("lenet5_o1_b16", "lenet5", 16, 1),
    # config 4: transformer
    ("transformer_o1_b2048", "transformer", 2048, 1),
    ("transformer_o1_b256", "transformer", 256, 1),
    ("transformer_o1_b1", "transformer", 1, 1),
    # configs 1 and 4 at -O3 (Gemm+Relu, MatMul+bias(+Relu), MatMul+scale+Softmax groups)
    ("lenet5_o3_b8192", "lenet5", 8192, 3),
    ("lenet5_o3_b16", "lenet5", 16, 3),
    ("transformer_o3_b2048", "transformer", 2048, 3),
    ("transformer_o3_b256", "transformer", 256, 3),
    ("transformer_o3_b1", "transformer", 1, 3),
    # debug builds (every intermediate tensor dumped; layer-by-layer parity)
    ("resnet18_o1_b1_debug", "resnet18", 1, 1),
    ("lenet5_o1_b1_debug", "lenet5", 1, 1),
]


def is_debug(d: str) -> bool:
    return d.endswith("_debug")


def generate(only: str | None = None) -> list[str]:
    from nnc_cuda import codegen, workloads

    done = []
    for d, model, batch, opt in CONFIGS:
        if only and d != only:
            continue
        codegen.compile_model(workloads.BUILDERS[model](batch), HERE / d, opt_level=opt, debug=is_debug(d))
        done.append(d)
    return done


if __name__ == "__main__":
    for d in generate(sys.argv[1] if len(sys.argv) > 1 else None):
        print("generated", d)

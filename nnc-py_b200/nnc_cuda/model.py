"""Runs a model library produced by the cuda target (``libmodel.so`` built
from the generated model.c / tensors.c / constants_loader.c /
model_runtime.c): device selection, constant upload, forward passes on
device buffers or host buffers.

    m = CudaModel("nnc-py_b200/models_gen/resnet18_o3_b256")
    m.init(device=0)
    m.load_constants(workloads.resnet18(256))
    logits = m.run_host(x)          # numpy in, numpy out
"""

from __future__ import annotations

import ctypes
import json
import pathlib

import numpy as np

from . import lib as L
from .workloads import Model, nncb_bytes

GEN_DIR = pathlib.Path(__file__).resolve().parent.parent / "models_gen"


class CudaModel:
    def __init__(self, path: str | pathlib.Path):
        p = pathlib.Path(path)
        if not p.is_absolute() and not p.exists():
            p = GEN_DIR / p
        self.dir = p
        self.manifest = json.loads((p / "manifest.json").read_text())
        so = p / "libmodel.so"
        if not so.exists():
            raise RuntimeError(f"{so} is missing: build with `make -C {GEN_DIR}`")
        self.rt = L.load()  # libnnc_cuda.so, shared with the model library
        self.lib = ctypes.CDLL(str(so))
        for name, res, args in (
            ("nnc_model_init", ctypes.c_int, [ctypes.c_int]),
            ("nnc_model_select", ctypes.c_int, [ctypes.c_int]),
            ("nnc_model_free", None, [ctypes.c_int]),
            ("nnc_load_constants", ctypes.c_int, [ctypes.c_char_p]),
            ("nnc_load_constants_from_memory", ctypes.c_int, [ctypes.c_void_p, ctypes.c_size_t]),
            ("nnc_model_arena_bytes", ctypes.c_size_t, []),
            ("nnc_model_const_bytes", ctypes.c_size_t, []),
            ("nnc_model_input", L.TensorP, [ctypes.c_int]),
            ("nnc_model_output", L.TensorP, [ctypes.c_int]),
            ("nnc_model_run_host", ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
            ("nnc_run", None, []),
        ):
            fn = getattr(self.lib, name)
            fn.restype = res
            fn.argtypes = args
        self.in_shape = tuple(self.manifest["inputs"][0]["shape"])
        self.out_shape = tuple(self.manifest["outputs"][0]["shape"])
        self.device = None

    @property
    def batch(self) -> int:
        return int(self.in_shape[0])

    def init(self, device: int = 0) -> None:
        if self.lib.nnc_model_init(device) != 0:
            raise RuntimeError(f"nnc_model_init({device}) failed: {self.rt.nnc_cuda_get_last_error_string()}")
        self.device = device

    def free(self) -> None:
        """Releases this device's arena and constant slab (init() again to
        reuse the model on it)."""
        if self.device is not None:
            self.release_graph()
            self.lib.nnc_model_free(self.device)
            self.device = None

    def select(self) -> None:
        if self.lib.nnc_model_select(self.device) != 0:
            raise RuntimeError("nnc_model_select failed")

    def set_stream(self, stream_handle: int) -> None:
        self.rt.nnc_cuda_set_stream(ctypes.c_void_p(stream_handle))

    def constants_blob(self, model: Model) -> bytes:
        """NNCB bytes in the generated table's order and symbol names."""
        syms = {c["name"]: c["symbol"] for c in self.manifest["constants"]}
        order = [c["name"] for c in self.manifest["constants"]]
        return nncb_bytes([(syms[n], model.constants[n]) for n in order])

    def load_constants(self, model: Model) -> None:
        blob = self.constants_blob(model)
        buf = ctypes.create_string_buffer(blob, len(blob))
        if self.lib.nnc_load_constants_from_memory(ctypes.cast(buf, ctypes.c_void_p), len(blob)) != 0:
            raise RuntimeError(f"constant upload failed: {self.rt.nnc_cuda_get_last_error_string()}")

    def input_ptr(self) -> int:
        return int(self.lib.nnc_model_input(0).contents.data or 0)

    def output_ptr(self) -> int:
        return int(self.lib.nnc_model_output(0).contents.data or 0)

    def run(self) -> None:
        """Enqueues one forward pass on the current stream (no sync)."""
        self.lib.nnc_run()

    def capture(self) -> None:
        """Records one forward pass on the library's current stream (set with
        set_stream) into a CUDA graph; replay() then enqueues it in one
        launch. Run the model once uncaptured first (workspace sizing)."""
        self.release_graph()
        if self.rt.nnc_cuda_graph_begin() != 0:
            raise RuntimeError(f"capture failed: {self.rt.nnc_cuda_get_last_error_string()}")
        self.lib.nnc_run()
        g = self.rt.nnc_cuda_graph_end()
        if not g:
            raise RuntimeError(f"capture failed: {self.rt.nnc_cuda_get_last_error_string()}")
        self.graph = g

    def replay(self) -> None:
        """Enqueues the captured forward pass on the current stream (no sync)."""
        if self.rt.nnc_cuda_graph_launch(self.graph) != 0:
            raise RuntimeError(f"graph launch failed: {self.rt.nnc_cuda_get_last_error_string()}")

    def release_graph(self) -> None:
        g = getattr(self, "graph", None)
        if g:
            self.rt.nnc_cuda_graph_destroy(g)
        self.graph = None

    def run_host(self, x: np.ndarray) -> np.ndarray:
        """Host-buffer forward (H2D, forward, D2H; synchronous)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.shape != self.in_shape:
            raise ValueError(f"input shape {x.shape} != compiled {self.in_shape}")
        out = np.empty(self.out_shape, dtype=np.float32)
        rc = self.lib.nnc_model_run_host(x.ctypes.data, out.ctypes.data)
        if rc != 0:
            raise RuntimeError(f"forward failed ({rc}): {self.rt.nnc_cuda_get_last_error_string()}")
        return out

"""Builds ``Tensor`` descriptors over torch device tensors and numpy arrays.

A descriptor owns its host shape array; keep the :class:`TensorRef` alive
for as long as the C side may read it.
"""

from __future__ import annotations

import ctypes
from typing import Any

import numpy as np

from . import lib as _lib

_NP_DTYPE = {np.dtype(np.float32): _lib.DTYPE_FLOAT32, np.dtype(np.int64): _lib.DTYPE_INT64,
             np.dtype(np.int32): _lib.DTYPE_INT32, np.dtype(np.uint8): _lib.DTYPE_BOOL}


class TensorRef:
    """A ctypes ``Tensor`` plus the objects that must outlive it."""

    def __init__(self, data_ptr: int, dtype: int, shape: tuple[int, ...], nbytes: int, owner: Any):
        self.shape_arr = (ctypes.c_int64 * max(len(shape), 1))(*shape)
        self.struct = _lib.Tensor(
            data=ctypes.c_void_p(data_ptr) if data_ptr else None,
            dtype=dtype,
            shape=ctypes.cast(self.shape_arr, ctypes.POINTER(ctypes.c_int64)),
            ndim=len(shape),
            nbytes=nbytes,
        )
        self.owner = owner
        self.logical_shape = tuple(shape)

    @property
    def ptr(self) -> ctypes._Pointer:
        return ctypes.pointer(self.struct)


def from_torch(t, tag: int = 0, shape: tuple[int, ...] | None = None) -> TensorRef:
    """Descriptor over a contiguous CUDA torch tensor.

    ``shape`` overrides the logical shape (e.g. NCHW extents of an NHWC-stored
    activation tagged with ``TAG_NHWC``).
    """
    import torch

    if not t.is_contiguous():
        raise ValueError("tensor must be contiguous")
    dt = {torch.float32: _lib.DTYPE_FLOAT32, torch.int64: _lib.DTYPE_INT64, torch.int32: _lib.DTYPE_INT32,
          torch.uint8: _lib.DTYPE_BOOL}[t.dtype]
    shp = tuple(int(s) for s in (shape if shape is not None else t.shape))
    return TensorRef(t.data_ptr(), dt | tag, shp, t.numel() * t.element_size(), t)


def from_numpy(a: np.ndarray) -> TensorRef:
    """Descriptor over a C-contiguous host array (used with the CPU oracle)."""
    if not a.flags["C_CONTIGUOUS"]:
        raise ValueError("array must be C-contiguous")
    return TensorRef(a.ctypes.data, _NP_DTYPE[a.dtype], tuple(int(s) for s in a.shape), a.nbytes, a)


def as_ptr(x) -> ctypes._Pointer | None:
    """Accepts a TensorRef, a torch tensor, a numpy array or None."""
    if x is None:
        return None
    if isinstance(x, TensorRef):
        return x.ptr
    if isinstance(x, np.ndarray):
        raise TypeError("wrap host arrays with from_numpy() and keep the ref alive")
    raise TypeError(f"unsupported tensor argument {type(x)!r}")


def tensor_array(refs: list[TensorRef]):
    """A ``Tensor**`` for concat/split."""
    arr = (_lib.TensorP * len(refs))(*[r.ptr for r in refs])
    return arr

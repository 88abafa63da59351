"""ctypes binding of libnnc_cuda.so, the B200 operator library.

Mirrors how nnc-py's own runtime tests drive the x86 operator library
(tests/test_x86_runtime.py:263-272: a ctypes ``Tensor`` and ``lib.nnc_*``
calls), except that ``Tensor.data`` holds a device pointer.

Loading is strict: if the shared library is missing or lacks a declared
symbol, :func:`load` raises — there is no CPU fallback behind this module.
"""

from __future__ import annotations

import ctypes
import os
import pathlib
import re

PKG_DIR = pathlib.Path(__file__).resolve().parent
REPO_ROOT = PKG_DIR.parent.parent
INCLUDE_DIR = REPO_ROOT / "include"
LIB_PATH = PKG_DIR / "libnnc_cuda.so"

# Element types (runtime/include/nnc_types.h:16-24 of the reference).
DTYPE_FLOAT32 = 0
DTYPE_INT32 = 2
DTYPE_BOOL = 5  # one byte per element (numpy / torch uint8)
DTYPE_INT64 = 6
# Storage tags (include/nnc_cuda.h).
TAG_NHWC = 0x100
TAG_PACKED_CONV = 0x200

OK = 0
ERR_INVALID = 1
ERR_UNSUPPORTED = 2
ERR_LAUNCH = 3
ERR_NOMEM = 4
ERR_DEVICE_TIMEOUT = 5

PRECISION_TF32 = 0
PRECISION_3XTF32 = 1


class Tensor(ctypes.Structure):
    """Same layout as ``Tensor`` in include/nnc_types.h."""

    _fields_ = [
        ("data", ctypes.c_void_p),
        ("dtype", ctypes.c_int),
        ("shape", ctypes.POINTER(ctypes.c_int64)),
        ("ndim", ctypes.c_int),
        ("nbytes", ctypes.c_int64),
    ]


TensorP = ctypes.POINTER(Tensor)

# Argument kinds used to build ctypes prototypes from the C headers.
_CTYPE_OF = {
    "Tensor*": TensorP,
    "Tensor**": ctypes.POINTER(TensorP),
    "const Tensor*": TensorP,
    "int": ctypes.c_int,
    "float": ctypes.c_float,
    "int64_t*": ctypes.POINTER(ctypes.c_int64),
    "void*": ctypes.c_void_p,
    "const void*": ctypes.c_void_p,
    "size_t": ctypes.c_size_t,
    "const char*": ctypes.c_char_p,
    "void": None,
    "long long": ctypes.c_longlong,
}

_PROTO_RE = re.compile(
    r"^\s*((?:const\s+)?(?:long\s+long|\w+)\s*\**)\s*(nnc_\w+)\s*\(([^)]*)\)\s*;", re.M | re.S
)


def header_prototypes(header: str) -> dict[str, tuple[str, list[str]]]:
    """Parses ``include/<header>`` into {name: (return type, [arg types])}."""
    text = (INCLUDE_DIR / header).read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    protos: dict[str, tuple[str, list[str]]] = {}
    for ret, name, args in _PROTO_RE.findall(text):
        ret = " ".join(ret.replace("*", " *").split()).replace(" *", "*")
        if ret not in _CTYPE_OF:
            raise ValueError(f"unsupported return type {ret!r} of {name}")
        args = " ".join(args.split())
        types: list[str] = []
        if args and args != "void":
            for a in args.split(","):
                a = a.strip()
                m = re.match(r"(const\s+)?(\w+)\s*(\**)\s*\w*$", a)
                if not m:
                    raise ValueError(f"cannot parse argument {a!r} of {name}")
                types.append(f"{m.group(1) or ''}{m.group(2)}{m.group(3)}")
        protos[name] = (ret, types)
    return protos


def declared_symbols() -> dict[str, tuple[str, list[str]]]:
    protos = {}
    for h in ("nnc_ops.h", "nnc_cuda.h"):
        protos.update(header_prototypes(h))
    return protos


_LIB: ctypes.CDLL | None = None


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Loads libnnc_cuda.so and types every symbol the headers declare."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    p = pathlib.Path(path) if path else LIB_PATH
    if not p.exists():
        raise RuntimeError(
            f"{p} is missing: build it with `make -C nnc-py_b200/csrc` "
            "(or __graft_entry__.build()); there is no fallback implementation"
        )
    lib = ctypes.CDLL(str(p))
    for name, (ret, args) in declared_symbols().items():
        fn = getattr(lib, name)  # AttributeError if the library lacks it
        fn.restype = _CTYPE_OF[ret] if ret != "void*" else ctypes.c_void_p
        fn.argtypes = [_CTYPE_OF[a] for a in args]
    if path is None:
        _LIB = lib
    return lib

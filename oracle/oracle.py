"""ctypes binding of the CPU checkers (TEST INFRASTRUCTURE ONLY).

* ``load_oracle()`` — liboracle.so, the restatement in nnc_oracle.c;
* ``load_reference()`` — _ref/libref_ops.so, the reference's own ops.c
  compiled from its sources (present only where it was built).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module. Both libraries take host pointers and export the reference's
``nnc_*`` names, typed here from include/nnc_ops.h.
"""

from __future__ import annotations

import ctypes
import pathlib
import sys

HERE = pathlib.Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libref_ops.so"

sys.path.insert(0, str(HERE.parent / "nnc-py_b200"))
from nnc_cuda import lib as _lib  # noqa: E402  (Tensor layout + header parser)


def _typed(path: pathlib.Path) -> ctypes.CDLL:
    so = ctypes.CDLL(str(path))
    for name, (ret, args) in _lib.header_prototypes("nnc_ops.h").items():
        fn = getattr(so, name, None)
        if fn is None:
            continue  # the reference lacks the fused entry points added here
        fn.restype = None if ret == "void" else _lib._CTYPE_OF[ret]
        fn.argtypes = [_lib._CTYPE_OF[a] for a in args]
    return so


def load_oracle() -> ctypes.CDLL:
    if not ORACLE_SO.exists():
        raise RuntimeError(f"{ORACLE_SO} missing: run `make -C oracle`")
    return _typed(ORACLE_SO)


def reference_available() -> bool:
    return REF_SO.exists()


def load_reference() -> ctypes.CDLL:
    if not REF_SO.exists():
        raise RuntimeError(f"{REF_SO} missing: run `make -C oracle ref` where the reference exists")
    return _typed(REF_SO)

"""nnc_cuda — host side of the B200 operator library for nnc-py.

* :mod:`nnc_cuda.lib`      ctypes binding of libnnc_cuda.so (strict loading)
* :mod:`nnc_cuda.tensor`   ``Tensor`` descriptors over torch / numpy buffers
* :mod:`nnc_cuda.workloads` BASELINE configs as layer lists + seeded weights
* :mod:`nnc_cuda.model`    runs a compiled ``-t cuda`` model library
* :mod:`nnc_cuda.codegen`  the ``cuda`` target for nnc-py's compiler
  (imports nnc-py, so it only works where nnc-py is importable)
"""

from . import lib  # noqa: F401
from .lib import load  # noqa: F401

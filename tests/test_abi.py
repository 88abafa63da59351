"""C-ABI checks that need no GPU: the library loads, exports every symbol the
headers declare, and the Tensor descriptor has the reference's layout."""

import ctypes
import subprocess

import pytest

from nnc_cuda import lib as L
from oracle import oracle as O


def test_headers_parse_and_cover_reference_hot_path():
    protos = L.declared_symbols()
    hot = {"nnc_add", "nnc_sub", "nnc_mul", "nnc_div", "nnc_relu", "nnc_sigmoid", "nnc_tanh", "nnc_clip",
           "nnc_add_relu", "nnc_add_sigmoid", "nnc_softmax", "nnc_layernorm", "nnc_reducemean", "nnc_reducesum",
           "nnc_maxpool2d", "nnc_avgpool2d", "nnc_reshape", "nnc_flatten", "nnc_transpose", "nnc_squeeze",
           "nnc_unsqueeze", "nnc_identity", "nnc_concat", "nnc_split", "nnc_matmul", "nnc_gemm", "nnc_gemm_nt",
           "nnc_conv", "nnc_conv1x1", "nnc_conv3x3_s1", "nnc_conv7x7_s2", "nnc_conv_relu", "nnc_conv_relu1x1",
           "nnc_conv_relu3x3_s1", "nnc_conv_relu7x7_s2", "nnc_conv_sigmoid", "nnc_conv_add_relu",
           "nnc_gemm_relu", "nnc_matmul_relu"}
    assert hot <= set(protos), sorted(hot - set(protos))
    assert protos["nnc_conv"] == ("void", ["Tensor*"] * 4 + ["int"] * 6)
    assert protos["nnc_gemm"] == ("void", ["Tensor*"] * 4 + ["float", "float", "int", "int"])
    assert protos["nnc_concat"] == ("void", ["Tensor**", "Tensor*", "int", "int"])


def test_library_loads_and_exports_every_declared_symbol():
    so = L.load()  # raises if a declared symbol is missing
    exported = subprocess.run(["nm", "-D", "--defined-only", str(L.LIB_PATH)], capture_output=True, text=True,
                              check=True).stdout.split()
    for name in L.declared_symbols():
        assert name in exported, name
        assert getattr(so, name) is not None


def test_oracle_exports_reference_names():
    orc = O.load_oracle()
    for name in L.header_prototypes("nnc_ops.h"):
        assert hasattr(orc, name), name


def test_tensor_layout_matches_c(tmp_path):
    src = tmp_path / "t.c"
    src.write_text('#include <stddef.h>\n#include <stdio.h>\n#include "nnc_types.h"\n'
                   'int main(void){printf("%zu %zu %zu %zu %zu %zu",sizeof(Tensor),offsetof(Tensor,data),'
                   'offsetof(Tensor,dtype),offsetof(Tensor,shape),offsetof(Tensor,ndim),offsetof(Tensor,nbytes));return 0;}\n')
    exe = tmp_path / "t"
    subprocess.run(["gcc", f"-I{L.INCLUDE_DIR}", str(src), "-o", str(exe)], check=True)
    vals = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    T = L.Tensor
    assert vals == [ctypes.sizeof(T), T.data.offset, T.dtype.offset, T.shape.offset, T.ndim.offset, T.nbytes.offset]


def test_status_api_without_device():
    so = L.load()
    so.nnc_cuda_clear_error()
    assert so.nnc_cuda_get_last_error() == 0
    so.nnc_cuda_set_precision(L.PRECISION_3XTF32)
    assert so.nnc_cuda_get_precision() == L.PRECISION_3XTF32
    so.nnc_cuda_set_precision(L.PRECISION_TF32)
    # A NULL tensor is rejected on the host before any device work.
    so.nnc_relu(None, None)
    assert so.nnc_cuda_get_last_error() == L.ERR_INVALID
    assert b"NULL" in so.nnc_cuda_get_last_error_string()
    so.nnc_cuda_clear_error()


def test_prepacked_weight_size():
    so = L.load()
    shape = (ctypes.c_int64 * 4)(64, 3, 7, 7)
    t = L.Tensor(None, 0, ctypes.cast(shape, ctypes.POINTER(ctypes.c_int64)), 4, 0)
    # C_in = 3 padded to 4 (chunk order): K = 7*7*4 = 196 -> 224; two planes of 64 x 224.
    assert so.nnc_cuda_prepacked_conv_weight_bytes(ctypes.byref(t)) == 2 * 64 * 224 * 4


def test_parser_sees_every_declaration():
    """Every nnc_* prototype in the headers is typed (a missed declaration
    would leave ctypes guessing its return type)."""
    import re

    for h in ("nnc_ops.h", "nnc_cuda.h"):
        text = re.sub(r"/\*.*?\*/", "", (L.INCLUDE_DIR / h).read_text(), flags=re.S)
        decls = set(re.findall(r"\b(nnc_\w+)\s*\(", text))
        assert decls == set(L.header_prototypes(h)), decls ^ set(L.header_prototypes(h))

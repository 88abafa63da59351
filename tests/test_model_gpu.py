"""Model-level parity on the GPU: cuda-target builds of the BASELINE graphs
(nnc-py_b200/models_gen) against the reference's own x86 build of the same
graphs on the same seeded inputs (tests/golden/models.npz)."""

import pathlib

import numpy as np
import pytest

import opcases as C
from nnc_cuda import lib as L
from nnc_cuda import workloads as W

pytestmark = pytest.mark.gpu

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "models.npz"
# End-to-end tolerances (normwise rtol, see opcases.assert_close and the
# measured figures beside opcases.MODEL_RTOL).
MODEL_RTOL = C.MODEL_RTOL


@pytest.fixture(scope="module")
def golden():
    z = np.load(GOLDEN)
    return {k: z[k] for k in z.files}


def _model(tag):
    from nnc_cuda.model import CudaModel

    m = CudaModel(tag)
    m.init(0)
    return m


@pytest.mark.parametrize("prec", [L.PRECISION_TF32, L.PRECISION_3XTF32])
@pytest.mark.parametrize("tag", ["resnet18_o3_b2", "resnet18_o1_b2"])
def test_resnet18_matches_reference_x86_build(cuda_lib, golden, tag, prec):
    m = _model(tag)
    m.load_constants(W.resnet18(2))
    cuda_lib.nnc_cuda_set_precision(prec)
    got = m.run_host(golden["resnet18_b2/input"])
    want = golden["resnet18_b2/output"]
    C.assert_close(got, want, MODEL_RTOL[prec], f"{tag} prec{prec}")
    assert np.array_equal(got.argmax(1), want.argmax(1))


@pytest.mark.parametrize("prec", [L.PRECISION_TF32, L.PRECISION_3XTF32])
def test_resnet18_batch_shards_agree(cuda_lib, golden, prec):
    """Sample independence (what batch sharding across GPUs relies on): the
    first two images of a batch-128 forward equal the batch-2 reference."""
    m = _model("resnet18_o3_b128")
    model = W.resnet18(128)
    m.load_constants(model)
    cuda_lib.nnc_cuda_set_precision(prec)
    got = m.run_host(model.input_array(128))
    C.assert_close(got[:2], golden["resnet18_b2/output"], MODEL_RTOL[prec], f"b128[:2] prec{prec}")


BENCH_GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "bench_resnet18_o3.npz"
GLOBAL_BATCH = 1024


@pytest.fixture(scope="module")
def bench_input():
    """The benchmark's seeded batch-1024 input (616 MB) and the reference
    logits of 32 of its images (the -O3 x86 build)."""
    z = np.load(BENCH_GOLDEN)
    return W.resnet18(1).input_array(GLOBAL_BATCH), z["indices"], z["logits"]


@pytest.mark.parametrize("prec", [L.PRECISION_TF32, L.PRECISION_3XTF32])
@pytest.mark.parametrize("per_gpu", [1024, 512, 256, 128])
def test_bench_config_matches_reference_x86_build(cuda_lib, bench_input, per_gpu, prec):
    """The benchmarked configuration itself: ResNet-18 -O3 over the global
    batch of 1024, compiled for the per-GPU batch of 1, 2, 4 and 8 GPUs and
    run shard by shard (as the ranks of `bench.py --gpus N` do), the shards'
    logits put together in rank order and compared at the fixture's indices
    (the first and last image of every 128-image shard and 16 others) with
    the reference's -O3 x86 build on the same images."""
    x, idx, want = bench_input
    m = _model(f"resnet18_o3_b{per_gpu}")
    try:
        m.load_constants(W.resnet18(per_gpu))
        cuda_lib.nnc_cuda_set_precision(prec)
        shards = [m.run_host(x[s:s + per_gpu]) for s in range(0, GLOBAL_BATCH, per_gpu)]
    finally:
        m.free()
    got = np.concatenate(shards)
    assert got.shape == (GLOBAL_BATCH, 1000)
    C.assert_close(got[idx], want, MODEL_RTOL[prec], f"resnet18_o3_b{per_gpu} prec{prec}")


@pytest.mark.parametrize("tag", ["lenet5_o1_b16", "lenet5_o3_b16"])
def test_lenet5_matches_reference_x86_build(cuda_lib, golden, tag):
    """-O1, and -O3 with the Gemm+Relu group (nnc_gemm_nt_relu)."""
    m = _model(tag)
    m.load_constants(W.lenet5(16))
    for prec in (L.PRECISION_TF32, L.PRECISION_3XTF32):
        cuda_lib.nnc_cuda_set_precision(prec)
        got = m.run_host(golden["lenet5_b16/input"])
        C.assert_close(got, golden["lenet5_b16/output"], MODEL_RTOL[prec], f"lenet5 prec{prec}")


@pytest.mark.parametrize("tag", ["transformer_o1_b1", "transformer_o3_b1"])
def test_transformer_matches_reference_x86_build(cuda_lib, golden, tag):
    """-O1, and -O3 with the MatMul epilogue groups (bias, bias+relu,
    scale+softmax); the reference's x86 build runs the unfused ops."""
    m = _model(tag)
    m.load_constants(W.transformer(1))
    for prec in (L.PRECISION_TF32, L.PRECISION_3XTF32):
        cuda_lib.nnc_cuda_set_precision(prec)
        got = m.run_host(golden["transformer_b1/input"])
        C.assert_close(got, golden["transformer_b1/output"], MODEL_RTOL[prec], f"transformer prec{prec}")


def test_graph_replay_matches_direct_run(cuda_lib, golden):
    """A forward pass captured into a CUDA graph (nnc_cuda_graph_*) and
    replayed gives bit-identical logits to direct runs on new inputs written
    into the same input tensor, and counts its kernels per replay."""
    import ctypes

    import torch

    m = _model("resnet18_o3_b2")
    m.load_constants(W.resnet18(2))
    cuda_lib.nnc_cuda_set_precision(L.PRECISION_TF32)
    stream = torch.cuda.Stream()
    m.set_stream(stream.cuda_stream)
    n_in = int(np.prod(m.in_shape))
    inp = torch.empty(n_in, dtype=torch.float32, device="cuda")
    out = torch.empty(int(np.prod(m.out_shape)), dtype=torch.float32, device="cuda")
    r = np.random.default_rng(3)
    xs = [golden["resnet18_b2/input"].ravel()] + [r.standard_normal(n_in).astype(np.float32) for _ in range(2)]

    def run(x, graph):
        inp.copy_(torch.from_numpy(x))
        torch.cuda.synchronize()
        cuda_lib.nnc_cuda_memcpy_async(ctypes.c_void_p(m.input_ptr()), ctypes.c_void_p(inp.data_ptr()), n_in * 4, 3)
        m.replay() if graph else m.run()
        cuda_lib.nnc_cuda_memcpy_async(ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(m.output_ptr()),
                                       out.numel() * 4, 3)
        stream.synchronize()
        assert cuda_lib.nnc_cuda_get_last_error() == 0, cuda_lib.nnc_cuda_get_last_error_string()
        return out.cpu().numpy().copy()

    direct = [run(x, False) for x in xs]
    before = cuda_lib.nnc_cuda_launch_count()
    m.capture()
    assert cuda_lib.nnc_cuda_launch_count() == before  # captured, not launched
    kernels = cuda_lib.nnc_cuda_graph_kernels(m.graph)
    assert kernels > 10
    try:
        for x, want in zip(xs, direct):
            c0 = cuda_lib.nnc_cuda_launch_count()
            got = run(x, True)
            assert cuda_lib.nnc_cuda_launch_count() - c0 == kernels
            assert np.array_equal(got, want)
    finally:
        m.release_graph()
        cuda_lib.nnc_cuda_set_stream(None)
    C.assert_close(direct[0].reshape(m.out_shape), golden["resnet18_b2/output"], MODEL_RTOL[L.PRECISION_TF32],
                   "direct run")

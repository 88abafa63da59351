// Host-side TMA tensor-map encoding through the driver entry point (no link
// dependency on libcuda; the runtime resolves cuTensorMapEncodeTiled once).
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "tc.cuh"

namespace nnc {

namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode_tiled = nullptr;
std::once_flag g_once;

void resolve() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
          cudaSuccess &&
      q == cudaDriverEntryPointSuccess) {
    g_encode_tiled = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
}
}  // namespace

bool encode_tmap_f32(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                     const uint64_t* strides_bytes, const uint32_t* box,
                     const uint32_t* elem_strides, const char* op) {
  std::call_once(g_once, resolve);
  if (!g_encode_tiled) {
    fail(NNC_CUDA_ERR_LAUNCH, op, "cuTensorMapEncodeTiled is unavailable");
    return false;
  }
  if (((uintptr_t)base & 15u) != 0) {
    fail(NNC_CUDA_ERR_UNSUPPORTED, op, "TMA base address %p is not 16-byte aligned", base);
    return false;
  }
  for (int i = 0; i + 1 < rank; ++i) {
    if (strides_bytes[i] % 16 != 0) {
      fail(NNC_CUDA_ERR_UNSUPPORTED, op, "TMA stride %llu is not a multiple of 16 bytes",
           (unsigned long long)strides_bytes[i]);
      return false;
    }
  }
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t bdim[5], estr[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estr[i] = elem_strides ? elem_strides[i] : 1;
  }
  for (int i = 0; i + 1 < rank; ++i) gstride[i] = strides_bytes[i];
  CUresult r = g_encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (cuuint32_t)rank,
                              const_cast<void*>(base), gdim, gstride, bdim, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    fail(NNC_CUDA_ERR_LAUNCH, op, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return false;
  }
  return true;
}

}  // namespace nnc

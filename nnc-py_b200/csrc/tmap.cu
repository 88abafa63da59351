// Host-side TMA tensor-map encoding through the driver entry points (no link
// dependency on libcuda; the runtime resolves the encoders once).
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "tc.cuh"

namespace nnc {

namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode_tiled = nullptr;
PFN_cuTensorMapEncodeIm2col_v12000 g_encode_im2col = nullptr;
std::once_flag g_once;

void resolve() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
          cudaSuccess &&
      q == cudaDriverEntryPointSuccess) {
    g_encode_tiled = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  fn = nullptr;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &fn, cudaEnableDefault, &q) ==
          cudaSuccess &&
      q == cudaDriverEntryPointSuccess) {
    g_encode_im2col = reinterpret_cast<PFN_cuTensorMapEncodeIm2col_v12000>(fn);
  }
}

bool check_base_and_strides(const void* base, int n, const uint64_t* strides, const char* op) {
  if (((uintptr_t)base & 15u) != 0) {
    fail(NNC_CUDA_ERR_UNSUPPORTED, op, "TMA base address %p is not 16-byte aligned", base);
    return false;
  }
  for (int i = 0; i < n; ++i) {
    if (strides[i] % 16 != 0) {
      fail(NNC_CUDA_ERR_UNSUPPORTED, op, "TMA stride %llu is not a multiple of 16 bytes",
           (unsigned long long)strides[i]);
      return false;
    }
  }
  return true;
}
}  // namespace

bool encode_tmap_f32(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                     const uint64_t* strides_bytes, const uint32_t* box,
                     const uint32_t* elem_strides, const char* op, int swizzle_bytes) {
  std::call_once(g_once, resolve);
  if (!g_encode_tiled) {
    fail(NNC_CUDA_ERR_LAUNCH, op, "cuTensorMapEncodeTiled is unavailable");
    return false;
  }
  if (!check_base_and_strides(base, rank - 1, strides_bytes, op)) return false;
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t bdim[5], estr[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estr[i] = elem_strides ? elem_strides[i] : 1;
  }
  for (int i = 0; i + 1 < rank; ++i) gstride[i] = strides_bytes[i];
  if (swizzle_bytes != 128 && swizzle_bytes != 64 && swizzle_bytes != kSwizzle128Atom32) {
    fail(NNC_CUDA_ERR_LAUNCH, op, "unsupported TMA swizzle span %d", swizzle_bytes);
    return false;
  }
  const CUtensorMapSwizzle swz = swizzle_bytes == 64                  ? CU_TENSOR_MAP_SWIZZLE_64B
                                 : swizzle_bytes == kSwizzle128Atom32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                                                                      : CU_TENSOR_MAP_SWIZZLE_128B;
  CUresult r = g_encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (cuuint32_t)rank,
                              const_cast<void*>(base), gdim, gstride, bdim, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    fail(NNC_CUDA_ERR_LAUNCH, op, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return false;
  }
  return true;
}

bool encode_tmap_im2col_f32(CUtensorMap* map, const void* base, const uint64_t* dims,
                            const uint64_t* strides_bytes, int lower, int upper,
                            uint32_t channels_per_pixel, uint32_t pixels_per_column,
                            uint32_t stride, bool swizzle128, const char* op) {
  std::call_once(g_once, resolve);
  if (!g_encode_im2col) {
    fail(NNC_CUDA_ERR_LAUNCH, op, "cuTensorMapEncodeIm2col is unavailable");
    return false;
  }
  if (!check_base_and_strides(base, 3, strides_bytes, op)) return false;
  cuuint64_t gdim[4] = {dims[0], dims[1], dims[2], dims[3]};
  cuuint64_t gstride[3] = {strides_bytes[0], strides_bytes[1], strides_bytes[2]};
  int lo[2] = {lower, lower};
  int up[2] = {upper, upper};
  cuuint32_t estr[4] = {1, stride, stride, 1};
  CUresult r = g_encode_im2col(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void*>(base),
                               gdim, gstride, lo, up, channels_per_pixel, pixels_per_column, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE,
                               swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    fail(NNC_CUDA_ERR_LAUNCH, op, "cuTensorMapEncodeIm2col failed (%d)", (int)r);
    return false;
  }
  return true;
}

}  // namespace nnc

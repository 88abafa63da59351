/*
 * nnc_types.h — tensor descriptor shared by generated model code and the
 * B200 operator library (libnnc_cuda.so).
 *
 * Binary-compatible with nnc-py's runtime/include/nnc_types.h:16-33, so a
 * model.c emitted by nnc-py links against this library unchanged:
 *   - same enum values for the element types;
 *   - same field order and types in `Tensor`.
 *
 * Differences in meaning on the CUDA target:
 *   - `data` is a DEVICE pointer (cudaMalloc'd or an offset into a device
 *     arena/constant slab);
 *   - `shape` stays a HOST array; launchers read it on the CPU;
 *   - the upper bits of `dtype` may carry a storage tag (see nnc_cuda.h:
 *     NNC_CUDA_TAG_*). Untagged tensors (the values below) are dense,
 *     row-major, exactly as in the reference.
 */
#ifndef NNC_TYPES_H
#define NNC_TYPES_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    NNC_DTYPE_FLOAT32 = 0,
    NNC_DTYPE_FLOAT16 = 1,
    NNC_DTYPE_INT32 = 2,
    NNC_DTYPE_INT8 = 3,
    NNC_DTYPE_UINT8 = 4,
    NNC_DTYPE_BOOL = 5,
    NNC_DTYPE_INT64 = 6,
} nnc_dtype_t;

typedef struct {
    void* data;        /* device pointer on the CUDA target */
    nnc_dtype_t dtype; /* element type (low byte) | optional storage tag */
    int64_t* shape;    /* host array of ndim extents (logical, NCHW for 4-D) */
    int ndim;
    int64_t nbytes;
} Tensor;

#ifdef __cplusplus
}
#endif

#endif /* NNC_TYPES_H */

// Internal data-movement helpers shared by the conv/gemm launchers.
#pragma once
#include <stdint.h>

namespace nnc {
// out[b][c][r] = in[b * in_batch_stride + r * C + c] for `batch` row-major
// R x C fp32 matrices (in_batch_stride < 0 means R * C), written densely;
// enqueued on the current stream. Returns false (status set) on launch error.
bool batched_transpose_f32(const float* in, float* out, int64_t batch, int64_t R, int64_t C,
                           const char* op, int64_t in_batch_stride = -1);
}  // namespace nnc

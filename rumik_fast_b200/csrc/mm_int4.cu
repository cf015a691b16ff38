// mm_int4.cu - int4-weight prefill matmul on tcgen05 tensor cores (in progress).
#include "common.cuh"
#include "kernels.h"

namespace rb {
int launch_mm_int4(const MmArgs&, int, cudaStream_t) { return RB_ERR_SHAPE; }
}  // namespace rb

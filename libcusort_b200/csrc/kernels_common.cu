// kernels_common.cu -- the init kernel (shared by every key width).
#include "cusort_dispatch.h"
#include "cusort_kernels.cuh"

namespace cusort_b200 {

// ---------------------------------------------------------------------------
// init: zero n16 16-byte words.  Launched with full stream ordering (it is the
// first kernel of a sort and may overwrite memory the caller's previous work
// used), it releases the histogram kernel early via PDL.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(512) init_kernel(const InitArgs a) {
  dev::pdl_launch_dependents();
  uint4* p = static_cast<uint4*>(a.ptr);
  const uint4 z = make_uint4(0, 0, 0, 0);
  for (uint64_t i = blockIdx.x * 512ull + threadIdx.x; i < a.n16; i += (uint64_t)gridDim.x * 512ull) p[i] = z;
}

const void* get_init_kernel() { return reinterpret_cast<const void*>(&init_kernel); }

}  // namespace cusort_b200

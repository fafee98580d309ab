// cusort_dispatch.h -- internal host-side interface between the dispatcher
// and the per-key-width kernel instantiation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace cusort_b200 {

struct KernelInfo {
  const void* func = nullptr;  // __global__ function
  int threads = 0;             // CTA size
  int tile = 0;                // items per tile (onesweep) / vectors per CTA step (histogram)
  size_t smem = 0;             // dynamic shared memory bytes
};

// One entry per key width; value bytes in {0,1,2,4,8,16}, off_bytes in {4,8}.
bool get_kernels_k1(int value_bytes, int off_bytes, KernelInfo* onesweep, KernelInfo* histogram);
bool get_kernels_k2(int value_bytes, int off_bytes, KernelInfo* onesweep, KernelInfo* histogram);
bool get_kernels_k4(int value_bytes, int off_bytes, KernelInfo* onesweep, KernelInfo* histogram);
bool get_kernels_k8(int value_bytes, int off_bytes, KernelInfo* onesweep, KernelInfo* histogram);
const void* get_init_kernel();

}  // namespace cusort_b200

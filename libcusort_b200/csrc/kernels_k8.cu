// kernels_k8.cu -- instantiates the histogram and onesweep kernels for
// 8-byte keys (all value widths, 32- and 64-bit offsets).
#include "cusort_instances.cuh"

namespace cusort_b200 {
bool get_kernels_k8(int value_bytes, int off_bytes, bool float_key, KernelInfo* onesweep,
                    KernelInfo* histogram) {
  return get_kernels_impl<8>(value_bytes, off_bytes, float_key, onesweep, histogram);
}
}  // namespace cusort_b200

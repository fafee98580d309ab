// kernels_k4.cu -- instantiates the histogram and onesweep kernels for
// 4-byte keys (all value widths, 32- and 64-bit offsets).
#include "cusort_instances.cuh"

namespace cusort_b200 {
bool get_kernels_k4(int value_bytes, int off_bytes, bool float_key, KernelInfo* onesweep,
                    KernelInfo* histogram) {
  return get_kernels_impl<4>(value_bytes, off_bytes, float_key, onesweep, histogram);
}
}  // namespace cusort_b200

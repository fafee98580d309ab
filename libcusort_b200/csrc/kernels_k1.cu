// kernels_k1.cu -- instantiates the histogram and onesweep kernels for
// 1-byte keys (all value widths, 32- and 64-bit offsets).
#include "cusort_instances.cuh"

namespace cusort_b200 {
bool get_kernels_k1(int value_bytes, int off_bytes, bool float_key, KernelInfo* onesweep,
                    KernelInfo* histogram) {
  return get_kernels_impl<1>(value_bytes, off_bytes, float_key, onesweep, histogram);
}
const void* get_fill_bytes_kernel(int off_bytes) {
  return off_bytes == 8 ? reinterpret_cast<const void*>(&fill_bytes_kernel<unsigned long long>)
                        : reinterpret_cast<const void*>(&fill_bytes_kernel<unsigned int>);
}
}  // namespace cusort_b200

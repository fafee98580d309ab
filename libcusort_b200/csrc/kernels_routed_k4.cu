// kernels_routed_k4.cu -- routed onesweep kernels (multi-GPU partition
// pass) for 4-byte keys.
#include "cusort_instances.cuh"

namespace cusort_b200 {
bool get_routed_k4(int value_bytes, int off_bytes, bool float_key, KernelInfo* onesweep) {
  return get_routed_impl<4>(value_bytes, off_bytes, float_key, onesweep);
}
}  // namespace cusort_b200

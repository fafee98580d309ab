// kernels_routed_k8.cu -- routed onesweep kernels (multi-GPU partition
// pass) for 8-byte keys.
#include "cusort_instances.cuh"

namespace cusort_b200 {
bool get_routed_k8(int value_bytes, int off_bytes, bool float_key, KernelInfo* onesweep) {
  return get_routed_impl<8>(value_bytes, off_bytes, float_key, onesweep);
}
}  // namespace cusort_b200

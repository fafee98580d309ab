// kernels_routed_k12.cu -- routed onesweep kernels (multi-GPU partition
// pass) for 1- and 2-byte keys.
#include "cusort_instances.cuh"

namespace cusort_b200 {
bool get_routed_k12(int key_bytes, int value_bytes, int off_bytes, bool float_key, KernelInfo* onesweep) {
  if (key_bytes == 1) return get_routed_impl<1>(value_bytes, off_bytes, float_key, onesweep);
  if (key_bytes == 2) return get_routed_impl<2>(value_bytes, off_bytes, float_key, onesweep);
  return false;
}
}  // namespace cusort_b200

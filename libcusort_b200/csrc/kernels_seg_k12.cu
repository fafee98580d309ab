// kernels_seg_k12.cu -- segmented-sort kernels (small-segment sorts,
// per-segment histogram and scan, segmented onesweep) for 1- and 2-byte keys.
#include "cusort_instances.cuh"

namespace cusort_b200 {
bool get_segmented_k12(int key_bytes, int value_bytes, int off_bytes, bool float_key, SegKernels* k) {
  if (key_bytes == 1) return get_segmented_impl<1>(value_bytes, off_bytes, float_key, k);
  if (key_bytes == 2) return get_segmented_impl<2>(value_bytes, off_bytes, float_key, k);
  return false;
}
}  // namespace cusort_b200

// kernels_seg_k4.cu -- segmented-sort kernels (small-segment sorts,
// per-segment histogram and scan, segmented onesweep) for 4-byte keys.
#include "cusort_instances.cuh"

namespace cusort_b200 {
bool get_segmented_k4(int value_bytes, int off_bytes, bool float_key, SegKernels* k) {
  return get_segmented_impl<4>(value_bytes, off_bytes, float_key, k);
}
}  // namespace cusort_b200

// kernels_small.cu -- smaller-tile onesweep kernels of 4-byte keys (keys-only
// and 4-byte values, 32-bit offsets) for sorts of few items: tier 0 with
// CUSORT_OS_KPT_SMALL_TILE items per thread, tier 1 with CUSORT_OS_KPT_MID_TILE.
#include "cusort_instances.cuh"

namespace cusort_b200 {
namespace {
template <int KPT>
bool small_for(int value_bytes, bool float_key, KernelInfo* os) {
  if (value_bytes == 0) {
    if (float_key) fill_onesweep_small<4, 0, true, KPT>(os);
    else fill_onesweep_small<4, 0, false, KPT>(os);
    return true;
  }
  if (value_bytes == 4) {
    if (float_key) fill_onesweep_small<4, 4, true, KPT>(os);
    else fill_onesweep_small<4, 4, false, KPT>(os);
    return true;
  }
  return false;
}
}  // namespace

bool get_small_onesweep(int key_bytes, int value_bytes, bool float_key, int tier, KernelInfo* onesweep) {
  if (key_bytes != 4) return false;
  return tier == 0 ? small_for<CUSORT_OS_KPT_SMALL_TILE>(value_bytes, float_key, onesweep)
                   : small_for<CUSORT_OS_KPT_MID_TILE>(value_bytes, float_key, onesweep);
}
}  // namespace cusort_b200

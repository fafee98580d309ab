// kernels_k2.cu -- instantiates the histogram and onesweep kernels for
// 2-byte keys (all value widths, 32- and 64-bit offsets), and the one-pass
// 16-bit-digit kernels (count, fill) of 2-byte keys-only full-range sorts.
#include "cusort_instances.cuh"

namespace cusort_b200 {
bool get_kernels_k2(int value_bytes, int off_bytes, bool float_key, KernelInfo* onesweep,
                    KernelInfo* histogram) {
  return get_kernels_impl<2>(value_bytes, off_bytes, float_key, onesweep, histogram);
}
bool get_fill16_kernels(int off_bytes, KernelInfo* hist, KernelInfo* fill) {
  const bool w = off_bytes == 8;
  hist->func = w ? reinterpret_cast<const void*>(&hist16_kernel<unsigned long long>)
                 : reinterpret_cast<const void*>(&hist16_kernel<unsigned int>);
  hist->threads = 1024;
  hist->tile = kHist16Readers;  // CTAs that read each key
  hist->smem = (size_t)kBins16 / 2 * 4;
  fill->func = w ? reinterpret_cast<const void*>(&fill16_kernel<unsigned long long>)
                 : reinterpret_cast<const void*>(&fill16_kernel<unsigned int>);
  fill->threads = 256;
  return true;
}
}  // namespace cusort_b200

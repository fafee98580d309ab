// cusort_noalloc.cu -- the sort entry point that allocates nothing.
//
// Some callers cannot allocate device memory at the moment they need to sort:
// a custom allocator or memory-pool hook that sorts its own free lists (an
// allocation from inside it would re-enter the allocator), a plugin living in
// a host process that reserved all device memory up front, or a latency-bound
// loop where cudaMalloc would synchronise the whole device.  For them this file
// keeps one fixed scratch array in device memory and runs the ordinary
// DoubleBuffer sort with that array as its temp storage.  It has no counterpart
// in the reference, which always takes temp storage from the caller.
#include <cuda_runtime.h>

#include <map>
#include <mutex>

#include "../../include/cusort_b200.h"
#include "cusort_dispatch.h"

namespace {

// The scratch itself: CUSORT_NOALLOC_SCRATCH_BYTES on every GPU whose context
// loads this module (under lazy loading, once this entry point runs there; with
// CUDA_MODULE_LOADING=EAGER, on every GPU that uses the library), held until
// the process exits.  Host code must not use
// the array's name as a device pointer: on the host it only names a stand-in,
// so its device address is looked up with cudaGetSymbolAddress below.
__device__ __align__(256) unsigned char g_noalloc_scratch[CUSORT_NOALLOC_SCRATCH_BYTES];

std::mutex& scratch_mutex() {
  static std::mutex* m = new std::mutex();
  return *m;
}
std::map<int, void*>& scratch_addresses() {
  static std::map<int, void*>* m = new std::map<int, void*>();
  return *m;
}

// Device address of the scratch on the current device, looked up once per
// device (the first call on a device does this; it must not be inside a
// stream capture) and kept for the life of the process.  A cudaDeviceReset
// between calls is therefore not supported: the module would be loaded again
// in a new context and the kept address could be stale.
cudaError_t scratch_on_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lk(scratch_mutex());
  auto& m = scratch_addresses();
  auto it = m.find(dev);
  if (it != m.end()) {
    *out = it->second;
    return cudaSuccess;
  }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess) return e;
  if (p == nullptr) return cudaErrorInvalidSymbol;
  m[dev] = p;
  *out = p;
  return cudaSuccess;
}

}  // namespace

extern "C" cudaError_t cusort_sort_db_noalloc(cusort_key_type key_type, cusort_double_buffer* d_keys,
                                              size_t value_bytes, cusort_double_buffer* d_values, int64_t num_items,
                                              int begin_bit, int end_bit, int descending, cudaStream_t stream) {
  void* scratch = nullptr;
  cudaError_t e = scratch_on_current_device(&scratch);
  if (e != cudaSuccess) return e;
  return cusort_b200::sort_db_in_scratch(scratch, CUSORT_NOALLOC_SCRATCH_BYTES, (int)key_type, value_bytes,
                                         descending != 0, d_keys, value_bytes ? d_values : nullptr, num_items,
                                         begin_bit, end_bit, stream);
}

// cusort_host.cu -- SortPairs of keys and values that live in HOST memory.
//
// A caller whose data is on the host pays two PCIe crossings per array around
// a device sort that takes a fraction of either.  This entry point orders the
// work so that the crossings overlap: the keys go up first and are sorted with
// their 32-bit input positions as values while the values go up; the sorted
// keys come down while the values are gathered through those positions and
// then come down too.  Upload and download use the two copy directions of the
// link at once, so a pinned-memory sort costs about (keys up + values up) or
// (keys up + sort + keys down + values down), whichever is longer, instead of
// their sum.  No reference counterpart: the reference sorts device memory only.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <map>
#include <mutex>

#include "../../include/cusort_b200.h"
#include "cusort_dispatch.h"

namespace {

constexpr size_t kAlign = 256;

int key_bytes(int kt) {
  switch (kt) {
    case CUSORT_KEY_U8: case CUSORT_KEY_I8: return 1;
    case CUSORT_KEY_U16: case CUSORT_KEY_I16: return 2;
    case CUSORT_KEY_U32: case CUSORT_KEY_I32: case CUSORT_KEY_F32: return 4;
    case CUSORT_KEY_U64: case CUSORT_KEY_I64: case CUSORT_KEY_F64: return 8;
    default: return 0;
  }
}
size_t align_up(size_t x) { return (x + kAlign - 1) & ~(kAlign - 1); }

__global__ void iota_u32_kernel(uint32_t* out, uint64_t n) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = (uint32_t)i;
}

// out[i] = in[perm[i]] for values of W bytes (T holds one value)
template <typename T>
__global__ void gather_kernel(const T* __restrict__ in, const uint32_t* __restrict__ perm, T* __restrict__ out,
                              uint64_t n) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = in[perm[i]];
}

// Two auxiliary streams per device (values upload, keys download), created
// once and kept for the life of the process.
struct AuxStreams {
  cudaStream_t up = nullptr, down = nullptr;
};
cudaError_t aux_streams(AuxStreams* out) {
  static std::mutex* mu = new std::mutex();
  static std::map<int, AuxStreams>* per_dev = new std::map<int, AuxStreams>();
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(*mu);
  auto it = per_dev->find(dev);
  if (it == per_dev->end()) {
    AuxStreams s;
    e = cudaStreamCreateWithFlags(&s.up, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s.down, cudaStreamNonBlocking);
    if (e != cudaSuccess) return e;
    it = per_dev->emplace(dev, s).first;
  }
  *out = it->second;
  return cudaSuccess;
}

int grid_for(uint64_t n) { return (int)std::max<uint64_t>(1, std::min<uint64_t>((n + 255) / 256, 148 * 8)); }

cudaError_t launch_gather(size_t vb, const void* in, const uint32_t* perm, void* out, uint64_t n, cudaStream_t s) {
  const int g = grid_for(n);
  switch (vb) {
    case 1: gather_kernel<uint8_t><<<g, 256, 0, s>>>(static_cast<const uint8_t*>(in), perm, static_cast<uint8_t*>(out), n); break;
    case 2: gather_kernel<uint16_t><<<g, 256, 0, s>>>(static_cast<const uint16_t*>(in), perm, static_cast<uint16_t*>(out), n); break;
    case 4: gather_kernel<uint32_t><<<g, 256, 0, s>>>(static_cast<const uint32_t*>(in), perm, static_cast<uint32_t*>(out), n); break;
    case 8: gather_kernel<unsigned long long><<<g, 256, 0, s>>>(static_cast<const unsigned long long*>(in), perm, static_cast<unsigned long long*>(out), n); break;
    case 16: gather_kernel<uint4><<<g, 256, 0, s>>>(static_cast<const uint4*>(in), perm, static_cast<uint4*>(out), n); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

#define HOST_TRY(x)                           \
  do {                                        \
    cudaError_t e_ = (x);                     \
    if (e_ != cudaSuccess) return e_;         \
  } while (0)

}  // namespace

extern "C" cudaError_t cusort_sort_pairs_host(void* d_temp_storage, size_t* temp_storage_bytes,
                                              cusort_key_type key_type, const void* h_keys_in, void* h_keys_out,
                                              size_t value_bytes, const void* h_values_in, void* h_values_out,
                                              int64_t num_items, int begin_bit, int end_bit, int descending,
                                              cudaStream_t stream) {
  const int kb = key_bytes((int)key_type);
  if (kb == 0 || temp_storage_bytes == nullptr || num_items < 0) return cudaErrorInvalidValue;
  if (value_bytes != 1 && value_bytes != 2 && value_bytes != 4 && value_bytes != 8 && value_bytes != 16)
    return cudaErrorInvalidValue;
  if ((uint64_t)num_items > 0xFFFFFFFFull) return cudaErrorInvalidValue;  // 32-bit input positions
  const uint64_t n = (uint64_t)num_items;
  const size_t vb = value_bytes;
  auto sort_call = [&](void* t, size_t* tb, const void* kin, void* kout, const void* vin, void* vout) {
    return descending ? cusort_sort_pairs_descending(t, tb, key_type, kin, kout, 4, vin, vout, num_items, begin_bit,
                                                     end_bit, stream)
                      : cusort_sort_pairs(t, tb, key_type, kin, kout, 4, vin, vout, num_items, begin_bit, end_bit,
                                          stream);
  };
  size_t sort_bytes = 0;
  HOST_TRY(sort_call(nullptr, &sort_bytes, nullptr, nullptr, nullptr, nullptr));
  // [sort temp][keys in][keys out][positions][sorted positions][values in][values out]
  const size_t o_kin = align_up(sort_bytes), o_kout = o_kin + align_up(n * kb), o_idx = o_kout + align_up(n * kb);
  const size_t o_perm = o_idx + align_up(n * 4), o_vin = o_perm + align_up(n * 4), o_vout = o_vin + align_up(n * vb);
  const size_t total = o_vout + align_up(n * vb);
  if (d_temp_storage == nullptr) {
    *temp_storage_bytes = total;
    return cudaSuccess;
  }
  if (*temp_storage_bytes < total) return cudaErrorInvalidValue;
  if (n == 0) return cudaSuccess;
  uint8_t* t = static_cast<uint8_t*>(d_temp_storage);
  void *kin = t + o_kin, *kout = t + o_kout, *vin = t + o_vin, *vout = t + o_vout;
  uint32_t* idx = reinterpret_cast<uint32_t*>(t + o_idx);
  uint32_t* perm = reinterpret_cast<uint32_t*>(t + o_perm);

  AuxStreams aux;
  HOST_TRY(aux_streams(&aux));
  cudaEvent_t ev[3];  // keys up (later: keys down), keys sorted, values up
  for (int i = 0; i < 3; ++i) {
    cudaError_t e = cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming);
    if (e != cudaSuccess) {
      for (int j = 0; j < i; ++j) cudaEventDestroy(ev[j]);
      return e;
    }
  }
  cudaError_t e = cudaSuccess;
  do {
    // keys up, then (upload engine) the values, while the keys sort with
    // their positions
    if ((e = cudaMemcpyAsync(kin, h_keys_in, n * kb, cudaMemcpyHostToDevice, stream))) break;
    if ((e = cudaEventRecord(ev[0], stream))) break;
    if ((e = cudaStreamWaitEvent(aux.up, ev[0], 0))) break;
    if ((e = cudaMemcpyAsync(vin, h_values_in, n * vb, cudaMemcpyHostToDevice, aux.up))) break;
    if ((e = cudaEventRecord(ev[2], aux.up))) break;
    iota_u32_kernel<<<grid_for(n), 256, 0, stream>>>(idx, n);
    if ((e = cudaGetLastError())) break;
    size_t sb = sort_bytes;
    if ((e = sort_call(t, &sb, kin, kout, idx, perm))) break;
    // sorted keys down (download engine) while the values finish coming up
    if ((e = cudaEventRecord(ev[1], stream))) break;
    if ((e = cudaStreamWaitEvent(aux.down, ev[1], 0))) break;
    if ((e = cudaMemcpyAsync(h_keys_out, kout, n * kb, cudaMemcpyDeviceToHost, aux.down))) break;
    // values gathered through the sorted positions, then down
    if ((e = cudaStreamWaitEvent(stream, ev[2], 0))) break;
    if ((e = launch_gather(vb, vin, perm, vout, n, stream))) break;
    if ((e = cudaMemcpyAsync(h_values_out, vout, n * vb, cudaMemcpyDeviceToHost, stream))) break;
    // the caller's stream ends after the keys' download too
    if ((e = cudaEventRecord(ev[0], aux.down))) break;
    if ((e = cudaStreamWaitEvent(stream, ev[0], 0))) break;
  } while (false);
  for (int i = 0; i < 3; ++i) cudaEventDestroy(ev[i]);
  return e;
}

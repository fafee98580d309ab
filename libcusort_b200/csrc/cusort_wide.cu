// cusort_wide.cu -- key/value sort for payloads of any width (including the
// > 16-byte payloads the reference cannot sort; it caps values at 16 bytes,
// libcusort.cuh:2854).  The keys are sorted together with their 32- or
// 64-bit input index (the ordinary pairs path), then the payload rows are
// gathered by that permutation.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "../../include/cusort_b200.h"
#include "cusort_device.cuh"
#include "cusort_dispatch.h"

namespace {

size_t a256(size_t x) { return (x + 255) & ~size_t(255); }

// out[i] = in[perm[i]] for rows of `words` elements of W bytes.  One thread
// per (row, word); a warp covers consecutive words of consecutive rows, so
// both the row reads and the writes are contiguous runs.
template <typename W, typename I>
__global__ void __launch_bounds__(256) gather_rows_kernel(const W* __restrict__ in, W* __restrict__ out,
                                                          const I* __restrict__ perm, uint64_t rows,
                                                          uint32_t words) {
  const uint64_t total = rows * words;
  for (uint64_t t = blockIdx.x * 256ull + threadIdx.x; t < total; t += (uint64_t)gridDim.x * 256ull) {
    const uint64_t r = t / words;
    const uint32_t w = (uint32_t)(t - r * words);
    out[t] = in[(uint64_t)perm[r] * words + w];
  }
}

// Index sequence 0..n-1.
template <typename I>
__global__ void __launch_bounds__(256) iota_kernel(I* out, uint64_t n) {
  for (uint64_t i = blockIdx.x * 256ull + threadIdx.x; i < n; i += (uint64_t)gridDim.x * 256ull) out[i] = (I)i;
}

int key_bytes(int kt) {
  switch (kt) {
    case CUSORT_KEY_U8: case CUSORT_KEY_I8: return 1;
    case CUSORT_KEY_U16: case CUSORT_KEY_I16: return 2;
    case CUSORT_KEY_U32: case CUSORT_KEY_I32: case CUSORT_KEY_F32: return 4;
    case CUSORT_KEY_U64: case CUSORT_KEY_I64: case CUSORT_KEY_F64: return 8;
    default: return 0;
  }
}

// Rows of exactly one W (8- or 16-byte values): each thread gathers R
// consecutive rows with R independent loads in flight (random 8/16-byte reads
// are latency-bound with one per thread), their positions read as one vector.
template <typename W, typename I, int R>
__global__ void __launch_bounds__(256) gather_words_kernel(const W* __restrict__ in, W* __restrict__ out,
                                                           const I* __restrict__ perm, uint64_t rows) {
  const uint64_t groups = rows / R;
  for (uint64_t gi = blockIdx.x * 256ull + threadIdx.x; gi < groups; gi += (uint64_t)gridDim.x * 256ull) {
    I p[R];
#pragma unroll
    for (int r = 0; r < R; ++r) p[r] = perm[gi * R + r];
    W v[R];
#pragma unroll
    for (int r = 0; r < R; ++r) v[r] = in[p[r]];
#pragma unroll
    for (int r = 0; r < R; ++r) out[gi * R + r] = v[r];
  }
  // the last rows % R rows
  for (uint64_t t = groups * R + blockIdx.x * 256ull + threadIdx.x; t < rows; t += (uint64_t)gridDim.x * 256ull)
    out[t] = in[perm[t]];
}

template <typename W, typename I>
cudaError_t gather(const void* in, void* out, const I* perm, uint64_t n, size_t vb, cudaStream_t s) {
  if (vb == sizeof(W) && sizeof(W) >= 8) {
    constexpr int R = 4;  // measured on B200: 8 rows per thread were slower
    const int grid = (int)std::max<uint64_t>(1, std::min<uint64_t>(148ull * 8, (n / R + 255) / 256));
    gather_words_kernel<W, I, R><<<grid, 256, 0, s>>>(static_cast<const W*>(in), static_cast<W*>(out), perm, n);
    return cudaGetLastError();
  }
  const uint32_t words = (uint32_t)(vb / sizeof(W));
  const uint64_t total = n * words;
  const int grid = (int)std::min<uint64_t>(148ull * 8, (total + 255) / 256);
  if (grid == 0) return cudaSuccess;
  gather_rows_kernel<W, I><<<grid, 256, 0, s>>>(static_cast<const W*>(in), static_cast<W*>(out), perm, n, words);
  return cudaGetLastError();
}

template <typename I>
cudaError_t gather_any(const void* in, void* out, const I* perm, uint64_t n, size_t vb, cudaStream_t s) {
  const uintptr_t al = reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out) | (uintptr_t)vb;
  if ((al & 15) == 0) return gather<uint4, I>(in, out, perm, n, vb, s);
  if ((al & 7) == 0) return gather<unsigned long long, I>(in, out, perm, n, vb, s);
  if ((al & 3) == 0) return gather<uint32_t, I>(in, out, perm, n, vb, s);
  if ((al & 1) == 0) return gather<uint16_t, I>(in, out, perm, n, vb, s);
  return gather<uint8_t, I>(in, out, perm, n, vb, s);
}

}  // namespace

namespace cusort_b200 {

cudaError_t sort_pairs_by_index(void* d_temp_storage, size_t* temp_storage_bytes, int key_type,
                                const void* d_keys_in, void* d_keys_out, size_t value_bytes, const void* d_values_in,
                                void* d_values_out, int64_t num_items, int begin_bit, int end_bit, int descending,
                                cudaStream_t stream) {
  const int kb = key_bytes(key_type);
  if (kb == 0 || temp_storage_bytes == nullptr || value_bytes == 0) return cudaErrorInvalidValue;
  if (begin_bit < 0 || end_bit < 0 || begin_bit > end_bit || end_bit > 8 * kb) return cudaErrorInvalidValue;
  const uint64_t n = num_items > 0 ? (uint64_t)num_items : 0;
  const bool idx64 = n > 0xffffffffull;
  const size_t ib = idx64 ? 8 : 4;
  // [index in][index out][sort temp]
  size_t sort_bytes = 0;
  cudaError_t e = sort_pairs_direct(nullptr, &sort_bytes, key_type, nullptr, nullptr, ib, nullptr, nullptr,
                                    num_items, begin_bit, end_bit, descending != 0, nullptr);
  if (e) return e;
  const size_t off_out = a256(n * ib), off_tmp = off_out + a256(n * ib);
  const size_t total = off_tmp + a256(std::max<size_t>(sort_bytes, 1));
  if (d_temp_storage == nullptr) {
    *temp_storage_bytes = total;
    return cudaSuccess;
  }
  if (*temp_storage_bytes < total) return cudaErrorInvalidValue;
  if (n == 0) return cudaSuccess;
  uint8_t* t = static_cast<uint8_t*>(d_temp_storage);
  void* idx_in = t;
  void* idx_out = t + off_out;
  const int grid = (int)std::min<uint64_t>(148ull * 8, (n + 255) / 256);
  if (idx64)
    iota_kernel<unsigned long long><<<grid, 256, 0, stream>>>(static_cast<unsigned long long*>(idx_in), n);
  else
    iota_kernel<uint32_t><<<grid, 256, 0, stream>>>(static_cast<uint32_t*>(idx_in), n);
  if ((e = cudaGetLastError())) return e;
  size_t sb = sort_bytes;
  e = sort_pairs_direct(t + off_tmp, &sb, key_type, d_keys_in, d_keys_out, ib, idx_in, idx_out, num_items,
                        begin_bit, end_bit, descending != 0, stream);
  if (e) return e;
  return idx64 ? gather_any<unsigned long long>(d_values_in, d_values_out,
                                                static_cast<const unsigned long long*>(idx_out), n, value_bytes,
                                                stream)
               : gather_any<uint32_t>(d_values_in, d_values_out, static_cast<const uint32_t*>(idx_out), n,
                                      value_bytes, stream);
}

}  // namespace cusort_b200

extern "C" cudaError_t cusort_sort_pairs_wide(void* d_temp_storage, size_t* temp_storage_bytes,
                                              cusort_key_type key_type, const void* d_keys_in, void* d_keys_out,
                                              size_t value_bytes, const void* d_values_in, void* d_values_out,
                                              int64_t num_items, int begin_bit, int end_bit, int descending,
                                              cudaStream_t stream) {
  return cusort_b200::sort_pairs_by_index(d_temp_storage, temp_storage_bytes, (int)key_type, d_keys_in, d_keys_out,
                                          value_bytes, d_values_in, d_values_out, num_items, begin_bit, end_bit,
                                          descending, stream);
}

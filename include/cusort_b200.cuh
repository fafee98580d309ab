// cusort_b200.cuh -- C++ drop-in for libcusort.cuh's public API.
//
// Replace `#include "libcusort.cuh"` with `#include "cusort_b200.cuh"` and
// link libcusort_b200.so: cusort::DoubleBuffer<T> and the eight
// cusort::DeviceRadixSort overloads (SortPairs, SortPairsDescending, SortKeys,
// SortKeysDescending; DoubleBuffer and in/out-pointer forms) keep the
// reference's signatures, defaults and semantics (libcusort.cuh:156-184,
// 2875-3105) and forward to the C ABI in cusort_b200.h.  Everything else of
// the reference header (internal namespaces, tuning macros) is not part of
// its public API and has no counterpart here.
#ifndef CUSORT_B200_CUH
#define CUSORT_B200_CUH 1

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <type_traits>

#include "cusort_b200.h"

#define LIBCUSORT_VERSION_MAJOR 1
#define LIBCUSORT_VERSION_MINOR 0
#define LIBCUSORT_VERSION_PATCH 1
#define LIBCUSORT_VERSION_STRING "1.0.1"

namespace cusort {

// Ping-pong buffer pair (same layout and members as the reference's).
template <typename T>
struct DoubleBuffer {
  T* d_buffers[2];
  int selector;

  __host__ __device__ __forceinline__ DoubleBuffer() : d_buffers{nullptr, nullptr}, selector(0) {}
  __host__ __device__ __forceinline__ DoubleBuffer(T* d_current, T* d_alternate)
      : d_buffers{d_current, d_alternate}, selector(0) {}
  __host__ __device__ __forceinline__ T* Current() const { return d_buffers[selector]; }
  __host__ __device__ __forceinline__ T* Alternate() const { return d_buffers[selector ^ 1]; }
};

namespace b200_detail {

// Key type tag by the same classification the reference's traits use
// (libcusort.cuh:321-429): floating point, signed integer, or unsigned.
template <typename K>
constexpr cusort_key_type key_type_of() {
  static_assert(std::is_arithmetic<K>::value &&
                    (sizeof(K) == 1 || sizeof(K) == 2 || sizeof(K) == 4 || sizeof(K) == 8),
                "KeyT must be an arithmetic type of 1, 2, 4, or 8 bytes");
  return std::is_floating_point<K>::value ? (sizeof(K) == 4 ? CUSORT_KEY_F32 : CUSORT_KEY_F64)
         : std::is_signed<K>::value
             ? (sizeof(K) == 1 ? CUSORT_KEY_I8
                               : sizeof(K) == 2 ? CUSORT_KEY_I16 : sizeof(K) == 4 ? CUSORT_KEY_I32 : CUSORT_KEY_I64)
             : (sizeof(K) == 1 ? CUSORT_KEY_U8
                               : sizeof(K) == 2 ? CUSORT_KEY_U16 : sizeof(K) == 4 ? CUSORT_KEY_U32 : CUSORT_KEY_U64);
}

template <typename V>
constexpr size_t value_bytes_of() {
  static_assert(sizeof(V) == 1 || sizeof(V) == 2 || sizeof(V) == 4 || sizeof(V) == 8 || sizeof(V) == 16,
                "ValueT must be a type of 1, 2, 4, 8, or 16 bytes");
  return sizeof(V);
}

template <typename T>
struct DbView {
  cusort_double_buffer c;
  DoubleBuffer<T>& ref;
  explicit DbView(DoubleBuffer<T>& r) : ref(r) {
    c.d_buffers[0] = r.d_buffers[0];
    c.d_buffers[1] = r.d_buffers[1];
    c.selector = r.selector;
  }
  ~DbView() { ref.selector = c.selector; }
};

template <typename N>
inline int64_t items(N n) {
  static_assert(std::is_integral<N>::value, "NumItemsT must be an integer type");
  return static_cast<int64_t>(n);
}

}  // namespace b200_detail

struct DeviceRadixSort {
  template <typename KeyT, typename ValueT, typename NumItemsT>
  static cudaError_t SortPairs(void* d_temp_storage, size_t& temp_storage_bytes, DoubleBuffer<KeyT>& d_keys,
                               DoubleBuffer<ValueT>& d_values, NumItemsT num_items, int begin_bit = 0,
                               int end_bit = sizeof(KeyT) * 8, cudaStream_t stream = 0) {
    b200_detail::DbView<KeyT> k(d_keys);
    b200_detail::DbView<ValueT> v(d_values);
    return cusort_sort_pairs_db(d_temp_storage, &temp_storage_bytes, b200_detail::key_type_of<KeyT>(), &k.c,
                                b200_detail::value_bytes_of<ValueT>(), &v.c, b200_detail::items(num_items),
                                begin_bit, end_bit, stream);
  }

  template <typename KeyT, typename ValueT, typename NumItemsT>
  static cudaError_t SortPairsDescending(void* d_temp_storage, size_t& temp_storage_bytes,
                                         DoubleBuffer<KeyT>& d_keys, DoubleBuffer<ValueT>& d_values,
                                         NumItemsT num_items, int begin_bit = 0, int end_bit = sizeof(KeyT) * 8,
                                         cudaStream_t stream = 0) {
    b200_detail::DbView<KeyT> k(d_keys);
    b200_detail::DbView<ValueT> v(d_values);
    return cusort_sort_pairs_descending_db(d_temp_storage, &temp_storage_bytes, b200_detail::key_type_of<KeyT>(),
                                           &k.c, b200_detail::value_bytes_of<ValueT>(), &v.c,
                                           b200_detail::items(num_items), begin_bit, end_bit, stream);
  }

  template <typename KeyT, typename NumItemsT>
  static cudaError_t SortKeys(void* d_temp_storage, size_t& temp_storage_bytes, DoubleBuffer<KeyT>& d_keys,
                              NumItemsT num_items, int begin_bit = 0, int end_bit = sizeof(KeyT) * 8,
                              cudaStream_t stream = 0) {
    b200_detail::DbView<KeyT> k(d_keys);
    return cusort_sort_keys_db(d_temp_storage, &temp_storage_bytes, b200_detail::key_type_of<KeyT>(), &k.c,
                               b200_detail::items(num_items), begin_bit, end_bit, stream);
  }

  template <typename KeyT, typename NumItemsT>
  static cudaError_t SortKeysDescending(void* d_temp_storage, size_t& temp_storage_bytes, DoubleBuffer<KeyT>& d_keys,
                                        NumItemsT num_items, int begin_bit = 0, int end_bit = sizeof(KeyT) * 8,
                                        cudaStream_t stream = 0) {
    b200_detail::DbView<KeyT> k(d_keys);
    return cusort_sort_keys_descending_db(d_temp_storage, &temp_storage_bytes, b200_detail::key_type_of<KeyT>(),
                                          &k.c, b200_detail::items(num_items), begin_bit, end_bit, stream);
  }

  template <typename KeyT, typename NumItemsT>
  static cudaError_t SortKeys(void* d_temp_storage, size_t& temp_storage_bytes, const KeyT* d_keys_in,
                              KeyT* d_keys_out, NumItemsT num_items, int begin_bit = 0,
                              int end_bit = sizeof(KeyT) * 8, cudaStream_t stream = 0) {
    return cusort_sort_keys(d_temp_storage, &temp_storage_bytes, b200_detail::key_type_of<KeyT>(), d_keys_in,
                            d_keys_out, b200_detail::items(num_items), begin_bit, end_bit, stream);
  }

  template <typename KeyT, typename NumItemsT>
  static cudaError_t SortKeysDescending(void* d_temp_storage, size_t& temp_storage_bytes, const KeyT* d_keys_in,
                                        KeyT* d_keys_out, NumItemsT num_items, int begin_bit = 0,
                                        int end_bit = sizeof(KeyT) * 8, cudaStream_t stream = 0) {
    return cusort_sort_keys_descending(d_temp_storage, &temp_storage_bytes, b200_detail::key_type_of<KeyT>(),
                                       d_keys_in, d_keys_out, b200_detail::items(num_items), begin_bit, end_bit,
                                       stream);
  }

  template <typename KeyT, typename ValueT, typename NumItemsT>
  static cudaError_t SortPairs(void* d_temp_storage, size_t& temp_storage_bytes, const KeyT* d_keys_in,
                               KeyT* d_keys_out, const ValueT* d_values_in, ValueT* d_values_out,
                               NumItemsT num_items, int begin_bit = 0, int end_bit = sizeof(KeyT) * 8,
                               cudaStream_t stream = 0) {
    return cusort_sort_pairs(d_temp_storage, &temp_storage_bytes, b200_detail::key_type_of<KeyT>(), d_keys_in,
                             d_keys_out, b200_detail::value_bytes_of<ValueT>(), d_values_in, d_values_out,
                             b200_detail::items(num_items), begin_bit, end_bit, stream);
  }

  template <typename KeyT, typename ValueT, typename NumItemsT>
  static cudaError_t SortPairsDescending(void* d_temp_storage, size_t& temp_storage_bytes, const KeyT* d_keys_in,
                                         KeyT* d_keys_out, const ValueT* d_values_in, ValueT* d_values_out,
                                         NumItemsT num_items, int begin_bit = 0, int end_bit = sizeof(KeyT) * 8,
                                         cudaStream_t stream = 0) {
    return cusort_sort_pairs_descending(d_temp_storage, &temp_storage_bytes, b200_detail::key_type_of<KeyT>(),
                                        d_keys_in, d_keys_out, b200_detail::value_bytes_of<ValueT>(), d_values_in,
                                        d_values_out, b200_detail::items(num_items), begin_bit, end_bit, stream);
  }
};

// Segmented sort (no counterpart in the reference beyond the name in its
// banner, libcusort.cuh:4): every segment [d_begin_offsets[s],
// d_end_offsets[s]) sorted independently and stably into the same positions
// of the output, CUB DeviceSegmentedRadixSort's argument order; offsets are
// int64 arrays in device memory.  Forwards to cusort_segmented_sort_keys /
// cusort_segmented_sort_pairs.
struct DeviceSegmentedRadixSort {
  template <typename KeyT, typename NumItemsT, typename NumSegmentsT>
  static cudaError_t SortKeys(void* d_temp_storage, size_t& temp_storage_bytes, const KeyT* d_keys_in,
                              KeyT* d_keys_out, NumItemsT num_items, NumSegmentsT num_segments,
                              const int64_t* d_begin_offsets, const int64_t* d_end_offsets, int begin_bit = 0,
                              int end_bit = sizeof(KeyT) * 8, cudaStream_t stream = 0) {
    return cusort_segmented_sort_keys(d_temp_storage, &temp_storage_bytes, b200_detail::key_type_of<KeyT>(),
                                      d_keys_in, d_keys_out, b200_detail::items(num_items),
                                      b200_detail::items(num_segments), d_begin_offsets, d_end_offsets, begin_bit,
                                      end_bit, 0, stream);
  }

  template <typename KeyT, typename NumItemsT, typename NumSegmentsT>
  static cudaError_t SortKeysDescending(void* d_temp_storage, size_t& temp_storage_bytes, const KeyT* d_keys_in,
                                        KeyT* d_keys_out, NumItemsT num_items, NumSegmentsT num_segments,
                                        const int64_t* d_begin_offsets, const int64_t* d_end_offsets,
                                        int begin_bit = 0, int end_bit = sizeof(KeyT) * 8, cudaStream_t stream = 0) {
    return cusort_segmented_sort_keys(d_temp_storage, &temp_storage_bytes, b200_detail::key_type_of<KeyT>(),
                                      d_keys_in, d_keys_out, b200_detail::items(num_items),
                                      b200_detail::items(num_segments), d_begin_offsets, d_end_offsets, begin_bit,
                                      end_bit, 1, stream);
  }

  template <typename KeyT, typename ValueT, typename NumItemsT, typename NumSegmentsT>
  static cudaError_t SortPairs(void* d_temp_storage, size_t& temp_storage_bytes, const KeyT* d_keys_in,
                               KeyT* d_keys_out, const ValueT* d_values_in, ValueT* d_values_out,
                               NumItemsT num_items, NumSegmentsT num_segments, const int64_t* d_begin_offsets,
                               const int64_t* d_end_offsets, int begin_bit = 0, int end_bit = sizeof(KeyT) * 8,
                               cudaStream_t stream = 0) {
    return cusort_segmented_sort_pairs(d_temp_storage, &temp_storage_bytes, b200_detail::key_type_of<KeyT>(),
                                       d_keys_in, d_keys_out, b200_detail::value_bytes_of<ValueT>(), d_values_in,
                                       d_values_out, b200_detail::items(num_items),
                                       b200_detail::items(num_segments), d_begin_offsets, d_end_offsets, begin_bit,
                                       end_bit, 0, stream);
  }

  template <typename KeyT, typename ValueT, typename NumItemsT, typename NumSegmentsT>
  static cudaError_t SortPairsDescending(void* d_temp_storage, size_t& temp_storage_bytes, const KeyT* d_keys_in,
                                         KeyT* d_keys_out, const ValueT* d_values_in, ValueT* d_values_out,
                                         NumItemsT num_items, NumSegmentsT num_segments,
                                         const int64_t* d_begin_offsets, const int64_t* d_end_offsets,
                                         int begin_bit = 0, int end_bit = sizeof(KeyT) * 8, cudaStream_t stream = 0) {
    return cusort_segmented_sort_pairs(d_temp_storage, &temp_storage_bytes, b200_detail::key_type_of<KeyT>(),
                                       d_keys_in, d_keys_out, b200_detail::value_bytes_of<ValueT>(), d_values_in,
                                       d_values_out, b200_detail::items(num_items),
                                       b200_detail::items(num_segments), d_begin_offsets, d_end_offsets, begin_bit,
                                       end_bit, 1, stream);
  }
};

}  // namespace cusort

#endif  // CUSORT_B200_CUH

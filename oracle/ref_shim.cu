// ref_shim.cu -- C entry points over the UNMODIFIED reference library, for
// parity tests and the benchmark's reference arm only (test infrastructure;
// never linked into libcusort_b200).
//
// It includes libcusort.cuh from the reference checkout (-I <reference dir>)
// and calls cusort::DeviceRadixSort's public overloads
// (libcusort.cuh:2972-3104) exactly as a user program would.  One object per
// key type (-DREF_KEY_T=<type> -DREF_KEY_ID=<cusort_key_type>) so the many
// template instantiations compile in parallel.
#include <cuda_runtime.h>
#include <cstdint>
#include "libcusort.cuh"

#ifndef REF_KEY_T
#error "define REF_KEY_T and REF_KEY_ID"
#endif

#define REF_CAT2(a, b) a##b
#define REF_CAT(a, b) REF_CAT2(a, b)

namespace {
using K = REF_KEY_T;

template <typename V>
cudaError_t run_pairs(int desc, int raw, void* t, size_t* tb, void* k0, void* k1, int* ks, void* v0, void* v1,
                      int* vs, int64_t n, int b, int e, cudaStream_t s) {
  using cusort::DeviceRadixSort;
  if (raw) {
    return desc ? DeviceRadixSort::SortPairsDescending(t, *tb, (const K*)k0, (K*)k1, (const V*)v0, (V*)v1, n, b, e, s)
                : DeviceRadixSort::SortPairs(t, *tb, (const K*)k0, (K*)k1, (const V*)v0, (V*)v1, n, b, e, s);
  }
  cusort::DoubleBuffer<K> kd((K*)k0, (K*)k1);
  kd.selector = *ks;
  cusort::DoubleBuffer<V> vd((V*)v0, (V*)v1);
  vd.selector = *vs;
  cudaError_t r = desc ? DeviceRadixSort::SortPairsDescending(t, *tb, kd, vd, n, b, e, s)
                       : DeviceRadixSort::SortPairs(t, *tb, kd, vd, n, b, e, s);
  *ks = kd.selector;
  *vs = vd.selector;
  return r;
}

cudaError_t run_keys(int desc, int raw, void* t, size_t* tb, void* k0, void* k1, int* ks, int64_t n, int b, int e,
                     cudaStream_t s) {
  using cusort::DeviceRadixSort;
  if (raw) {
    return desc ? DeviceRadixSort::SortKeysDescending(t, *tb, (const K*)k0, (K*)k1, n, b, e, s)
                : DeviceRadixSort::SortKeys(t, *tb, (const K*)k0, (K*)k1, n, b, e, s);
  }
  cusort::DoubleBuffer<K> kd((K*)k0, (K*)k1);
  kd.selector = *ks;
  cudaError_t r = desc ? DeviceRadixSort::SortKeysDescending(t, *tb, kd, n, b, e, s)
                       : DeviceRadixSort::SortKeys(t, *tb, kd, n, b, e, s);
  *ks = kd.selector;
  return r;
}
}  // namespace

// raw != 0: (k0, k1) = (in, out), (v0, v1) = (in, out); selectors ignored.
// raw == 0: DoubleBuffer form, *ks / *vs updated as the reference leaves them.
extern "C" int REF_CAT(ref_sort_k, REF_KEY_ID)(int value_bytes, int desc, int raw, void* t, size_t* tb, void* k0,
                                               void* k1, int* ks, void* v0, void* v1, int* vs, int64_t n, int b,
                                               int e, void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (value_bytes) {
    case 0: return (int)run_keys(desc, raw, t, tb, k0, k1, ks, n, b, e, s);
    case 1: return (int)run_pairs<uint8_t>(desc, raw, t, tb, k0, k1, ks, v0, v1, vs, n, b, e, s);
    case 2: return (int)run_pairs<uint16_t>(desc, raw, t, tb, k0, k1, ks, v0, v1, vs, n, b, e, s);
    case 4: return (int)run_pairs<uint32_t>(desc, raw, t, tb, k0, k1, ks, v0, v1, vs, n, b, e, s);
    case 8: return (int)run_pairs<uint64_t>(desc, raw, t, tb, k0, k1, ks, v0, v1, vs, n, b, e, s);
    case 16: return (int)run_pairs<ulonglong2>(desc, raw, t, tb, k0, k1, ks, v0, v1, vs, n, b, e, s);
    default: return (int)cudaErrorInvalidValue;
  }
}

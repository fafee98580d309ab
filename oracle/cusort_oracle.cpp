// cusort_oracle.cpp -- CPU restatement of libcusort's radix-sort semantics.
//
// TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA sort in
// libcusort_b200; it is never linked into, loaded by, or called from the
// product library.  Only tests/, __graft_entry__.smoke() and bench.py's
// cpu_baseline leg load it.
//
// What it restates (reference = IlyaGrebnov/libcusort 1.0.1, libcusort.cuh):
//   * key bit-twiddle  : traits::RadixTraits::Twiddle (libcusort.cuh:398-429)
//       unsigned -> identity; signed -> flip the sign bit; float/double ->
//       flip every bit when the sign bit is set, else flip only the sign bit;
//       descending -> additionally invert every bit.
//   * digit extraction : (twiddled >> begin_bit) masked to end_bit-begin_bit
//       bits (histogram kernel libcusort.cuh:1753, onesweep digit mask
//       libcusort.cuh:2665).
//   * ordering         : one stable LSD pass per 8-bit digit is equivalent to a
//       single stable sort on the masked twiddled key (libcusort.cuh:2662-2686);
//       equal keys keep input order in BOTH directions.
//   * argument checks  : DeviceRadixSort::DispatchSort (libcusort.cuh:2908-2931).
//
// The sort itself is std::stable_sort (or libstdc++ parallel-mode
// __gnu_parallel::stable_sort over OpenMP threads for the timed CPU baseline)
// on (masked twiddled key, input index) -- deliberately NOT a radix sort, so
// the oracle shares no algorithm with the code under test.

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <numeric>
#include <vector>
#include <parallel/algorithm>
#include <omp.h>

namespace {

enum KeyType {
  KT_U8 = 0, KT_I8 = 1, KT_U16 = 2, KT_I16 = 3, KT_U32 = 4,
  KT_I32 = 5, KT_U64 = 6, KT_I64 = 7, KT_F32 = 8, KT_F64 = 9
};

int key_bytes(int kt) {
  switch (kt) {
    case KT_U8: case KT_I8: return 1;
    case KT_U16: case KT_I16: return 2;
    case KT_U32: case KT_I32: case KT_F32: return 4;
    case KT_U64: case KT_I64: case KT_F64: return 8;
    default: return 0;
  }
}
bool key_signed(int kt) { return kt == KT_I8 || kt == KT_I16 || kt == KT_I32 || kt == KT_I64; }
bool key_float(int kt) { return kt == KT_F32 || kt == KT_F64; }

uint64_t load_bits(const void* p, int kb, int64_t i) {
  const uint8_t* b = static_cast<const uint8_t*>(p) + i * kb;
  uint64_t v = 0;
  std::memcpy(&v, b, kb);  // little-endian host
  return v;
}

// Restatement of RadixTraits::TwiddleForward (libcusort.cuh:417-429), written
// from the ordering rules rather than from the xor-table form.
uint64_t twiddle(uint64_t bits, int kt, int descending) {
  const int nb = 8 * key_bytes(kt);
  const uint64_t all = (nb == 64) ? ~0ull : ((1ull << nb) - 1);
  const uint64_t sign = 1ull << (nb - 1);
  uint64_t t = bits;
  if (key_float(kt)) {
    // IEEE totalOrder as unsigned: negatives reversed below positives.
    t = (bits & sign) ? (~bits & all) : (bits | sign);
  } else if (key_signed(kt)) {
    t = bits ^ sign;
  }
  if (descending) t = ~t & all;
  return t;
}

uint64_t digit_key(uint64_t bits, int kt, int descending, int begin_bit, int end_bit) {
  uint64_t t = twiddle(bits, kt, descending);
  const int w = end_bit - begin_bit;
  if (w <= 0) return 0;
  t >>= begin_bit;
  if (w < 64) t &= (1ull << w) - 1;
  return t;
}

}  // namespace

extern "C" {

// Stable-sort permutation: perm[i] = input index of the i-th output item.
// threads <= 1 -> std::stable_sort; otherwise __gnu_parallel::stable_sort.
int oracle_sort_permutation(int key_type, const void* keys, int64_t n, int begin_bit,
                            int end_bit, int descending, int threads, int64_t* perm) {
  const int kb = key_bytes(key_type);
  if (kb == 0) return 1;
  if (begin_bit < 0 || end_bit < 0 || begin_bit > end_bit || end_bit > 8 * kb) return 1;
  if (n <= 0) return 0;
  struct Item { uint64_t k; int64_t i; };
  std::vector<Item> items(static_cast<size_t>(n));
  for (int64_t i = 0; i < n; ++i)
    items[i] = {digit_key(load_bits(keys, kb, i), key_type, descending, begin_bit, end_bit), i};
  auto less = [](const Item& a, const Item& b) { return a.k < b.k; };
  if (threads > 1) {
    omp_set_num_threads(threads);
    __gnu_parallel::stable_sort(items.begin(), items.end(), less);
  } else {
    std::stable_sort(items.begin(), items.end(), less);
  }
  for (int64_t i = 0; i < n; ++i) perm[i] = items[i].i;
  return 0;
}

// Full sort: gathers keys (and values of value_bytes each, may be 0) by the
// stable permutation.  Output buffers must not alias inputs.
int oracle_sort(int key_type, const void* keys_in, void* keys_out, int64_t value_bytes,
                const void* values_in, void* values_out, int64_t n, int begin_bit,
                int end_bit, int descending, int threads) {
  const int kb = key_bytes(key_type);
  if (kb == 0) return 1;
  if (begin_bit < 0 || end_bit < 0 || begin_bit > end_bit || end_bit > 8 * kb) return 1;
  if (n <= 0) return 0;
  std::vector<int64_t> perm(static_cast<size_t>(n));
  int rc = oracle_sort_permutation(key_type, keys_in, n, begin_bit, end_bit, descending,
                                   threads, perm.data());
  if (rc) return rc;
  const uint8_t* ki = static_cast<const uint8_t*>(keys_in);
  uint8_t* ko = static_cast<uint8_t*>(keys_out);
  const uint8_t* vi = static_cast<const uint8_t*>(values_in);
  uint8_t* vo = static_cast<uint8_t*>(values_out);
#pragma omp parallel for num_threads(threads > 1 ? threads : 1) schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    std::memcpy(ko + i * kb, ki + perm[i] * kb, kb);
    if (value_bytes > 0) std::memcpy(vo + i * value_bytes, vi + perm[i] * value_bytes, value_bytes);
  }
  return 0;
}

// Twiddled, masked digit key of one element (exposed for host-logic tests).
uint64_t oracle_digit_key(int key_type, uint64_t bits, int descending, int begin_bit, int end_bit) {
  return digit_key(bits, key_type, descending, begin_bit, end_bit);
}

// Per-pass 8-bit digit histogram, counts[pass*256 + digit], passes =
// ceil((end-begin)/8); the last pass is masked to the remaining bits
// (libcusort.cuh:2586-2588, 2665).
int oracle_digit_histogram(int key_type, const void* keys, int64_t n, int begin_bit,
                           int end_bit, int descending, uint64_t* counts) {
  const int kb = key_bytes(key_type);
  if (kb == 0) return 1;
  const int nbits = end_bit - begin_bit;
  const int passes = (nbits + 7) / 8;
  std::fill(counts, counts + passes * 256, 0ull);
  for (int64_t i = 0; i < n; ++i) {
    uint64_t t = twiddle(load_bits(keys, kb, i), key_type, descending);
    for (int p = 0; p < passes; ++p) {
      int sh = begin_bit + 8 * p;
      int w = std::min(8, end_bit - sh);
      counts[p * 256 + ((t >> sh) & ((1ull << w) - 1))]++;
    }
  }
  return 0;
}

}  // extern "C"

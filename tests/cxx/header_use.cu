// Compile-and-link check of include/cusort_b200.cuh: every public template is
// instantiated for several key/value types and linked against the library.
// Built by tests/test_cxx_header.py (no GPU needed; the program is not run
// there).  With a GPU, running it sorts a small array through every form and
// prints "ok".
#include <cstdio>
#include <vector>

#include "cusort_b200.cuh"

template <typename K, typename V>
static int all_forms(int n) {
  K *k0, *k1;
  V *v0, *v1;
  int64_t *b, *e;
  if (cudaMalloc(&k0, n * sizeof(K)) || cudaMalloc(&k1, n * sizeof(K)) || cudaMalloc(&v0, n * sizeof(V)) ||
      cudaMalloc(&v1, n * sizeof(V)) || cudaMalloc(&b, sizeof(int64_t)) || cudaMalloc(&e, sizeof(int64_t)))
    return 1;
  cudaMemset(k0, 0, n * sizeof(K));
  const int64_t hb = 0, he = n;
  cudaMemcpy(b, &hb, sizeof(hb), cudaMemcpyHostToDevice);
  cudaMemcpy(e, &he, sizeof(he), cudaMemcpyHostToDevice);
  cusort::DoubleBuffer<K> dk(k0, k1);
  cusort::DoubleBuffer<V> dv(v0, v1);
  size_t bytes = 0, m = 0;
  void* t = nullptr;
  int rc = 0;
  auto need = [&](size_t x) { m = x > m ? x : m; };
  rc |= cusort::DeviceRadixSort::SortPairs(nullptr, bytes, dk, dv, n); need(bytes);
  rc |= cusort::DeviceRadixSort::SortPairsDescending(nullptr, bytes, dk, dv, n, 0, 8 * (int)sizeof(K)); need(bytes);
  rc |= cusort::DeviceRadixSort::SortKeys(nullptr, bytes, dk, n); need(bytes);
  rc |= cusort::DeviceRadixSort::SortKeysDescending(nullptr, bytes, dk, n); need(bytes);
  rc |= cusort::DeviceRadixSort::SortKeys(nullptr, bytes, k0, k1, n); need(bytes);
  rc |= cusort::DeviceRadixSort::SortKeysDescending(nullptr, bytes, k0, k1, n); need(bytes);
  rc |= cusort::DeviceRadixSort::SortPairs(nullptr, bytes, k0, k1, v0, v1, n); need(bytes);
  rc |= cusort::DeviceRadixSort::SortPairsDescending(nullptr, bytes, k0, k1, v0, v1, n); need(bytes);
  rc |= cusort::DeviceSegmentedRadixSort::SortKeys(nullptr, bytes, k0, k1, n, 1, b, e); need(bytes);
  rc |= cusort::DeviceSegmentedRadixSort::SortKeysDescending(nullptr, bytes, k0, k1, n, 1, b, e); need(bytes);
  rc |= cusort::DeviceSegmentedRadixSort::SortPairs(nullptr, bytes, k0, k1, v0, v1, n, 1, b, e); need(bytes);
  rc |= cusort::DeviceSegmentedRadixSort::SortPairsDescending(nullptr, bytes, k0, k1, v0, v1, n, 1, b, e);
  need(bytes);
  if (rc || cudaMalloc(&t, m)) return 1;
  bytes = m;
  rc |= cusort::DeviceRadixSort::SortPairs(t, bytes, dk, dv, n);
  rc |= cusort::DeviceRadixSort::SortKeys(t, bytes, k0, k1, n);
  rc |= cusort::DeviceRadixSort::SortPairsDescending(t, bytes, k0, k1, v0, v1, n);
  rc |= cusort::DeviceSegmentedRadixSort::SortPairs(t, bytes, k0, k1, v0, v1, n, 1, b, e);
  rc |= cudaDeviceSynchronize();
  cudaFree(t); cudaFree(k0); cudaFree(k1); cudaFree(v0); cudaFree(v1); cudaFree(b); cudaFree(e);
  return rc;
}

int main() {
  int rc = all_forms<unsigned int, int>(1000) | all_forms<float, double>(1000) | all_forms<short, char>(1000) |
           all_forms<long long, unsigned long long>(1000);
  std::printf(rc ? "failed\n" : "ok\n");
  return rc ? 1 : 0;
}

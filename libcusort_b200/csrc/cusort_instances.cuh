// cusort_instances.cuh -- kernel configuration table and the instantiation
// macro used by kernels_k{1,2,4,8}.cu (one translation unit per key width so
// the build compiles them in parallel).
//
// Tile shapes are chosen for B200 (148 SMs, 228 KB shared memory per SM,
// 64K registers per SM): 512-thread CTAs, two resident per SM, with the
// per-thread item count (KPT) set so keys + values + rank words stay in
// registers without spilling.  Reference counterpart: the RTX 5090 tuning
// table (libcusort.cuh:2433-2484), whose values do not carry over.
#pragma once

#include "cusort_dispatch.h"
#include "cusort_kernels.cuh"

namespace cusort_b200 {

template <int KB, int VB>
struct TileShape {
  static constexpr int THREADS = 512;
  static constexpr int BYTES = KB + VB;
  static constexpr int KPT = (KB == 8 && VB >= 8) ? 8 : (BYTES > 16) ? 8 : (BYTES > 8) ? 12 : 16;
  static constexpr int MINB = 2;
};

constexpr int kHistThreads = 1024;
constexpr int kHistUnroll = 4;

template <int KB, int VB, typename Off>
inline void fill_onesweep(KernelInfo* os) {
  using S = TileShape<KB, VB>;
  using CFG = OnesweepCfg<KB, VB, Off, S::THREADS, S::KPT, S::MINB>;
  os->func = reinterpret_cast<const void*>(&onesweep_kernel<CFG>);
  os->threads = CFG::THREADS;
  os->tile = CFG::TILE;
  os->smem = CFG::SMEM_BYTES;
}

template <int KB, typename Off>
inline void fill_histogram(KernelInfo* h) {
  h->func = reinterpret_cast<const void*>(&histogram_kernel<KB, Off, kHistThreads, kHistUnroll>);
  h->threads = kHistThreads;
  h->tile = kHistThreads * kHistUnroll;
  h->smem = HistShape<KB>::SMEM;
}

template <int KB, typename Off>
inline bool fill_for_value(int vb, KernelInfo* os) {
  switch (vb) {
    case 0: fill_onesweep<KB, 0, Off>(os); return true;
    case 1: fill_onesweep<KB, 1, Off>(os); return true;
    case 2: fill_onesweep<KB, 2, Off>(os); return true;
    case 4: fill_onesweep<KB, 4, Off>(os); return true;
    case 8: fill_onesweep<KB, 8, Off>(os); return true;
    case 16: fill_onesweep<KB, 16, Off>(os); return true;
    default: return false;
  }
}

template <int KB>
inline bool get_kernels_impl(int vb, int offb, KernelInfo* os, KernelInfo* h) {
  if (offb == 4) {
    fill_histogram<KB, unsigned int>(h);
    return fill_for_value<KB, unsigned int>(vb, os);
  }
  if (offb == 8) {
    fill_histogram<KB, unsigned long long>(h);
    return fill_for_value<KB, unsigned long long>(vb, os);
  }
  return false;
}

}  // namespace cusort_b200

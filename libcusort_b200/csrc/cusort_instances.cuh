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
#include "cusort_segmented.cuh"

namespace cusort_b200 {

#ifndef CUSORT_OS_THREADS
#define CUSORT_OS_THREADS 512
#endif
#ifndef CUSORT_OS_MINB
#define CUSORT_OS_MINB 2
#endif
// Items per thread (KPT) by bytes per item; overridable for tuning.  Larger
// tiles amortise the per-tile work (column scan, block scan, lookback,
// ticket) over more keys; the limit is 64 registers per thread at two 512-
// thread CTAs per SM.  Measured on B200 at 2^26 items (onesweep launch, 32-bit
// counters, pipelined loads for 4-byte keys): keys-only 32 (230 us; 28: 235,
// 36: 243, 40: 246 with spills); 4-byte keys with 4-byte values 16 (341 us;
// 12: 356, 14: 345, 18: 366, 20: 367 with spills).  The staged kernel of the
// other widths was tuned at 20 items per thread for pairs of up to 8 bytes.
#ifndef CUSORT_OS_KPT_KEYS4
#define CUSORT_OS_KPT_KEYS4 32
#endif
#ifndef CUSORT_OS_KPT_K4V4
#define CUSORT_OS_KPT_K4V4 16
#endif
// The staged kernel (routed multi-GPU partition passes, segmented passes, and
// keys-only sorts of 1-2 byte keys) keeps the sizes it was tuned at: 36 items
// per thread keys-only (32 -> 36: u32 keys-only sort 1.045 -> 1.026 ms), 20
// for 8-byte items (16 -> 20: int32+uint32 pass 0.369 -> 0.356 ms).
#ifndef CUSORT_OS_KPT_KEYS_STAGED
#define CUSORT_OS_KPT_KEYS_STAGED 36
#endif
#ifndef CUSORT_OS_KPT_LE8
#define CUSORT_OS_KPT_LE8 20
#endif
#ifndef CUSORT_OS_KPT_LE16
#define CUSORT_OS_KPT_LE16 12
#endif
#ifndef CUSORT_OS_KPT_GT16
#define CUSORT_OS_KPT_GT16 8
#endif

// 8-byte keys with 8- or 16-byte values: smaller tiles than the byte-size
// rule, which would spill registers (measured on B200, 2^26 items: u64 + 16 B
// 8.07 -> 6.67 ms at KPT 6, u64 + 8 B 5.83 -> 4.66 ms at KPT 10; the other
// shapes were equal or slower with smaller tiles).
#ifndef CUSORT_OS_KPT_K8V16
#define CUSORT_OS_KPT_K8V16 6
#endif
#ifndef CUSORT_OS_KPT_K8V8
#define CUSORT_OS_KPT_K8V8 10
#endif

// Keys of up to 4 bytes with 1-2 byte values keep their values in shared
// memory (OnesweepCfg::VSMEM), so the register budget allows larger tiles,
// as large as two CTAs per SM fit in shared memory: 32 items per thread for
// 1-2 byte keys (2+2: 28), 28 for 4+1 and 22 for 4+2.  Measured on B200 at
// 2^26: u8+u8 0.327 -> 0.296 ms, u16+u8 0.668 -> 0.599, u16+u16 0.688 ->
// 0.646, u32+u8 1.384 -> 1.292, u32+u16 1.451 -> 1.415.
#ifndef CUSORT_OS_KPT_SMALLV
#define CUSORT_OS_KPT_SMALLV 32
#endif
#ifndef CUSORT_OS_KPT_K2V2
#define CUSORT_OS_KPT_K2V2 28
#endif
#ifndef CUSORT_OS_KPT_K4V1
#define CUSORT_OS_KPT_K4V1 28
#endif
#ifndef CUSORT_OS_KPT_K4V2
#define CUSORT_OS_KPT_K4V2 22
#endif

// Small sorts of 4-byte keys (keys-only or with 4-byte values): a 2^20-key
// sort has only 57 tiles of 512 x 36 keys, so most of the 148 SMs would sit
// idle in every pass.  Up to kSmallTileMaxItems items the tiles hold 8 items
// per thread, up to kMidTileMaxItems 16.  Measured on B200 (u32 keys-only /
// int32+uint32 pairs, us per sort, tile 36 or 20 -> 8 -> 16): 2^16 82 / 64 ->
// 33 / 35 -> 39 / 43; 2^20 72 / 81 -> 53 / 59 -> 59 / 72; 2^21 99 / 88 -> 80
// / 92 -> 66 / 78; 2^23 213 / 239 -> 233 / 268 -> 176 / 218; 2^24 309 / 417
// -> 430 / 514 -> 328 / 422.
#ifndef CUSORT_OS_KPT_SMALL_TILE
#define CUSORT_OS_KPT_SMALL_TILE 8
#endif
#ifndef CUSORT_OS_KPT_MID_TILE
#define CUSORT_OS_KPT_MID_TILE 16
#endif

template <int KB, int VB, bool STAGED = false>
struct TileShape {
  static constexpr int THREADS = CUSORT_OS_THREADS;
  static constexpr int BYTES = KB + VB;
  static constexpr bool SMALLV = CUSORT_VSMEM && KB <= CUSORT_VSMEM_MAXKB && VB > 0 && VB <= 2;
  static constexpr int KPT = (SMALLV && KB == 4 && VB == 2) ? CUSORT_OS_KPT_K4V2
                             : (SMALLV && KB == 4)          ? CUSORT_OS_KPT_K4V1
                             : (SMALLV && KB == 2 && VB == 2) ? CUSORT_OS_KPT_K2V2
                             : SMALLV                       ? CUSORT_OS_KPT_SMALLV
                             : (KB == 8 && VB == 16)  ? CUSORT_OS_KPT_K8V16
                             : (KB == 8 && VB == 8) ? CUSORT_OS_KPT_K8V8
                             : (VB == 0 && KB <= 4 && (STAGED || KB < 4)) ? CUSORT_OS_KPT_KEYS_STAGED
                             : (VB == 0 && KB <= 4) ? CUSORT_OS_KPT_KEYS4
                             : (KB == 4 && VB == 4 && !STAGED) ? CUSORT_OS_KPT_K4V4
                             : (BYTES > 16)         ? CUSORT_OS_KPT_GT16
                             : (BYTES > 8)          ? CUSORT_OS_KPT_LE16
                                                    : CUSORT_OS_KPT_LE8;
  static constexpr int MINB = CUSORT_OS_MINB;
};

constexpr int kHistThreads = 1024;
constexpr int kHistUnroll = 4;

// Largest items-per-thread count <= KPT at which the preferred rank mode's
// per-warp tables still fit the CTA's share of shared memory.  Without it a
// shape whose tables overflow keeps its tile and falls back to the packed
// 16-bit counters of mode 4 -- and routed shapes overflowed the share even
// then (one CTA per SM).  Measured on B200 (ms per sort, 64-bit offsets,
// uint32 + uint32 pairs, 20 items per thread in mode 4 -> 19 in mode 6):
// 2^31 uniform 43.3 -> 43.3, 2^31 Zipf(1.1) over 2^24 values 67.0 -> 50.5;
// 2^30 uniform 21.7 -> 21.4, Zipf 33.5 -> 25.2.
#ifndef CUSORT_FIT_RANK_MODE
#define CUSORT_FIT_RANK_MODE 1
#endif
template <int KB, int VB, typename Off, int THREADS, int KPT, int MINB, bool FK, bool ROUTED, bool SEG>
constexpr int fit_kpt() {
  using CFG = OnesweepCfg<KB, VB, Off, THREADS, KPT, MINB, FK, ROUTED, SEG>;
  if constexpr (!CUSORT_FIT_RANK_MODE || KPT <= 4 || CFG::RANK_MODE == CFG::PREF_RANK_MODE) return KPT;
  else return fit_kpt<KB, VB, Off, THREADS, KPT - 1, MINB, FK, ROUTED, SEG>();
}

// Routed partition pass (multi-GPU): CTAs per SM, tile size in percent of
// the plain staged shape's, and whether the tile is fitted to the 32-bit
// warp counters.  One CTA per SM with 1.4x the items per thread (128
// registers): measured on 2 B200s, 2^31 int32+uint32 pairs per GPU, routed
// pass ms: two CTAs per SM, fitted (17 items per thread) 18.3, not fitted
// (20 items, 16-bit counters; its tables overflowed the two-CTA share, so
// one CTA per SM) 15.8, one CTA 20 / 28 / 36 items 15.7 / 15.5 / 15.5.
// Writing each owner's run of a tile with 16-byte stores instead of one
// item per thread measured 15.5 -> 15.7-18.9 ms, so the per-item scatter
// stays: the pass is bound by the peer link, not by store instructions.
#ifndef CUSORT_ROUTED_MINB
#define CUSORT_ROUTED_MINB 1
#endif
#ifndef CUSORT_ROUTED_KPT_PCT
#define CUSORT_ROUTED_KPT_PCT 140
#endif
// Items of fewer than 8 bytes keep the plain shape (two CTAs per SM): their
// larger tiles spilled registers at one CTA per SM.
#ifndef CUSORT_ROUTED_MIN_ITEM_BYTES
#define CUSORT_ROUTED_MIN_ITEM_BYTES 8
#endif
#ifndef CUSORT_FIT_ROUTED
#define CUSORT_FIT_ROUTED 1
#endif

template <int KB, int VB, typename Off, bool FK, bool ROUTED = false, bool SEG = false>
inline void fill_onesweep(KernelInfo* os) {
  using S = TileShape<KB, VB, ROUTED || SEG || (sizeof(Off) == 8 && !CUSORT_PIPE_WIDE_OFFSETS)>;
  constexpr bool ROUTED_WIDE = ROUTED && KB + VB >= CUSORT_ROUTED_MIN_ITEM_BYTES;
  constexpr int MINB = ROUTED_WIDE ? CUSORT_ROUTED_MINB : S::MINB;
  constexpr int KPT0 = ROUTED_WIDE ? S::KPT * CUSORT_ROUTED_KPT_PCT / 100 : S::KPT;
  constexpr int KPT = (ROUTED && !CUSORT_FIT_ROUTED) ? KPT0 : fit_kpt<KB, VB, Off, S::THREADS, KPT0, MINB, FK, ROUTED, SEG>();
  using CFG = OnesweepCfg<KB, VB, Off, S::THREADS, KPT, MINB, FK, ROUTED, SEG>;
  if constexpr (CFG::PIPE) os->func = reinterpret_cast<const void*>(&onesweep_pipe_kernel<CFG>);
  else os->func = reinterpret_cast<const void*>(&onesweep_kernel<CFG>);
  os->threads = CFG::THREADS;
  os->tile = CFG::TILE;
  os->smem = CFG::SMEM_BYTES;
}

template <int KB, int VB, bool FK, int KPT>
inline void fill_onesweep_small(KernelInfo* os) {
  using CFG = OnesweepCfg<KB, VB, unsigned int, CUSORT_OS_THREADS, KPT, CUSORT_OS_MINB, FK>;
  if constexpr (CFG::PIPE) os->func = reinterpret_cast<const void*>(&onesweep_pipe_kernel<CFG>);
  else os->func = reinterpret_cast<const void*>(&onesweep_kernel<CFG>);
  os->threads = CFG::THREADS;
  os->tile = CFG::TILE;
  os->smem = CFG::SMEM_BYTES;
}

template <int KB, typename Off, bool FK>
inline void fill_histogram(KernelInfo* h) {
  h->func = reinterpret_cast<const void*>(&histogram_kernel<KB, Off, kHistThreads, kHistUnroll, FK>);
  h->threads = kHistThreads;
  h->tile = kHistThreads * kHistUnroll;
  h->smem = HistShape<KB>::SMEM;
}

template <int KB, typename Off, bool FK, bool ROUTED = false>
inline bool fill_for_value(int vb, KernelInfo* os) {
  switch (vb) {
    case 0: fill_onesweep<KB, 0, Off, FK, ROUTED>(os); return true;
    case 1: fill_onesweep<KB, 1, Off, FK, ROUTED>(os); return true;
    case 2: fill_onesweep<KB, 2, Off, FK, ROUTED>(os); return true;
    case 4: fill_onesweep<KB, 4, Off, FK, ROUTED>(os); return true;
    case 8: fill_onesweep<KB, 8, Off, FK, ROUTED>(os); return true;
    case 16: fill_onesweep<KB, 16, Off, FK, ROUTED>(os); return true;
    default: return false;
  }
}

// Floating-point keys exist only at 4 and 8 bytes.
template <int KB, bool FK>
inline bool get_kernels_fk(int vb, int offb, KernelInfo* os, KernelInfo* h) {
  if (offb == 4) {
    fill_histogram<KB, unsigned int, FK>(h);
    return fill_for_value<KB, unsigned int, FK>(vb, os);
  }
  if (offb == 8) {
    fill_histogram<KB, unsigned long long, FK>(h);
    return fill_for_value<KB, unsigned long long, FK>(vb, os);
  }
  return false;
}

template <int KB>
inline bool get_kernels_impl(int vb, int offb, bool float_key, KernelInfo* os, KernelInfo* h) {
  if constexpr (KB == 4 || KB == 8) {
    if (float_key) return get_kernels_fk<KB, true>(vb, offb, os, h);
  } else {
    if (float_key) return false;
  }
  return get_kernels_fk<KB, false>(vb, offb, os, h);
}

// Routed onesweep kernels (single partition pass of the multi-GPU sort).
template <int KB>
inline bool get_routed_impl(int vb, int offb, bool float_key, KernelInfo* os) {
  if constexpr (KB == 4 || KB == 8) {
    if (float_key) {
      if (offb == 4) return fill_for_value<KB, unsigned int, true, true>(vb, os);
      if (offb == 8) return fill_for_value<KB, unsigned long long, true, true>(vb, os);
      return false;
    }
  } else {
    if (float_key) return false;
  }
  if (offb == 4) return fill_for_value<KB, unsigned int, false, true>(vb, os);
  if (offb == 8) return fill_for_value<KB, unsigned long long, false, true>(vb, os);
  return false;
}

// Segmented sort kernels for one (key width, value width, offset width, float).
template <int KB, int VB, typename Off, bool FK>
inline void fill_segmented(SegKernels* k) {
  fill_onesweep<KB, VB, Off, FK, false, true>(&k->onesweep);
  k->hist.func = reinterpret_cast<const void*>(&seg_hist_kernel<KB, Off, FK>);
  k->hist.threads = 512;
  k->hist.smem = (size_t)KB * kRadix * kSegHistReplicas * 4;  // at most KB passes
  k->scan.func = reinterpret_cast<const void*>(&seg_scan_kernel<Off>);
  k->scan.threads = 256;
  constexpr int KPT = SegSmallShape<KB, VB>::KPT;
  k->small_warp.func = reinterpret_cast<const void*>(&seg_small_kernel<KB, VB, FK, 1, KPT>);
  k->small_warp.threads = 256;
  k->small_warp.tile = SegSmallLayout<KB, VB, FK, 1, KPT>::CAP;
  k->small_warp.smem = SegSmallLayout<KB, VB, FK, 1, KPT>::SMEM;
  // shapes of 16 items per thread: a one-warp class of 8 first (no register
  // spills; the shorter half of the one-warp lengths)
  if constexpr (KPT > 8) {
    k->small_warp8.func = reinterpret_cast<const void*>(&seg_small_kernel<KB, VB, FK, 1, 8>);
    k->small_warp8.threads = 256;
    k->small_warp8.tile = SegSmallLayout<KB, VB, FK, 1, 8>::CAP;
    k->small_warp8.smem = SegSmallLayout<KB, VB, FK, 1, 8>::SMEM;
  } else {
    k->small_warp8 = KernelInfo{};
  }
  static_assert(kTinyClasses == 2 && sizeof(k->tiny) / sizeof(k->tiny[0]) == kTinyClasses, "tiny classes");
  k->tiny[0].func = reinterpret_cast<const void*>(&seg_tiny_kernel<KB, VB, FK, kTinySlotsOf[0]>);
  k->tiny[1].func = reinterpret_cast<const void*>(&seg_tiny_kernel<KB, VB, FK, kTinySlotsOf[1]>);
  for (int t = 0; t < kTinyClasses; ++t) {
    k->tiny[t].threads = 256;
    k->tiny[t].tile = 32 * kTinySlotsOf[t];
    k->tiny[t].smem = 0;
  }
  k->small_2warps.func = reinterpret_cast<const void*>(&seg_small_kernel<KB, VB, FK, 2, KPT>);
  k->small_2warps.threads = 256;
  k->small_2warps.tile = SegSmallLayout<KB, VB, FK, 2, KPT>::CAP;
  k->small_2warps.smem = SegSmallLayout<KB, VB, FK, 2, KPT>::SMEM;
  k->small_4warps.func = reinterpret_cast<const void*>(&seg_small_kernel<KB, VB, FK, 4, KPT>);
  k->small_4warps.threads = 256;
  k->small_4warps.tile = SegSmallLayout<KB, VB, FK, 4, KPT>::CAP;
  k->small_4warps.smem = SegSmallLayout<KB, VB, FK, 4, KPT>::SMEM;
  k->small_block.func = reinterpret_cast<const void*>(&seg_small_kernel<KB, VB, FK, 8, KPT>);
  k->small_block.threads = 256;
  k->small_block.tile = SegSmallLayout<KB, VB, FK, 8, KPT>::CAP;
  k->small_block.smem = SegSmallLayout<KB, VB, FK, 8, KPT>::SMEM;
  k->small_block2.func = reinterpret_cast<const void*>(&seg_small_kernel<KB, VB, FK, 8, 2 * KPT>);
  k->small_block2.threads = 256;
  k->small_block2.tile = SegSmallLayout<KB, VB, FK, 8, 2 * KPT>::CAP;
  k->small_block2.smem = SegSmallLayout<KB, VB, FK, 8, 2 * KPT>::SMEM;
}

template <int KB, typename Off, bool FK>
inline bool fill_segmented_vb(int vb, SegKernels* k) {
  switch (vb) {
    case 0: fill_segmented<KB, 0, Off, FK>(k); return true;
    case 1: fill_segmented<KB, 1, Off, FK>(k); return true;
    case 2: fill_segmented<KB, 2, Off, FK>(k); return true;
    case 4: fill_segmented<KB, 4, Off, FK>(k); return true;
    case 8: fill_segmented<KB, 8, Off, FK>(k); return true;
    case 16: fill_segmented<KB, 16, Off, FK>(k); return true;
    default: return false;
  }
}

template <int KB>
inline bool get_segmented_impl(int vb, int offb, bool float_key, SegKernels* k) {
  if constexpr (KB == 4 || KB == 8) {
    if (float_key) {
      if (offb == 4) return fill_segmented_vb<KB, unsigned int, true>(vb, k);
      if (offb == 8) return fill_segmented_vb<KB, unsigned long long, true>(vb, k);
      return false;
    }
  } else {
    if (float_key) return false;
  }
  if (offb == 4) return fill_segmented_vb<KB, unsigned int, false>(vb, k);
  if (offb == 8) return fill_segmented_vb<KB, unsigned long long, false>(vb, k);
  return false;
}

}  // namespace cusort_b200

// cusort_segmented.cuh -- kernels of the segmented sort (each segment
// [begin[s], end[s]) of the input sorted independently, stable, into the same
// positions of the output).  The reference names segmented sorting in its
// banner (libcusort.cuh:4) but implements none; the interface follows CUB's
// DeviceSegmentedRadixSort (begin/end offset arrays in device memory).
//
// Segments are handled by length class, with no host synchronisation:
//   * up to 128 items: one warp per segment, one item per lane (up to 32
//     items) or four, stable rank of the whole masked key by all-pairs
//     comparison (seg_tiny_kernel);
//   * up to 32*KPT items: one warp per segment, every pass in shared memory
//     (seg_small_kernel<..., WPS = 1>; where KPT is 16, a kernel of 8 items
//     per thread takes the lengths up to 256 first);
//   * up to 64*KPT, 128*KPT, 256*KPT items: groups of 2, 4 or 8 warps per
//     segment (four, two or one per CTA), same scheme
//     (seg_small_kernel<..., WPS = 2, 4, 8>);
//   * up to 512*KPT items: one CTA per segment with 2*KPT items per thread
//     (seg_small_kernel<..., WPS = 8, 2*KPT>, two CTAs per SM);
//   * longer: cut into onesweep tiles that never straddle a segment.  The
//     planner (seg_plan_kernel) gives each such segment a slot and a run of
//     tile numbers, seg_hist_kernel counts every pass's digits per segment,
//     seg_scan_kernel turns the counts into segment-local digit bases, and
//     each pass is onesweep_kernel with SEG = true (lookback stops at the
//     segment's first tile).
#pragma once

#include <type_traits>

#include "cusort_device.cuh"
#include "cusort_types.h"

namespace cusort_b200 {

enum : uint32_t { kStatusSegOverflow = 8u };  // more tiles/segments than planned (overlapping segments)

// Items per thread of the small-segment sorts, by bytes per item.
template <int KB, int VB>
struct SegSmallShape {
  static constexpr int BYTES = KB + VB;
  static constexpr int KPT = BYTES <= 8 ? 16 : (BYTES <= 16 ? 8 : 4);
};

// ---------------------------------------------------------------------------
// small segments: WPS warps sort one segment of at most WPS*32*KPT items, all
// passes in shared memory, then one coalesced write.  Per pass: each warp
// ranks its slots in order with a ballot match (rank among equal digits =
// earlier slots' count + lower lanes of this slot), the group turns the
// per-warp digit counts into offsets (digit-major, warp-minor: stable), and
// every item is stored at its offset (in place: all items are in registers).
// ---------------------------------------------------------------------------
template <int KB, int VB, bool FK, int WPS, int KPT>
struct SegSmallLayout {
  static constexpr int CAP = WPS * 32 * KPT;
  static constexpr size_t KEYS = ((size_t)CAP * KB + 15) / 16 * 16;
  static constexpr size_t VALS = ((size_t)CAP * (VB ? VB : 1) + 15) / 16 * 16;
  static constexpr size_t CNT = (size_t)WPS * kRadix * 4;
  static constexpr size_t SCAN = 16 * 4;
  static constexpr size_t QUAL = 8 * 4;  // the qualifying segments of a chunk, one mask per warp
  static constexpr size_t GROUP = KEYS + VALS + CNT + SCAN + QUAL;
  static constexpr int GROUPS = 8 / WPS;
  static constexpr size_t SMEM = GROUP * GROUPS;
};

// Resident CTAs per SM the small-segment kernels are compiled for (4: at most
// 64 registers per thread).  The large CTA class (twice the items per thread
// of its shape) is compiled for 2.
#ifndef CUSORT_SEG_SMALL_MIN_CTAS
#define CUSORT_SEG_SMALL_MIN_CTAS 4
#endif

template <int KB, int VB, bool FK, int WPS, int KPT>
__global__ void __launch_bounds__(256, (KPT > SegSmallShape<KB, VB>::KPT) ? 2 : CUSORT_SEG_SMALL_MIN_CTAS)
    seg_small_kernel(const SegSmallArgs a) {
  using K = typename dev::UIntOf<KB>::T;
  using V = typename dev::UIntOf<(VB ? VB : 1)>::T;
  using L = SegSmallLayout<KB, VB, FK, WPS, KPT>;
  constexpr bool HAS_V = VB > 0;
  constexpr int GT = WPS * 32;  // threads per group
  extern __shared__ __align__(16) uint8_t smem[];

  const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
  const uint32_t g = warp / WPS, wg = warp % WPS, gtid = tid % GT;
  uint8_t* gb = smem + (size_t)g * L::GROUP;
  K* sk = reinterpret_cast<K*>(gb);
  V* sv = reinterpret_cast<V*>(gb + L::KEYS);
  uint32_t* cnt = reinterpret_cast<uint32_t*>(gb + L::KEYS + L::VALS);  // [WPS][256]
  uint32_t* scan = reinterpret_cast<uint32_t*>(gb + L::KEYS + L::VALS + L::CNT);
  uint32_t* qual = reinterpret_cast<uint32_t*>(gb + L::KEYS + L::VALS + L::CNT + L::SCAN);
  // the group's barrier: its warp, the CTA, or (2 or 4 warps) named barrier
  // 1 + g, so the groups of a CTA advance independently
  auto gsync = [&]() {
    if constexpr (WPS == 1) {
      __syncwarp();
    } else if constexpr (WPS == 8) {
      __syncthreads();
    } else {
      asm volatile("bar.sync %0, %1;" ::"r"(1u + g), "r"((uint32_t)GT) : "memory");
    }
  };
  const K* keys_in = static_cast<const K*>(a.keys_in);
  K* keys_out = static_cast<K*>(a.keys_out);
  const V* vals_in = static_cast<const V*>(a.vals_in);
  V* vals_out = static_cast<V*>(a.vals_out);
  const K tc = (K)a.tw_c, tf = (K)a.tw_f;
  const uint32_t lt = dev::lanemask_lt();

  auto length_of = [&](uint64_t s) -> uint64_t {
    const int64_t b = a.begin_offsets[s], e = a.end_offsets[s];
    return e > b ? (uint64_t)(e - b) : 0;
  };
  auto sort_segment = [&](uint64_t s) {
    const int64_t b = a.begin_offsets[s];
    const uint32_t n = (uint32_t)length_of(s);
    for (uint32_t i = gtid; i < n; i += GT) {
      sk[i] = keys_in[b + i];
      if constexpr (HAS_V) sv[i] = vals_in[b + i];
    }
    gsync();
    for (uint32_t p = 0; p < a.passes; ++p) {
      const uint32_t shift = a.begin_bit + 8u * p;
      const uint32_t mask = (p + 1 == a.passes) ? a.last_mask : 0xffu;
      uint32_t* wc = cnt + wg * kRadix;
      for (uint32_t d = lane; d < kRadix; d += 32) wc[d] = 0;
      __syncwarp();
      K key[KPT];
      V val[HAS_V ? KPT : 1];
      uint32_t rd[KPT];  // digit (9 bits, 0x100 = past the end) | rank within the warp << 9
      const uint32_t wfirst = wg * KPT * 32;
      // slots past the segment's end (warp-uniform) are skipped: short
      // segments cost their own length, not the group's capacity
#pragma unroll
      for (int sl = 0; sl < KPT; ++sl) {
        rd[sl] = 0x100u;
        if (wfirst + sl * 32 >= n) continue;
        const uint32_t i = wfirst + sl * 32 + lane;
        const bool in = i < n;
        key[sl] = in ? sk[i] : K(0);
        if constexpr (HAS_V) val[sl] = in ? sv[i] : V{};
        const uint32_t d = in ? dev::digit_k<FK, K>(key[sl], tc, tf, shift, mask) : 0x100u;
        // peers: 8 ballots (about twice the rate of match.any on B200),
        // restricted to the lanes inside the segment
        const uint32_t peers = dev::match_digit_ballot<8>(d) & __ballot_sync(0xffffffffu, in);
        uint32_t before = 0;
        if (in) before = wc[d];
        __syncwarp();
        if (in && (peers & lt) == 0) wc[d] = before + __popc(peers);
        __syncwarp();
        rd[sl] = d | ((before + __popc(peers & lt)) << 9);
      }
      gsync();
      // digit totals -> offsets[w][d] = start of digit d + items of d in lower warps
      if constexpr (WPS == 8) {
        const uint32_t d = tid;  // 256 threads, one digit each
        uint32_t tot = 0;
#pragma unroll
        for (int w = 0; w < WPS; ++w) tot += cnt[w * kRadix + d];
        const uint32_t incl = dev::warp_inclusive_scan(tot, lane);
        if (lane == 31) scan[warp] = incl;
        __syncthreads();
        uint32_t start = incl - tot;
        for (uint32_t w = 0; w < warp; ++w) start += scan[w];
#pragma unroll
        for (int w = 0; w < WPS; ++w) {
          const uint32_t c = cnt[w * kRadix + d];
          cnt[w * kRadix + d] = start;
          start += c;
        }
      } else if constexpr (WPS > 1) {
        // 64 or 128 threads, DPT consecutive digits each
        constexpr int DPT = kRadix / GT;
        const uint32_t d0 = gtid * DPT;
        uint32_t tot[DPT], sum = 0;
#pragma unroll
        for (int j = 0; j < DPT; ++j) {
          tot[j] = 0;
#pragma unroll
          for (int w = 0; w < WPS; ++w) tot[j] += cnt[w * kRadix + d0 + j];
          sum += tot[j];
        }
        const uint32_t incl = dev::warp_inclusive_scan(sum, lane);
        if (lane == 31) scan[wg] = incl;
        gsync();
        uint32_t start = incl - sum;
        for (uint32_t w = 0; w < wg; ++w) start += scan[w];
#pragma unroll
        for (int j = 0; j < DPT; ++j) {
          uint32_t run = start;
#pragma unroll
          for (int w = 0; w < WPS; ++w) {
            const uint32_t c = cnt[w * kRadix + d0 + j];
            cnt[w * kRadix + d0 + j] = run;
            run += c;
          }
          start += tot[j];
        }
      } else {
        // one warp: lane handles digits 8*lane .. 8*lane+7
        uint32_t c[8], sum = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          c[j] = cnt[lane * 8 + j];
          sum += c[j];
        }
        uint32_t start = dev::warp_inclusive_scan(sum, lane) - sum;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          cnt[lane * 8 + j] = start;
          start += c[j];
        }
      }
      gsync();
#pragma unroll
      for (int sl = 0; sl < KPT; ++sl) {
        const uint32_t d = rd[sl] & 0x1ffu;
        if (d < kRadix) {  // 0x100: past the end
          const uint32_t pos = cnt[wg * kRadix + d] + (rd[sl] >> 9);
          sk[pos] = key[sl];
          if constexpr (HAS_V) sv[pos] = val[sl];
        }
      }
      gsync();
    }
    for (uint32_t i = gtid; i < n; i += GT) {
      keys_out[b + i] = sk[i];
      if constexpr (HAS_V) vals_out[b + i] = sv[i];
    }
    gsync();  // the buffers are reused by the next segment
  };

  // Group G owns segments G, G + groups, G + 2 groups, ...  It examines GT of
  // them at a time, one per thread, and then sorts the ones of its length
  // class in order: finding them costs one round trip per GT segments, not
  // one per segment (with millions of short segments, mostly of other
  // classes, that round trip dominated), and the work stays spread over the
  // groups as before.
  const uint64_t groups = (uint64_t)gridDim.x * L::GROUPS;
  const uint64_t G = (uint64_t)blockIdx.x * L::GROUPS + g;
  auto seg_at = [&](uint64_t base, uint32_t t) { return base + (uint64_t)t * groups + G; };
  for (uint64_t base = 0; base + G < a.num_segments; base += groups * GT) {
    const uint64_t mine = seg_at(base, gtid);
    uint64_t len = 0;
    if (mine < a.num_segments) len = length_of(mine);
    const uint32_t qm = __ballot_sync(0xffffffffu, len != 0 && len >= a.min_len && len <= a.max_len);
    if constexpr (WPS == 1) {
      for (uint32_t m = qm; m; m &= m - 1) sort_segment(seg_at(base, (uint32_t)(__ffs(m) - 1)));
    } else {
      if (lane == 0) qual[wg] = qm;
      gsync();
      for (int w = 0; w < WPS; ++w)
        for (uint32_t m = qual[w]; m; m &= m - 1) sort_segment(seg_at(base, (uint32_t)w * 32 + (uint32_t)(__ffs(m) - 1)));
      gsync();  // every thread of the group has read qual[] before it is rewritten
    }
  }
}

// ---------------------------------------------------------------------------
// planner: a slot and a run of tile numbers for every segment longer than
// min_len (atomic allocation: each segment's tiles are consecutive, which is
// all the lookback needs).  Capacity is checked; an overflow (only possible
// with overlapping segments) sets kStatusSegOverflow and ctl->pad[0], and the
// tiled kernels then do nothing.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) seg_plan_kernel(const SegPlanArgs a);

// ---------------------------------------------------------------------------
// per-segment digit counts of every pass, one tile at a time
// ---------------------------------------------------------------------------
// Replicas of the per-segment counters: lane l counts into replica l % R
// ([pass][digit][replica]), so a warp's shared atomics rarely collide.
constexpr int kSegHistReplicas = 8;

template <int KB, typename Off, bool FK>
__global__ void __launch_bounds__(512) seg_hist_kernel(const SegHistArgs a) {
  using K = typename dev::UIntOf<KB>::T;
  constexpr int R = kSegHistReplicas;
  constexpr int PER = 16 / KB;  // keys per 16-byte load
  extern __shared__ __align__(16) uint32_t s_cnt[];  // [passes][256][R]
  dev::pdl_wait();
  dev::pdl_launch_dependents();
  const uint32_t tid = threadIdx.x;
  const uint32_t P = a.passes;
  const uint32_t num_tiles = a.ctl->pad[0] ? 0u : a.ctl->num_tiles;
  const K* keys = static_cast<const K*>(a.keys);
  const K tc = (K)a.tw_c, tf = (K)a.tw_f;
  Off* hist = static_cast<Off*>(a.seg_hist);
  uint32_t* my = s_cnt + (tid % R);
  auto count = [&](K k) {
    const K tw = dev::twiddle_k<FK, K>(k, tc, tf);
    for (uint32_t p = 0; p < P; ++p) {
      const uint32_t m = (p + 1 == P) ? a.last_mask : 0xffu;
      atomicAdd(my + (p * kRadix + ((uint32_t)(tw >> (a.begin_bit + 8 * p)) & m)) * R, 1u);
    }
  };
  // Each CTA counts a contiguous range of tiles and flushes its counts when
  // the segment changes (and at the end), so a long segment costs one flush
  // per CTA, not one per tile.
  const uint32_t per = (num_tiles + gridDim.x - 1) / gridDim.x;
  const uint32_t t0 = blockIdx.x * per, t1 = min(num_tiles, t0 + per);
  for (uint32_t i = tid; i < P * kRadix * R; i += blockDim.x) s_cnt[i] = 0;
  __syncthreads();
  uint32_t cur_slot = 0xffffffffu;
  auto flush = [&]() {
    Off* h = hist + (size_t)cur_slot * P * kRadix;
    for (uint32_t i = tid; i < P * kRadix; i += blockDim.x) {
      uint32_t c = 0;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const uint32_t x = i * R + ((r + i) % R);  // rotated: conflict-free
        c += s_cnt[x];
        s_cnt[x] = 0;
      }
      if (c) atomicAdd(h + i, (Off)c);
    }
    __syncthreads();
  };
  for (uint32_t t = t0; t < t1; ++t) {
    const uint32_t slot = a.tile_slot[t];
    if (slot != cur_slot) {
      if (cur_slot != 0xffffffffu) flush();
      cur_slot = slot;
    }
    const SegRecord r = a.recs[slot];
    const uint64_t off = (uint64_t)(t - r.tile_first) * a.tile;
    const uint64_t base = r.begin + off;
    const uint32_t valid = (uint32_t)((r.len - off) < (uint64_t)a.tile ? (r.len - off) : (uint64_t)a.tile);
    // 16-byte loads between the unaligned head and the ragged tail
    const K* kp = keys + base;
    uint32_t head = (uint32_t)(((16 - (reinterpret_cast<uintptr_t>(kp) & 15)) & 15) / KB);
    if (head > valid) head = valid;
    const uint32_t nvec = (valid - head) / PER;
    const uint4* vec = reinterpret_cast<const uint4*>(kp + head);
    for (uint32_t v = tid; v < nvec; v += blockDim.x) {
      const uint4 x = dev::ld_stream_v4(vec + v);
      const K* kk = reinterpret_cast<const K*>(&x);
#pragma unroll
      for (int e = 0; e < PER; ++e) count(kk[e]);
    }
    for (uint32_t j = tid; j < head; j += blockDim.x) count(kp[j]);
    for (uint32_t j = head + nvec * PER + tid; j < valid; j += blockDim.x) count(kp[j]);
    __syncthreads();
  }
  if (cur_slot != 0xffffffffu) flush();
}

// counts -> segment begin + exclusive digit prefix, per (slot, pass), in place
template <typename Off>
__global__ void __launch_bounds__(256) seg_scan_kernel(const SegHistArgs a) {
  __shared__ Off s_part[8];
  dev::pdl_wait();
  dev::pdl_launch_dependents();
  const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
  const uint32_t slots = a.ctl->pad[0] ? 0u : a.ctl->num_slots;
  Off* hist = static_cast<Off*>(a.seg_hist);
  for (uint64_t x = blockIdx.x; x < (uint64_t)slots * a.passes; x += gridDim.x) {
    const uint64_t slot = x / a.passes;
    Off* h = hist + x * kRadix;
    const Off c = h[tid];
    Off incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const Off t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= (uint32_t)o) incl += t;
    }
    if (lane == 31) s_part[warp] = incl;
    __syncthreads();
    Off pre = (Off)a.recs[slot].begin;
    for (uint32_t w = 0; w < warp; ++w) pre += s_part[w];
    h[tid] = pre + incl - c;
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// tiny segments (at most 32 * S items): one warp per segment, up to S items
// per lane (item sl * 32 + lane in slot sl), every pass at once: an item's
// output position is the number of items whose masked key (all bits of
// [begin_bit, end_bit), twiddled) is smaller, or equal and earlier in the
// segment -- a stable rank by all-pairs comparison over warp shuffles, then
// one store per item.  Work is (length / 32) x length shuffle-compares,
// whatever the number of passes: up to 128 items that is less than the
// per-pass digit counts and scans of the warp class (at 200-256 items it was
// more).  Two instances: S = 1 for 1-32 items and S = 4 for 33-128; the
// one-slot kernel keeps four segments' loads in flight per warp.
// ---------------------------------------------------------------------------
constexpr int kTinyClasses = 2;
constexpr int kTinySlotsOf[kTinyClasses] = {1, 4};

// Ranks of the U occupied slots: every valid item (slot ss, lane l) of the
// segment is broadcast once and compared with each own item.
template <int U, int S, typename M>
__device__ __forceinline__ void tiny_rank(const M (&mk)[S], uint32_t (&rank)[S], uint32_t n, uint32_t lane) {
#pragma unroll
  for (int ss = 0; ss < U; ++ss) {
    const uint32_t cnt = min(32u, n - (uint32_t)ss * 32u);
#pragma unroll 4
    for (uint32_t l = 0; l < cnt; ++l) {
      const M o = __shfl_sync(0xffffffffu, mk[ss], l);
#pragma unroll
      for (int si = 0; si < U; ++si) {
        // item (ss, l) precedes item (si, lane) in the segment when ss < si,
        // or ss == si and l < lane
        bool lt;
        if (ss < si) lt = o <= mk[si];
        else if (ss > si) lt = o < mk[si];
        else lt = o < mk[si] || (o == mk[si] && l < lane);
        rank[si] += lt ? 1u : 0u;
      }
    }
  }
}

// tiny_rank<used> for the warp-uniform number of occupied slots
template <int U, int S, typename M>
__device__ __forceinline__ void tiny_rank_used(uint32_t used, const M (&mk)[S], uint32_t (&rank)[S], uint32_t n,
                                               uint32_t lane) {
  if constexpr (U < S) {
    if (used <= (uint32_t)U) {
      tiny_rank<U, S>(mk, rank, n, lane);
      return;
    }
    tiny_rank_used<U + 1, S>(used, mk, rank, n, lane);
  } else {
    tiny_rank<S, S>(mk, rank, n, lane);
  }
}

template <int KB, int VB, bool FK, int S>
__global__ void __launch_bounds__(256) seg_tiny_kernel(const SegSmallArgs a) {
  using K = typename dev::UIntOf<KB>::T;
  using V = typename dev::UIntOf<(VB ? VB : 1)>::T;
  constexpr bool HAS_V = VB > 0;
  // the masked key, compared as 32 bits when the key fits (one shuffle)
  using M = typename std::conditional<(KB <= 4), uint32_t, unsigned long long>::type;
  const uint32_t lane = threadIdx.x & 31u;
  const K* keys_in = static_cast<const K*>(a.keys_in);
  K* keys_out = static_cast<K*>(a.keys_out);
  const V* vals_in = static_cast<const V*>(a.vals_in);
  V* vals_out = static_cast<V*>(a.vals_out);
  const K tc = (K)a.tw_c, tf = (K)a.tw_f;
  const uint32_t nbits = 8u * (a.passes - 1u) + (uint32_t)__popc(a.last_mask);
  const unsigned long long range = nbits >= 64 ? ~0ull : ((1ull << nbits) - 1ull);
  // Warp W examines segments W*32 .. W*32+31 (one per lane, coalesced), then
  // the next chunk NW*32 further on, and sorts the ones of its class P at a
  // time: the P segments' loads are in flight together, and skipping the
  // segments of other classes costs one round trip per 32 of them.
  constexpr int P = S == 1 ? 4 : (S <= 4 ? 2 : 1);
  const uint64_t nw = (uint64_t)gridDim.x * (blockDim.x >> 5);
  for (uint64_t base = ((uint64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 32u; base < a.num_segments;
       base += nw * 32u) {
    int64_t mb = 0, me = 0;
    if (base + lane < a.num_segments) {
      mb = a.begin_offsets[base + lane];
      me = a.end_offsets[base + lane];
    }
    const uint64_t len = me > mb ? (uint64_t)(me - mb) : 0;
    uint32_t m = __ballot_sync(0xffffffffu, len != 0 && len >= a.min_len && len <= a.max_len &&
                                                len <= (uint64_t)(32 * S));
    while (m) {  // warp-uniform
      int64_t sb[P];
      uint32_t sn[P];
#pragma unroll
      for (int p = 0; p < P; ++p) {
        sb[p] = 0;
        sn[p] = 0;
        if (m) {
          const int j = __ffs(m) - 1;
          m &= m - 1;
          sb[p] = __shfl_sync(0xffffffffu, mb, j);
          sn[p] = (uint32_t)(__shfl_sync(0xffffffffu, me, j) - sb[p]);
        }
      }
      K k[P][S];
      V v[P][HAS_V ? S : 1];
#pragma unroll
      for (int p = 0; p < P; ++p) {
#pragma unroll
        for (int sl = 0; sl < S; ++sl) {
          const uint32_t i = (uint32_t)sl * 32u + lane;
          k[p][sl] = K(0);
          if constexpr (HAS_V) v[p][sl] = V{};
          if (i < sn[p]) {
            k[p][sl] = keys_in[sb[p] + i];
            if constexpr (HAS_V) v[p][sl] = vals_in[sb[p] + i];
          }
        }
      }
#pragma unroll
      for (int p = 0; p < P; ++p) {
        const uint32_t n = sn[p];
        if (n == 0) continue;  // warp-uniform
        M mk[S];
        uint32_t rank[S];
#pragma unroll
        for (int sl = 0; sl < S; ++sl) {
          mk[sl] = (M)(((unsigned long long)dev::twiddle_k<FK, K>(k[p][sl], tc, tf) >> a.begin_bit) & range);
          rank[sl] = 0;
        }
        tiny_rank_used<1, S>((n + 31u) / 32u, mk, rank, n, lane);
#pragma unroll
        for (int sl = 0; sl < S; ++sl) {
          if ((uint32_t)sl * 32u + lane < n) {
            keys_out[sb[p] + rank[sl]] = k[p][sl];
            if constexpr (HAS_V) vals_out[sb[p] + rank[sl]] = v[p][sl];
          }
        }
      }
    }
  }
}

// begin_bit == end_bit: every segment is copied as it is
template <int BYTES>
__global__ void __launch_bounds__(256) seg_copy_kernel(const SegSmallArgs a) {
  using T = typename dev::UIntOf<BYTES>::T;
  (void)sizeof(T);
  const T* in = static_cast<const T*>(a.keys_in);
  T* out = static_cast<T*>(a.keys_out);
  for (uint64_t s = blockIdx.x; s < a.num_segments; s += gridDim.x) {
    const int64_t b = a.begin_offsets[s], e = a.end_offsets[s];
    for (int64_t i = b + threadIdx.x; i < e; i += blockDim.x) out[i] = in[i];
  }
}

}  // namespace cusort_b200

// cusort_kernels.cuh -- the three kernels of one sort, as templates.
//
//   init_kernel       zero the control block + lookback descriptors
//   histogram_kernel  one read of the keys -> digit counts of every pass
//   onesweep_kernel   one stable 8-bit LSD pass (persistent CTAs, TMA tile
//                     staging, shared-memory ranking, decoupled lookback,
//                     shared-memory reorder, coalesced scatter)
//
// Reference counterparts: RadixSortHistogramKernel (libcusort.cuh:1679-1841),
// RadixSortOnesweepKernel (libcusort.cuh:1843-2415), the temp memset
// (libcusort.cuh:2650).  The algorithm (Onesweep: one upfront histogram, one
// binning kernel per digit with decoupled lookback) is the same; the kernels
// are re-designed for sm_100a (see the per-kernel comments).
#pragma once

#include <type_traits>

#include "cusort_device.cuh"

namespace cusort_b200 {

__host__ __device__ constexpr size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// ---------------------------------------------------------------------------
// histogram: digit counts of every pass from ONE read of the keys.
// 16-byte streaming loads (ld.global.nc.L1::no_allocate.v4), UNROLL vectors in
// flight per thread, one persistent CTA per SM.  Shared-memory counters are
// replicated R times and laid out [pass][digit][replica] so that lane l always
// increments replica l % R: with R = 32 every lane of a warp hits its own bank
// and the P shared atomics per key are conflict-free (a single 256-bin table
// costs ~3.5 wavefronts per warp atomic for random digits).  The replicas are
// summed once per CTA into one global atomic per (pass, digit).  The global
// atomics wait for the init kernel (PDL); reads and counting overlap it.
// ---------------------------------------------------------------------------
template <int KB>
struct HistShape {
  static constexpr int MAXP = KB;  // 8-bit digits: at most one pass per key byte
  static constexpr int R = (KB == 8) ? 16 : 32;
  static constexpr size_t SMEM = (size_t)MAXP * kRadix * R * 4;
};

template <int KB, typename Off, int THREADS, int UNROLL, bool FLOAT_KEY>
__global__ void __launch_bounds__(THREADS, 1) histogram_kernel(const HistArgs a) {
  using K = typename dev::UIntOf<KB>::T;
  using HS = HistShape<KB>;
  constexpr int MAXP = HS::MAXP, R = HS::R;
  constexpr int PER = 16 / KB;  // keys per 16-byte vector
  extern __shared__ __align__(16) uint32_t s_hist[];

  dev::pdl_launch_dependents();
  const uint32_t tid = threadIdx.x;
  const uint32_t rep = tid % R;
  for (uint32_t i = tid; i < MAXP * kRadix * R; i += THREADS) s_hist[i] = 0;
  __syncthreads();

  const K tc = (K)a.tw_c, tf = (K)a.tw_f;
  const uint32_t P = a.num_passes;
  uint32_t* my_hist = s_hist + rep;

  const K* keys = static_cast<const K*>(a.keys);
  const uint64_t n = a.n;
  const uintptr_t addr = reinterpret_cast<uintptr_t>(keys);
  uint64_t head = ((16 - (addr & 15)) & 15) / KB;
  if (head > n) head = n;
  const uint64_t nvec = (n - head) / PER;
  const uint4* vec = reinterpret_cast<const uint4*>(keys + head);
  const uint64_t gthreads = (uint64_t)gridDim.x * THREADS;
  const uint64_t gtid = (uint64_t)blockIdx.x * THREADS + tid;

  // FULL: every byte of the key is one pass (begin_bit 0, all passes 8 bits
  // wide) -- the common case -- so digits are constant byte extractions and
  // the counter offsets compile-time constants.
  auto run = [&](auto full_tag) {
    constexpr bool FULL = decltype(full_tag)::value;
    auto count = [&](K k) {
      const K t = dev::twiddle_k<FLOAT_KEY, K>(k, tc, tf);
#pragma unroll
      for (int p = 0; p < MAXP; ++p) {
        if constexpr (FULL) {
          const uint32_t d = (uint32_t)(t >> (8 * p)) & 0xffu;
          atomicAdd(my_hist + (p * kRadix + d) * R, 1u);
        } else if (p < (int)P) {
          const uint32_t m = (p + 1 == (int)P) ? a.last_mask : 0xffu;
          const uint32_t d = (uint32_t)(t >> (a.begin_bit + 8 * p)) & m;
          atomicAdd(my_hist + (p * kRadix + d) * R, 1u);
        }
      }
    };
    uint64_t v = gtid;
    for (; v + (UNROLL - 1) * gthreads < nvec; v += UNROLL * gthreads) {
      uint4 x[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) x[u] = dev::ld_stream_v4(vec + v + u * gthreads);
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const K* kk = reinterpret_cast<const K*>(&x[u]);
#pragma unroll
        for (int e = 0; e < PER; ++e) count(kk[e]);
      }
    }
    for (; v < nvec; v += gthreads) {
      uint4 x = dev::ld_stream_v4(vec + v);
      const K* kk = reinterpret_cast<const K*>(&x);
#pragma unroll
      for (int e = 0; e < PER; ++e) count(kk[e]);
    }
    // Unaligned head and ragged tail, element by element.
    for (uint64_t i = gtid; i < head; i += gthreads) count(keys[i]);
    for (uint64_t i = head + nvec * PER + gtid; i < n; i += gthreads) count(keys[i]);
  };
  if (P == (uint32_t)MAXP && a.begin_bit == 0 && a.last_mask == 0xffu)
    run(std::integral_constant<bool, true>{});
  else
    run(std::integral_constant<bool, false>{});
  __syncthreads();

  dev::pdl_wait();  // g_hist zeroed by init_kernel
  Off* g = static_cast<Off*>(a.g_hist);
  for (uint32_t i = tid; i < P * kRadix; i += THREADS) {
    uint32_t c = 0;
#pragma unroll 8
    for (int r = 0; r < R; ++r) c += s_hist[i * R + ((r + i) % R)];  // rotated: conflict-free
    if (c) atomicAdd(g + i, (Off)c);
  }
}

// ---------------------------------------------------------------------------
// fill (1-byte keys-only, all 8 bits sorted): the digit is the whole key, so
// keys with equal digits are bit-identical and the sorted output is every key
// value repeated by its count -- one histogram read plus this write-only
// kernel, instead of a ranking pass.  out[i] = (d ^ c) for the digit d whose
// range [start[d], start[d+1]) holds i.
// ---------------------------------------------------------------------------
template <typename Off>
__global__ void __launch_bounds__(256) fill_bytes_kernel(const FillArgs a) {
  __shared__ Off s_start[kRadix + 1];
  __shared__ Off s_part[8];
  const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
  dev::pdl_wait();  // counts from the histogram kernel
  const Off c = static_cast<const Off*>(a.counts)[tid];
  Off incl = c;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const Off t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= (uint32_t)o) incl += t;
  }
  if (lane == 31) s_part[warp] = incl;
  __syncthreads();
  Off pre = 0;
  for (uint32_t w = 0; w < warp; ++w) pre += s_part[w];
  s_start[tid] = pre + incl - c;
  if (tid == 0) s_start[kRadix] = (Off)a.n;
  __syncthreads();
  uint8_t* out = static_cast<uint8_t*>(a.out);
  const uint8_t xc = (uint8_t)a.xor_c;
  auto digit_at = [&](uint64_t i) {  // largest d with start[d] <= i
    uint32_t lo = 0;
#pragma unroll
    for (uint32_t step = 128; step; step >>= 1)
      if ((uint64_t)s_start[lo + step] <= i) lo += step;
    return lo;
  };
  const uint64_t head = (16 - (reinterpret_cast<uintptr_t>(out) & 15)) & 15;
  const uint64_t h = head < a.n ? head : a.n;
  const uint64_t nvec = (a.n - h) / 16;
  const uint64_t gthreads = (uint64_t)gridDim.x * 256, gtid = (uint64_t)blockIdx.x * 256 + tid;
  for (uint64_t v = gtid; v < nvec; v += gthreads) {
    const uint64_t p = h + v * 16;
    const uint32_t d = digit_at(p);
    if ((uint64_t)s_start[d + 1] >= p + 16) {
      const uint32_t b = (uint32_t)(uint8_t)(d ^ xc) * 0x01010101u;
      *reinterpret_cast<uint4*>(out + p) = make_uint4(b, b, b, b);
    } else {
      for (int e = 0; e < 16; ++e) out[p + e] = (uint8_t)(digit_at(p + e) ^ xc);
    }
  }
  for (uint64_t i = gtid; i < h; i += gthreads) out[i] = (uint8_t)(digit_at(i) ^ xc);
  for (uint64_t i = h + nvec * 16 + gtid; i < a.n; i += gthreads) out[i] = (uint8_t)(digit_at(i) ^ xc);
}

// ---------------------------------------------------------------------------
// 16-bit digits for 16-bit keys-only sorts over all 16 bits (a one-pass
// schedule: equal digits are equal keys, so counting is sorting).
//   hist16_kernel: one 1024-thread CTA per SM counts its share of the keys
//     (16-byte loads, four in flight per thread) into all 65536 bins held as
//     packed 16-bit counters (two bins per shared word, 128 KB).  An add
//     that flips bit 14 of its half moves 0x4000 of the half to the global
//     count, so a counter never carries into its neighbour (see count_vec).
//     At the end one global atomic per nonzero
//     bin and one per nonzero group of 256 bins.  (CUSORT_HIST16_PACKED=0:
//     32-bit counters, CTA pairs splitting the bins, every key read by both
//     CTAs of a pair.)
//   fill16_kernel: each CTA owns one group of 256 consecutive bins (a
//     contiguous output range, a quarter of it per CTA): its start is the sum
//     of the lower groups' totals, the bins' starts a 256-wide scan; it writes
//     every position's key, 8 keys (16 bytes) per store inside a run, warps on
//     contiguous shares.
// ---------------------------------------------------------------------------
constexpr int kBins16 = 65536;
#ifndef CUSORT_HIST16_PACKED
#define CUSORT_HIST16_PACKED 1
#endif
// CTAs that read each key: 1 with packed counters, 2 (a pair) with 32-bit ones
constexpr int kHist16Readers = CUSORT_HIST16_PACKED ? 1 : 2;

template <typename Off>
__global__ void __launch_bounds__(1024, 1) hist16_kernel(const Fill16Args a) {
  extern __shared__ __align__(16) uint32_t s_cnt16[];  // [32768]
  __shared__ uint32_t s_grp[256];
  constexpr bool PACKED = CUSORT_HIST16_PACKED != 0;
  dev::pdl_launch_dependents();
  const uint32_t tid = threadIdx.x, lane = tid & 31u;
  const uint32_t half = PACKED ? 0u : (blockIdx.x & 1u);
  const uint32_t part = PACKED ? blockIdx.x : (blockIdx.x >> 1);
  const uint32_t parts = PACKED ? gridDim.x : (gridDim.x >> 1);
  for (uint32_t i = tid; i < kBins16 / 2; i += 1024) s_cnt16[i] = 0;
  if (tid < 256) s_grp[tid] = 0;
  Off* g = static_cast<Off*>(a.counts);
  Off* gg = static_cast<Off*>(a.groups);
  // packed counters move overflow chunks to the global counts while counting,
  // so those must be zeroed (init kernel) first
  if constexpr (PACKED) dev::pdl_wait();
  __syncthreads();
  const uint16_t* keys = static_cast<const uint16_t*>(a.keys);
  const uint32_t xc = a.xor_c & 0xffffu;
  // m (<= 0x4000) more copies of key k
  auto count_m = [&](uint32_t k, uint32_t m) {
    const uint32_t t = (k ^ xc) & 0xffffu;
    if constexpr (PACKED) {
      const uint32_t sh = (t & 1u) << 4, inc = m << sh;
      const uint32_t old = atomicAdd(s_cnt16 + (t >> 1), inc);
      if ((old ^ (old + inc)) & 0x40004000u) {
        atomicSub(s_cnt16 + (t >> 1), 0x4000u << sh);
        atomicAdd(g + t, (Off)0x4000u);
        atomicAdd(gg + (t >> 8), (Off)0x4000u);
      }
    } else {
      if ((t >> 15) == half) atomicAdd(s_cnt16 + (t & 0x7fffu), m);
    }
  };
  auto count = [&](uint32_t k) { count_m(k, 1u); };
  const uintptr_t addr = reinterpret_cast<uintptr_t>(keys);
  uint64_t head = ((16 - (addr & 15)) & 15) / 2;
  if (head > a.n) head = a.n;
  const uint64_t nvec = (a.n - head) / 8;
  const uint4* vec = reinterpret_cast<const uint4*>(keys + head);
  const uint64_t stride = (uint64_t)parts * 1024;
  auto count_vec = [&](const uint4& x) {
    const uint32_t w[4] = {x.x, x.y, x.z, x.w};
    if constexpr (PACKED) {
      // the 8 adds first (8 atomics in flight), then the 8 tests: an add that
      // flipped bit 14 of its half moves 0x4000 of the half to the global
      // count.  Every such move follows an add that took the half to 0x4000
      // or more, so the half never borrows; and until the move lands the half
      // can take another 0xbfff adds before it would carry into its
      // neighbour -- far more than the 8 per thread that are in flight here
      uint32_t t[8], sh[8], old[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        t[e] = ((e & 1 ? w[e >> 1] >> 16 : w[e >> 1]) ^ xc) & 0xffffu;
        sh[e] = (t[e] & 1u) << 4;
        old[e] = atomicAdd(s_cnt16 + (t[e] >> 1), 1u << sh[e]);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if ((old[e] ^ (old[e] + (1u << sh[e]))) & 0x40004000u) {
          atomicSub(s_cnt16 + (t[e] >> 1), 0x4000u << sh[e]);
          atomicAdd(g + t[e], (Off)0x4000u);
          atomicAdd(gg + (t[e] >> 8), (Off)0x4000u);
        }
      }
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        count(w[e] & 0xffffu);
        count(w[e] >> 16);
      }
    }
  };
  // four independent 16-byte loads in flight per thread (one CTA of 1024
  // threads per SM: with one load each, DRAM latency capped the read rate)
  constexpr int U = 4;
  uint64_t v = (uint64_t)part * 1024 + tid;
  // while every lane of the warp has U vectors left (a warp-uniform test: the
  // loop body uses warp collectives); the rest vector by vector
  for (; (v - lane) + 31 + (U - 1) * stride < nvec; v += U * stride) {
    uint4 x[U];
#pragma unroll
    for (int u = 0; u < U; ++u) x[u] = dev::ld_stream_v4(vec + v + u * stride);
    if constexpr (PACKED) {
      // the warp's 32 x 8U keys all equal (one heavy value): one add for all,
      // instead of 32-way same-address atomics
      const uint32_t ref = __shfl_sync(0xffffffffu, x[0].x & 0xffffu, 0) * 0x10001u;
      uint32_t d = 0;
#pragma unroll
      for (int u = 0; u < U; ++u) d |= (x[u].x ^ ref) | (x[u].y ^ ref) | (x[u].z ^ ref) | (x[u].w ^ ref);
      if (__all_sync(0xffffffffu, d == 0u)) {
        if (lane == 0) count_m(ref & 0xffffu, 32u * 8u * U);
        continue;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) count_vec(x[u]);
  }
  for (; v < nvec; v += stride) count_vec(dev::ld_stream_v4(vec + v));
  if (part == 0) {
    for (uint64_t i = tid; i < head; i += 1024) count(keys[i]);
    for (uint64_t i = head + nvec * 8 + tid; i < a.n; i += 1024) count(keys[i]);
  }
  __syncthreads();
  if constexpr (!PACKED) dev::pdl_wait();  // counts zeroed by the init kernel
  // coalesced flush (a warp's bins share one line); each warp's bins lie in
  // one group of 256, whose total is gathered in shared memory first
  for (uint32_t i = tid; i < kBins16 / 2; i += 1024) {
    const uint32_t c = s_cnt16[i];
    uint32_t w;
    if constexpr (PACKED) {
      const uint32_t lo = c & 0xffffu, hi = c >> 16;
      if (lo) atomicAdd(g + 2 * i, (Off)lo);
      if (hi) atomicAdd(g + 2 * i + 1, (Off)hi);
      w = lo + hi;
    } else {
      if (c) atomicAdd(g + (size_t)half * (kBins16 / 2) + i, (Off)c);
      w = c;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) w += __shfl_xor_sync(0xffffffffu, w, o);
    if (lane == 0 && w) atomicAdd(s_grp + (PACKED ? (i >> 7) : (half * 128 + (i >> 8))), w);
  }
  __syncthreads();
  if (tid < 256 && s_grp[tid]) atomicAdd(gg + tid, (Off)s_grp[tid]);
}

// fill16_kernel: the output is split evenly over the CTAs whatever the key
// distribution (a heavy value is written by every CTA its positions reach,
// not by the one CTA that owns its bin).  A CTA walks its positions in
// windows: a window's bin starts -- 2048 bins from a group boundary -- come
// from a block-wide scan of their counts on top of the group starts (the
// exclusive scan of the 256 group totals); the warps split the window's
// 8-key vectors, lanes on consecutive vectors.
constexpr int kFill16Chunk = 2048;

template <typename Off>
__global__ void __launch_bounds__(256) fill16_kernel(const Fill16Args a) {
  __shared__ Off s_gstart[kRadix + 1];
  __shared__ Off s_bs[kFill16Chunk + 1];
  __shared__ Off s_wsum[8];
  __shared__ unsigned long long s_w[2];
  dev::pdl_wait();  // counts from hist16_kernel
  const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
  const Off* counts = static_cast<const Off*>(a.counts);
  auto block_excl_scan = [&](Off v, Off* total) {  // all 256 threads
    Off incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const Off t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= (uint32_t)o) incl += t;
    }
    if (lane == 31) s_wsum[warp] = incl;
    __syncthreads();
    Off pre = 0, all = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      pre += (w < (int)warp) ? s_wsum[w] : Off(0);
      all += s_wsum[w];
    }
    __syncthreads();  // s_wsum is reused by the next scan
    *total = all;
    return pre + incl - v;
  };
  {
    Off total;
    const Off g = static_cast<const Off*>(a.groups)[tid];
    s_gstart[tid] = block_excl_scan(g, &total);
    if (tid == 0) s_gstart[kRadix] = total;
    __syncthreads();
  }
  uint16_t* out = static_cast<uint16_t*>(a.out);
  const uint32_t xc = a.xor_c & 0xffffu;
  auto key_of = [&](uint32_t bin) { return (uint16_t)(bin ^ xc); };
  auto group_of = [&](uint64_t p) {  // largest g with s_gstart[g] <= p (p < n)
    uint32_t g = 0;
#pragma unroll
    for (uint32_t step = 128; step; step >>= 1)
      if ((uint64_t)s_gstart[g + step] <= p) g += step;
    return g;
  };
  // bin of position p, the whole warp with the same p: the group's 256
  // counts, 8 per lane, scanned across the lanes
  auto bin_of = [&](uint64_t p) -> uint32_t {
    const uint32_t g = group_of(p);
    Off c[8], sum = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      c[i] = counts[(size_t)g * kRadix + lane * 8 + i];
      sum += c[i];
    }
    Off incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const Off t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= (uint32_t)o) incl += t;
    }
    const uint64_t lo = (uint64_t)s_gstart[g] + (uint64_t)(incl - sum);
    const bool mine = lo <= p && p < lo + (uint64_t)sum;
    uint32_t e = 0;
    if (mine) {
      uint64_t at = lo;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (at <= p && p < at + (uint64_t)c[i]) e = (uint32_t)i;
        at += (uint64_t)c[i];
      }
    }
    const uint32_t who = __ffs(__ballot_sync(0xffffffffu, mine)) - 1;
    return g * kRadix + who * 8 + __shfl_sync(0xffffffffu, e, who);
  };
  const uint64_t n = a.n;
  const uint64_t mis = (reinterpret_cast<uintptr_t>(out) & 15) / 2;
  const uint64_t h = min(n, mis ? 8 - mis : (uint64_t)0);
  const uint64_t nvec = (n - h) / 8, tail0 = h + nvec * 8;
  // unaligned head (first CTA) and ragged tail (last CTA), element by element
  if (warp == 0 && blockIdx.x == 0)
    for (uint64_t i = 0; i < h; ++i) {
      const uint32_t b = bin_of(i);
      if (lane == 0) out[i] = key_of(b);
    }
  if (warp == 0 && blockIdx.x == gridDim.x - 1)
    for (uint64_t i = tail0; i < n; ++i) {
      const uint32_t b = bin_of(i);
      if (lane == 0) out[i] = key_of(b);
    }
  const uint64_t p0 = h + 8 * (nvec * blockIdx.x / gridDim.x);
  const uint64_t p1 = h + 8 * (nvec * (blockIdx.x + 1) / gridDim.x);
  uint64_t w0 = p0;
  while (w0 < p1) {
    // window: the chunk of bins from the group of w0's bin
    if (warp == 0) {
      const uint32_t b = bin_of(w0);
      if (lane == 0) s_w[0] = b & ~(uint32_t)(kRadix - 1);
    }
    __syncthreads();
    const uint32_t cb = (uint32_t)s_w[0];
    Off c[8], sum = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t bin = cb + tid * 8 + i;
      c[i] = bin < (uint32_t)kBins16 ? counts[bin] : Off(0);
      sum += c[i];
    }
    Off total;
    Off at = s_gstart[cb / kRadix] + block_excl_scan(sum, &total);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      s_bs[tid * 8 + i] = at;
      at += c[i];
    }
    if (tid == 0) s_bs[kFill16Chunk] = s_gstart[cb / kRadix] + total;
    __syncthreads();
    // vectors wholly inside the chunk's positions
    uint64_t w1 = min(p1, (uint64_t)s_bs[kFill16Chunk]);
    w1 = w1 > h ? h + (w1 - h) / 8 * 8 : h;
    if (w1 <= w0) {
      // one vector reaches past the chunk (empty bins between its keys): by element
      if (warp == 0)
        for (int e = 0; e < 8; ++e) {
          const uint32_t b = bin_of(w0 + e);
          if (lane == 0) out[w0 + e] = key_of(b);
        }
      w0 += 8;
      __syncthreads();  // s_w, s_bs reused
      continue;
    }
    const uint64_t nv = (w1 - w0) / 8;
    const uint64_t per = (nv + 7) / 8, u0 = min(nv, per * warp), u1 = min(nv, u0 + per);
    uint32_t b = 0;
    bool found = false;
    for (uint64_t v = u0 + lane; v < u1; v += 32) {
      const uint64_t p = w0 + v * 8;
      if (!found) {  // largest local bin with start <= p
        uint32_t lo = 0;
#pragma unroll
        for (uint32_t step = kFill16Chunk / 2; step; step >>= 1)
          if ((uint64_t)s_bs[lo + step] <= p) lo += step;
        b = lo;
        found = true;
      }
      while ((uint64_t)s_bs[b + 1] <= p) ++b;
      if ((uint64_t)s_bs[b + 1] >= p + 8) {
        const uint32_t k2 = (uint32_t)key_of(cb + b) * 0x10001u;
        *reinterpret_cast<uint4*>(out + p) = make_uint4(k2, k2, k2, k2);
      } else {
        uint32_t bb = b;
        uint32_t k[4];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          while ((uint64_t)s_bs[bb + 1] <= p + e) ++bb;
          const uint32_t ke = key_of(cb + bb);
          if (e & 1) k[e >> 1] |= ke << 16;
          else k[e >> 1] = ke;
        }
        *reinterpret_cast<uint4*>(out + p) = make_uint4(k[0], k[1], k[2], k[3]);
      }
    }
    w0 = w1;
    __syncthreads();  // s_w, s_bs reused
  }
}

// ---------------------------------------------------------------------------
// onesweep: one stable LSD pass over digit (shift, mask).
//
// Persistent CTAs take tiles from a global ticket counter (so the lookback
// only ever waits on tiles that a running CTA already owns).  Per tile:
//   1. TMA bulk copy of the tile's keys (and values) into shared memory
//      (cooperative loads for the ragged last tile or unaligned pointers);
//   2. each warp ranks its 32*KPT keys slot by slot with the shared-memory
//      match (dev::warp_rank_slot), keys/values held in registers;
//   3. per-digit counts -> aggregate descriptor published at once; tile-local
//      exclusive digit offsets by a 256-wide block scan;
//   4. keys/values are written back to shared memory in sorted order;
//   5. decoupled lookback over earlier tiles' descriptors (bounded wait), the
//      inclusive descriptor is published;
//   6. coalesced global scatter: consecutive threads write consecutive
//      positions of each digit run.
// Out-of-range slots of the last tile take the top digit and are never
// written (their sorted positions are >= the tile's valid count).
// ---------------------------------------------------------------------------
// Warp ranking variants (see WarpCounters): 0 = shared-memory match,
// 1 = ballot match with 16-bit per-warp counters, 2 = hybrid ballot/shared
// match, 3 = hybrid with rotating tables and no branches, 4 = mode 3 after a
// counting pre-pass (early aggregate publish, ranks are final positions).
#ifndef CUSORT_RANK_MODE
#define CUSORT_RANK_MODE -1  // per key/value width, see OnesweepCfg::RANK_MODE
#endif

template <int MODE>
struct WarpCounters;

// Shared-memory match (dev::warp_rank_slot): one 64-bit [count | lane mask]
// word per (warp, digit).
template <>
struct WarpCounters<0> {
  using Word = unsigned long long;
  static constexpr size_t BYTES_PER_WARP = kRadix * 8;
  __device__ __forceinline__ static void zero(uint8_t* tab, uint32_t warp, uint32_t lane) {
    Word* w = reinterpret_cast<Word*>(tab) + warp * kRadix;
#pragma unroll
    for (int i = 0; i < kRadix / 32; ++i) w[lane + 32 * i] = 0ull;
  }
  __device__ __forceinline__ static uint32_t rank(uint8_t* tab, uint32_t warp, uint32_t d, uint32_t lane,
                                                  uint32_t lt) {
    return dev::warp_rank_slot(reinterpret_cast<Word*>(tab) + warp * kRadix, d, lane, lt);
  }
  __device__ __forceinline__ static uint32_t count(const uint8_t* tab, uint32_t w, uint32_t t) {
    return (uint32_t)(reinterpret_cast<const Word*>(tab)[w * kRadix + t] >> 32);
  }
  __device__ __forceinline__ static uint32_t get(const uint8_t* tab, uint32_t w, uint32_t t) {
    return (uint32_t)reinterpret_cast<const Word*>(tab)[w * kRadix + t];
  }
  __device__ __forceinline__ static void put(uint8_t* tab, uint32_t w, uint32_t t, uint32_t v) {
    reinterpret_cast<Word*>(tab)[w * kRadix + t] = v;
  }
};

// Ballot match (8 vote.ballot per slot, no shared-memory traffic) plus one
// 16-bit counter per (warp, digit): the highest peer lane adds the group size
// with a 32-bit shared atomic on the word holding two counters and shuffles
// the previous count to its peers.
template <>
struct WarpCounters<1> {
  static constexpr size_t BYTES_PER_WARP = kRadix * 2;
  __device__ __forceinline__ static void zero(uint8_t* tab, uint32_t warp, uint32_t lane) {
    uint32_t* w = reinterpret_cast<uint32_t*>(tab) + warp * (kRadix / 2);
#pragma unroll
    for (int i = 0; i < kRadix / 64; ++i) w[lane + 32 * i] = 0u;
  }
  __device__ __forceinline__ static uint32_t rank(uint8_t* tab, uint32_t warp, uint32_t d, uint32_t lane,
                                                  uint32_t lt) {
    uint32_t* w = reinterpret_cast<uint32_t*>(tab) + warp * (kRadix / 2);
    const uint32_t peers = dev::match_digit_ballot<8>(d);
    const uint32_t below = __popc(peers & lt);
    const uint32_t leader = 31u - __clz(peers);
    const uint32_t sh = (d & 1u) << 4;
    uint32_t old = 0;
    if (lane == leader) old = atomicAdd(w + (d >> 1), (below + 1u) << sh);
    old = __shfl_sync(0xffffffffu, old, leader);
    return ((old >> sh) & 0xffffu) + below;
  }
  __device__ __forceinline__ static uint32_t count(const uint8_t* tab, uint32_t w, uint32_t t) {
    return reinterpret_cast<const uint16_t*>(tab)[w * kRadix + t];
  }
  __device__ __forceinline__ static uint32_t get(const uint8_t* tab, uint32_t w, uint32_t t) {
    return reinterpret_cast<const uint16_t*>(tab)[w * kRadix + t];
  }
  __device__ __forceinline__ static void put(uint8_t* tab, uint32_t w, uint32_t t, uint32_t v) {
    reinterpret_cast<uint16_t*>(tab)[w * kRadix + t] = (uint16_t)v;
  }
};

// Hybrid: the low 2 digit bits by ballot, the high 6 bits by a shared-memory
// match on a 64-word per-warp table (two bank rows, so far fewer bank
// conflicts than a 256-entry table), then the 16-bit counters of mode 1.
template <>
struct WarpCounters<2> {
  static constexpr size_t MASK_WORDS = 64;
  static constexpr size_t BYTES_PER_WARP = kRadix * 2 + MASK_WORDS * 4;
  __device__ __forceinline__ static uint32_t* masks(uint8_t* tab, uint32_t warp) {
    return reinterpret_cast<uint32_t*>(tab + (size_t)warp * BYTES_PER_WARP + kRadix * 2);
  }
  __device__ __forceinline__ static void zero(uint8_t* tab, uint32_t warp, uint32_t lane) {
    uint32_t* w = reinterpret_cast<uint32_t*>(tab + (size_t)warp * BYTES_PER_WARP);
#pragma unroll
    for (int i = 0; i < (int)(BYTES_PER_WARP / 4 / 32); ++i) w[lane + 32 * i] = 0u;
  }
  __device__ __forceinline__ static uint32_t rank(uint8_t* tab, uint32_t warp, uint32_t d, uint32_t lane,
                                                  uint32_t lt) {
    uint32_t* cnt = reinterpret_cast<uint32_t*>(tab + (size_t)warp * BYTES_PER_WARP);
    uint32_t* msk = masks(tab, warp);
    const uint32_t hi = d >> 2;
    atomicOr(msk + hi, 1u << lane);
    const uint32_t pl = dev::match_digit_ballot<2>(d);
    __syncwarp();
    const uint32_t ph = msk[hi];
    __syncwarp();
    if ((ph >> lane) == 1u) msk[hi] = 0u;
    const uint32_t peers = pl & ph;
    const uint32_t below = __popc(peers & lt);
    const uint32_t leader = 31u - __clz(peers);
    const uint32_t sh = (d & 1u) << 4;
    uint32_t old = 0;
    if (lane == leader) old = atomicAdd(cnt + (d >> 1), (below + 1u) << sh);
    old = __shfl_sync(0xffffffffu, old, leader);
    __syncwarp();
    return ((old >> sh) & 0xffffu) + below;
  }
  __device__ __forceinline__ static uint32_t count(const uint8_t* tab, uint32_t w, uint32_t t) {
    return reinterpret_cast<const uint16_t*>(tab + (size_t)w * BYTES_PER_WARP)[t];
  }
  __device__ __forceinline__ static uint32_t get(const uint8_t* tab, uint32_t w, uint32_t t) {
    return reinterpret_cast<const uint16_t*>(tab + (size_t)w * BYTES_PER_WARP)[t];
  }
  __device__ __forceinline__ static void put(uint8_t* tab, uint32_t w, uint32_t t, uint32_t v) {
    reinterpret_cast<uint16_t*>(tab + (size_t)w * BYTES_PER_WARP)[t] = (uint16_t)v;
  }
};

// Mode 3: the hybrid of mode 2 with three mask tables used in rotation, so a
// slot clears the table of the slot before it and one warp barrier per slot
// suffices; the clears are unconditional stores and the counter update is a
// predicated atomic (no branches).  rank() takes the slot index and carries the
// previous slot's table word index per lane.
template <>
struct WarpCounters<3> {
  static constexpr int NT = 3;
  static constexpr size_t MASK_WORDS = 64;
  static constexpr size_t BYTES_PER_WARP = kRadix * 2 + NT * MASK_WORDS * 4;
  __device__ __forceinline__ static void zero(uint8_t* tab, uint32_t warp, uint32_t lane) {
    uint32_t* w = reinterpret_cast<uint32_t*>(tab + (size_t)warp * BYTES_PER_WARP);
#pragma unroll
    for (int i = 0; i < (int)(BYTES_PER_WARP / 4 / 32); ++i) w[lane + 32 * i] = 0u;
  }
  template <int S>
  __device__ __forceinline__ static uint32_t rank_slot(uint8_t* tab, uint32_t warp, uint32_t d, uint32_t lane,
                                                       uint32_t lt, uint32_t& prev_word) {
    uint32_t* base = reinterpret_cast<uint32_t*>(tab + (size_t)warp * BYTES_PER_WARP);
    uint32_t* cnt = base;
    uint32_t* msk = base + kRadix / 2;
    const uint32_t word = (uint32_t)(S % NT) * MASK_WORDS + (d >> 2);
    atomicOr(msk + word, 1u << lane);
    const uint32_t pl = dev::match_digit_ballot<2>(d);
    __syncwarp();
    const uint32_t ph = msk[word];
    if (S > 0) msk[prev_word] = 0u;  // previous slot's table: read by all lanes before the barrier above
    prev_word = word;
    const uint32_t peers = pl & ph;
    const uint32_t below = __popc(peers & lt);
    const uint32_t leader = 31u - __clz(peers);
    const uint32_t sh = (d & 1u) << 4;
    uint32_t old = dev::atom_add_shared_if(lane == leader, cnt + (d >> 1), (below + 1u) << sh, 0u);
    old = __shfl_sync(0xffffffffu, old, leader);
    return ((old >> sh) & 0xffffu) + below;
  }
  __device__ __forceinline__ static uint32_t count(const uint8_t* tab, uint32_t w, uint32_t t) {
    return reinterpret_cast<const uint16_t*>(tab + (size_t)w * BYTES_PER_WARP)[t];
  }
  __device__ __forceinline__ static uint32_t get(const uint8_t* tab, uint32_t w, uint32_t t) {
    return reinterpret_cast<const uint16_t*>(tab + (size_t)w * BYTES_PER_WARP)[t];
  }
  __device__ __forceinline__ static void put(uint8_t* tab, uint32_t w, uint32_t t, uint32_t v) {
    reinterpret_cast<uint16_t*>(tab + (size_t)w * BYTES_PER_WARP)[t] = (uint16_t)v;
  }
};

// Mode 4: per-warp digit counts are taken first (one shared atomic per key on
// the 16-bit counters), so the tile's aggregate can be published before the
// expensive ranking; the counters are then turned into each warp's final tile
// positions and the ranking atomics of mode 3 return positions directly.
template <>
struct WarpCounters<4> : WarpCounters<3> {
  __device__ __forceinline__ static void count_key(uint8_t* tab, uint32_t warp, uint32_t d) {
    uint32_t* cnt = reinterpret_cast<uint32_t*>(tab + (size_t)warp * BYTES_PER_WARP);
    atomicAdd(cnt + (d >> 1), 1u << ((d & 1u) << 4));
  }
};

// Mode 5: mode 4's counting pre-pass and position counters with the peer set
// found by 8 ballots (ALU only, no shared-memory match table).
template <>
struct WarpCounters<5> : WarpCounters<1> {
  __device__ __forceinline__ static void count_key(uint8_t* tab, uint32_t warp, uint32_t d) {
    uint32_t* cnt = reinterpret_cast<uint32_t*>(tab) + warp * (kRadix / 2);
    atomicAdd(cnt + (d >> 1), 1u << ((d & 1u) << 4));
  }
  template <int S>
  __device__ __forceinline__ static uint32_t rank_slot(uint8_t* tab, uint32_t warp, uint32_t d, uint32_t lane,
                                                       uint32_t lt, uint32_t&) {
    uint32_t* cnt = reinterpret_cast<uint32_t*>(tab) + warp * (kRadix / 2);
    const uint32_t peers = dev::match_digit_ballot<8>(d);
    const uint32_t below = __popc(peers & lt);
    const uint32_t leader = 31u - __clz(peers);
    const uint32_t sh = (d & 1u) << 4;
    uint32_t old = dev::atom_add_shared_if(lane == leader, cnt + (d >> 1), (below + 1u) << sh, 0u);
    old = __shfl_sync(0xffffffffu, old, leader);
    return ((old >> sh) & 0xffffu) + below;
  }
};

// Modes 6-8: mode 4 with one 32-bit counter per (warp, digit) instead of
// two 16-bit counters per word: the counting and position atomics add 1 or
// the group size to the digit's own word (no shift or mask arithmetic per
// key, and two different digits never share an atomic's address), at 1 KB
// instead of 512 B of counters per warp.  BB of the digit's bits are matched
// by ballot and the other 8 - BB by the shared-memory table of 2^(8-BB)
// words (mode 6: BB = 2, mode 7: BB = 1, mode 8: BB = 3).
template <int BB>
struct WarpCounters32 {
  static constexpr int NT = 3;
  static constexpr size_t MASK_WORDS = (size_t)kRadix >> BB;
  static constexpr size_t BYTES_PER_WARP = kRadix * 4 + NT * MASK_WORDS * 4;
  static_assert(BYTES_PER_WARP % 16 == 0, "16-byte zeroing");
  __device__ __forceinline__ static void zero(uint8_t* tab, uint32_t warp, uint32_t lane) {
    uint4* w = reinterpret_cast<uint4*>(tab + (size_t)warp * BYTES_PER_WARP);
    constexpr int V = (int)(BYTES_PER_WARP / 16);
#pragma unroll
    for (int i = 0; i < (V + 31) / 32; ++i)
      if (i * 32 + (int)lane < V) w[lane + 32 * i] = make_uint4(0u, 0u, 0u, 0u);
  }
  __device__ __forceinline__ static void count_key(uint8_t* tab, uint32_t warp, uint32_t d) {
    atomicAdd(reinterpret_cast<uint32_t*>(tab + (size_t)warp * BYTES_PER_WARP) + d, 1u);
  }
  template <int S>
  __device__ __forceinline__ static uint32_t rank_slot(uint8_t* tab, uint32_t warp, uint32_t d, uint32_t lane,
                                                       uint32_t lt, uint32_t& prev_word) {
    uint32_t* base = reinterpret_cast<uint32_t*>(tab + (size_t)warp * BYTES_PER_WARP);
    uint32_t* cnt = base;
    uint32_t* msk = base + kRadix;
    const uint32_t word = (uint32_t)(S % NT) * MASK_WORDS + (d >> BB);
    atomicOr(msk + word, 1u << lane);
    const uint32_t pl = dev::match_digit_ballot<BB>(d);
    __syncwarp();
    const uint32_t ph = msk[word];
    if (S > 0) msk[prev_word] = 0u;  // previous slot's table: read by all lanes before the barrier above
    prev_word = word;
    const uint32_t peers = pl & ph;
    const uint32_t below = __popc(peers & lt);
    const uint32_t leader = 31u - __clz(peers);
    uint32_t old = dev::atom_add_shared_if(lane == leader, cnt + d, below + 1u, 0u);
    old = __shfl_sync(0xffffffffu, old, leader);
    return old + below;
  }
  __device__ __forceinline__ static uint32_t count(const uint8_t* tab, uint32_t w, uint32_t t) {
    return reinterpret_cast<const uint32_t*>(tab + (size_t)w * BYTES_PER_WARP)[t];
  }
  __device__ __forceinline__ static uint32_t get(const uint8_t* tab, uint32_t w, uint32_t t) {
    return reinterpret_cast<const uint32_t*>(tab + (size_t)w * BYTES_PER_WARP)[t];
  }
  __device__ __forceinline__ static void put(uint8_t* tab, uint32_t w, uint32_t t, uint32_t v) {
    reinterpret_cast<uint32_t*>(tab + (size_t)w * BYTES_PER_WARP)[t] = v;
  }
};
template <>
struct WarpCounters<6> : WarpCounters32<2> {};

template <>
struct WarpCounters<7> : WarpCounters32<1> {};
template <>
struct WarpCounters<8> : WarpCounters32<3> {};

template <int S, int N, class F>
__device__ __forceinline__ void static_for(F&& f) {
  if constexpr (S < N) {
    f(std::integral_constant<int, S>{});
    static_for<S + 1, N>(f);
  }
}

template <int MODE, int S>
struct RankStep {
  __device__ __forceinline__ static uint32_t run(uint8_t* tab, uint32_t warp, uint32_t d, uint32_t lane, uint32_t lt,
                                                 uint32_t& prev) {
    if constexpr (MODE == 3) return WarpCounters<3>::rank_slot<S>(tab, warp, d, lane, lt, prev);
    else return WarpCounters<MODE>::rank(tab, warp, d, lane, lt);
  }
};

// Unrolled slot loop with the slot index as a compile-time constant.
template <int MODE, int S, int KPT>
struct RankSlots {
  __device__ __forceinline__ static void run(uint8_t* tab, uint32_t warp, uint32_t* dr, uint32_t lane, uint32_t lt,
                                             uint32_t& prev) {
    if constexpr (S < KPT) {
      const uint32_t r = RankStep<MODE, S>::run(tab, warp, dr[S], lane, lt, prev);
      dr[S] |= r << 8;
      RankSlots<MODE, S + 1, KPT>::run(tab, warp, dr, lane, lt, prev);
    }
  }
};

// Tile input path: 1 = streaming loads straight into registers, 0 = TMA bulk
// copy into shared memory first (default: with the large tiles TMA staging
// is as fast or faster for every width measured), -1 = direct loads for
// 4-byte keys-only only.
#ifndef CUSORT_DIRECT_LOAD
#define CUSORT_DIRECT_LOAD 0
#endif

// Tile prefetch: 1 = take the next tile's ticket one tile ahead and TMA-load
// it into a second buffer while the current tile is processed.  Off by
// default: on B200 the early tickets delay those tiles' descriptors and the
// longer lookback waits cost more than the hidden load latency (u32 keys
// 0.306 -> 0.335 ms per pass at 2^26).
#ifndef CUSORT_PREFETCH
#define CUSORT_PREFETCH 0
#endif

// Bank swizzle of the sorted tile in shared memory: sorted position p lives
// at p ^ ((p >> 5) & 31), a permutation inside each aligned block of 32, so
// 32 consecutive positions (the scatter's reads) stay conflict-free while
// positions 32k apart -- the same rank in digit runs of equal length, which
// a slot of sorted or evenly spread keys writes at once -- fall into
// different banks instead of one.  1 = on.
#ifndef CUSORT_TILE_SWIZZLE
#define CUSORT_TILE_SWIZZLE 1
#endif
// Full tiles whose keys all share one digit skip the ranking and go out in
// input order (the reference's per-tile short-circuit): 1 = on.
#ifndef CUSORT_ONE_DIGIT_TILES
#define CUSORT_ONE_DIGIT_TILES 1
#endif
// Full tiles whose digits never decrease in input order (sorted input, runs
// of equal keys) are already in stable digit order: they skip the ranking
// too.  The whole-tile check runs only when every warp's first and last
// slots are non-decreasing across their lanes (a few instructions per warp
// and tile).  1 = on.
#ifndef CUSORT_SORTED_TILES
#define CUSORT_SORTED_TILES 1
#endif
// this warp's 32 values non-decreasing from lane 0 to lane 31
__device__ __forceinline__ bool warp_nondecreasing(uint32_t d, uint32_t lane) {
  const uint32_t p = __shfl_up_sync(0xffffffffu, d, 1);
  return __ballot_sync(0xffffffffu, lane != 0u && p > d) == 0u;
}
__device__ __forceinline__ uint32_t tile_swz(uint32_t p) {
  return CUSORT_TILE_SWIZZLE ? p ^ ((p >> 5) & 31u) : p;
}
// tile_swz(tid + i * THREADS) for the scatter's i-th item of thread tid
template <int THREADS>
__device__ __forceinline__ uint32_t tile_swz_at(uint32_t tid, uint32_t i) {
  if constexpr (CUSORT_TILE_SWIZZLE && THREADS == 512) {
    // (p >> 5) & 31 = warp + 16 (i & 1) with 16 warps: only the lane bits change
    return (tid ^ (tid >> 5) ^ ((i & 1u) << 4)) + i * THREADS;
  } else {
    return tile_swz(tid + i * THREADS);
  }
}

// Rank mode per key/value width (measured on B200, see OnesweepCfg).
#ifndef CUSORT_KEYS_RANK_MODE
#define CUSORT_KEYS_RANK_MODE 6
#endif
#ifndef CUSORT_OTHER_RANK_MODE
#define CUSORT_OTHER_RANK_MODE 6
#endif
#define CUSORT_RANK_MODE_OF(KB, VB) \
  (CUSORT_RANK_MODE >= 0 ? CUSORT_RANK_MODE                   \
                         : (((VB) == 0 && (KB) <= 4) ? CUSORT_KEYS_RANK_MODE : CUSORT_OTHER_RANK_MODE))

template <int KB_, int VB_, typename Off_, int THREADS_, int KPT_, int MINB_, bool FLOAT_KEY_, bool ROUTED_ = false,
          bool SEG_ = false>
struct OnesweepCfg {
  static constexpr int KB = KB_, VB = VB_, THREADS = THREADS_, KPT = KPT_, MINB = MINB_;
  static constexpr bool FLOAT_KEY = FLOAT_KEY_;
  // Routed pass (multi-GPU partition): digit bases and destinations come from
  // a RouteTable, stores may target peers' memory.
  static constexpr bool ROUTED = ROUTED_;
  // Segmented pass: tiles of multi-tile segments (SegOnesweepArgs).
  static constexpr bool SEG = SEG_;
  static_assert(!(ROUTED && SEG), "one special mode at a time");
  using Args = typename std::conditional<SEG, SegOnesweepArgs, OnesweepArgs>::type;
  using Off = Off_;
  static constexpr int WARPS = THREADS / 32;
  static constexpr int TILE = THREADS * KPT;
  // One staging buffer = the tile's keys + values.  Two buffers when they fit
  // in this CTA's share of shared memory: the next tile is then loaded by TMA
  // while the current one is processed.
  static constexpr size_t KEYS_BYTES = align_up((size_t)TILE * KB, 128);
  static constexpr size_t BUF_BYTES = KEYS_BYTES + align_up((size_t)TILE * VB, 128);
  static constexpr size_t SMEM_PER_CTA = (227 * 1024) / MINB - 1024;
  static constexpr bool PREFETCH = CUSORT_PREFETCH != 0;
  static constexpr bool DIRECT_LOAD = CUSORT_DIRECT_LOAD >= 0 ? (CUSORT_DIRECT_LOAD == 1) : (VB_ == 0 && KB_ <= 4);
  // 4-byte keys with 4-byte values move through shared memory as one 8-byte
  // item (one 64-bit store when scattering, one 64-bit load when writing out).
  static constexpr bool PACKED_KV = (KB_ == 4 && VB_ == 4);
  // Keys of up to 4 bytes with 1- or 2-byte values: the values stay in shared
  // memory (copied from the staged tile straight to their sorted position in
  // a second buffer), which frees KPT registers for larger tiles.
#ifndef CUSORT_VSMEM
#define CUSORT_VSMEM 1
#endif
#ifndef CUSORT_VSMEM_MAXKB
#define CUSORT_VSMEM_MAXKB 4
#endif
  static constexpr bool VSMEM = CUSORT_VSMEM && VB_ > 0 && VB_ <= 2 && KB_ <= CUSORT_VSMEM_MAXKB;
  // Pipelined register loads (onesweep_pipe_kernel): the next tile's keys and
  // values are loaded from global memory straight into registers while the
  // current tile is scattered out of shared memory; no staging copy.
// Measured on B200 at 2^26 items (onesweep launch, 32-bit counters): 4-byte
// keys-only 239 -> 230 us, int32 + uint32 pairs 342 -> 341 us (at 32 and 16
// items per thread), float keys 259 -> 240 us; the next tile's aggregate is
// published later, which the lookback timer sees (about 4 descriptor-window
// rounds per tile instead of 3.6).  Other key widths keep the staged kernel.
#ifndef CUSORT_PIPE
#define CUSORT_PIPE 1
#endif
#ifndef CUSORT_PIPE_MAXKB
#define CUSORT_PIPE_MAXKB 4
#endif
#ifndef CUSORT_PIPE_MINKB
#define CUSORT_PIPE_MINKB 4
#endif
#ifndef CUSORT_PIPE_MAXVB
#define CUSORT_PIPE_MAXVB 4
#endif
// 64-bit offsets (2^30 items and more) keep the staged kernel: with 64-bit
// descriptor words the lookback window is half as wide, and the pipelined
// kernel's smaller tiles mean more tiles to look back over.  Measured on B200
// (ms per sort, pipelined -> staged): 2^30 int32+uint32 pairs 23.5 -> 21.7,
// 2^30 int32 keys 15.5 -> 14.5, 2^31 pairs 46.9 -> 43.3.
#ifndef CUSORT_PIPE_WIDE_OFFSETS
#define CUSORT_PIPE_WIDE_OFFSETS 0
#endif
  static constexpr bool PIPE_OK = CUSORT_PIPE && !ROUTED_ && !SEG_ && !VSMEM && !(CUSORT_PREFETCH != 0) &&
                                  KB_ <= CUSORT_PIPE_MAXKB && KB_ >= CUSORT_PIPE_MINKB && VB_ <= CUSORT_PIPE_MAXVB &&
                                  (sizeof(Off_) == 4 || CUSORT_PIPE_WIDE_OFFSETS);
  // Routed passes' tables (layout below).
  static constexpr size_t ROUTE_LAYOUT_BYTES =
      ROUTED ? (kRadix + 4 * 8 * kMaxRouteRanks + 8 * (kRadix + 8) + 2 * 4 * kMaxRouteRanks + 2 * 8 * kRadix) : 0;
  // Everything but the per-warp tables (one staging buffer).
  static constexpr size_t NON_WTAB_BYTES = BUF_BYTES + 16 + kRadix * 4 + 2 * kRadix * sizeof(Off) + 16 * 4 + 32 +
                                           (VSMEM ? align_up((size_t)TILE * VB, 16) : 0) + ROUTE_LAYOUT_BYTES;
  // Rank mode (WarpCounters): the preferred one for the key/value width --
  // measured on B200 at 2^26 items, the 32-bit counters of mode 6 beat the
  // packed 16-bit counters of mode 4 for every 4-byte-key shape (2-5 % on
  // uniform keys, 18-26 % on skewed ones) -- unless its larger tables would
  // push the CTA past its share of shared memory (MINB CTAs per SM), where
  // mode 4 keeps the tile shape's occupancy.
  static constexpr int PREF_RANK_MODE = CUSORT_RANK_MODE_OF(KB_, VB_);
  static constexpr int RANK_MODE =
      (PREF_RANK_MODE >= 6 && NON_WTAB_BYTES + (size_t)WARPS * WarpCounters<(PREF_RANK_MODE >= 6 ? PREF_RANK_MODE : 6)>::BYTES_PER_WARP >
                                  SMEM_PER_CTA)
          ? 4
          : PREF_RANK_MODE;
  using WC = WarpCounters<RANK_MODE>;
  static constexpr size_t REST_BYTES = align_up((size_t)WARPS * WC::BYTES_PER_WARP, 16) + kRadix * 4 +
                                       2 * kRadix * sizeof(Off) + 16 * 4 + 32;
  // Mode 4 needs a key's digit twice (count, rank); recomputing it from the
  // key instead of keeping a digit array frees KPT registers, which buys
  // larger tiles (2 = every width, 1 = keys-only, 0 = never).
#ifndef CUSORT_RECOMPUTE_DIGIT
#define CUSORT_RECOMPUTE_DIGIT 2
#endif
  static constexpr bool RECOMPUTE_DIGIT =
      RANK_MODE >= 4 && (CUSORT_RECOMPUTE_DIGIT == 2 || (CUSORT_RECOMPUTE_DIGIT == 1 && VB_ == 0));
  static constexpr bool PIPE = PIPE_OK && RANK_MODE >= 4;
  static constexpr int NBUF = (PREFETCH && 2 * BUF_BYTES + REST_BYTES <= SMEM_PER_CTA) ? 2 : 1;
  static constexpr size_t OFF_WTAB = NBUF * BUF_BYTES;
  static constexpr size_t OFF_TSTART = align_up(OFF_WTAB + (size_t)WARPS * WC::BYTES_PER_WARP, 16);
  static constexpr size_t OFF_GBASE = OFF_TSTART + kRadix * 4;
  static constexpr size_t OFF_GOFF = OFF_GBASE + kRadix * sizeof(Off);
  static constexpr size_t OFF_MISC = OFF_GOFF + kRadix * sizeof(Off);
  static constexpr size_t OFF_MBAR = OFF_MISC + 16 * 4;
  // routed: owner[256] (u8); kptr/vptr/cap/base[kMaxRouteRanks] (u64); the
  // tile's digit prefix of earlier tiles' counts pre[256] + 8 warp totals
  // (u64); each owner's first and last digit [2][kMaxRouteRanks] (u32); per
  // digit the tile's destination addresses dk/dv[256] (u64)
  static constexpr size_t OFF_VOUT = align_up(OFF_MBAR + 2 * 8, 16);  // VSMEM: sorted values
  static constexpr size_t VOUT_BYTES = VSMEM ? align_up((size_t)TILE * VB, 16) : 0;
  static constexpr size_t OFF_ROUTE = OFF_VOUT + VOUT_BYTES;
  static constexpr size_t OFF_RPTR = OFF_ROUTE + kRadix;
  static constexpr size_t OFF_RPRE = OFF_RPTR + 4 * 8 * kMaxRouteRanks;
  static constexpr size_t OFF_RFIRST = OFF_RPRE + 8 * (kRadix + 8);
  static constexpr size_t OFF_RDST = OFF_RFIRST + 2 * 4 * kMaxRouteRanks;
  static constexpr size_t ROUTE_BYTES = ROUTED ? (OFF_RDST + 2 * 8 * kRadix - OFF_ROUTE) : 0;
  static_assert(ROUTE_BYTES == ROUTE_LAYOUT_BYTES, "routed table layout");
  static_assert(!(ROUTED && PREFETCH), "routed passes take tickets one tile at a time");
  static constexpr size_t SMEM_BYTES = OFF_ROUTE + ROUTE_BYTES;
  static_assert(THREADS >= kRadix && THREADS % 32 == 0, "need >= 256 threads");
  static_assert(TILE * (KB + VB) < (1 << 20), "mbarrier tx-count limit");
  static_assert(32 * KPT < (1 << 24), "rank packing");
  static_assert(TILE <= 65536, "16-bit tile positions");
};

// Predecessor words read per lookback round trip: 8 with 32-bit words; 4 with
// 64-bit words (n >= 2^30), where 8 would make the pass spill registers.
#ifndef CUSORT_LOOKBACK_WINDOW
#define CUSORT_LOOKBACK_WINDOW 8
#endif
template <typename Off>
constexpr int lookback_window() {
  return sizeof(Off) == 8 ? CUSORT_LOOKBACK_WINDOW / 2 : CUSORT_LOOKBACK_WINDOW;
}

template <typename Off>
struct DescBits {
  static constexpr int SH = sizeof(Off) * 8 - 2;
  static constexpr Off COUNT_MASK = (Off(1) << SH) - 1;
  __device__ __forceinline__ static Off make(uint32_t pass, uint32_t state, Off count) {
    return (Off((2u * pass + state) & 3u) << SH) | count;
  }
  __device__ __forceinline__ static uint32_t state(Off w, uint32_t pass) {
    return ((uint32_t)(w >> SH) - 2u * pass) & 3u;
  }
};

// Exclusive prefix over earlier tiles of this digit's counts (decoupled
// lookback; reference LookbackComputePrefixAndPublishComplete,
// libcusort.cuh:1340-1382, walks one tile per L2 round trip).  Here each
// digit's thread reads a window of W predecessor words per round trip
// (independent loads), adds aggregates from the nearest outward and stops at
// the first INCLUSIVE word; an EMPTY word ends the window and is re-polled
// (bounded wait).  Tile `floor` (0, or a segment's first tile) has no
// predecessors.
template <typename Off, int W>
__device__ __forceinline__ Off lookback_prefix(const Off* desc, uint32_t tile, uint32_t digit, uint32_t pass,
                                               uint32_t* status, uint64_t limit_ns, int64_t floor = 0,
                                               uint32_t* rounds = nullptr, uint32_t* empties = nullptr) {
  using DB = DescBits<Off>;
  Off excl = 0;
  int64_t j = (int64_t)tile - 1;  // nearest predecessor not yet accounted for
  dev::SpinGuard guard;
  while (j >= floor) {  // floor: first tile of the prefix (a segment's first tile)
    if (rounds) ++*rounds;
    Off w[W];
#pragma unroll
    for (int k = 0; k < W; ++k)
      w[k] = (j - k >= floor) ? dev::ld_relaxed(desc + (size_t)(j - k) * kRadix + digit)
                              : DB::make(pass, kDescInclusive, Off(0));
    int consumed = 0;
    bool done = false;
#pragma unroll
    for (int k = 0; k < W; ++k) {
      if (done || consumed < k) continue;  // stopped earlier in this window
      const uint32_t st = DB::state(w[k], pass);
      if (st == kDescEmpty) continue;
      excl += w[k] & DB::COUNT_MASK;
      consumed = k + 1;
      done = (st == kDescInclusive);
    }
    if (done) break;
    j -= consumed;
    if (empties && consumed == 0) ++*empties;
    if (consumed == 0 && guard.expired(status, limit_ns)) {
      atomicOr(status, kStatusLookbackTimeout);
      break;
    }
  }
  return excl;
}

// Opt-in lookback timer (compile with CUSORT_LOOKBACK_TIMER=1; plain passes).
// Adds to u64 words of the control block (zeroed by the init kernel with the
// rest of it, so they cover every pass of one sort): +128 the sum over tiles
// of the longest time any digit-owning thread of the tile spent in
// lookback_prefix (ns), +136 descriptor-window rounds summed over all digit
// threads and tiles, +144 tiles, +152 the rounds among those that re-polled
// because the nearest unaccounted predecessor had published nothing yet.
#ifndef CUSORT_LOOKBACK_TIMER
#define CUSORT_LOOKBACK_TIMER 0
#endif
constexpr uint32_t kLookbackTimerOffset = 128;

struct LookbackTimer {
  uint32_t t0 = 0;  // low word of %globaltimer (a lookback takes far less than 4 s)
  uint32_t r = 0, e = 0;
  __device__ __forceinline__ void begin() {
    if constexpr (CUSORT_LOOKBACK_TIMER) {
      r = 0;
      e = 0;
      t0 = (uint32_t)dev::globaltimer_ns();
    }
  }
  // digit-owning warps (all lanes) after their lookback
  __device__ __forceinline__ void end(uint32_t* s, uint32_t lane, uint32_t* status) {
    if constexpr (CUSORT_LOOKBACK_TIMER) {
      const uint32_t dt = __reduce_max_sync(0xffffffffu, (uint32_t)dev::globaltimer_ns() - t0);
      const uint32_t rs = __reduce_add_sync(0xffffffffu, r);
      const uint32_t es = __reduce_add_sync(0xffffffffu, e);
      if (lane == 0) {
        atomicMax(s, dt);
        unsigned long long* w = reinterpret_cast<unsigned long long*>(reinterpret_cast<uint8_t*>(status) +
                                                                      kLookbackTimerOffset);
        atomicAdd(w + 1, (unsigned long long)rs);
        atomicAdd(w + 3, (unsigned long long)es);
      }
    }
  }
  // thread 0, after a barrier that follows every end() of the tile
  __device__ __forceinline__ void tile_done(uint32_t* s, uint32_t* status) {
    if constexpr (CUSORT_LOOKBACK_TIMER) {
      unsigned long long* w = reinterpret_cast<unsigned long long*>(reinterpret_cast<uint8_t*>(status) +
                                                                    kLookbackTimerOffset);
      atomicAdd(w, (unsigned long long)s[0]);
      atomicAdd(w + 2, 1ull);
      s[0] = 0;
    }
  }
};

template <class CFG>
__global__ void __launch_bounds__(CFG::THREADS, CFG::MINB) onesweep_kernel(const typename CFG::Args a) {
  using K = typename dev::UIntOf<CFG::KB>::T;
  using V = typename dev::UIntOf<(CFG::VB ? CFG::VB : 1)>::T;
  using Off = typename CFG::Off;
  using DB = DescBits<Off>;
  using WC = typename CFG::WC;
  constexpr int THREADS = CFG::THREADS, KPT = CFG::KPT, TILE = CFG::TILE, WARPS = CFG::WARPS;
  constexpr int NBUF = CFG::NBUF;
  constexpr bool HAS_V = CFG::VB > 0;

  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* s_wtab = smem + CFG::OFF_WTAB;
  uint32_t* s_tstart = reinterpret_cast<uint32_t*>(smem + CFG::OFF_TSTART);
  Off* s_gbase = reinterpret_cast<Off*>(smem + CFG::OFF_GBASE);
  Off* s_goff = reinterpret_cast<Off*>(smem + CFG::OFF_GOFF);
  // [0] first ticket, [1] next ticket, [2] abort flag, [3] prefetch in flight, [4..11] scan partials
  uint32_t* s_misc = reinterpret_cast<uint32_t*>(smem + CFG::OFF_MISC);
  uint64_t* s_mbar = reinterpret_cast<uint64_t*>(smem + CFG::OFF_MBAR);

  const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
  const K tc = (K)a.tw_c, tf = (K)a.tw_f;
  const K* keys_in = static_cast<const K*>(a.keys_in);
  K* keys_out = static_cast<K*>(a.keys_out);
  const V* vals_in = static_cast<const V*>(a.vals_in);
  V* vals_out = static_cast<V*>(a.vals_out);
  Off* desc = static_cast<Off*>(a.desc);
  uint32_t num_tiles = a.num_tiles;  // segmented: the planner's count, read after the PDL wait
  const bool tma_ok = a.tma_keys && (!HAS_V || a.tma_vals);
  const uint64_t pol = dev::l2_policy_evict_first();
  auto kdigit = [&](K k) -> uint32_t { return dev::digit_k<CFG::FLOAT_KEY, K>(k, tc, tf, a.shift, a.mask); };

  // A tile is staged by TMA when it is full and both inputs are 16-byte aligned.
  auto tma_tile = [&](uint32_t t) {
    if constexpr (CFG::SEG) return false;  // per tile, below (segment tiles start anywhere)
    return !CFG::DIRECT_LOAD && tma_ok && t < num_tiles && (uint64_t)(t + 1) * TILE <= a.n;
  };
  auto issue_tma_at = [&](uint64_t base, int buf) {
    uint8_t* bp = smem + (size_t)buf * CFG::BUF_BYTES;
    dev::mbar_arrive_expect_tx(s_mbar + buf, (uint32_t)TILE * (CFG::KB + CFG::VB));
    dev::tma_load_1d(bp, keys_in + base, (uint32_t)TILE * CFG::KB, s_mbar + buf, pol);
    if constexpr (HAS_V) dev::tma_load_1d(bp + CFG::KEYS_BYTES, vals_in + base, (uint32_t)TILE * CFG::VB, s_mbar + buf, pol);
  };
  auto issue_tma = [&](uint32_t t, int buf) { issue_tma_at((uint64_t)t * TILE, buf); };
  // Bounded wait for a buffer's bulk copy; false if it timed out.
  auto wait_tma = [&](int buf, uint32_t parity) {
    dev::SpinGuard guard;
    while (!dev::mbar_try_wait(s_mbar + buf, parity))
      if (guard.expired(nullptr, a.spin_limit_ns)) return false;
    return true;
  };

  constexpr bool TIMED = CUSORT_LOOKBACK_TIMER && !CFG::ROUTED && !CFG::SEG;
  LookbackTimer lbt;
  if (tid == 0) {
    dev::mbar_init(s_mbar, 1);
    dev::mbar_init(s_mbar + 1, 1);
    dev::fence_mbar_init();
    s_misc[2] = 0;
    s_misc[3] = 0;
    s_misc[14] = 0;  // lookback timer: the tile's maxima
    s_misc[15] = 0;
  }
  dev::pdl_wait();
  dev::pdl_launch_dependents();

  // Global exclusive offset of every digit for this pass (from the upfront
  // histogram), computed once per CTA; the first tile ticket is taken here.
  if constexpr (CFG::SEG) {
    // per-segment digit bases are loaded per tile; nothing to do after a
    // planner overflow (overlapping segments)
    num_tiles = a.ctl->pad[0] ? 0u : a.ctl->num_tiles;
    if (tid == 0) s_misc[0] = atomicAdd(a.tile_counter, 1u);
    __syncthreads();
  } else if constexpr (CFG::ROUTED) {
    // Destinations: owner of each digit; per owner its buffers, capacity,
    // this rank's offset in it and its first digit.
    unsigned char* s_owner = smem + CFG::OFF_ROUTE;
    unsigned long long* s_rptr = reinterpret_cast<unsigned long long*>(smem + CFG::OFF_RPTR);
    uint32_t* s_rfirst = reinterpret_cast<uint32_t*>(smem + CFG::OFF_RFIRST);
    const RouteTable* route = static_cast<const RouteTable*>(a.g_hist_pass);
    if (tid == 0) s_misc[0] = atomicAdd(a.tile_counter, 1u);
    if (tid < kRadix) s_owner[tid] = route->owner[tid];
    if (tid < kMaxRouteRanks) {
      s_rptr[tid] = route->kptr[tid];
      s_rptr[kMaxRouteRanks + tid] = route->vptr[tid];
      s_rptr[2 * kMaxRouteRanks + tid] = route->cap[tid];
      s_rptr[3 * kMaxRouteRanks + tid] = route->base[tid];
      s_rfirst[tid] = route->first_digit[tid];
      s_rfirst[kMaxRouteRanks + tid] = route->last_digit[tid];
    }
    __syncthreads();
  } else {
    if (tid == 0) s_misc[0] = atomicAdd(a.tile_counter, 1u);
    Off cv = (tid < kRadix) ? static_cast<const Off*>(a.g_hist_pass)[tid] : Off(0);
    Off incl = cv;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      Off t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= (uint32_t)o) incl += t;
    }
    if (lane == 31 && warp < 8) s_goff[warp] = incl;
    __syncthreads();
    if (tid < kRadix) {
      Off pre = 0;
      for (uint32_t w = 0; w < warp; ++w) pre += s_goff[w];
      s_gbase[tid] = pre + incl - cv;
    }
  }
  uint32_t cur = s_misc[0];
  uint32_t pending = 0;  // thread 0: ticket requested one tile ahead (prefetch mode)
  if (CFG::PREFETCH && tid == 0) {
    if (NBUF == 2 && tma_tile(cur)) issue_tma(cur, 0);
    pending = atomicAdd(a.tile_counter, 1u);
  }
  uint32_t parity = 0u;  // bit b: phase parity of buffer b's mbarrier
  int b = 0;
  const uint32_t lt = dev::lanemask_lt();

  for (bool first = true;; first = false) {
    if constexpr (!CFG::PREFETCH) {
      // Ticket for this tile, taken when the CTA is ready for it.
      if (!first) {
        if (tid == 0) s_misc[0] = atomicAdd(a.tile_counter, 1u);
        WC::zero(s_wtab, warp, lane);
        __syncthreads();
        cur = s_misc[0];
      } else {
        WC::zero(s_wtab, warp, lane);
        __syncthreads();
      }
    }
    if (cur >= num_tiles) break;
    uint32_t nxt = 0;
    if constexpr (CFG::PREFETCH) {
      WC::zero(s_wtab, warp, lane);
      if (tid == 0) {
        s_misc[1] = pending;
        s_misc[3] = 0;
      }
      __syncthreads();  // previous tile fully written out; next ticket visible
      nxt = s_misc[1];
      if (tid == 0) {
        if (NBUF == 2 && tma_tile(nxt)) {
          issue_tma(nxt, b ^ 1);  // its buffer held the previous tile, consumed before the barrier
          s_misc[3] = 1;
        }
        pending = atomicAdd(a.tile_counter, 1u);
      }
    }
    const uint32_t tile = cur;
    uint64_t base;
    uint32_t valid;
    uint32_t floor = 0;  // first tile of this tile's prefix chain
    if constexpr (CFG::SEG) {
      // the tile's segment, its place in it, and the segment's digit bases
      const uint32_t slot = a.tile_slot[tile];
      const SegRecord r = a.recs[slot];
      const uint64_t i = (uint64_t)(tile - r.tile_first) * TILE;
      base = r.begin + i;
      valid = (uint32_t)((r.len - i) < (uint64_t)TILE ? (r.len - i) : (uint64_t)TILE);
      floor = r.tile_first;
      if (tid < kRadix)
        s_gbase[tid] = static_cast<const Off*>(a.seg_gbase)[((size_t)slot * a.seg_passes + a.seg_pass) * kRadix + tid];
    } else {
      base = (uint64_t)tile * TILE;
      valid = (uint32_t)((a.n - base) < (uint64_t)TILE ? (a.n - base) : (uint64_t)TILE);
    }
    const bool publish = (int64_t)tile != a.skip_tile;
    K* s_keys = reinterpret_cast<K*>(smem + (size_t)b * CFG::BUF_BYTES);
    V* s_vals = reinterpret_cast<V*>(smem + (size_t)b * CFG::BUF_BYTES + CFG::KEYS_BYTES);
    // values in sorted tile order (the staged buffer itself unless VSMEM)
    V* s_vsort = CFG::VSMEM ? reinterpret_cast<V*>(smem + CFG::OFF_VOUT) : s_vals;
    constexpr bool VREG = HAS_V && !CFG::VSMEM;  // values held in registers

    // ---- 1. the tile's keys/values in shared memory
    bool use_tma = tma_tile(tile);
    if constexpr (CFG::SEG) {
      // a full tile whose start is 16-byte aligned in both inputs
      use_tma = !CFG::DIRECT_LOAD && NBUF == 1 && tma_ok && valid == (uint32_t)TILE &&
                ((reinterpret_cast<uintptr_t>(keys_in + base) | (HAS_V ? reinterpret_cast<uintptr_t>(vals_in + base)
                                                                       : uintptr_t(0))) & 15u) == 0;
    }
    if (use_tma) {
      if (NBUF == 1 && tid == 0) issue_tma_at(base, 0);
      const bool ok = wait_tma(b, (parity >> b) & 1u);
      parity ^= 1u << b;
      if (!ok) {
        atomicOr(a.status, kStatusTmaTimeout);
        s_misc[2] = 1;
      }
      __syncthreads();
      if (s_misc[2]) {
        // Give the other buffer's copy, if one is in flight, a bounded wait.
        if (NBUF == 2 && s_misc[3]) wait_tma(b ^ 1, (parity >> (b ^ 1)) & 1u);
        break;
      }
    } else if constexpr (!CFG::DIRECT_LOAD) {
      for (uint32_t i = tid; i < valid; i += THREADS) {
        s_keys[i] = keys_in[base + i];
        if constexpr (HAS_V) s_vals[i] = vals_in[base + i];
      }
      __syncthreads();
    }

    // ---- 2. registers, digits, warp ranking
    const uint32_t wfirst_c = warp * (KPT * 32);
    K key[KPT];
    constexpr bool RECOMP = CFG::RECOMPUTE_DIGIT;
    uint32_t dr[RECOMP ? 1 : KPT];  // digit | (rank within warp << 8)
    // digit of slot s (the top digit for slots past the end of the tile)
    auto digit_at = [&](int s) -> uint32_t {
      const uint32_t idx = wfirst_c + s * 32 + lane;
      return (idx < valid) ? kdigit(key[s]) : a.mask;
    };
    V val[VREG ? KPT : 1];
    const uint32_t wfirst = wfirst_c;
    if constexpr (CFG::DIRECT_LOAD) {
      const K* kin = keys_in + base + wfirst + lane;
      const V* vin = vals_in + base + wfirst + lane;
      if (valid == (uint32_t)TILE) {
#pragma unroll
        for (int s = 0; s < KPT; ++s) {
          key[s] = dev::ld_cs(kin + s * 32);
          if constexpr (VREG) val[s] = dev::ld_cs(vin + s * 32);
        }
      } else {
#pragma unroll
        for (int s = 0; s < KPT; ++s) {
          const bool in = wfirst + s * 32 + lane < valid;
          key[s] = in ? dev::ld_cs(kin + s * 32) : K(0);
          if constexpr (VREG) {
            if (in) val[s] = dev::ld_cs(vin + s * 32);
          }
        }
      }
      if constexpr (!RECOMP) {
#pragma unroll
        for (int s = 0; s < KPT; ++s) dr[s] = digit_at(s);
      }
    } else {
#pragma unroll
      for (int s = 0; s < KPT; ++s) {
        const uint32_t idx = wfirst + s * 32 + lane;
        key[s] = s_keys[idx];
        if constexpr (!RECOMP) dr[s] = digit_at(s);
        if constexpr (VREG) val[s] = s_vals[idx];
      }
    }
    uint2* s_kv = reinterpret_cast<uint2*>(s_keys);  // PACKED_KV view of the same buffer
    constexpr bool EARLY = CFG::RANK_MODE >= 4;
    // sorted-tile check (see the pipelined pass): plain passes, staged tiles
    constexpr bool SORTED = CUSORT_SORTED_TILES && CFG::RANK_MODE == 6 && !CFG::ROUTED && !CFG::SEG &&
                            !CFG::DIRECT_LOAD;
    bool hint = false;
    if constexpr (SORTED) {
      hint = warp_nondecreasing(RECOMP ? digit_at(0) : dr[0], lane) &&
             warp_nondecreasing(RECOMP ? digit_at(KPT - 1) : dr[KPT - 1], lane);
    }
    if constexpr (EARLY) {
#pragma unroll
      for (int s = 0; s < KPT; ++s) WC::count_key(s_wtab, warp, RECOMP ? digit_at(s) : dr[s]);
    } else {
      static_assert(!RECOMP, "digit recomputation needs the early-count rank modes");
      uint32_t prev = 0;
      RankSlots<CFG::RANK_MODE, 0, KPT>::run(s_wtab, warp, dr, lane, lt, prev);
    }
    const bool all_hint = __syncthreads_and(hint) != 0;

    // ---- 3. per-digit counts, aggregate publish, tile-local digit offsets
    uint32_t cnt = 0;
    if (tid < kRadix) {
#pragma unroll 4
      for (int w = 0; w < WARPS; ++w) {
        const uint32_t c = WC::count(s_wtab, w, tid);
        WC::put(s_wtab, w, tid, cnt);
        cnt += c;
      }
      if (tid == a.mask) cnt -= (uint32_t)TILE - valid;
      if (publish)
        dev::st_relaxed(desc + (size_t)tile * kRadix + tid,
                        DB::make(a.pass, tile == floor ? kDescInclusive : kDescAggregate, (Off)cnt));
    }
    uint32_t incl = 0;
    if (warp < kRadix / 32) {
      incl = dev::warp_inclusive_scan(cnt, lane);
      if (lane == 31) s_misc[4 + warp] = incl;
    }
    // a full tile whose keys all share one digit is already in sorted order
    // (plain passes: the tile then goes out from the registers, unranked)
    constexpr bool PLAIN = CUSORT_ONE_DIGIT_TILES && !CFG::ROUTED && !CFG::SEG;
    const bool one_digit = __syncthreads_or(PLAIN && tid < kRadix && cnt == (uint32_t)TILE) != 0;
    if (tid < kRadix) {
      uint32_t pre = 0;
      for (uint32_t w = 0; w < warp; ++w) pre += s_misc[4 + w];
      const uint32_t ts = pre + incl - cnt;
      s_tstart[tid] = ts;
#pragma unroll 4
      for (int w = 0; w < WARPS; ++w) WC::put(s_wtab, w, tid, WC::get(s_wtab, w, tid) + ts);
    }
    __syncthreads();
    // a tile whose digits never decrease in input order: no ranking either
    bool sorted_tile = false;
    if (SORTED && all_hint && !one_digit && valid == (uint32_t)TILE) {
      // neighbours compared in the staged tile (input order)
      bool ok = true;
      for (uint32_t j = tid + 1; j < (uint32_t)TILE; j += THREADS) ok = ok && kdigit(s_keys[j - 1]) <= kdigit(s_keys[j]);
      sorted_tile = __syncthreads_and(ok) != 0;
    }

    // ---- 4. reorder in shared memory (tile sorted by digit, stable)
    auto reorder = [&]() {
      if constexpr (EARLY) {
        // rank against the per-warp position counters, store at once
        auto store = [&](auto sc, uint32_t pos) {
          constexpr int S = decltype(sc)::value;
          pos = tile_swz(pos);
          if constexpr (CFG::PACKED_KV) {
            s_kv[pos] = make_uint2((uint32_t)key[S], (uint32_t)val[S]);
          } else {
            s_keys[pos] = key[S];
            if constexpr (VREG) s_vals[pos] = val[S];
            if constexpr (CFG::VSMEM) s_vsort[pos] = s_vals[wfirst_c + S * 32 + lane];
          }
        };
        uint32_t prev = 0;
        static_for<0, KPT>([&](auto sc) {
          constexpr int S = decltype(sc)::value;
          store(sc, WC::template rank_slot<S>(s_wtab, warp, RECOMP ? digit_at(S) : dr[S], lane, lt, prev));
        });
      } else {
#pragma unroll
        for (int s = 0; s < KPT; ++s) {
          const uint32_t pos = tile_swz(WC::get(s_wtab, warp, dr[s] & 0xffu) + (dr[s] >> 8));
          if constexpr (CFG::PACKED_KV) {
            s_kv[pos] = make_uint2((uint32_t)key[s], (uint32_t)val[s]);
          } else {
            s_keys[pos] = key[s];
            if constexpr (VREG) s_vals[pos] = val[s];
            if constexpr (CFG::VSMEM) s_vsort[pos] = s_vals[wfirst_c + s * 32 + lane];
          }
        }
      }
    };

    // ---- 5. decoupled lookback.  The warps that own a digit (0-7) run it
    // before their own reorder, so its L2 round trips overlap the other
    // warps' reorder work instead of trailing it.
    if (tid < kRadix) {
      Off excl = 0;
      if (tile > floor) {
        if constexpr (TIMED) lbt.begin();
        excl = lookback_prefix<Off, lookback_window<Off>()>(desc, tile, tid, a.pass, a.status, a.spin_limit_ns, floor,
                                                            TIMED ? &lbt.r : nullptr, TIMED ? &lbt.e : nullptr);
        if constexpr (TIMED) lbt.end(s_misc + 14, lane, a.status);
        if (publish)
          dev::st_relaxed(desc + (size_t)tile * kRadix + tid, DB::make(a.pass, kDescInclusive, excl + (Off)cnt));
      }
      if constexpr (CFG::ROUTED) {
        // Inclusive prefix over digits of the earlier tiles' counts (warp
        // part here, warp totals added after the barrier): the items of an
        // owner in earlier tiles are a difference of two prefixes.
        unsigned long long* s_pre = reinterpret_cast<unsigned long long*>(smem + CFG::OFF_RPRE);
        const unsigned long long incl_x = dev::warp_inclusive_scan<unsigned long long>(excl, lane);
        s_pre[tid] = incl_x;
        if (lane == 31) s_pre[kRadix + warp] = incl_x;
      } else {
        s_goff[tid] = s_gbase[tid] + excl - (Off)s_tstart[tid];
      }
    }
    if (PLAIN && (one_digit || sorted_tile)) {
      __syncthreads();
      if constexpr (TIMED) {
        if (tid == 0) lbt.tile_done(s_misc + 14, a.status);
      }
      if constexpr (CFG::DIRECT_LOAD) {
        const Off dst = s_goff[kdigit(key[0])] + (Off)(wfirst_c + lane);  // one digit only
#pragma unroll
        for (int s = 0; s < KPT; ++s) {
          keys_out[dst + (Off)(s * 32)] = key[s];
          if constexpr (VREG) vals_out[dst + (Off)(s * 32)] = val[s];
        }
      } else {
        // from the staged copy of the tile, which the reorder has not touched
#pragma unroll 4
        for (uint32_t j = tid; j < (uint32_t)TILE; j += THREADS) {
          const K k = s_keys[j];
          const Off dst = s_goff[kdigit(k)] + (Off)j;
          keys_out[dst] = k;
          if constexpr (HAS_V) vals_out[dst] = s_vals[j];
        }
      }
      dev::fence_proxy_async_smem();  // before the buffer is refilled by TMA
      if constexpr (CFG::PREFETCH) {
        cur = nxt;
        if (NBUF == 2) b ^= 1;
      }
      continue;
    }
    reorder();
    __syncthreads();
    if constexpr (TIMED) {
      if (tid == 0) lbt.tile_done(s_misc + 14, a.status);
    }
    if constexpr (CFG::ROUTED) {
      // Owner q receives, per source rank, that rank's tiles in order, each
      // tile's items of q in the tile's (digit-sorted) order: one contiguous
      // run per (tile, owner).  Resolve each digit's address once (dst(j) =
      // addr + j for tile position j); a run that would not fit is dropped
      // and flagged.
      if (tid < kRadix) {
        const unsigned long long* s_rptr = reinterpret_cast<const unsigned long long*>(smem + CFG::OFF_RPTR);
        const unsigned long long* s_pre = reinterpret_cast<const unsigned long long*>(smem + CFG::OFF_RPRE);
        const uint32_t* s_rfirst = reinterpret_cast<const uint32_t*>(smem + CFG::OFF_RFIRST);
        unsigned long long* s_dst = reinterpret_cast<unsigned long long*>(smem + CFG::OFF_RDST);
        const uint32_t q = smem[CFG::OFF_ROUTE + tid];
        const uint32_t lo = s_rfirst[q], hi = s_rfirst[kMaxRouteRanks + q];  // owner's digits [lo, hi]
        // inclusive digit prefix at x (over all 8 warps' parts)
        auto prefix = [&](uint32_t x) {
          unsigned long long v = s_pre[x];
          for (uint32_t w = 0; w < (x >> 5); ++w) v += s_pre[kRadix + w];
          return v;
        };
        const unsigned long long earlier = prefix(hi) - (lo ? prefix(lo - 1) : 0ull);
        // position of the owner's run in its buffer, and of this digit in it
        const unsigned long long run = s_rptr[3 * kMaxRouteRanks + q] + earlier;
        const unsigned long long rel = run - (unsigned long long)s_tstart[lo];  // modulo 2^64
        const unsigned long long first = rel + s_tstart[tid];
        unsigned long long dk = 0, dv = 0;
        if (first + cnt <= s_rptr[2 * kMaxRouteRanks + q]) {
          dk = s_rptr[q] + rel * sizeof(K);
          if constexpr (HAS_V) dv = s_rptr[kMaxRouteRanks + q] + rel * sizeof(V);
        } else if (cnt) {
          atomicOr(a.status, kStatusRouteOverflow);
        }
        s_dst[tid] = dk;
        s_dst[kRadix + tid] = dv;
      }
      __syncthreads();
    }

    // ---- 6. coalesced scatter
    // sorted position j, read from its swizzled slot p
    auto put_one = [&](uint32_t j, uint32_t p) {
      if constexpr (CFG::ROUTED) {
        K k;
        V v;
        if constexpr (CFG::PACKED_KV) {
          const uint2 kv = s_kv[p];
          k = (K)kv.x;
          v = (V)kv.y;
        } else {
          k = s_keys[p];
          if constexpr (HAS_V) v = s_vsort[p];
        }
        const unsigned long long* s_dst = reinterpret_cast<const unsigned long long*>(smem + CFG::OFF_RDST);
        const uint32_t d = dev::digit_k<CFG::FLOAT_KEY, K>(k, tc, tf, a.shift, a.mask);
        const unsigned long long dk = s_dst[d];
        if (dk != 0ull) {  // 0: the run did not fit (flagged above)
          reinterpret_cast<K*>(dk)[j] = k;
          if constexpr (HAS_V) reinterpret_cast<V*>(s_dst[kRadix + d])[j] = v;
        }
      } else if constexpr (CFG::PACKED_KV) {
        const uint2 kv = s_kv[p];
        const K k = (K)kv.x;
        const Off dst = s_goff[kdigit(k)] + (Off)j;
        keys_out[dst] = k;
        vals_out[dst] = (V)kv.y;
      } else {
        const K k = s_keys[p];
        const Off dst = s_goff[kdigit(k)] + (Off)j;
        keys_out[dst] = k;
        if constexpr (HAS_V) vals_out[dst] = s_vsort[p];
      }
    };
    if (valid == (uint32_t)TILE) {
#pragma unroll
      for (int i = 0; i < KPT; ++i) put_one(tid + i * THREADS, tile_swz_at<THREADS>(tid, i));
    } else {
      for (uint32_t j = tid; j < valid; j += THREADS) put_one(j, tile_swz(j));
    }
    dev::fence_proxy_async_smem();  // before the buffer is refilled by TMA
    if constexpr (CFG::PREFETCH) {
      cur = nxt;
      if (NBUF == 2) b ^= 1;
    }
  }
  if constexpr (CFG::ROUTED) __threadfence_system();  // peer stores visible before the kernel ends
}

// ---------------------------------------------------------------------------
// onesweep, pipelined register loads (CFG::PIPE; plain passes).  The same
// stable pass as onesweep_kernel, re-ordered so that no CTA waits for its
// tile's data:
//   prologue   ticket t0; issue t0's loads (global -> registers)
//   per tile   count digits (registers) -> aggregate publish -> block scan ->
//              lookback + rank/reorder into the shared-memory tile ->
//              ticket t+1 -> ISSUE t+1's loads into the now free registers ->
//              scatter tile t from shared memory (the loads land meanwhile)
// Slots past the end of the last tile hold a sentinel key whose twiddled
// bits are all ones, so every slot's digit is computed the same way (the
// sentinels take the top digit and sort behind the tile's valid items, which
// are the only ones written).  The next ticket is taken once the tile is
// reordered, so the next tile's aggregate is published about one scatter
// later -- the same delay as a tile load, which it replaces.
// ---------------------------------------------------------------------------
#ifndef CUSORT_PIPE_SCATTER_UNROLL
#define CUSORT_PIPE_SCATTER_UNROLL 4
#endif
// Issues the global loads of tile t for one thread (slot s = item first + 32 s
// of the tile) into registers; slots past the end get the sentinel key.
template <class CFG, typename K, typename V, int NV>
__device__ __forceinline__ void pipe_load_tile(K (&key)[CFG::KPT], V (&val)[NV], const K* keys_in, const V* vals_in,
                                               uint64_t n, uint32_t t, uint32_t first, K sentinel) {
  constexpr int KPT = CFG::KPT, TILE = CFG::TILE;
  const uint64_t base = (uint64_t)t * TILE;
  const uint32_t valid = (uint32_t)((n - base) < (uint64_t)TILE ? (n - base) : (uint64_t)TILE);
  const K* kin = keys_in + base + first;
  const V* vin = vals_in + base + first;
  if (valid == (uint32_t)TILE) {
#pragma unroll
    for (int s = 0; s < KPT; ++s) {
      key[s] = __ldcs(kin + s * 32);
      if constexpr (CFG::VB > 0) val[s] = __ldcs(vin + s * 32);
    }
  } else {
#pragma unroll
    for (int s = 0; s < KPT; ++s) {
      const bool in = first + s * 32 < valid;
      key[s] = in ? __ldcs(kin + s * 32) : sentinel;
      if constexpr (CFG::VB > 0) {
        if (in) val[s] = __ldcs(vin + s * 32);
      }
    }
  }
}
template <class CFG>
__global__ void __launch_bounds__(CFG::THREADS, CFG::MINB) onesweep_pipe_kernel(const OnesweepArgs a) {
  using K = typename dev::UIntOf<CFG::KB>::T;
  using V = typename dev::UIntOf<(CFG::VB ? CFG::VB : 1)>::T;
  using Off = typename CFG::Off;
  using DB = DescBits<Off>;
  using WC = typename CFG::WC;
  constexpr int THREADS = CFG::THREADS, KPT = CFG::KPT, TILE = CFG::TILE, WARPS = CFG::WARPS;
  constexpr bool HAS_V = CFG::VB > 0;
  static_assert(CFG::PIPE && CFG::RANK_MODE >= 4, "pipelined pass: early-count rank modes only");
  constexpr bool SORTED = CUSORT_SORTED_TILES && CFG::RANK_MODE == 6;

  extern __shared__ __align__(128) uint8_t smem[];
  K* s_keys = reinterpret_cast<K*>(smem);  // the tile in sorted order
  V* s_vals = reinterpret_cast<V*>(smem + CFG::KEYS_BYTES);
  uint2* s_kv = reinterpret_cast<uint2*>(smem);  // PACKED_KV view
  uint8_t* s_wtab = smem + CFG::OFF_WTAB;
  uint32_t* s_tstart = reinterpret_cast<uint32_t*>(smem + CFG::OFF_TSTART);
  Off* s_gbase = reinterpret_cast<Off*>(smem + CFG::OFF_GBASE);
  Off* s_goff = reinterpret_cast<Off*>(smem + CFG::OFF_GOFF);
  uint32_t* s_misc = reinterpret_cast<uint32_t*>(smem + CFG::OFF_MISC);  // [0],[1] tickets, [4..11] scan

  const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
  const K tc = (K)a.tw_c, tf = (K)a.tw_f;
  // a key whose twiddled bits are all ones (dev::twiddle): ~c when c's sign
  // bit is set (the key's own sign bit is then clear), else ~(c ^ f)
  constexpr int NB = CFG::KB * 8;
  const K sentinel = ((tc >> (NB - 1)) & 1) ? (K)~tc : (K)~(tc ^ tf);
  auto kdigit = [&](K k) -> uint32_t { return dev::digit_k<CFG::FLOAT_KEY, K>(k, tc, tf, a.shift, a.mask); };
  const K* keys_in = static_cast<const K*>(a.keys_in);
  K* keys_out = static_cast<K*>(a.keys_out);
  const V* vals_in = static_cast<const V*>(a.vals_in);
  V* vals_out = static_cast<V*>(a.vals_out);
  Off* desc = static_cast<Off*>(a.desc);
  const uint32_t num_tiles = a.num_tiles;

  LookbackTimer lbt;
  dev::pdl_wait();
  dev::pdl_launch_dependents();
  if (tid == 0) {
    s_misc[0] = atomicAdd(a.tile_counter, 1u);
    s_misc[14] = 0;  // lookback timer: the tile's maxima
    s_misc[15] = 0;
  }
  {
    // global exclusive offset of every digit (upfront histogram)
    Off cv = (tid < kRadix) ? static_cast<const Off*>(a.g_hist_pass)[tid] : Off(0);
    Off incl = cv;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      Off t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= (uint32_t)o) incl += t;
    }
    if (lane == 31 && warp < 8) s_goff[warp] = incl;
    WC::zero(s_wtab, warp, lane);
    __syncthreads();
    if (tid < kRadix) {
      Off pre = 0;
      for (uint32_t w = 0; w < warp; ++w) pre += s_goff[w];
      s_gbase[tid] = pre + incl - cv;
    }
  }
  uint32_t cur = s_misc[0];
  const uint32_t lt = dev::lanemask_lt();
  const uint32_t wfirst = warp * (KPT * 32);
  K key[KPT];
  V val[HAS_V ? KPT : 1];

  // issue the loads of tile t into key[] / val[] (consumed later)
  auto load_tile = [&](uint32_t t) {
    pipe_load_tile<CFG>(key, val, keys_in, vals_in, a.n, t, wfirst + lane, sentinel);
  };
  if (cur < num_tiles) load_tile(cur);

  while (cur < num_tiles) {
    const uint32_t tile = cur;
    const uint64_t base = (uint64_t)tile * TILE;
    const uint32_t valid = (uint32_t)((a.n - base) < (uint64_t)TILE ? (a.n - base) : (uint64_t)TILE);
    const bool publish = (int64_t)tile != a.skip_tile;
    auto digit = [&](int s) -> uint32_t { return kdigit(key[s]); };

    // ---- counting pre-pass (per-warp digit counts).  The digit is taken from
    // an opaque copy of the key: otherwise the compiler keeps every slot's
    // digit live until the ranking recomputes it, and spills registers.
    bool hint = false;  // this warp's first and last slots non-decreasing (sorted-tile check)
    if constexpr (SORTED) {
      hint = warp_nondecreasing(kdigit(dev::opaque(key[0])), lane) &&
             warp_nondecreasing(kdigit(dev::opaque(key[KPT - 1])), lane);
    }
#pragma unroll
    for (int s = 0; s < KPT; ++s)
      WC::count_key(s_wtab, warp, kdigit(dev::opaque(key[s])));
    const bool all_hint = __syncthreads_and(hint) != 0;

    // ---- per-digit counts, aggregate publish, tile-local digit offsets
    uint32_t cnt = 0;
    if (tid < kRadix) {
#pragma unroll 4
      for (int w = 0; w < WARPS; ++w) {
        const uint32_t c = WC::count(s_wtab, w, tid);
        WC::put(s_wtab, w, tid, cnt);
        cnt += c;
      }
      if (tid == a.mask) cnt -= (uint32_t)TILE - valid;  // the sentinels
      if (publish)
        dev::st_relaxed(desc + (size_t)tile * kRadix + tid,
                        DB::make(a.pass, tile == 0 ? kDescInclusive : kDescAggregate, (Off)cnt));
    }
    uint32_t incl = 0;
    if (warp < kRadix / 32) {
      incl = dev::warp_inclusive_scan(cnt, lane);
      if (lane == 31) s_misc[4 + warp] = incl;
    }
    // a full tile whose keys all share one digit is already in sorted order
    const bool one_digit =
        __syncthreads_or(CUSORT_ONE_DIGIT_TILES && tid < kRadix && cnt == (uint32_t)TILE) != 0;
    if (tid < kRadix) {
      uint32_t pre = 0;
      for (uint32_t w = 0; w < warp; ++w) pre += s_misc[4 + w];
      const uint32_t ts = pre + incl - cnt;
      s_tstart[tid] = ts;
#pragma unroll 4
      for (int w = 0; w < WARPS; ++w) WC::put(s_wtab, w, tid, WC::get(s_wtab, w, tid) + ts);
    }
    __syncthreads();
    // a tile whose digits never decrease in input order: no ranking either
    bool sorted_tile = false;
    if (SORTED && all_hint && !one_digit && valid == (uint32_t)TILE) {
      bool ok = true;
      uint32_t last = 0;  // previous slot's lane-31 digit
      static_for<0, KPT>([&](auto sc) {
        constexpr int S = decltype(sc)::value;
        const uint32_t d = digit(S);
        ok = ok && warp_nondecreasing(d, lane) && (S == 0 || __shfl_sync(0xffffffffu, d, 0) >= last);
        last = __shfl_sync(0xffffffffu, d, 31);
      });
      // warp edges through the (still unused) sorted-tile buffer
      uint32_t* s_edge = reinterpret_cast<uint32_t*>(s_keys);
      if (lane == 0) s_edge[warp] = digit(0);
      if (lane == 31) s_edge[WARPS + warp] = digit(KPT - 1);
      __syncthreads();
      ok = ok && (warp == 0 || s_edge[WARPS + warp - 1] <= s_edge[warp]);
      sorted_tile = __syncthreads_and(ok) != 0;
    }

    // ---- decoupled lookback and rank + reorder: the digit-owning warps look
    // back first, so their L2 round trips overlap the other warps' reordering
    // (with a window small enough to fit beside the tile's keys in registers)
    {
      constexpr int W = lookback_window<Off>();
      if (tid < kRadix) {
        Off excl = 0;
        if (tile > 0) {
          lbt.begin();
          excl = lookback_prefix<Off, W>(desc, tile, tid, a.pass, a.status, a.spin_limit_ns, 0,
                                         CUSORT_LOOKBACK_TIMER ? &lbt.r : nullptr,
                                         CUSORT_LOOKBACK_TIMER ? &lbt.e : nullptr);
          lbt.end(s_misc + 14, lane, a.status);
          if (publish)
            dev::st_relaxed(desc + (size_t)tile * kRadix + tid, DB::make(a.pass, kDescInclusive, excl + (Off)cnt));
        }
        s_goff[tid] = s_gbase[tid] + excl - (Off)s_tstart[tid];
      }
    }
    if (one_digit || sorted_tile) {
      // no ranking: the tile goes out from the registers in input order
      if (tid == 0) s_misc[1] = atomicAdd(a.tile_counter, 1u);
      __syncthreads();
      if (tid == 0) lbt.tile_done(s_misc + 14, a.status);
#pragma unroll
      for (int s = 0; s < KPT; ++s) {
        const Off dst = s_goff[kdigit(key[s])] + (Off)(wfirst + s * 32 + lane);
        keys_out[dst] = key[s];
        if constexpr (HAS_V) vals_out[dst] = val[s];
      }
      const uint32_t nxt = s_misc[1];
      if (nxt < num_tiles) load_tile(nxt);
      WC::zero(s_wtab, warp, lane);
      cur = nxt;
      continue;
    }
    {
      auto store = [&](auto sc, uint32_t pos) {
        constexpr int S = decltype(sc)::value;
        pos = tile_swz(pos);
        if constexpr (CFG::PACKED_KV) {
          s_kv[pos] = make_uint2((uint32_t)key[S], (uint32_t)val[S]);
        } else {
          s_keys[pos] = key[S];
          if constexpr (HAS_V) s_vals[pos] = val[S];
        }
      };
      uint32_t prev = 0;
      static_for<0, KPT>([&](auto sc) {
        constexpr int S = decltype(sc)::value;
        store(sc, WC::template rank_slot<S>(s_wtab, warp, digit(S), lane, lt, prev));
      });
    }
    if (tid == 0) s_misc[1] = atomicAdd(a.tile_counter, 1u);
    __syncthreads();
    if (tid == 0) lbt.tile_done(s_misc + 14, a.status);

    // ---- next tile's loads in flight while this tile is written out
    const uint32_t nxt = s_misc[1];
    if (nxt < num_tiles) load_tile(nxt);
    WC::zero(s_wtab, warp, lane);  // this warp's table: its ranking is done

    // ---- coalesced scatter
    // sorted position j, read from its swizzled slot p
    auto put_one = [&](uint32_t j, uint32_t p) {
      if constexpr (CFG::PACKED_KV) {
        const uint2 kv = s_kv[p];
        const K k = (K)kv.x;
        const Off dst = s_goff[kdigit(k)] + (Off)j;
        keys_out[dst] = k;
        vals_out[dst] = (V)kv.y;
      } else {
        const K k = s_keys[p];
        const Off dst = s_goff[kdigit(k)] + (Off)j;
        keys_out[dst] = k;
        if constexpr (HAS_V) vals_out[dst] = s_vals[p];
      }
    };
    if (valid == (uint32_t)TILE) {
      constexpr int SU = CUSORT_PIPE_SCATTER_UNROLL;
#pragma unroll SU
      for (int i = 0; i < KPT; ++i) put_one(tid + i * THREADS, tile_swz_at<THREADS>(tid, i));
    } else {
      for (uint32_t j = tid; j < valid; j += THREADS) put_one(j, tile_swz(j));
    }
    cur = nxt;
  }
}

}  // namespace cusort_b200

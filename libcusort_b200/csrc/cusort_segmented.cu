// cusort_segmented.cu -- host side of the segmented sort (C ABI
// cusort_segmented_sort_keys / cusort_segmented_sort_pairs) and the planner
// kernel.  No counterpart in the reference beyond the name in its banner
// (libcusort.cuh:4); semantics as CUB's DeviceSegmentedRadixSort: every
// segment [d_begin_offsets[s], d_end_offsets[s]) is sorted independently and
// stably into the same positions of the output, positions outside every
// segment are not written, end <= begin is an empty segment, segments must
// not overlap.
//
// Temp storage (size independent of the offsets' contents, so the two-phase
// protocol needs no host synchronisation):
//   [control 256 B: status u32 @0, tile counters u32[8] @64, SegControl @128]
//   [per-segment digit counts: slots x passes x 256 x OffsetT]   zeroed
//   [lookback descriptors: tiles x 256 x OffsetT]                zeroed
//   [segment records: slots x SegRecord][tile -> slot: tiles x u32]
//   [staging keys n x K][staging values n x V]                  (passes >= 2)
// where slots (segments longer than the small-sort capacity) are at most
// n / (capacity + 1) and tiles at most n / tile + slots.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "../../include/cusort_b200.h"
#include "cusort_dispatch.h"
#include "cusort_segmented.cuh"
#include "cusort_types.h"

namespace cusort_b200 {

__global__ void __launch_bounds__(256) seg_plan_kernel(const SegPlanArgs a) {
  dev::pdl_wait();  // control block zeroed by the init kernel
  dev::pdl_launch_dependents();
  // one segment per thread; the tile -> slot entries of the warp's segments
  // are then written by the whole warp (one long segment would otherwise be
  // written by a single thread)
  const uint64_t gthreads = (uint64_t)gridDim.x * blockDim.x;
  const uint32_t lane = threadIdx.x & 31u;
  const uint64_t first_s = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x - lane;
  for (uint64_t s0 = first_s; s0 < a.num_segments; s0 += gthreads) {
    const uint64_t s = s0 + lane;
    uint32_t slot = 0, first = 0, nt = 0;
    if (s < a.num_segments) {
      const int64_t b = a.begin_offsets[s], e = a.end_offsets[s];
      const uint64_t len = e > b ? (uint64_t)(e - b) : 0;
      if (len > a.min_len) {
        const uint64_t ntl = (len + a.tile - 1) / a.tile;
        slot = atomicAdd(&a.ctl->num_slots, 1u);
        first = atomicAdd(&a.ctl->num_tiles, (uint32_t)ntl);
        if (slot >= a.max_slots || (uint64_t)first + ntl > a.max_tiles) {
          atomicOr(a.status, kStatusSegOverflow);
          atomicOr(&a.ctl->pad[0], 1u);
        } else {
          SegRecord r;
          r.begin = (uint64_t)b;
          r.len = len;
          r.tile_first = first;
          r.pad = 0;
          a.recs[slot] = r;
          nt = (uint32_t)ntl;
        }
      }
    }
    for (uint32_t j = 0; j < 32; ++j) {
      const uint32_t nt_j = __shfl_sync(0xffffffffu, nt, j);
      const uint32_t first_j = __shfl_sync(0xffffffffu, first, j);
      const uint32_t slot_j = __shfl_sync(0xffffffffu, slot, j);
      for (uint32_t t = lane; t < nt_j; t += 32) a.tile_slot[first_j + t] = slot_j;
    }
  }
}

template <int BYTES>
static const void* copy_kernel() {
  return reinterpret_cast<const void*>(&seg_copy_kernel<BYTES>);
}

const void* get_seg_plan_kernel() { return reinterpret_cast<const void*>(&seg_plan_kernel); }

const void* get_seg_copy_kernel(int bytes) {
  switch (bytes) {
    case 1: return copy_kernel<1>();
    case 2: return copy_kernel<2>();
    case 4: return copy_kernel<4>();
    case 8: return copy_kernel<8>();
    case 16: return copy_kernel<16>();
    default: return nullptr;
  }
}

namespace {

int key_bytes(int kt) {
  switch (kt) {
    case CUSORT_KEY_U8: case CUSORT_KEY_I8: return 1;
    case CUSORT_KEY_U16: case CUSORT_KEY_I16: return 2;
    case CUSORT_KEY_U32: case CUSORT_KEY_I32: case CUSORT_KEY_F32: return 4;
    case CUSORT_KEY_U64: case CUSORT_KEY_I64: case CUSORT_KEY_F64: return 8;
    default: return 0;
  }
}
size_t a256(size_t x) { return (x + 255) & ~size_t(255); }

cudaError_t launch(const void* func, int grid, int threads, size_t smem, bool pdl, void* args, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)std::max(grid, 1));
  cfg.blockDim = dim3((unsigned)threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  void* argv[1] = {args};
  return cudaLaunchKernelExC(&cfg, func, argv);
}

struct SegLayout {
  uint64_t max_slots, max_tiles;
  size_t hist, desc, zero_end, recs, tile_slot, stage_k, stage_v, total;
};

cudaError_t seg_sort(void* d_temp, size_t* temp_bytes, int kt, size_t vb, bool desc, const void* kin, void* kout,
                     const void* vin, void* vout, int64_t n, int64_t num_segments, const int64_t* bo,
                     const int64_t* eo, int begin_bit, int end_bit, cudaStream_t stream) {
  const int kb = key_bytes(kt);
  if (kb == 0 || temp_bytes == nullptr || n < 0 || num_segments < 0) return cudaErrorInvalidValue;
  if (vb != 0 && vb != 1 && vb != 2 && vb != 4 && vb != 8 && vb != 16) return cudaErrorInvalidValue;
  if (begin_bit < 0 || end_bit < 0 || begin_bit > end_bit || end_bit > 8 * kb) return cudaErrorInvalidValue;
  const uint32_t nbits = (uint32_t)(end_bit - begin_bit);
  const uint32_t P = (nbits + 7) / 8;
  const uint32_t last_mask = P ? (1u << (nbits - (P - 1) * 8)) - 1u : 0u;
  const int offb = ((uint64_t)n < (1ull << 30) && !force_wide_offsets()) ? 4 : 8;
  const bool fk = (kt == CUSORT_KEY_F32 || kt == CUSORT_KEY_F64);
  SegKernels k;
  bool ok = false;
  switch (kb) {
    case 1: case 2: ok = get_segmented_k12(kb, (int)vb, offb, fk, &k); break;
    case 4: ok = get_segmented_k4((int)vb, offb, fk, &k); break;
    case 8: ok = get_segmented_k8((int)vb, offb, fk, &k); break;
    default: ok = false;
  }
  if (!ok) return cudaErrorInvalidValue;

  // temp layout (see the file comment)
  const uint64_t nn = (uint64_t)n;
  const uint64_t small_cap = (uint64_t)k.small_block2.tile;  // longer segments are tiled
  SegLayout L;
  L.max_slots = nn / (small_cap + 1) + 1;
  L.max_tiles = nn / (uint64_t)k.onesweep.tile + L.max_slots + 1;
  if (L.max_tiles >= (1ull << 32)) return cudaErrorInvalidValue;
  size_t o = 256;
  L.hist = o;
  o += a256((size_t)L.max_slots * std::max<uint32_t>(P, 1) * kRadix * offb);
  L.desc = o;
  o += a256((size_t)L.max_tiles * kRadix * offb);
  L.zero_end = o;
  L.recs = o;
  o += a256((size_t)L.max_slots * sizeof(SegRecord));
  L.tile_slot = o;
  o += a256((size_t)L.max_tiles * 4);
  const bool staging = P >= 2;
  L.stage_k = o;
  o += staging ? a256((size_t)nn * kb) : 0;
  L.stage_v = o;
  o += (staging && vb) ? a256((size_t)nn * vb) : 0;
  L.total = o;
  if (d_temp == nullptr) {
    *temp_bytes = L.total;
    return cudaSuccess;
  }
  if (*temp_bytes < L.total || (reinterpret_cast<uintptr_t>(d_temp) & 15) != 0) return cudaErrorInvalidValue;
  if (n == 0 || num_segments == 0) return cudaSuccess;
  if (bo == nullptr || eo == nullptr || kin == nullptr || kout == nullptr) return cudaErrorInvalidValue;
  if (vb && (vin == nullptr || vout == nullptr)) return cudaErrorInvalidValue;

  uint8_t* t = static_cast<uint8_t*>(d_temp);
  uint32_t* status = reinterpret_cast<uint32_t*>(t);
  uint32_t* counters = reinterpret_cast<uint32_t*>(t + 64);
  SegControl* ctl = reinterpret_cast<SegControl*>(t + 128);
  int sms = 0, occ = 0;
  {
    cudaError_t e = occupancy_of(k.onesweep, &sms, &occ);
    if (e) return e;
  }
  const int init_grid_cap = 4 * sms;
  uint64_t tw_c = 0, tw_f = 0;
  twiddle_constants_of(kt, desc, &tw_c, &tw_f);
  const int seg_grid = (int)std::min<int64_t>(num_segments, 1 << 20);

  if (P == 0) {  // zero-width key range: every segment copied as it is
    cudaError_t z = cudaMemsetAsync(d_temp, 0, 256, stream);  // status word
    if (z) return z;
    SegSmallArgs c = {};
    c.keys_in = kin;
    c.keys_out = kout;
    c.begin_offsets = bo;
    c.end_offsets = eo;
    c.num_segments = (uint64_t)num_segments;
    cudaError_t e = launch(get_seg_copy_kernel(kb), seg_grid, 256, 0, false, &c, stream);
    if (e || !vb) return e;
    c.keys_in = vin;
    c.keys_out = vout;
    return launch(get_seg_copy_kernel((int)vb), seg_grid, 256, 0, false, &c, stream);
  }

  // 1. small segments: one warp per segment up to 128 items (all-pairs rank)
  //    and up to the warp capacity (passes in shared memory), groups of 2 and
  //    4 warps, then one CTA per segment up to the block capacity
  SegSmallArgs sa = {};
  sa.keys_in = kin;
  sa.keys_out = kout;
  sa.vals_in = vb ? vin : nullptr;
  sa.vals_out = vb ? vout : nullptr;
  sa.begin_offsets = bo;
  sa.end_offsets = eo;
  sa.num_segments = (uint64_t)num_segments;
  sa.tw_c = tw_c;
  sa.tw_f = tw_f;
  sa.begin_bit = (uint32_t)begin_bit;
  sa.passes = P;
  sa.last_mask = last_mask;
  {
    // all-pairs classes: 1-32 and 33-128 items
    cudaError_t e = cudaSuccess;
    uint64_t lo = 1;
    for (const KernelInfo& ki : k.tiny) {
      e = occupancy_of(ki, &sms, &occ);
      if (e) return e;
      sa.min_len = lo;
      sa.max_len = (uint64_t)ki.tile;
      // 8 warps per CTA, 32 segments per warp and round
      e = launch(ki.func, (int)std::min<int64_t>((num_segments + 255) / 256, (int64_t)sms * occ), 256, 0, false, &sa,
                 stream);
      if (e) return e;
      lo = (uint64_t)ki.tile + 1;
    }
    const int64_t want = (num_segments + 7) / 8;
    if (k.small_warp8.func != nullptr) {  // one warp, 8 items per thread, before the 16-item shape
      e = occupancy_of(k.small_warp8, &sms, &occ);
      if (e) return e;
      sa.min_len = lo;
      sa.max_len = (uint64_t)k.small_warp8.tile;
      e = launch(k.small_warp8.func, (int)std::min<int64_t>(want, (int64_t)sms * occ), 256, k.small_warp8.smem,
                 false, &sa, stream);
      if (e) return e;
      lo = std::max<uint64_t>(lo, (uint64_t)k.small_warp8.tile + 1);
    }
    e = occupancy_of(k.small_warp, &sms, &occ);
    if (e) return e;
    sa.min_len = lo;
    sa.max_len = (uint64_t)k.small_warp.tile;
    e = launch(k.small_warp.func, (int)std::min<int64_t>(want, (int64_t)sms * occ), 256, k.small_warp.smem, false,
               &sa, stream);
    if (e) return e;
    // groups of 2 and 4 warps (four and two per CTA) for the middle lengths
    const KernelInfo* mids[2] = {&k.small_2warps, &k.small_4warps};
    lo = std::max<uint64_t>(lo, (uint64_t)k.small_warp.tile + 1);
    for (int m = 0; m < 2; ++m) {
      const KernelInfo& ki = *mids[m];
      e = occupancy_of(ki, &sms, &occ);
      if (e) return e;
      sa.min_len = lo;
      sa.max_len = (uint64_t)ki.tile;
      const int64_t groups_per_cta = 4 >> m;
      e = launch(ki.func, (int)std::min<int64_t>((num_segments + groups_per_cta - 1) / groups_per_cta,
                                                 (int64_t)sms * occ),
                 256, ki.smem, false, &sa, stream);
      if (e) return e;
      lo = (uint64_t)ki.tile + 1;
    }
    e = occupancy_of(k.small_block, &sms, &occ);
    if (e) return e;
    sa.min_len = lo;
    sa.max_len = (uint64_t)k.small_block.tile;
    e = launch(k.small_block.func, (int)std::min<int64_t>(num_segments, (int64_t)sms * occ), 256,
               k.small_block.smem, false, &sa, stream);
    if (e) return e;
    e = occupancy_of(k.small_block2, &sms, &occ);
    if (e) return e;
    sa.min_len = (uint64_t)k.small_block.tile + 1;
    sa.max_len = small_cap;
    e = launch(k.small_block2.func, (int)std::min<int64_t>(num_segments, (int64_t)sms * occ), 256,
               k.small_block2.smem, false, &sa, stream);
    if (e) return e;
  }

  // 2. long segments: zero control/counts/descriptors, plan, count, scan
  {
    InitArgs ia;
    ia.ptr = d_temp;
    ia.n16 = L.zero_end / 16;
    cudaError_t e = launch(get_init_kernel(), (int)std::min<uint64_t>((uint64_t)init_grid_cap, (ia.n16 + 511) / 512), 512, 0,
                           false, &ia, stream);
    if (e) return e;
    SegPlanArgs pa = {};
    pa.begin_offsets = bo;
    pa.end_offsets = eo;
    pa.num_segments = (uint64_t)num_segments;
    pa.min_len = small_cap;
    pa.tile = (uint32_t)k.onesweep.tile;
    pa.max_slots = (uint32_t)L.max_slots;
    pa.max_tiles = (uint32_t)L.max_tiles;
    pa.recs = reinterpret_cast<SegRecord*>(t + L.recs);
    pa.tile_slot = reinterpret_cast<uint32_t*>(t + L.tile_slot);
    pa.ctl = ctl;
    pa.status = status;
    e = launch(get_seg_plan_kernel(), (int)std::min<int64_t>((num_segments + 255) / 256, 4096), 256, 0, true, &pa,
               stream);
    if (e) return e;
    SegHistArgs ha = {};
    ha.keys = kin;
    ha.recs = pa.recs;
    ha.tile_slot = pa.tile_slot;
    ha.ctl = ctl;
    ha.seg_hist = t + L.hist;
    ha.tw_c = tw_c;
    ha.tw_f = tw_f;
    ha.tile = (uint32_t)k.onesweep.tile;
    ha.begin_bit = (uint32_t)begin_bit;
    ha.passes = P;
    ha.last_mask = last_mask;
    e = occupancy_of(k.hist, &sms, &occ);
    if (e) return e;
    e = launch(k.hist.func, (int)std::min<uint64_t>((uint64_t)sms * occ, L.max_tiles), 512,
               (size_t)P * kRadix * kSegHistReplicas * 4, true, &ha, stream);
    if (e) return e;
    e = launch(k.scan.func, (int)std::min<uint64_t>((uint64_t)sms * 8, L.max_slots * P), 256, 0, true, &ha, stream);
    if (e) return e;
  }

  // 3. one segmented onesweep pass per digit; the last one writes the output
  {
    cudaError_t e = occupancy_of(k.onesweep, &sms, &occ);
    if (e) return e;
    const void* ks = kin;
    const void* vs = vin;
    for (uint32_t p = 0; p < P; ++p) {
      const bool to_out = ((P - 1 - p) & 1u) == 0;
      SegOnesweepArgs a;
      std::memset(&a, 0, sizeof(a));
      a.keys_in = ks;
      a.keys_out = to_out ? kout : static_cast<void*>(t + L.stage_k);
      a.vals_in = vb ? vs : nullptr;
      a.vals_out = vb ? (to_out ? vout : static_cast<void*>(t + L.stage_v)) : nullptr;
      a.n = nn;
      a.tw_c = tw_c;
      a.tw_f = tw_f;
      a.shift = (uint32_t)begin_bit + 8u * p;
      a.mask = (p + 1 == P) ? last_mask : 0xffu;
      a.pass = p;
      a.num_tiles = (uint32_t)L.max_tiles;
      a.desc = t + L.desc;
      a.g_hist_pass = nullptr;
      a.tile_counter = counters + p;
      a.status = status;
      a.spin_limit_ns = wait_limit_ns();
      a.skip_tile = -1;
      // TMA tile loads where a tile starts 16-byte aligned (checked per tile)
      const size_t tile_k = (size_t)k.onesweep.tile * kb, tile_v = (size_t)k.onesweep.tile * vb;
      a.tma_keys = (tile_k & 15) == 0 ? 1u : 0u;
      a.tma_vals = (vb == 0 || (tile_v & 15) == 0) ? 1u : 0u;
      a.recs = reinterpret_cast<const SegRecord*>(t + L.recs);
      a.tile_slot = reinterpret_cast<const uint32_t*>(t + L.tile_slot);
      a.ctl = ctl;
      a.seg_gbase = t + L.hist;
      a.seg_pass = p;
      a.seg_passes = P;
      e = launch(k.onesweep.func, sms * occ, k.onesweep.threads, k.onesweep.smem, true, &a, stream);
      if (e) return e;
      ks = a.keys_out;
      vs = a.vals_out;
    }
  }
  return cudaSuccess;
}

}  // namespace
}  // namespace cusort_b200

extern "C" {

cudaError_t cusort_segmented_sort_keys(void* d_temp_storage, size_t* temp_storage_bytes, cusort_key_type key_type,
                                       const void* d_keys_in, void* d_keys_out, int64_t num_items,
                                       int64_t num_segments, const int64_t* d_begin_offsets,
                                       const int64_t* d_end_offsets, int begin_bit, int end_bit, int descending,
                                       cudaStream_t stream) {
  return cusort_b200::seg_sort(d_temp_storage, temp_storage_bytes, (int)key_type, 0, descending != 0, d_keys_in,
                               d_keys_out, nullptr, nullptr, num_items, num_segments, d_begin_offsets,
                               d_end_offsets, begin_bit, end_bit, stream);
}

cudaError_t cusort_segmented_sort_pairs(void* d_temp_storage, size_t* temp_storage_bytes, cusort_key_type key_type,
                                        const void* d_keys_in, void* d_keys_out, size_t value_bytes,
                                        const void* d_values_in, void* d_values_out, int64_t num_items,
                                        int64_t num_segments, const int64_t* d_begin_offsets,
                                        const int64_t* d_end_offsets, int begin_bit, int end_bit, int descending,
                                        cudaStream_t stream) {
  if (value_bytes == 0) return cudaErrorInvalidValue;
  return cusort_b200::seg_sort(d_temp_storage, temp_storage_bytes, (int)key_type, value_bytes, descending != 0,
                               d_keys_in, d_keys_out, d_values_in, d_values_out, num_items, num_segments,
                               d_begin_offsets, d_end_offsets, begin_bit, end_bit, stream);
}

}  // extern "C"

// cusort_types.h -- structures shared by the host dispatcher and the kernels.
#pragma once

#include <stdint.h>

namespace cusort_b200 {

constexpr int kRadixBits = 8;
constexpr int kRadix = 256;
constexpr int kMaxPasses = 8;

// Device status bits (written into the control block of the temp storage).
enum : uint32_t {
  kStatusLookbackTimeout = 1u,  // a decoupled-lookback wait ran out of time
  kStatusTmaTimeout = 2u,       // a bulk-copy (TMA) completion wait ran out of time
  kStatusRouteOverflow = 4u,    // a routed store fell outside its destination buffer (skipped)
};

// Routing of a partition pass straight into several destination buffers
// (the multi-GPU exchange).  Digit d belongs to destination q = owner[d]
// (q < kMaxRouteRanks; each destination owns the contiguous digit range
// [first_digit[q], last_digit[q]]).  Destination q receives, from item offset
// base[q] on, every tile's items of its digits: tile by tile, each tile's in
// the tile's stable digit order.  A tile's run that would reach cap[q] items
// is skipped and flagged.
constexpr int kMaxRouteRanks = 64;
struct RouteTable {
  unsigned long long base[kMaxRouteRanks];
  unsigned long long kptr[kMaxRouteRanks];
  unsigned long long vptr[kMaxRouteRanks];
  unsigned long long cap[kMaxRouteRanks];
  unsigned int first_digit[kMaxRouteRanks];
  unsigned int last_digit[kMaxRouteRanks];
  unsigned char owner[256];
};

// Descriptor state, stored in the top two bits of each (tile, digit) word as
// (2*pass + state) mod 4.  After pass p every word is INCLUSIVE(p), which
// decodes as EMPTY in pass p+1, so descriptors are zeroed once per sort.
enum : uint32_t { kDescEmpty = 0u, kDescAggregate = 1u, kDescInclusive = 2u };

struct InitArgs {
  void* ptr;      // 16-byte aligned
  uint64_t n16;   // number of 16-byte words to zero
};

struct HistArgs {
  const void* keys;
  uint64_t n;
  uint64_t tw_c, tw_f;     // twiddle constants (see dev::twiddle)
  uint32_t begin_bit;
  uint32_t num_passes;
  uint32_t last_mask;      // digit mask of the last pass
  void* g_hist;            // OffsetT[num_passes * 256]
};

struct FillArgs {
  const void* counts;  // OffsetT[256] digit counts
  void* out;           // n bytes
  uint64_t n;
  uint32_t xor_c;      // key = digit ^ xor_c (1-byte keys have no float twiddle)
};

// 16-bit keys-only sorts over all 16 bits: one 16-bit digit (65536 bins).
// hist16: counts of the twiddled keys and of each group of 256 bins; each CTA
// counts one half of the bins (blockIdx.x & 1) over its share of the keys.
// fill16: the output is every key value repeated by its count.
struct Fill16Args {
  const void* keys;    // hist16: n 2-byte keys
  void* counts;        // OffsetT[65536], zeroed by the init kernel
  void* groups;        // OffsetT[256]: items per group of 256 bins, zeroed
  void* out;           // fill16: n 2-byte keys
  uint64_t n;
  uint32_t xor_c;      // twiddled key = key ^ xor_c (2-byte keys have no float twiddle)
  uint32_t pad;
};

struct OnesweepArgs {
  const void* keys_in;
  void* keys_out;
  const void* vals_in;
  void* vals_out;
  uint64_t n;
  uint64_t tw_c, tw_f;
  uint32_t shift;          // first bit of this pass's digit
  uint32_t mask;           // digit mask (255, or smaller on a partial last pass)
  uint32_t pass;
  uint32_t num_tiles;
  void* desc;              // OffsetT[num_tiles * 256], shared by all passes
  const void* g_hist_pass; // OffsetT[256] digit counts of this pass; routed kernels: the RouteTable
  uint32_t* tile_counter;  // dynamic tile ticket of this pass
  uint32_t* status;        // device status word
  uint64_t spin_limit_ns;  // bound on every wait
  int64_t skip_tile;       // fault injection: tile that never publishes (-1 = off)
  uint32_t tma_keys;       // keys_in/keys_out 16-byte aligned -> TMA tile loads
  uint32_t tma_vals;
};

// Segmented sort: a segment longer than one small-sort block is cut into
// onesweep tiles that never straddle segments.  One record per such segment
// (index = its slot): first item, length, index of its first tile.
struct SegRecord {
  uint64_t begin;
  uint64_t len;
  uint32_t tile_first;
  uint32_t pad;
};

// Planner output and counters of a segmented sort (device memory).
struct SegControl {
  uint32_t num_tiles;  // tiles of all multi-tile segments
  uint32_t num_slots;  // multi-tile segments
  uint32_t pad[2];
};

// Onesweep pass over the tiles of multi-tile segments: each tile's segment,
// per-segment digit bases instead of one global histogram, and a lookback
// that stops at the segment's first tile.
struct SegOnesweepArgs : OnesweepArgs {
  const SegRecord* recs;
  const uint32_t* tile_slot;     // per tile: slot of its segment
  const SegControl* ctl;         // num_tiles (written by the planner)
  const void* seg_gbase;         // OffsetT[slot][passes][256]: segment begin + exclusive digit prefix
  uint32_t seg_pass;             // index of this pass in seg_gbase
  uint32_t seg_passes;
};

// Small-segment sorts and the planner.
struct SegSmallArgs {
  const void* keys_in;
  void* keys_out;
  const void* vals_in;
  void* vals_out;
  const int64_t* begin_offsets;
  const int64_t* end_offsets;
  uint64_t num_segments;
  uint64_t min_len, max_len;     // this kernel sorts segments with min_len <= len <= max_len
  uint64_t tw_c, tw_f;
  uint32_t begin_bit, passes, last_mask;
  uint32_t pad;
};

struct SegPlanArgs {
  const int64_t* begin_offsets;
  const int64_t* end_offsets;
  uint64_t num_segments;
  uint64_t min_len;              // segments longer than this are tiled
  uint32_t tile;                 // items per onesweep tile
  uint32_t max_slots, max_tiles; // capacity of recs / tile_slot (bounds-checked)
  SegRecord* recs;
  uint32_t* tile_slot;
  SegControl* ctl;
  uint32_t* status;
};

struct SegHistArgs {
  const void* keys;
  const SegRecord* recs;
  const uint32_t* tile_slot;
  const SegControl* ctl;
  void* seg_hist;                // OffsetT[slot][passes][256], zeroed; scanned in place by seg_scan
  uint64_t tw_c, tw_f;
  uint32_t tile, begin_bit, passes, last_mask;
};

}  // namespace cusort_b200

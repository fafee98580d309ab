// cusort_dispatch.h -- internal host-side interface between the dispatcher
// and the per-key-width kernel instantiation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

struct cusort_double_buffer;

#ifndef CUSORT_SMALL_TILE_MAX_ITEMS
#define CUSORT_SMALL_TILE_MAX_ITEMS (1ull << 20)
#endif
#ifndef CUSORT_MID_TILE_MAX_ITEMS
#define CUSORT_MID_TILE_MAX_ITEMS (1ull << 23)
#endif

namespace cusort_b200 {

struct KernelInfo {
  const void* func = nullptr;  // __global__ function
  int threads = 0;             // CTA size
  int tile = 0;                // items per tile (onesweep) / vectors per CTA step (histogram)
  size_t smem = 0;             // dynamic shared memory bytes
};

// One entry per key width; value bytes in {0,1,2,4,8,16}, off_bytes in {4,8};
// float_key selects the floating-point twiddle (4- and 8-byte keys only).
bool get_kernels_k1(int value_bytes, int off_bytes, bool float_key, KernelInfo* onesweep, KernelInfo* histogram);
bool get_kernels_k2(int value_bytes, int off_bytes, bool float_key, KernelInfo* onesweep, KernelInfo* histogram);
bool get_kernels_k4(int value_bytes, int off_bytes, bool float_key, KernelInfo* onesweep, KernelInfo* histogram);
bool get_kernels_k8(int value_bytes, int off_bytes, bool float_key, KernelInfo* onesweep, KernelInfo* histogram);
// Smaller-tile onesweep kernels (32-bit offsets) for sorts of at most
// kSmallTileMaxItems (tier 0) or kMidTileMaxItems (tier 1) items; false where
// the key/value widths have none (kernels_small.cu).
constexpr uint64_t kSmallTileMaxItems = CUSORT_SMALL_TILE_MAX_ITEMS;
constexpr uint64_t kMidTileMaxItems = CUSORT_MID_TILE_MAX_ITEMS;
static_assert(kSmallTileMaxItems <= kMidTileMaxItems && kMidTileMaxItems < (1ull << 30),
              "smaller-tile kernels use 32-bit offsets");
bool get_small_onesweep(int key_bytes, int value_bytes, bool float_key, int tier, KernelInfo* onesweep);
// Routed onesweep kernels (kernels_routed_*.cu): the multi-GPU partition pass.
bool get_routed_k12(int key_bytes, int value_bytes, int off_bytes, bool float_key, KernelInfo* onesweep);
bool get_routed_k4(int value_bytes, int off_bytes, bool float_key, KernelInfo* onesweep);
bool get_routed_k8(int value_bytes, int off_bytes, bool float_key, KernelInfo* onesweep);
// Segmented-sort kernels (kernels_seg_*.cu; cusort_segmented.cuh).
struct SegKernels {
  KernelInfo onesweep, hist, scan, small_warp, small_2warps, small_4warps, small_block;
  KernelInfo small_block2;  // one CTA per segment, twice small_block's items per thread
  KernelInfo small_warp8;   // one warp per segment, 8 items per thread (func null where small_warp has <= 8)
  KernelInfo tiny[2];  // all-pairs rank, 1 and 4 items per lane (capacity in .tile)
};
bool get_segmented_k12(int key_bytes, int value_bytes, int off_bytes, bool float_key, SegKernels* k);
bool get_segmented_k4(int value_bytes, int off_bytes, bool float_key, SegKernels* k);
bool get_segmented_k8(int value_bytes, int off_bytes, bool float_key, SegKernels* k);
const void* get_seg_plan_kernel();
const void* get_seg_copy_kernel(int bytes);
const void* get_init_kernel();
// Count-and-fill kernel of 1-byte keys-only full-range sorts (kernels_k1.cu).
const void* get_fill_bytes_kernel(int off_bytes);
// 16-bit-digit count and fill kernels of 2-byte keys-only full-range sorts
// (kernels_k2.cu).
bool get_fill16_kernels(int off_bytes, KernelInfo* hist, KernelInfo* fill);

// DoubleBuffer sort with `scratch` as its temp storage (cusort_api.cu).
cudaError_t sort_db_in_scratch(void* scratch, size_t scratch_bytes, int key_type, size_t value_bytes, bool descending,
                               struct cusort_double_buffer* keys, struct cusort_double_buffer* values,
                               int64_t num_items, int begin_bit, int end_bit, cudaStream_t stream);

// In/out-pointer SortPairs without the index-path choice below
// (cusort_api.cu).
cudaError_t sort_pairs_direct(void* d_temp, size_t* temp_bytes, int key_type, const void* keys_in,
                              void* keys_out, size_t value_bytes, const void* values_in, void* values_out,
                              int64_t num_items, int begin_bit, int end_bit, bool descending, cudaStream_t stream);
// SortPairs as the keys with their input positions, then the values gathered
// through the sorted positions (cusort_wide.cu): any value width.
cudaError_t sort_pairs_by_index(void* d_temp, size_t* temp_bytes, int key_type, const void* keys_in,
                                void* keys_out, size_t value_bytes, const void* values_in, void* values_out,
                                int64_t num_items, int begin_bit, int end_bit, int descending, cudaStream_t stream);

// CUSORT_WIDE_OFFSETS=1 in the environment: sorts of any size use the 64-bit
// offset kernels (cusort_api.cu; a test hook).
bool force_wide_offsets();

// Single-digit counts (u64[256]) of the twiddled keys (cusort_api.cu).
cudaError_t digit_counts_u64(int key_type, bool descending, const void* keys, int64_t num_items, int begin_bit,
                             int end_bit, unsigned long long* d_counts, cudaStream_t stream);

// Twiddle constants of a key type (cusort_api.cu) and the calling thread's
// bound on device-side waits (cusort_set_wait_limit_ns).
void twiddle_constants_of(int key_type, bool descending, uint64_t* c, uint64_t* f);
uint64_t wait_limit_ns();
// Resident CTAs per SM of a kernel on the current device (cached).
cudaError_t occupancy_of(const KernelInfo& k, int* sms, int* ctas_per_sm);

struct RouteTable;
// One stable partition pass over the digit [begin_bit, end_bit) (at most 8
// bits) whose write-out goes straight to route->kptr/vptr[owner[d]] at
// route->base[d] + (rank of the item among this call's items of digit d):
// the fused partition + exchange of the multi-GPU sort.  `d_route` is device
// memory.  wide_offsets selects 64-bit offsets (destinations >= 2^32 items).
// With d_temp == nullptr only *temp_bytes is set (cusort_api.cu).  keep_status
// leaves the status word of d_temp as earlier passes left it.
cudaError_t routed_partition(int key_type, size_t value_bytes, bool descending, const void* keys, const void* values,
                             int64_t num_items, int begin_bit, int end_bit, bool wide_offsets,
                             const RouteTable* d_route, void* d_temp, size_t* temp_bytes, cudaStream_t stream,
                             bool keep_status = false);

}  // namespace cusort_b200

/* cusort_b200.h -- C ABI of the B200-native LSD radix sort.
 *
 * Drop-in boundary for cusort::DeviceRadixSort (IlyaGrebnov/libcusort 1.0.1,
 * libcusort.cuh).  The reference is a header-only C++ template library; the
 * eight public overloads of DeviceRadixSort map one-to-one onto the eight
 * sort entry points below, with the key type passed as a tag and the value
 * type by its size (the reference itself maps values to uint8/16/32/64 or
 * ulonglong2 by size, libcusort.cuh:2942-2953).  include/cusort_b200.cuh puts
 * the reference's C++ templates (cusort::DoubleBuffer,
 * cusort::DeviceRadixSort) back on top of these symbols.
 *
 * Semantics kept from the reference:
 *   - d_temp_storage == NULL only writes *temp_storage_bytes and makes no
 *     CUDA call (libcusort.cuh:2609-2613); trivial calls (num_items <= 1 or
 *     begin_bit == end_bit) report 0 bytes, or 1 for the in/out-pointer form
 *     with num_items > 0 (libcusort.cuh:2914-2919).
 *   - DoubleBuffer form: both buffers are clobbered; afterwards each selector
 *     is flipped once per 8-bit pass, i.e. selector ^= (passes & 1)
 *     (libcusort.cuh:2685).
 *   - In/out-pointer form: the result is in *_out, *_in is never written
 *     (libcusort.cuh:2637-2641, 2668-2672); trivial calls copy in -> out.
 *   - Stable; key order is the unsigned order of the twiddled key bits in
 *     [begin_bit, end_bit) (signed: sign bit flipped; float/double: IEEE
 *     total order, -0.0 < +0.0, NaN payloads kept; descending inverts the
 *     bits, equal keys keep input order).
 *   - cudaErrorInvalidValue when begin_bit < 0, end_bit < 0,
 *     begin_bit > end_bit or end_bit > 8*sizeof(key) (libcusort.cuh:2908).
 *   - Asynchronous on `stream`; no host synchronisation.
 * Differences (stricter): an unknown key type, a value size outside
 * {1,2,4,8,16}, a NULL temp_storage_bytes pointer, a temp_storage_bytes
 * below the size this library reported, or a d_temp_storage that is not
 * 16-byte aligned (cudaMalloc'd memory always is) returns
 * cudaErrorInvalidValue.
 *
 * All pointers are device pointers, naturally aligned for their element
 * type.  The library allocates no device memory.
 */
#ifndef CUSORT_B200_H
#define CUSORT_B200_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Key types of DeviceRadixSort (libcusort.cuh:2853: 1/2/4/8-byte arithmetic). */
typedef enum cusort_key_type {
  CUSORT_KEY_U8 = 0,
  CUSORT_KEY_I8 = 1,
  CUSORT_KEY_U16 = 2,
  CUSORT_KEY_I16 = 3,
  CUSORT_KEY_U32 = 4,
  CUSORT_KEY_I32 = 5,
  CUSORT_KEY_U64 = 6,
  CUSORT_KEY_I64 = 7,
  CUSORT_KEY_F32 = 8,
  CUSORT_KEY_F64 = 9
} cusort_key_type;

/* Same layout as cusort::DoubleBuffer<T> (libcusort.cuh:156-184). */
typedef struct cusort_double_buffer {
  void* d_buffers[2];
  int selector;
} cusort_double_buffer;

/* ---- DoubleBuffer overloads ------------------------------------------- */

/* DeviceRadixSort::SortKeys(temp, bytes, DoubleBuffer<K>&, n, begin, end, stream)
 * (libcusort.cuh:3004-3016). */
cudaError_t cusort_sort_keys_db(void* d_temp_storage, size_t* temp_storage_bytes, cusort_key_type key_type,
                                cusort_double_buffer* d_keys, int64_t num_items, int begin_bit, int end_bit,
                                cudaStream_t stream);

/* DeviceRadixSort::SortKeysDescending, DoubleBuffer (libcusort.cuh:3019-3031). */
cudaError_t cusort_sort_keys_descending_db(void* d_temp_storage, size_t* temp_storage_bytes,
                                           cusort_key_type key_type, cusort_double_buffer* d_keys,
                                           int64_t num_items, int begin_bit, int end_bit, cudaStream_t stream);

/* DeviceRadixSort::SortPairs(temp, bytes, DoubleBuffer<K>&, DoubleBuffer<V>&, n, ...)
 * (libcusort.cuh:2972-2984); value_bytes = sizeof(V). */
cudaError_t cusort_sort_pairs_db(void* d_temp_storage, size_t* temp_storage_bytes, cusort_key_type key_type,
                                 cusort_double_buffer* d_keys, size_t value_bytes, cusort_double_buffer* d_values,
                                 int64_t num_items, int begin_bit, int end_bit, cudaStream_t stream);

/* DeviceRadixSort::SortPairsDescending, DoubleBuffer (libcusort.cuh:2988-3000). */
cudaError_t cusort_sort_pairs_descending_db(void* d_temp_storage, size_t* temp_storage_bytes,
                                            cusort_key_type key_type, cusort_double_buffer* d_keys,
                                            size_t value_bytes, cusort_double_buffer* d_values,
                                            int64_t num_items, int begin_bit, int end_bit, cudaStream_t stream);

/* ---- in/out-pointer overloads ------------------------------------------ */

/* DeviceRadixSort::SortKeys(temp, bytes, const K* in, K* out, n, ...)
 * (libcusort.cuh:3035-3048). */
cudaError_t cusort_sort_keys(void* d_temp_storage, size_t* temp_storage_bytes, cusort_key_type key_type,
                             const void* d_keys_in, void* d_keys_out, int64_t num_items, int begin_bit,
                             int end_bit, cudaStream_t stream);

/* DeviceRadixSort::SortKeysDescending, in/out (libcusort.cuh:3052-3065). */
cudaError_t cusort_sort_keys_descending(void* d_temp_storage, size_t* temp_storage_bytes,
                                        cusort_key_type key_type, const void* d_keys_in, void* d_keys_out,
                                        int64_t num_items, int begin_bit, int end_bit, cudaStream_t stream);

/* DeviceRadixSort::SortPairs(temp, bytes, const K*, K*, const V*, V*, n, ...)
 * (libcusort.cuh:3070-3085). */
cudaError_t cusort_sort_pairs(void* d_temp_storage, size_t* temp_storage_bytes, cusort_key_type key_type,
                              const void* d_keys_in, void* d_keys_out, size_t value_bytes,
                              const void* d_values_in, void* d_values_out, int64_t num_items, int begin_bit,
                              int end_bit, cudaStream_t stream);

/* DeviceRadixSort::SortPairsDescending, in/out (libcusort.cuh:3089-3104). */
cudaError_t cusort_sort_pairs_descending(void* d_temp_storage, size_t* temp_storage_bytes,
                                         cusort_key_type key_type, const void* d_keys_in, void* d_keys_out,
                                         size_t value_bytes, const void* d_values_in, void* d_values_out,
                                         int64_t num_items, int begin_bit, int end_bit, cudaStream_t stream);

/* ---- payloads of any width (the reference caps values at 16 bytes,
 *      libcusort.cuh:2854) ----------------------------------------------
 * Sorts the keys together with their input index, then gathers the payload
 * rows (value_bytes each, any size >= 1) by that permutation.  Same ordering,
 * stability and in/out semantics as cusort_sort_pairs[_descending]; two-phase
 * temp protocol. */
cudaError_t cusort_sort_pairs_wide(void* d_temp_storage, size_t* temp_storage_bytes, cusort_key_type key_type,
                                   const void* d_keys_in, void* d_keys_out, size_t value_bytes,
                                   const void* d_values_in, void* d_values_out, int64_t num_items, int begin_bit,
                                   int end_bit, int descending, cudaStream_t stream);

/* ---- pairs held in host memory ---------------------------------------
 * No counterpart in the reference (which sorts device memory only).  Sorts
 * (keys, values) that live in HOST memory: h_keys_in / h_values_in are read,
 * h_keys_out / h_values_out written (page-locked memory lets the copies run
 * asynchronously and overlap).  The keys go up first and are sorted with their
 * 32-bit input positions while the values go up; the sorted keys come down
 * while the values are gathered through those positions, then the values come
 * down.  Same ordering, stability and bit-range semantics as
 * cusort_sort_pairs[_descending]; value_bytes 1, 2, 4, 8 or 16; num_items <
 * 2^32.  d_temp_storage is DEVICE memory (two-phase size query as elsewhere).
 * All work is ordered on `stream`: synchronise it before reading the host
 * outputs. */
cudaError_t cusort_sort_pairs_host(void* d_temp_storage, size_t* temp_storage_bytes, cusort_key_type key_type,
                                   const void* h_keys_in, void* h_keys_out, size_t value_bytes,
                                   const void* h_values_in, void* h_values_out, int64_t num_items, int begin_bit,
                                   int end_bit, int descending, cudaStream_t stream);

/* ---- sorting without any device allocation ----------------------------
 * No counterpart in the reference (which always takes temp storage from the
 * caller).  For callers that cannot allocate device memory when they need to
 * sort: a custom allocator or memory-pool hook sorting its own bookkeeping
 * (allocating from inside it would re-enter the allocator), a plugin in a host
 * process that has reserved all device memory up front, or a latency-bound
 * loop where cudaMalloc would synchronise the device.
 *
 * Sorts a DoubleBuffer of keys (value_bytes == 0, d_values may be NULL) or of
 * key/value pairs (value_bytes 1, 2, 4, 8 or 16), ascending or descending
 * (`descending` != 0), exactly like cusort_sort_keys_db / cusort_sort_pairs_db
 * (same results, same selector updates), but its temp storage is one fixed
 * array of CUSORT_NOALLOC_SCRATCH_BYTES that the library keeps in device
 * memory.  It calls no cudaMalloc, cudaFree or allocating library routine.
 *   - Limit: a call whose temp storage would exceed the array returns
 *     cudaErrorInvalidValue and does nothing.  The temp storage is about
 *     1 KiB per tile (2 KiB from 2^30 items on) plus a few KiB, a tile being
 *     4096 to 18432 items by key and value width (e.g. 2^26 32-bit keys, or
 *     2^25 32-bit keys with 32-bit values, fit in 4 MiB).
 *   - The array occupies CUSORT_NOALLOC_SCRATCH_BYTES on every GPU whose
 *     context loads this library's device code, until the process exits:
 *     under lazy module loading (the CUDA default) only once this entry point
 *     has run there; with CUDA_MODULE_LOADING=EAGER on every GPU that uses
 *     the library at all.
 *   - The first call on each device looks up the array's device address
 *     (cudaGetSymbolAddress) and keeps it; make that first call before any
 *     stream capture.  A device reset (cudaDeviceReset) between calls is not
 *     supported: the kept address would belong to the old context.
 *   - All calls share the one array and it keeps the last call's contents:
 *     calls whose GPU work can overlap (other streams, other host threads on
 *     the same device) race on it and corrupt each other's results, so
 *     serialise them (e.g. one stream). */
#define CUSORT_NOALLOC_SCRATCH_BYTES (4u << 20)
cudaError_t cusort_sort_db_noalloc(cusort_key_type key_type, cusort_double_buffer* d_keys, size_t value_bytes,
                                   cusort_double_buffer* d_values, int64_t num_items, int begin_bit, int end_bit,
                                   int descending, cudaStream_t stream);

/* ---- segmented sort ----------------------------------------------------
 * The reference names segmented sorting in its banner (libcusort.cuh:4) but
 * implements none; the interface follows CUB's DeviceSegmentedRadixSort.
 * Every segment [d_begin_offsets[s], d_end_offsets[s]) of the input is sorted
 * independently and stably (same key order, bit range and direction rules as
 * cusort_sort_keys / cusort_sort_pairs) into the same positions of the
 * output.  Positions outside every segment are not written; end <= begin is
 * an empty segment; segments must not overlap (overlap that exceeds the
 * planned work sets status bit 3, value 8, and leaves the long segments
 * unsorted).  Offsets are int64 arrays in device memory.  Two-phase temp
 * protocol; the size depends only on num_items, the key/value types and the
 * bit range, not on the offsets, and no call synchronises the stream.
 * Segments of up to a few thousand items are sorted in one warp or one CTA
 * (every pass in shared memory); longer ones by onesweep passes whose tiles
 * never straddle a segment. */
cudaError_t cusort_segmented_sort_keys(void* d_temp_storage, size_t* temp_storage_bytes, cusort_key_type key_type,
                                       const void* d_keys_in, void* d_keys_out, int64_t num_items,
                                       int64_t num_segments, const int64_t* d_begin_offsets,
                                       const int64_t* d_end_offsets, int begin_bit, int end_bit, int descending,
                                       cudaStream_t stream);
cudaError_t cusort_segmented_sort_pairs(void* d_temp_storage, size_t* temp_storage_bytes, cusort_key_type key_type,
                                        const void* d_keys_in, void* d_keys_out, size_t value_bytes,
                                        const void* d_values_in, void* d_values_out, int64_t num_items,
                                        int64_t num_segments, const int64_t* d_begin_offsets,
                                        const int64_t* d_end_offsets, int begin_bit, int end_bit, int descending,
                                        cudaStream_t stream);

/* ---- sharded multi-GPU sort over NCCL (no counterpart in the reference,
 *      which is single-GPU only) ------------------------------------------
 * One process (or thread) per GPU.  Rank r passes its contiguous slice of
 * the global input (global order = rank-major, then local index); it gets
 * back a contiguous part of the globally sorted sequence (ranks' outputs
 * concatenated in rank order are the global result), stable by global index.
 * Steps: most-significant-digit counts, ncclAllGather of G x 256 counts, a
 * digit -> owner plan computed identically on every rank, one stable
 * partition pass whose stores go straight into the owning ranks' output
 * buffers over NVLink (peer memory mapped through CUDA IPC; fenced by a
 * one-word ncclAllReduce), and a stable local sort of the received items.
 * Environment CUSORT_MGPU_EXCHANGE=copy|nccl (or a rank whose buffers cannot
 * be mapped) selects a local partition pass followed by copy-engine pushes
 * or grouped ncclSend/ncclRecv instead.  The output buffers are written by
 * other ranks' kernels: they must be device allocations (cudaMalloc or a
 * caching allocator over it) and must not be used from other streams while a
 * call runs.
 *
 * cusort_mgpu_unique_id: on one rank; the caller broadcasts the 128 bytes.
 * cusort_mgpu_comm_init: every rank, with its GPU current.
 * cusort_mgpu_plan: host-only planning step (exposed for tests and tools):
 *   all_counts[r*256 + d] = rank r's count of owner digit d; fills the digit
 *   owners (256), this rank's send and receive counts per peer, and every
 *   rank's receive total.  Returns 0 on success.
 * cusort_mgpu_sort: two-phase temp protocol as the single-GPU calls (the size
 *   depends on the communicator's size, n_local and out_capacity).  It
 *   waits on the host once (for the gathered counts).  Returns
 *   cudaErrorInvalidValue on every rank, before any data exchange, when some
 *   rank's share would exceed out_capacity.  *n_out receives this rank's
 *   item count.  value_bytes 0 = keys only.
 *
 * Failure handling (no reference counterpart: the reference is single-GPU and
 * its only wait is an unbounded lookback spin, libcusort.cuh:1360-1374).  The
 * communicator is non-blocking and every host wait of the library is bounded
 * by the communicator's limit (default 30 s): joining in
 * cusort_mgpu_comm_init, the gathered counts inside cusort_mgpu_sort, each
 * NCCL call being issued, and cusort_mgpu_wait.  When a limit passes or NCCL
 * reports an asynchronous error (a rank that left, a broken connection), the
 * communicator is aborted (ncclCommAbort: NCCL kernels still waiting for a
 * peer give up), the call returns cudaErrorTimeout (or the mapped NCCL
 * error), every later call on that communicator returns cudaErrorTimeout at
 * once, and cusort_mgpu_comm_destroy only frees the handle.
 * cusort_mgpu_set_timeout_ns: that limit, per communicator.
 * cusort_mgpu_wait: bounded host wait for all work queued on `stream` so far
 *   (the exchange's fence collective and the local sort included); use it in
 *   place of cudaStreamSynchronize to learn of a peer's failure. */
cudaError_t cusort_mgpu_unique_id(unsigned char* id128);
cudaError_t cusort_mgpu_comm_init(void** comm, const unsigned char* id128, int nranks, int rank);
cudaError_t cusort_mgpu_comm_destroy(void* comm);
int cusort_mgpu_plan(const uint64_t* all_counts, int nranks, int rank, int* digit_owner, int64_t* send_counts,
                     int64_t* recv_counts, int64_t* recv_totals);
cudaError_t cusort_mgpu_sort(void* comm, void* d_temp_storage, size_t* temp_storage_bytes, cusort_key_type key_type,
                             size_t value_bytes, const void* d_keys_in, const void* d_values_in, int64_t n_local,
                             void* d_keys_out, void* d_values_out, int64_t out_capacity, int64_t* n_out,
                             int begin_bit, int end_bit, int descending, cudaStream_t stream);
cudaError_t cusort_mgpu_set_timeout_ns(void* comm, uint64_t ns);
cudaError_t cusort_mgpu_wait(void* comm, cudaStream_t stream);

/* Phase times of this host thread's last cusort_mgpu_sort call, measured with
 * CUDA events on its stream while timing is on (cusort_mgpu_set_timing(1), per
 * host thread; returns the previous setting).  With timing on, each call
 * waits for its own last phase before returning.  cusort_mgpu_get_phase_times
 * fills up to `capacity` (ms, name) pairs -- names are static strings such as
 * "counts+gather", "host", "routed-pass", "exchange", "local-sort" -- and
 * returns how many it filled. */
int cusort_mgpu_set_timing(int enable);
int cusort_mgpu_get_phase_times(float* ms, const char** names, int capacity);

/* ---- library state, status and diagnostics (no reference counterpart;
 *      the reference has compile-time macros only, libcusort.cuh:119-148) -- */

/* "1.0.1-b200.N": reference API version this build is a drop-in for. */
const char* cusort_version(void);

/* Launch modes: 0 = one launch per kernel with programmatic dependent launch
 * (default), 1 = CUDA graph per (device, kernel set, grid) replayed with
 * updated parameters (reference GraphCache, libcusort.cuh:192-225, 2693-2834).
 * Per host thread.  Returns the previous mode. */
int cusort_set_launch_mode(int mode);

/* Device status word of the last sort that used this temp storage:
 * 0 = ok, bit 0 = a lookback wait timed out, bit 1 = a tile-copy wait timed
 * out, bit 2 = (cusort_mgpu_sort temp storage) a partition store fell outside
 * its destination buffer and was skipped, bit 3 = (segmented sort temp
 * storage) the segments needed more work than planned (overlapping segments).
 * Synchronises `stream`. */
cudaError_t cusort_read_device_status(const void* d_temp_storage, uint32_t* status, cudaStream_t stream);

/* Bound on every device-side wait, in nanoseconds (default 2e9).  Per host
 * thread.  Returns the previous value. */
uint64_t cusort_set_wait_limit_ns(uint64_t ns);

/* Fault injection for tests: tile `tile` of every pass never publishes its
 * lookback descriptors (-1 = off, the default).  Per host thread. */
int64_t cusort_debug_set_skip_tile(int64_t tile);

/* Per-kernel timing for the benchmark: when enabled, every sort records CUDA
 * events around each of its kernels on `stream`; cusort_get_kernel_times
 * synchronises on the last event and returns the durations (ms) of the last
 * sort in launch order with kind codes 0 = init, 1 = histogram,
 * 2 = onesweep.  Per host thread. */
int cusort_set_kernel_timing(int enable);
int cusort_get_kernel_times(float* ms, int* kinds, int capacity);

/* Kernel geometry chosen for a call (tile items, passes, CTAs per grid) --
 * used by tests and the benchmark's roofline arithmetic. */
cudaError_t cusort_query_plan(cusort_key_type key_type, size_t value_bytes, int64_t num_items, int begin_bit,
                              int end_bit, int* passes, int* tile_items, int* onesweep_grid,
                              int* histogram_grid, int* offset_bytes);

#ifdef __cplusplus
}
#endif

#endif /* CUSORT_B200_H */

// cusort_mgpu.cu -- sharded multi-GPU sort over NCCL (one process or thread
// per GPU).  No counterpart in the reference, which is single-GPU only.
//
// Every rank holds a contiguous slice of the global input (global index =
// rank-major, then local index).  Per call:
//   1. count the most significant (up to 8-bit) digit of the twiddled keys;
//   2. all-gather the G x 256 counts (ncclAllGather);
//   3. on the host, every rank derives the same digit -> owner plan
//      (cusort_mgpu_plan): digits go to ranks in order, each by the midpoint
//      of its share of the global count, so rank q owns a contiguous digit
//      range and the ranks' outputs concatenate to the global order;
//   4+5. partition the local slice by that digit and exchange it, all-to-all.
//      Default ("routed"): ONE onesweep pass over the digit whose write-out
//      stores, per tile and owner, the tile's (digit-sorted) items of that
//      owner as one contiguous run straight into the owner's receive buffer
//      over NVLink (peer buffers mapped once through CUDA IPC), tiles in
//      order after the runs of lower source ranks.  Long runs keep the
//      remote stores efficient.  A one-word ncclAllReduce then fences the
//      exchange.  CUSORT_MGPU_EXCHANGE=pipe runs the routed pass chunk by
//      chunk (up to 8 chunks of >= 2^24 items), this rank's own items straight
//      into its receive buffer and each peer's into one contiguous staging run
//      per chunk, which the copy engines push into the peer's buffer while the
//      next chunk is partitioned (measured equal to "routed" at 2 GPUs).
//      Fallbacks, chosen when a rank cannot map its buffers (or by
//      CUSORT_MGPU_EXCHANGE=copy|nccl): a local partition pass, then
//      copy-engine pushes into the mapped peer buffers ("copy") or grouped
//      ncclSend/ncclRecv ("nccl"), pieces laid out by source rank;
//   6. stably sort the received items on all key bits.
// In every layout, equal keys (which share the digit) arrive in global input
// order, so they end up in global input order (stable across ranks).
#include <cuda_runtime.h>
#include <nccl.h>

#include <time.h>

#include <algorithm>
#include <cstddef>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <utility>
#include <vector>

#include "../../include/cusort_b200.h"
#include "cusort_dispatch.h"
#include "cusort_types.h"

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

// Pinned host buffer for the gathered counts (per host thread, grown on
// demand): a copy into pageable memory would block the host until it lands.
struct PinnedCounts {
  uint64_t* p = nullptr;
  size_t cap = 0;
  ~PinnedCounts() {
    if (p) cudaFreeHost(p);
  }
  cudaError_t reserve(size_t n) {
    if (n <= cap) return cudaSuccess;
    if (p) cudaFreeHost(p);
    p = nullptr;
    cap = 0;
    cudaError_t e = cudaMallocHost(reinterpret_cast<void**>(&p), n * sizeof(uint64_t));
    if (e == cudaSuccess) cap = n;
    return e;
  }
};
thread_local PinnedCounts g_pinned_counts;

// The handle behind `void* comm`: the NCCL communicator plus the receive
// buffers of peers already mapped through CUDA IPC (opened once, closed when
// the communicator is destroyed).
struct MgpuComm {
  ncclComm_t nccl = nullptr;
  // Bound on every host wait of a call (the gathered counts, a non-blocking
  // NCCL call being issued, cusort_mgpu_wait); on expiry the communicator is
  // aborted and the call returns cudaErrorTimeout.
  uint64_t timeout_ns = 30000000000ull;
  bool aborted = false;  // after ncclCommAbort: every later call fails at once
  cudaEvent_t done = nullptr;  // cusort_mgpu_wait
  std::map<std::pair<int, std::string>, void*> mapped;  // (peer, IPC handle) -> local address
  // pipelined exchange: copy streams (one per peer, up to kMaxCopyStreams) and events
  std::vector<cudaStream_t> copy_streams;
  std::vector<cudaEvent_t> events;
  ~MgpuComm() {
    for (cudaStream_t s : copy_streams) cudaStreamDestroy(s);
    for (cudaEvent_t e : events) cudaEventDestroy(e);
    if (done) cudaEventDestroy(done);
  }
};

uint64_t now_ns() {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return (uint64_t)ts.tv_sec * 1000000000ull + (uint64_t)ts.tv_nsec;
}

void pause_briefly() {
  timespec ts = {0, 20000};  // 20 us between polls
  nanosleep(&ts, nullptr);
}

// Ends the communicator after a failed or expired wait: NCCL kernels still
// waiting for a peer give up, and every later call on it fails at once.
cudaError_t abort_comm(MgpuComm* mc, cudaError_t why) {
  if (!mc->aborted) {
    ncclCommAbort(mc->nccl);
    mc->aborted = true;
  }
  return why;
}

cudaError_t nccl_to_cuda(ncclResult_t r);

// The communicator is non-blocking: an NCCL call may return ncclInProgress
// while it is still being issued.  Polls until it has been (bounded), and
// aborts the communicator on an error or when the limit passes.
cudaError_t settle(MgpuComm* mc, ncclResult_t r) {
  if (r != ncclSuccess && r != ncclInProgress) return abort_comm(mc, nccl_to_cuda(r));
  const uint64_t t0 = now_ns();
  while (r == ncclInProgress) {
    if (ncclCommGetAsyncError(mc->nccl, &r) != ncclSuccess) return abort_comm(mc, cudaErrorUnknown);
    if (r == ncclSuccess) break;
    if (r != ncclInProgress) return abort_comm(mc, nccl_to_cuda(r));
    if (now_ns() - t0 > mc->timeout_ns) return abort_comm(mc, cudaErrorTimeout);
    pause_briefly();
  }
  return cudaSuccess;
}

// Host wait for `ev` (work on the stream, NCCL collectives included), bounded
// by the communicator's limit; an asynchronous NCCL error (a peer that left,
// a broken connection) or the limit aborts the communicator.
cudaError_t wait_event(MgpuComm* mc, cudaEvent_t ev) {
  const uint64_t t0 = now_ns();
  for (;;) {
    const cudaError_t q = cudaEventQuery(ev);
    if (q == cudaSuccess) return cudaSuccess;
    if (q != cudaErrorNotReady) return q;
    ncclResult_t st = ncclSuccess;
    if (ncclCommGetAsyncError(mc->nccl, &st) != ncclSuccess) return abort_comm(mc, cudaErrorUnknown);
    if (st != ncclSuccess && st != ncclInProgress) return abort_comm(mc, nccl_to_cuda(st));
    if (now_ns() - t0 > mc->timeout_ns) return abort_comm(mc, cudaErrorTimeout);
    pause_briefly();
  }
}

// Exchange modes, ordered: the call uses the lowest mode any rank asks for.
enum : unsigned long long { kXchgNccl = 0, kXchgCopy = 1, kXchgRouted = 2, kXchgPipe = 3 };

// Pipelined exchange: the local slice is partitioned in chunks of at least
// 2^24 items (at most kMaxChunks); chunk c's pieces for peers are copied by
// the copy engines while chunk c+1 is partitioned.
constexpr int kMaxChunks = 8;
constexpr int kMaxCopyStreams = 8;
int chunks_for(int64_t n_local) {
  const char* force = std::getenv("CUSORT_MGPU_CHUNKS");  // tests: pipeline small inputs too
  if (force && std::atoi(force) >= 1)
    return (int)std::min<int64_t>(std::min(kMaxChunks, std::atoi(force)), std::max<int64_t>(1, n_local));
  return (int)std::min<int64_t>(kMaxChunks, std::max<int64_t>(1, n_local >> 24));
}

__global__ void sum_chunk_counts_kernel(const unsigned long long* chunk_counts, int chunks, unsigned long long* out) {
  unsigned long long s = 0;
  for (int c = 0; c < chunks; ++c) s += chunk_counts[c * 256 + threadIdx.x];
  out[threadIdx.x] = s;
}

cudaError_t comm_resources(MgpuComm* mc, int streams, int events) {
  while ((int)mc->copy_streams.size() < streams) {
    cudaStream_t s;
    cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
    if (e) return e;
    mc->copy_streams.push_back(s);
  }
  while ((int)mc->events.size() < events) {
    cudaEvent_t ev;
    cudaError_t e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
    if (e) return e;
    mc->events.push_back(ev);
  }
  return cudaSuccess;
}

// Per-rank record all-gathered before the exchange.
struct RankRecord {
  unsigned long long counts[256];
  cudaIpcMemHandle_t hk, hv;   // receive buffers (keys, values) of this rank
  unsigned long long mode;     // kXchg*: highest exchange mode this rank supports
  unsigned long long off_k, off_v;  // receive buffers' offsets inside their allocations
  unsigned long long cap;      // receive capacity (items) of this rank
};
static_assert(sizeof(RankRecord) % 8 == 0, "record layout");

// Allocation base of a device pointer (driver entry point, no link-time
// dependency on libcuda).
cudaError_t allocation_base(const void* p, void** base) {
  typedef int (*GetRangeFn)(unsigned long long*, size_t*, unsigned long long);
  static GetRangeFn fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !f) return cudaErrorNotSupported;
    fn = reinterpret_cast<GetRangeFn>(f);
  }
  unsigned long long b = 0;
  size_t sz = 0;
  if (fn(&b, &sz, reinterpret_cast<unsigned long long>(p)) != 0) return cudaErrorInvalidValue;
  *base = reinterpret_cast<void*>(b);
  return cudaSuccess;
}

// IPC handle + offset of a receive buffer; ok = false if it cannot be shared.
bool export_buffer(const void* p, cudaIpcMemHandle_t* h, unsigned long long* off) {
  std::memset(h, 0, sizeof(*h));
  *off = 0;
  if (!p) return true;  // nothing to receive into (keys-only values slot)
  void* base = nullptr;
  if (allocation_base(p, &base) != cudaSuccess) return false;
  if (cudaIpcGetMemHandle(h, base) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  *off = (unsigned long long)(static_cast<const uint8_t*>(p) - static_cast<const uint8_t*>(base));
  return true;
}

cudaError_t peer_address(MgpuComm* c, int peer, const cudaIpcMemHandle_t& h, unsigned long long off, uint8_t** out) {
  const std::string key(reinterpret_cast<const char*>(&h), sizeof(h));
  auto it = c->mapped.find({peer, key});
  if (it == c->mapped.end()) {
    void* base = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return e;
    it = c->mapped.emplace(std::make_pair(peer, key), base).first;
  }
  *out = static_cast<uint8_t*>(it->second) + off;
  return cudaSuccess;
}

// Phase timing of one call (cusort_mgpu_set_timing(1), per host thread, or
// environment CUSORT_MGPU_TIMING=1): events on the stream at each phase
// boundary; when the call returns the host waits for the last one and keeps
// the phase times for cusort_mgpu_get_phase_times (the environment variable
// also prints them to stderr).
thread_local int g_timing = 0;
struct PhaseRecord {
  int n = 0;
  const char* name[8];
  float ms[8];
};
thread_local PhaseRecord g_last_phases;

struct PhaseTimer {
  static constexpr int kMax = 8;
  bool on = false, print = false;
  cudaStream_t stream = nullptr;
  int n = 0, rank = 0;
  cudaEvent_t ev[kMax];
  const char* name[kMax];
  PhaseTimer(cudaStream_t s, int r) : stream(s), rank(r) {
    const char* v = std::getenv("CUSORT_MGPU_TIMING");
    print = v && v[0] == '1';
    on = print || g_timing;
    if (on) g_last_phases.n = 0;
  }
  void mark(const char* what) {
    if (!on || n >= kMax) return;
    if (cudaEventCreate(&ev[n]) != cudaSuccess) return;
    name[n] = what;
    cudaEventRecord(ev[n], stream);
    ++n;
  }
  ~PhaseTimer() {
    if (!on || n == 0) return;
    if (cudaEventSynchronize(ev[n - 1]) == cudaSuccess) {
      g_last_phases.n = n - 1;
      for (int i = 1; i < n; ++i) {
        float ms = 0.f;
        cudaEventElapsedTime(&ms, ev[i - 1], ev[i]);
        g_last_phases.name[i - 1] = name[i];
        g_last_phases.ms[i - 1] = ms;
      }
      if (print) {
        std::fprintf(stderr, "cusort_mgpu rank %d:", rank);
        for (int i = 0; i < g_last_phases.n; ++i)
          std::fprintf(stderr, " %s %.3f", g_last_phases.name[i], g_last_phases.ms[i]);
        std::fprintf(stderr, " (ms)\n");
      }
    }
    for (int i = 0; i < n; ++i) cudaEventDestroy(ev[i]);
  }
};

cudaError_t nccl_to_cuda(ncclResult_t r) {
  if (r == ncclSuccess) return cudaSuccess;
  if (r == ncclInvalidArgument || r == ncclInvalidUsage) return cudaErrorInvalidValue;
  return cudaErrorUnknown;
}

struct MgpuLayout {
  size_t route_tmp, route_tmp_bytes, route, chunk_counts, counts, all_counts, part_k, part_v, alt_k, alt_v,
      sort_tmp, sort_tmp_bytes, total;
};

// Temp storage of one call; the local sorts' sizes come from this library's
// own size queries.
// CUSORT_MGPU_FORCE_EXCHANGE=1: a 1-rank communicator runs the whole
// pipeline (counts, all-gather, partition + exchange to itself, fence, local
// sort) instead of a plain sort -- a test hook for the exchange kernels on
// one GPU.
bool force_exchange() {
  const char* v = std::getenv("CUSORT_MGPU_FORCE_EXCHANGE");
  return v && v[0] == '1';
}

cudaError_t layout(int kt, size_t vb, int64_t n_local, int64_t cap, int nranks, int begin, int end, bool desc,
                   MgpuLayout* L) {
  const int kb = key_bytes(kt);
  const int msd_begin = std::max(begin, end - 8);
  size_t part_tmp = 0, final_tmp = 0, single_tmp = 0;
  cusort_double_buffer kd = {}, vd = {};
  cudaError_t e;
  if (nranks == 1 && !force_exchange()) {  // a plain single-GPU sort in the temp storage
    e = vb ? cusort_sort_pairs(nullptr, &single_tmp, (cusort_key_type)kt, nullptr, nullptr, vb, nullptr, nullptr,
                               n_local, begin, end, nullptr)
           : cusort_sort_keys(nullptr, &single_tmp, (cusort_key_type)kt, nullptr, nullptr, n_local, begin, end,
                              nullptr);
    if (e) return e;
    std::memset(L, 0, sizeof(*L));
    L->sort_tmp_bytes = std::max<size_t>(single_tmp, 1);
    L->total = a256(L->sort_tmp_bytes);
    return cudaSuccess;
  }
  if (vb) {
    e = desc ? cusort_sort_pairs_descending(nullptr, &part_tmp, (cusort_key_type)kt, nullptr, nullptr, vb, nullptr,
                                            nullptr, n_local, msd_begin, end, nullptr)
             : cusort_sort_pairs(nullptr, &part_tmp, (cusort_key_type)kt, nullptr, nullptr, vb, nullptr, nullptr,
                                 n_local, msd_begin, end, nullptr);
    if (e) return e;
    e = desc ? cusort_sort_pairs_descending_db(nullptr, &final_tmp, (cusort_key_type)kt, &kd, vb, &vd, cap, begin,
                                               end, nullptr)
             : cusort_sort_pairs_db(nullptr, &final_tmp, (cusort_key_type)kt, &kd, vb, &vd, cap, begin, end, nullptr);
  } else {
    e = cusort_sort_keys(nullptr, &part_tmp, (cusort_key_type)kt, nullptr, nullptr, n_local, msd_begin, end, nullptr);
    if (e) return e;
    e = cusort_sort_keys_db(nullptr, &final_tmp, (cusort_key_type)kt, &kd, cap, begin, end, nullptr);
  }
  if (e) return e;
  size_t route_tmp = 0;
  e = cusort_b200::routed_partition(kt, vb, desc, nullptr, nullptr, n_local, msd_begin, end, true, nullptr, nullptr,
                                    &route_tmp, nullptr);
  if (e) return e;
  size_t o = 0;
  L->route_tmp = o;  // first, so that the status word at d_temp is the routed pass's
  L->route_tmp_bytes = route_tmp;
  o += a256(route_tmp);
  L->route = o;  // one route table per chunk
  o += a256(kMaxChunks * sizeof(cusort_b200::RouteTable));
  L->chunk_counts = o;
  o += a256((size_t)kMaxChunks * 256 * sizeof(unsigned long long));
  L->counts = o;  // this rank's RankRecord (counts first), then the fence word
  o += a256(sizeof(RankRecord) + 16);
  L->all_counts = o;  // every rank's RankRecord
  o += a256((size_t)nranks * sizeof(RankRecord));
  L->part_k = o;
  o += a256((size_t)n_local * kb);
  L->part_v = o;
  o += a256((size_t)n_local * vb);
  L->alt_k = o;
  o += a256((size_t)cap * kb);
  L->alt_v = o;
  o += a256((size_t)cap * vb);
  L->sort_tmp = o;
  L->sort_tmp_bytes = std::max(std::max(part_tmp, final_tmp), size_t(1));
  o += a256(L->sort_tmp_bytes);
  L->total = o;
  return cudaSuccess;
}

}  // namespace

extern "C" {

int cusort_mgpu_plan(const uint64_t* all_counts, int nranks, int rank, int* digit_owner, int64_t* send_counts,
                     int64_t* recv_counts, int64_t* recv_totals) {
  if (!all_counts || nranks < 1 || rank < 0 || rank >= nranks) return 1;
  uint64_t total[256] = {};
  uint64_t N = 0;
  for (int r = 0; r < nranks; ++r)
    for (int d = 0; d < 256; ++d) total[d] += all_counts[(size_t)r * 256 + d];
  for (int d = 0; d < 256; ++d) N += total[d];
  int owner[256];
  uint64_t cum = 0;
  for (int d = 0; d < 256; ++d) {
    // owner by the midpoint of the digit's share of the global count
    const long double mid = (long double)cum + (long double)total[d] / 2.0L;
    int q = (N == 0) ? 0 : (int)((mid * nranks) / (long double)N);
    owner[d] = std::min(std::max(q, 0), nranks - 1);
    cum += total[d];
  }
  for (int d = 1; d < 256; ++d) owner[d] = std::max(owner[d], owner[d - 1]);  // monotone
  if (digit_owner) std::memcpy(digit_owner, owner, sizeof(owner));
  if (send_counts)
    for (int q = 0; q < nranks; ++q) {
      int64_t s = 0;
      for (int d = 0; d < 256; ++d)
        if (owner[d] == q) s += (int64_t)all_counts[(size_t)rank * 256 + d];
      send_counts[q] = s;
    }
  if (recv_counts)
    for (int p = 0; p < nranks; ++p) {
      int64_t s = 0;
      for (int d = 0; d < 256; ++d)
        if (owner[d] == rank) s += (int64_t)all_counts[(size_t)p * 256 + d];
      recv_counts[p] = s;
    }
  if (recv_totals)
    for (int q = 0; q < nranks; ++q) {
      int64_t s = 0;
      for (int d = 0; d < 256; ++d)
        if (owner[d] == q) s += (int64_t)total[d];
      recv_totals[q] = s;
    }
  return 0;
}

cudaError_t cusort_mgpu_unique_id(unsigned char* id) {
  if (!id) return cudaErrorInvalidValue;
  ncclUniqueId u;
  ncclResult_t r = ncclGetUniqueId(&u);
  if (r != ncclSuccess) return nccl_to_cuda(r);
  static_assert(sizeof(u) == 128, "NCCL unique id size");
  std::memcpy(id, &u, sizeof(u));
  return cudaSuccess;
}

cudaError_t cusort_mgpu_comm_init(void** comm, const unsigned char* id, int nranks, int rank) {
  if (!comm || !id || nranks < 1 || rank < 0 || rank >= nranks) return cudaErrorInvalidValue;
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof(u));
  // Non-blocking communicator: every wait on it is bounded (settle,
  // wait_event) and can end in ncclCommAbort.
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclComm_t c = nullptr;
  ncclResult_t r = ncclCommInitRankConfig(&c, nranks, u, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    if (c) ncclCommAbort(c);
    return nccl_to_cuda(r);
  }
  MgpuComm* mc = new MgpuComm();
  mc->nccl = c;
  const cudaError_t e = settle(mc, r);  // every rank must join within the limit
  if (e != cudaSuccess) {
    delete mc;
    return e;
  }
  *comm = mc;
  return cudaSuccess;
}

cudaError_t cusort_mgpu_set_timeout_ns(void* comm, uint64_t ns) {
  if (!comm || ns == 0) return cudaErrorInvalidValue;
  static_cast<MgpuComm*>(comm)->timeout_ns = ns;
  return cudaSuccess;
}

cudaError_t cusort_mgpu_wait(void* comm, cudaStream_t stream) {
  if (!comm) return cudaErrorInvalidValue;
  MgpuComm* mc = static_cast<MgpuComm*>(comm);
  if (mc->aborted) return cudaErrorTimeout;
  if (!mc->done) {
    const cudaError_t e = cudaEventCreateWithFlags(&mc->done, cudaEventDisableTiming);
    if (e) return e;
  }
  const cudaError_t e = cudaEventRecord(mc->done, stream);
  if (e) return e;
  return wait_event(mc, mc->done);
}

int cusort_mgpu_set_timing(int enable) {
  const int prev = g_timing;
  g_timing = enable ? 1 : 0;
  return prev;
}

int cusort_mgpu_get_phase_times(float* ms, const char** names, int capacity) {
  const int m = std::min(g_last_phases.n, std::max(capacity, 0));
  for (int i = 0; i < m; ++i) {
    if (ms) ms[i] = g_last_phases.ms[i];
    if (names) names[i] = g_last_phases.name[i];
  }
  return m;
}

cudaError_t cusort_mgpu_comm_destroy(void* comm) {
  if (!comm) return cudaErrorInvalidValue;
  MgpuComm* mc = static_cast<MgpuComm*>(comm);
  for (cudaStream_t st : mc->copy_streams) cudaStreamSynchronize(st);
  for (auto& kv : mc->mapped) cudaIpcCloseMemHandle(kv.second);
  cudaError_t e = cudaSuccess;
  if (!mc->aborted) {
    // non-blocking communicator: finish outstanding work, then free it
    ncclResult_t r = ncclCommFinalize(mc->nccl);
    e = settle(mc, r);
    if (!mc->aborted) {
      r = ncclCommDestroy(mc->nccl);
      if (r != ncclSuccess && r != ncclInProgress) e = nccl_to_cuda(r);
    }
  }
  delete mc;
  return e;
}

cudaError_t cusort_mgpu_sort(void* comm, void* d_temp, size_t* temp_bytes, cusort_key_type key_type,
                             size_t value_bytes, const void* d_keys_in, const void* d_values_in, int64_t n_local,
                             void* d_keys_out, void* d_values_out, int64_t out_capacity, int64_t* n_out,
                             int begin_bit, int end_bit, int descending, cudaStream_t stream) {
  const int kt = (int)key_type;
  const int kb = key_bytes(kt);
  const size_t vb = value_bytes;
  if (!comm || !temp_bytes || kb == 0) return cudaErrorInvalidValue;
  if (vb != 0 && vb != 1 && vb != 2 && vb != 4 && vb != 8 && vb != 16) return cudaErrorInvalidValue;
  if (begin_bit < 0 || end_bit < 0 || begin_bit > end_bit || end_bit > 8 * kb) return cudaErrorInvalidValue;
  if (n_local < 0 || out_capacity < 0) return cudaErrorInvalidValue;
  MgpuComm* mc = static_cast<MgpuComm*>(comm);
  if (mc->aborted) return cudaErrorTimeout;
  ncclComm_t nc = mc->nccl;
  int nranks = 0, rank = 0;
  cudaError_t e = nccl_to_cuda(ncclCommCount(nc, &nranks));
  if (e) return e;
  e = nccl_to_cuda(ncclCommUserRank(nc, &rank));
  if (e) return e;
  const bool desc = descending != 0;

  if (begin_bit == end_bit) {
    // Zero-width key range: the global order is the input order; every rank
    // keeps its slice.
    if (!d_temp) {
      *temp_bytes = 1;
      return cudaSuccess;
    }
    if (n_local > out_capacity) return cudaErrorInvalidValue;
    if (n_local > 0) {
      e = cudaMemcpyAsync(d_keys_out, d_keys_in, (size_t)n_local * kb, cudaMemcpyDeviceToDevice, stream);
      if (!e && vb) e = cudaMemcpyAsync(d_values_out, d_values_in, (size_t)n_local * vb, cudaMemcpyDeviceToDevice, stream);
      if (e) return e;
    }
    if (n_out) *n_out = n_local;
    return cudaSuccess;
  }

  MgpuLayout L;
  e = layout(kt, vb, n_local, out_capacity, nranks, begin_bit, end_bit, desc, &L);
  if (e) return e;
  if (!d_temp) {
    *temp_bytes = L.total;
    return cudaSuccess;
  }
  if (*temp_bytes < L.total || (reinterpret_cast<uintptr_t>(d_temp) & 15) != 0) return cudaErrorInvalidValue;
  uint8_t* t = static_cast<uint8_t*>(d_temp);
  void* stmp = t + L.sort_tmp;
  size_t stmp_bytes = L.sort_tmp_bytes;

  if (nranks == 1 && !force_exchange()) {
    if (n_local > out_capacity) return cudaErrorInvalidValue;
    if (vb)
      e = desc ? cusort_sort_pairs_descending(stmp, &stmp_bytes, key_type, d_keys_in, d_keys_out, vb, d_values_in,
                                              d_values_out, n_local, begin_bit, end_bit, stream)
               : cusort_sort_pairs(stmp, &stmp_bytes, key_type, d_keys_in, d_keys_out, vb, d_values_in, d_values_out,
                                   n_local, begin_bit, end_bit, stream);
    else
      e = desc ? cusort_sort_keys_descending(stmp, &stmp_bytes, key_type, d_keys_in, d_keys_out, n_local, begin_bit,
                                             end_bit, stream)
               : cusort_sort_keys(stmp, &stmp_bytes, key_type, d_keys_in, d_keys_out, n_local, begin_bit, end_bit,
                                  stream);
    if (e) return e;
    if (n_out) *n_out = n_local;
    return cudaSuccess;
  }

  // Receive buffers: chosen so that the final sort's last pass lands in the
  // caller's output (pieces arrive in source-rank order).
  const int passes = (end_bit - begin_bit + 7) / 8;
  const bool recv_in_out = (passes % 2) == 0;
  uint8_t* rk = static_cast<uint8_t*>(recv_in_out ? d_keys_out : (void*)(t + L.alt_k));
  uint8_t* ok_ = static_cast<uint8_t*>(recv_in_out ? (void*)(t + L.alt_k) : d_keys_out);
  uint8_t* rv = static_cast<uint8_t*>(recv_in_out ? d_values_out : (void*)(t + L.alt_v));
  uint8_t* ov = static_cast<uint8_t*>(recv_in_out ? (void*)(t + L.alt_v) : d_values_out);

  // 1-2. this rank's record (digit counts, receive capacity, exchange mode,
  //      IPC handles of its receive buffers), all-gathered
  const int msd_begin = std::max(begin_bit, end_bit - 8);
  PhaseTimer timer(stream, rank);
  timer.mark("start");
  RankRecord* rec = reinterpret_cast<RankRecord*>(t + L.counts);
  RankRecord* all_rec = reinterpret_cast<RankRecord*>(t + L.all_counts);
  int* fence = reinterpret_cast<int*>(t + L.counts + sizeof(RankRecord));
  // CUSORT_MGPU_EXCHANGE=pipe|copy|nccl selects another exchange than the
  // routed pass (the mode is all-gathered, so every rank takes the same path).
  const char* ex = std::getenv("CUSORT_MGPU_EXCHANGE");
  unsigned long long want = kXchgRouted;
  if (ex && std::strcmp(ex, "pipe") == 0) want = kXchgPipe;
  if (ex && std::strcmp(ex, "copy") == 0) want = kXchgCopy;
  if (ex && std::strcmp(ex, "nccl") == 0) want = kXchgNccl;
  const int chunks = chunks_for(n_local);
  if (want == kXchgPipe && chunks == 1) want = kXchgRouted;  // nothing to overlap
  if (want >= kXchgRouted && nranks > cusort_b200::kMaxRouteRanks) want = kXchgCopy;
  const int64_t chunk_items = (n_local + chunks - 1) / chunks;
  unsigned long long* d_cc = reinterpret_cast<unsigned long long*>(t + L.chunk_counts);
  if (want == kXchgPipe) {
    // per-chunk digit counts, and their sum for the record
    for (int c = 0; c < chunks && !e; ++c) {
      const int64_t c0 = c * chunk_items, cn = std::max<int64_t>(0, std::min(n_local - c0, chunk_items));
      e = cusort_b200::digit_counts_u64(kt, desc, static_cast<const uint8_t*>(d_keys_in) + c0 * kb, cn, msd_begin,
                                        end_bit, d_cc + c * 256, stream);
    }
    if (e) return e;
    sum_chunk_counts_kernel<<<1, 256, 0, stream>>>(d_cc, chunks, rec->counts);
    e = cudaGetLastError();
  } else {
    e = cusort_b200::digit_counts_u64(kt, desc, d_keys_in, n_local, msd_begin, end_bit, rec->counts, stream);
  }
  if (e) return e;
  const size_t tail = sizeof(RankRecord) - offsetof(RankRecord, hk);
  const size_t rec_words = ((size_t)nranks * sizeof(RankRecord) + tail + 7) / 8;
  e = g_pinned_counts.reserve(rec_words + (size_t)kMaxChunks * 256);
  if (e) return e;
  RankRecord* h_all = reinterpret_cast<RankRecord*>(g_pinned_counts.p);
  uint8_t* h_tail = reinterpret_cast<uint8_t*>(h_all + nranks);
  unsigned long long* h_cc = reinterpret_cast<unsigned long long*>(g_pinned_counts.p + rec_words);
  unsigned long long my_mode = kXchgNccl;
  {
    RankRecord mine;
    const bool ok = want != kXchgNccl && export_buffer(rk, &mine.hk, &mine.off_k) &&
                    (vb == 0 || export_buffer(rv, &mine.hv, &mine.off_v));
    if (vb == 0) {
      std::memset(&mine.hv, 0, sizeof(mine.hv));
      mine.off_v = 0;
    }
    my_mode = ok ? want : kXchgNccl;
    mine.mode = my_mode;
    mine.cap = (unsigned long long)out_capacity;
    std::memcpy(h_tail, reinterpret_cast<const uint8_t*>(&mine) + offsetof(RankRecord, hk), tail);
  }
  e = cudaMemcpyAsync(reinterpret_cast<uint8_t*>(rec) + offsetof(RankRecord, hk), h_tail, tail,
                      cudaMemcpyHostToDevice, stream);
  if (e) return e;
  e = settle(mc, ncclAllGather(rec, all_rec, sizeof(RankRecord), ncclUint8, nc, stream));
  if (e) return e;
  e = cudaMemcpyAsync(h_all, all_rec, (size_t)nranks * sizeof(RankRecord), cudaMemcpyDeviceToHost, stream);
  if (e) return e;
  if (want == kXchgPipe) {
    e = cudaMemcpyAsync(h_cc, d_cc, (size_t)chunks * 256 * sizeof(unsigned long long), cudaMemcpyDeviceToHost,
                        stream);
    if (e) return e;
  }
  cudaEvent_t counts_ready;
  e = cudaEventCreateWithFlags(&counts_ready, cudaEventDisableTiming);
  if (e) return e;
  e = cudaEventRecord(counts_ready, stream);
  if (e) {
    cudaEventDestroy(counts_ready);
    return e;
  }
  timer.mark("counts+gather");

  // 4 (fallback modes). stable partition by the owner digit into part_k/v.
  //    When this rank asked for a fallback exchange, it is enqueued before
  //    the host waits for the records, so the host round trip overlaps this
  //    pass.  (It does not depend on the plan: owners are contiguous digit
  //    ranges.)
  void* part_k = t + L.part_k;
  void* part_v = t + L.part_v;
  auto partition = [&]() -> cudaError_t {
    if (vb)
      return desc ? cusort_sort_pairs_descending(stmp, &stmp_bytes, key_type, d_keys_in, part_k, vb, d_values_in,
                                                 part_v, n_local, msd_begin, end_bit, stream)
                  : cusort_sort_pairs(stmp, &stmp_bytes, key_type, d_keys_in, part_k, vb, d_values_in, part_v,
                                      n_local, msd_begin, end_bit, stream);
    return desc ? cusort_sort_keys_descending(stmp, &stmp_bytes, key_type, d_keys_in, part_k, n_local, msd_begin,
                                              end_bit, stream)
                : cusort_sort_keys(stmp, &stmp_bytes, key_type, d_keys_in, part_k, n_local, msd_begin, end_bit,
                                   stream);
  };
  bool partitioned = false;
  if (my_mode == kXchgCopy || my_mode == kXchgNccl) {
    e = partition();
    if (e) {
      cudaEventDestroy(counts_ready);
      return e;
    }
    partitioned = true;
  }

  // 3. plan (identical on every rank); the wait is bounded and aborts the
  //    communicator when a rank never arrives
  e = wait_event(mc, counts_ready);
  cudaEventDestroy(counts_ready);
  if (e) return e;
  std::vector<uint64_t> all_counts((size_t)nranks * 256);
  unsigned long long mode = kXchgRouted;
  for (int q = 0; q < nranks; ++q) {
    std::memcpy(&all_counts[(size_t)q * 256], h_all[q].counts, 256 * 8);
    mode = std::min(mode, h_all[q].mode);
  }
  std::vector<int64_t> send((size_t)nranks), recv((size_t)nranks), totals((size_t)nranks);
  std::vector<int> owner(256);
  if (cusort_mgpu_plan(all_counts.data(), nranks, rank, owner.data(), send.data(), recv.data(), totals.data()))
    return cudaErrorInvalidValue;
  for (int q = 0; q < nranks; ++q)  // every rank sees the same records: no rank enters NCCL
    if (totals[q] > (int64_t)h_all[q].cap) return cudaErrorInvalidValue;
  const int64_t n_recv = totals[rank];

  // 5. all-to-all
  timer.mark("host");
  if (mode == kXchgPipe) {
    // Pipelined: chunk c is partitioned by the routed pass -- this rank's own
    // items straight into its receive buffer, each peer's into one staging
    // run -- and the copy engines push chunk c's staging runs into the peers'
    // receive buffers while chunk c+1 is partitioned.  Peer q's buffer gets
    // this rank's chunks in order after the items of lower source ranks.
    const int peers = nranks - 1;
    const int ns = std::min(peers, kMaxCopyStreams);
    e = comm_resources(mc, ns, chunks + ns);
    if (e) return e;
    std::vector<int64_t> cnt((size_t)chunks * nranks, 0);  // [c][q]
    for (int c = 0; c < chunks; ++c)
      for (int d = 0; d < 256; ++d) cnt[(size_t)c * nranks + owner[d]] += (int64_t)h_cc[c * 256 + d];
    std::vector<int64_t> at((size_t)nranks, 0);  // this rank's offset in q's buffer
    for (int q = 0; q < nranks; ++q)
      for (int p = 0; p < rank; ++p)
        for (int d = 0; d < 256; ++d)
          if (owner[d] == q) at[q] += (int64_t)all_counts[(size_t)p * 256 + d];
    std::vector<uint8_t*> pk((size_t)nranks, nullptr), pv((size_t)nranks, nullptr);
    for (int q = 0; q < nranks && !e; ++q) {
      if (q == rank) continue;
      e = peer_address(mc, q, h_all[q].hk, h_all[q].off_k, &pk[q]);
      if (!e && vb) e = peer_address(mc, q, h_all[q].hv, h_all[q].off_v, &pv[q]);
    }
    if (e) return e;
    std::vector<cusort_b200::RouteTable> rts((size_t)chunks);
    std::vector<int64_t> stage((size_t)chunks * nranks, 0), dst((size_t)chunks * nranks, 0);
    int64_t so = 0;
    std::vector<int64_t> run = at;  // next free offset per destination
    for (int c = 0; c < chunks; ++c) {
      cusort_b200::RouteTable& rt = rts[c];
      std::memset(&rt, 0, sizeof(rt));
      for (int d = 255; d >= 0; --d) {
        rt.owner[d] = (unsigned char)owner[d];
        rt.first_digit[owner[d]] = (unsigned int)d;
      }
      for (int d = 0; d < 256; ++d) rt.last_digit[owner[d]] = (unsigned int)d;
      for (int q = 0; q < nranks; ++q) {
        const int64_t m = cnt[(size_t)c * nranks + q];
        dst[(size_t)c * nranks + q] = run[q];
        if (q == rank) {
          rt.kptr[q] = reinterpret_cast<unsigned long long>(rk);
          rt.vptr[q] = vb ? reinterpret_cast<unsigned long long>(rv) : 0ull;
          rt.cap[q] = (unsigned long long)out_capacity;
          rt.base[q] = (unsigned long long)run[q];
        } else {
          rt.kptr[q] = reinterpret_cast<unsigned long long>(part_k);
          rt.vptr[q] = vb ? reinterpret_cast<unsigned long long>(part_v) : 0ull;
          rt.cap[q] = (unsigned long long)n_local;
          rt.base[q] = (unsigned long long)so;
          stage[(size_t)c * nranks + q] = so;
          so += m;
        }
        run[q] += m;
      }
    }
    const bool wide = (uint64_t)out_capacity > 0xFFFFFFFFull || (uint64_t)n_local > 0xFFFFFFFFull;
    auto* d_rt = reinterpret_cast<cusort_b200::RouteTable*>(t + L.route);
    // pageable source: staged before the call returns; the stream is idle here
    e = cudaMemcpyAsync(d_rt, rts.data(), (size_t)chunks * sizeof(cusort_b200::RouteTable), cudaMemcpyHostToDevice,
                        stream);
    if (e) return e;
    std::vector<bool> used((size_t)ns, false);
    for (int c = 0; c < chunks && !e; ++c) {
      const int64_t c0 = c * chunk_items, cn = std::max<int64_t>(0, std::min(n_local - c0, chunk_items));
      size_t rtb = L.route_tmp_bytes;
      e = cusort_b200::routed_partition(kt, vb, desc, static_cast<const uint8_t*>(d_keys_in) + c0 * kb,
                                        vb ? static_cast<const uint8_t*>(d_values_in) + c0 * vb : nullptr, cn,
                                        msd_begin, end_bit, wide, d_rt + c, t + L.route_tmp, &rtb, stream, c > 0);
      if (!e) e = cudaEventRecord(mc->events[c], stream);
      for (int q = 0; q < nranks && !e; ++q) {
        const int64_t m = cnt[(size_t)c * nranks + q];
        if (q == rank || m == 0) continue;
        const int j = (q < rank ? q : q - 1) % ns;
        cudaStream_t cs = mc->copy_streams[j];
        e = cudaStreamWaitEvent(cs, mc->events[c], 0);
        used[j] = true;
        const int64_t sidx = stage[(size_t)c * nranks + q], didx = dst[(size_t)c * nranks + q];
        if (!e)
          e = cudaMemcpyAsync(pk[q] + didx * kb, static_cast<uint8_t*>(part_k) + sidx * kb, (size_t)m * kb,
                              cudaMemcpyDeviceToDevice, cs);
        if (!e && vb)
          e = cudaMemcpyAsync(pv[q] + didx * vb, static_cast<uint8_t*>(part_v) + sidx * vb, (size_t)m * vb,
                              cudaMemcpyDeviceToDevice, cs);
      }
    }
    // join the copy streams, then fence
    for (int j = 0; j < ns && !e; ++j) {
      if (!used[j]) continue;
      e = cudaEventRecord(mc->events[chunks + j], mc->copy_streams[j]);
      if (!e) e = cudaStreamWaitEvent(stream, mc->events[chunks + j], 0);
    }
    timer.mark("routed-pass");
    if (!e) e = cudaMemsetAsync(fence, 0, sizeof(int), stream);
    if (!e) e = settle(mc, ncclAllReduce(fence, fence, 1, ncclInt32, ncclSum, nc, stream));
    if (e) return e;
  } else if (mode == kXchgRouted) {
    // Fused partition + exchange: this rank's items for q go after the items
    // q receives from lower source ranks, tile by tile.
    cusort_b200::RouteTable rt;
    std::memset(&rt, 0, sizeof(rt));
    for (int d = 255; d >= 0; --d) {
      rt.owner[d] = (unsigned char)owner[d];
      rt.first_digit[owner[d]] = (unsigned int)d;
    }
    for (int d = 0; d < 256; ++d) rt.last_digit[owner[d]] = (unsigned int)d;
    for (int q = 0; q < nranks; ++q)
      for (int p = 0; p < rank; ++p)
        for (int d = 0; d < 256; ++d)
          if (owner[d] == q) rt.base[q] += all_counts[(size_t)p * 256 + d];
    bool wide = false;
    for (int q = 0; q < nranks && !e; ++q) {
      uint8_t* dk = rk;
      uint8_t* dv = rv;
      if (q != rank) {
        e = peer_address(mc, q, h_all[q].hk, h_all[q].off_k, &dk);
        if (!e && vb) e = peer_address(mc, q, h_all[q].hv, h_all[q].off_v, &dv);
      }
      rt.kptr[q] = reinterpret_cast<unsigned long long>(dk);
      rt.vptr[q] = vb ? reinterpret_cast<unsigned long long>(dv) : 0ull;
      rt.cap[q] = h_all[q].cap;
      wide = wide || (uint64_t)totals[q] > 0xFFFFFFFFull;
    }
    if (e) return e;
    // Pageable source: staged by the driver before the call returns, and the
    // stream has no pending work here (the records were just waited for).
    e = cudaMemcpyAsync(t + L.route, &rt, sizeof(rt), cudaMemcpyHostToDevice, stream);
    if (e) return e;
    size_t rtb = L.route_tmp_bytes;
    e = cusort_b200::routed_partition(kt, vb, desc, d_keys_in, d_values_in, n_local, msd_begin, end_bit, wide,
                                      reinterpret_cast<const cusort_b200::RouteTable*>(t + L.route),
                                      t + L.route_tmp, &rtb, stream);
    timer.mark("routed-pass");
    // Fence: once every rank's routed pass (earlier on its stream) is done,
    // the all-reduce completes everywhere and the received data is complete.
    if (!e) e = cudaMemsetAsync(fence, 0, sizeof(int), stream);
    if (!e) e = settle(mc, ncclAllReduce(fence, fence, 1, ncclInt32, ncclSum, nc, stream));
    if (e) return e;
  } else {
    if (!partitioned) {
      e = partition();
      if (e) return e;
    }
    if (mode == kXchgCopy) {
      // Push this rank's piece for q into q's receive buffers at the offset of
      // source `rank` (the pieces of lower ranks come first).
      int64_t so = 0;
      for (int q = 0; q < nranks && !e; ++q) {
        if (send[q] > 0) {
          int64_t at = 0;  // items q receives from the ranks below this one
          for (int p = 0; p < rank; ++p)
            for (int d = 0; d < 256; ++d)
              if (owner[d] == q) at += (int64_t)all_counts[(size_t)p * 256 + d];
          uint8_t* dk = rk;
          uint8_t* dv = rv;
          if (q != rank) {
            e = peer_address(mc, q, h_all[q].hk, h_all[q].off_k, &dk);
            if (!e && vb) e = peer_address(mc, q, h_all[q].hv, h_all[q].off_v, &dv);
          }
          if (!e)
            e = cudaMemcpyAsync(dk + at * kb, static_cast<uint8_t*>(part_k) + so * kb, (size_t)send[q] * kb,
                                cudaMemcpyDeviceToDevice, stream);
          if (!e && vb)
            e = cudaMemcpyAsync(dv + at * vb, static_cast<uint8_t*>(part_v) + so * vb, (size_t)send[q] * vb,
                                cudaMemcpyDeviceToDevice, stream);
        }
        so += send[q];
      }
      if (!e) e = cudaMemsetAsync(fence, 0, sizeof(int), stream);
      if (!e) e = settle(mc, ncclAllReduce(fence, fence, 1, ncclInt32, ncclSum, nc, stream));
      if (e) return e;
    } else {
      ncclResult_t r = ncclGroupStart();
      int64_t so = 0, ro = 0;
      for (int q = 0; q < nranks && r == ncclSuccess; ++q) {
        if (send[q] > 0) {
          r = ncclSend(static_cast<uint8_t*>(part_k) + so * kb, (size_t)send[q] * kb, ncclUint8, q, nc, stream);
          if (r == ncclSuccess && vb)
            r = ncclSend(static_cast<uint8_t*>(part_v) + so * vb, (size_t)send[q] * vb, ncclUint8, q, nc, stream);
        }
        if (r == ncclSuccess && recv[q] > 0) {
          r = ncclRecv(rk + ro * kb, (size_t)recv[q] * kb, ncclUint8, q, nc, stream);
          if (r == ncclSuccess && vb) r = ncclRecv(rv + ro * vb, (size_t)recv[q] * vb, ncclUint8, q, nc, stream);
        }
        so += send[q];
        ro += recv[q];
      }
      ncclResult_t r2 = ncclGroupEnd();
      e = (r != ncclSuccess && r != ncclInProgress) ? abort_comm(mc, nccl_to_cuda(r)) : settle(mc, r2);
      if (e) return e;
    }
  }

  timer.mark("exchange");
  // 6. stable local sort of the received items on every key bit
  if (n_recv >= 2) {
    cusort_double_buffer kd = {{rk, ok_}, 0};
    cusort_double_buffer vd = {{rv, ov}, 0};
    if (vb)
      e = desc ? cusort_sort_pairs_descending_db(stmp, &stmp_bytes, key_type, &kd, vb, &vd, n_recv, begin_bit,
                                                 end_bit, stream)
               : cusort_sort_pairs_db(stmp, &stmp_bytes, key_type, &kd, vb, &vd, n_recv, begin_bit, end_bit, stream);
    else
      e = desc ? cusort_sort_keys_descending_db(stmp, &stmp_bytes, key_type, &kd, n_recv, begin_bit, end_bit, stream)
               : cusort_sort_keys_db(stmp, &stmp_bytes, key_type, &kd, n_recv, begin_bit, end_bit, stream);
    if (e) return e;
  } else if (n_recv == 1 && !recv_in_out) {
    e = cudaMemcpyAsync(d_keys_out, rk, kb, cudaMemcpyDeviceToDevice, stream);
    if (!e && vb) e = cudaMemcpyAsync(d_values_out, rv, vb, cudaMemcpyDeviceToDevice, stream);
    if (e) return e;
  }
  timer.mark("local-sort");
  if (n_out) *n_out = n_recv;
  return cudaSuccess;
}

}  // extern "C"

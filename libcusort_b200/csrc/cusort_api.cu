// cusort_api.cu -- host dispatcher and C ABI of the B200 radix sort.
//
// Reference counterparts: DeviceRadixSort::DispatchSort (libcusort.cuh:2896-2965),
// DispatchRadixSort::Dispatch/Invoke (libcusort.cuh:2553-2872), GraphCache
// (libcusort.cuh:192-225) and the cached device queries of utils
// (libcusort.cuh:227-312).  Differences by design:
//   * device queries and occupancy are cached per (device, kernel), thread-safe;
//   * only the control block, digit histogram and lookback descriptors are
//     zeroed (never the staging buffers of the in/out-pointer form);
//   * kernels are chained with programmatic dependent launch (PDL), either as
//     direct cudaLaunchKernelEx launches or as a cached CUDA graph whose edges
//     are programmatic;
//   * onesweep grids are persistent (SMs x resident CTAs) with a tile ticket.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <utility>
#include <vector>

#include "../../include/cusort_b200.h"
#include "cusort_dispatch.h"
#include "cusort_types.h"

#define CUSORT_TRY(x)                     \
  do {                                    \
    cudaError_t e__ = (x);                \
    if (e__ != cudaSuccess) return e__;   \
  } while (0)

namespace cusort_b200 {

// ---------------------------------------------------------------------------
// per-device caches (thread-safe)
// ---------------------------------------------------------------------------
struct DeviceCache {
  std::mutex mu;
  std::map<int, int> sm_count;
  std::map<std::pair<int, const void*>, int> occupancy;
};
static DeviceCache& dcache() {
  static DeviceCache* c = new DeviceCache();  // never destroyed: safe at exit
  return *c;
}

static cudaError_t get_sm_count(int dev, int* out) {
  DeviceCache& c = dcache();
  std::lock_guard<std::mutex> lk(c.mu);
  auto it = c.sm_count.find(dev);
  if (it != c.sm_count.end()) {
    *out = it->second;
    return cudaSuccess;
  }
  int v = 0;
  CUSORT_TRY(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev));
  c.sm_count[dev] = v;
  *out = v;
  return cudaSuccess;
}

// Resident CTAs per SM for `k`; raises the kernel's dynamic shared-memory
// limit on first use on this device.
static cudaError_t get_occupancy(int dev, const KernelInfo& k, int* out) {
  DeviceCache& c = dcache();
  std::lock_guard<std::mutex> lk(c.mu);
  auto key = std::make_pair(dev, k.func);
  auto it = c.occupancy.find(key);
  if (it != c.occupancy.end()) {
    *out = it->second;
    return cudaSuccess;
  }
  if (k.smem > 48 * 1024)
    CUSORT_TRY(cudaFuncSetAttribute(k.func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)k.smem));
  int occ = 0;
  CUSORT_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k.func, k.threads, k.smem));
  if (occ < 1) return cudaErrorInvalidConfiguration;
  c.occupancy[key] = occ;
  *out = occ;
  return cudaSuccess;
}

// ---------------------------------------------------------------------------
// key traits
// ---------------------------------------------------------------------------
static int key_bytes_of(int kt) {
  switch (kt) {
    case CUSORT_KEY_U8: case CUSORT_KEY_I8: return 1;
    case CUSORT_KEY_U16: case CUSORT_KEY_I16: return 2;
    case CUSORT_KEY_U32: case CUSORT_KEY_I32: case CUSORT_KEY_F32: return 4;
    case CUSORT_KEY_U64: case CUSORT_KEY_I64: case CUSORT_KEY_F64: return 8;
    default: return 0;
  }
}
static bool value_bytes_ok(size_t vb) { return vb == 1 || vb == 2 || vb == 4 || vb == 8 || vb == 16; }

// Twiddle constants (C, F) of dev::twiddle; reference RadixTraits::Twiddle
// (libcusort.cuh:417-429).
static void twiddle_constants(int kt, int kb, bool desc, uint64_t* c, uint64_t* f) {
  const uint64_t all = (kb == 8) ? ~0ull : ((1ull << (8 * kb)) - 1);
  const uint64_t sb = 1ull << (8 * kb - 1);
  const bool is_float = kt == CUSORT_KEY_F32 || kt == CUSORT_KEY_F64;
  const bool is_signed = kt == CUSORT_KEY_I8 || kt == CUSORT_KEY_I16 || kt == CUSORT_KEY_I32 || kt == CUSORT_KEY_I64;
  uint64_t cc = 0, ff = 0;
  if (is_float) {
    cc = sb;
    ff = all ^ sb;
  } else if (is_signed) {
    cc = sb;
  }
  if (desc) cc ^= all;
  *c = cc;
  *f = ff;
}

// ---------------------------------------------------------------------------
// plan: kernels, grids and temp-storage layout
//   [control 256 B: status u32 @0, tile counters u32[8] @64]
//   [digit histogram: passes x 256 x OffsetT]
//   [lookback descriptors: tiles x 256 x OffsetT]     <- zeroed by init
//   [staging keys n x K][staging values n x V]        <- in/out form, passes >= 2
// (2-byte keys-only full-range sorts: control + counts[65536] + group
// totals[256], all zeroed; nothing else)
// ---------------------------------------------------------------------------
struct Plan {
  int kt = 0, kb = 0, vb = 0, offb = 4;
  bool desc = false;
  uint64_t n = 0;
  int begin = 0, end = 0;
  uint32_t passes = 0, last_mask = 0;
  uint64_t tw_c = 0, tw_f = 0;
  KernelInfo os, hist;
  uint64_t tiles = 0;
  size_t off_hist = 0, off_desc = 0, off_stage_k = 0, off_stage_v = 0, zero_bytes = 0, total = 0;
  bool staging = false;
  // 2-byte keys-only over all 16 bits: one 16-bit digit (count, fill); the
  // histogram region then holds counts[65536] and group totals[256]
  bool fill16 = false;
  KernelInfo h16, f16;
};

constexpr size_t kCtrlBytes = 256;
static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// CUSORT_WIDE_OFFSETS=1: every sort uses the 64-bit offset kernels that
// 2^30 items and more select -- a test hook that checks those kernels against
// the oracle on inputs it can sort.
bool force_wide_offsets() {
  const char* v = std::getenv("CUSORT_WIDE_OFFSETS");
  return v && v[0] == '1';
}

static bool make_plan(int kt, size_t vb, bool desc, uint64_t n, int begin, int end, bool raw, Plan* p) {
  p->kt = kt;
  p->kb = key_bytes_of(kt);
  p->vb = (int)vb;
  p->desc = desc;
  p->n = n;
  p->begin = begin;
  p->end = end;
  // 30 count bits per descriptor word with 32-bit offsets (2 state bits).
  p->offb = (n < (1ull << 30) && !force_wide_offsets()) ? 4 : 8;
  const uint32_t nbits = (uint32_t)(end - begin);
  p->passes = (nbits + kRadixBits - 1) / kRadixBits;
  p->last_mask = (1u << (nbits - (p->passes - 1) * kRadixBits)) - 1u;
  twiddle_constants(kt, p->kb, desc, &p->tw_c, &p->tw_f);
  bool ok = false;
  const bool fk = (kt == CUSORT_KEY_F32 || kt == CUSORT_KEY_F64);
  switch (p->kb) {
    case 1: ok = get_kernels_k1(p->vb, p->offb, fk, &p->os, &p->hist); break;
    case 2: ok = get_kernels_k2(p->vb, p->offb, fk, &p->os, &p->hist); break;
    case 4: ok = get_kernels_k4(p->vb, p->offb, fk, &p->os, &p->hist); break;
    case 8: ok = get_kernels_k8(p->vb, p->offb, fk, &p->os, &p->hist); break;
    default: ok = false;
  }
  if (!ok) return false;
  if (p->kb == 2 && p->vb == 0 && begin == 0 && end == 16) {
    p->fill16 = get_fill16_kernels(p->offb, &p->h16, &p->f16);
    if (p->fill16) {
      p->tiles = 0;
      p->off_hist = kCtrlBytes;
      p->zero_bytes = kCtrlBytes + align256((size_t)(65536 + 256) * p->offb);
      p->off_desc = p->zero_bytes;
      p->staging = false;
      p->off_stage_k = p->off_stage_v = p->off_desc;
      p->total = p->off_desc;
      return true;
    }
  }
  // Fewer items: smaller tiles, so the persistent grid still covers the SMs.
  if (n <= kMidTileMaxItems && p->offb == 4) {
    KernelInfo small;
    if (get_small_onesweep(p->kb, p->vb, fk, n <= kSmallTileMaxItems ? 0 : 1, &small)) p->os = small;
  }
  p->tiles = (n + p->os.tile - 1) / p->os.tile;
  p->off_hist = kCtrlBytes;
  p->off_desc = p->off_hist + align256((size_t)p->passes * kRadix * p->offb);
  const size_t end_desc = p->off_desc + align256((size_t)p->tiles * kRadix * p->offb);
  p->zero_bytes = end_desc;
  p->staging = raw && p->passes >= 2;
  p->off_stage_k = end_desc;
  p->off_stage_v = p->off_stage_k + (p->staging ? align256((size_t)n * p->kb) : 0);
  p->total = p->off_stage_v + ((p->staging && p->vb) ? align256((size_t)n * p->vb) : 0);
  return true;
}

// ---------------------------------------------------------------------------
// per-thread settings, timing and graph cache
// ---------------------------------------------------------------------------
struct GraphEntry {
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  std::vector<cudaGraphNode_t> nodes;  // init, histogram, onesweep[0..P-1]
};
using GraphKey = std::tuple<int, const void*, const void*, uint32_t, int, int, int>;

struct ThreadState {
  int launch_mode = 0;
  uint64_t wait_limit_ns = 2000000000ull;
  int64_t skip_tile = -1;
  int timing = 0;
  std::vector<cudaEvent_t> events;
  std::vector<int> kinds;
  int recorded = 0;
  std::map<GraphKey, GraphEntry> graphs;
  ~ThreadState() {
    // Best effort: the CUDA context may already be gone at process exit.
    for (auto& kv : graphs) {
      if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
      if (kv.second.graph) cudaGraphDestroy(kv.second.graph);
    }
    for (cudaEvent_t e : events) cudaEventDestroy(e);
  }
};
static thread_local ThreadState g_ts;

static void timing_begin(cudaStream_t s, int kind) {
  if (!g_ts.timing) return;
  const size_t need = (size_t)(g_ts.recorded + 1) * 2;
  while (g_ts.events.size() < need) {
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) return;
    g_ts.events.push_back(e);
  }
  if ((int)g_ts.kinds.size() <= g_ts.recorded) g_ts.kinds.resize(g_ts.recorded + 1);
  g_ts.kinds[g_ts.recorded] = kind;
  cudaEventRecord(g_ts.events[2 * g_ts.recorded], s);
}
static void timing_end(cudaStream_t s) {
  if (!g_ts.timing) return;
  if ((size_t)(2 * g_ts.recorded + 1) >= g_ts.events.size()) return;
  cudaEventRecord(g_ts.events[2 * g_ts.recorded + 1], s);
  g_ts.recorded++;
}

// ---------------------------------------------------------------------------
// launch sequence
// ---------------------------------------------------------------------------
struct Launch {
  const void* func;
  int grid, threads;
  size_t smem;
  bool pdl;
  int kind;
  union {
    InitArgs init;
    HistArgs hist;
    OnesweepArgs os;
    FillArgs fill;
    Fill16Args f16;
  } args;
};

struct PassBuffers {
  const void* k_src[kMaxPasses];
  void* k_dst[kMaxPasses];
  const void* v_src[kMaxPasses];
  void* v_dst[kMaxPasses];
};

static cudaError_t build_launches(const Plan& p, void* d_temp, const PassBuffers& b, std::vector<Launch>* out) {
  int dev = 0;
  CUSORT_TRY(cudaGetDevice(&dev));
  int sms = 0, occ_os = 0, occ_h = 0;
  CUSORT_TRY(get_sm_count(dev, &sms));
  CUSORT_TRY(get_occupancy(dev, p.os, &occ_os));
  CUSORT_TRY(get_occupancy(dev, p.hist, &occ_h));

  uint8_t* t = static_cast<uint8_t*>(d_temp);
  uint32_t* status = reinterpret_cast<uint32_t*>(t);
  uint32_t* counters = reinterpret_cast<uint32_t*>(t + 64);
  uint8_t* g_hist = t + p.off_hist;
  void* desc = t + p.off_desc;

  out->clear();
  {
    Launch l{};
    l.func = get_init_kernel();
    const uint64_t n16 = p.zero_bytes / 16;
    l.grid = (int)std::min<uint64_t>((uint64_t)sms * 4, std::max<uint64_t>(1, (n16 + 511) / 512));
    l.threads = 512;
    l.smem = 0;
    l.pdl = false;  // first kernel: full ordering after the caller's work
    l.kind = 0;
    l.args.init.ptr = d_temp;
    l.args.init.n16 = n16;
    out->push_back(l);
  }
  if (p.fill16) {
    // one 16-bit digit: count, then fill the
    // final destination (the last pass's output of the 8-bit schedule)
    Fill16Args f;
    f.keys = b.k_src[0];
    f.counts = g_hist;
    f.groups = g_hist + (size_t)65536 * p.offb;
    f.out = b.k_dst[p.passes - 1];
    f.n = p.n;
    f.xor_c = (uint32_t)p.tw_c;
    f.pad = 0;
    int occ16 = 0;
    CUSORT_TRY(get_occupancy(dev, p.h16, &occ16));
    Launch l{};
    l.func = p.h16.func;
    const int readers = std::max(1, p.h16.tile);  // CTAs that read each key (a pair splits the bins)
    l.grid = readers * (int)std::max<uint64_t>(1, std::min<uint64_t>((uint64_t)sms * occ16 / readers,
                                                                      p.n / (8192 * (uint64_t)readers) + 1));
    l.threads = p.h16.threads;
    l.smem = p.h16.smem;
    l.pdl = true;
    l.kind = 1;
    l.args.f16 = f;
    out->push_back(l);
    Launch l3{};
    l3.func = p.f16.func;
    // the output split evenly: at least 32768 keys per CTA, at most 8 CTAs per SM
    l3.grid = (int)std::max<uint64_t>(1, std::min<uint64_t>((uint64_t)sms * 8, (p.n + 32767) / 32768));
    l3.threads = p.f16.threads;
    l3.pdl = true;
    l3.kind = 2;
    l3.args.f16 = f;
    out->push_back(l3);
    return cudaSuccess;
  }
  {
    Launch l{};
    l.func = p.hist.func;
    const uint64_t vec = p.n * p.kb / 16 + 1;
    const uint64_t want = (vec + p.hist.tile - 1) / p.hist.tile;
    l.grid = (int)std::max<uint64_t>(1, std::min<uint64_t>((uint64_t)sms * occ_h, want));
    l.threads = p.hist.threads;
    l.smem = p.hist.smem;
    l.pdl = true;
    l.kind = 1;
    HistArgs& h = l.args.hist;
    h.keys = b.k_src[0];
    h.n = p.n;
    h.tw_c = p.tw_c;
    h.tw_f = p.tw_f;
    h.begin_bit = (uint32_t)p.begin;
    h.num_passes = p.passes;
    h.last_mask = p.last_mask;
    h.g_hist = g_hist;
    out->push_back(l);
  }
  // 1-byte keys, no values, every key bit sorted in one pass: count and fill.
  if (p.kb == 1 && p.vb == 0 && p.begin == 0 && p.end == 8) {
    Launch l{};
    l.func = get_fill_bytes_kernel(p.offb);
    l.grid = (int)std::max<uint64_t>(1, std::min<uint64_t>((uint64_t)sms * 8, (p.n / 16 + 255) / 256));
    l.threads = 256;
    l.smem = 0;
    l.pdl = true;
    l.kind = 2;
    l.args.fill.counts = g_hist;
    l.args.fill.out = b.k_dst[0];
    l.args.fill.n = p.n;
    l.args.fill.xor_c = (uint32_t)p.tw_c;
    out->push_back(l);
    return cudaSuccess;
  }
  const int os_grid = (int)std::max<uint64_t>(1, std::min<uint64_t>((uint64_t)sms * occ_os, p.tiles));
  for (uint32_t pass = 0; pass < p.passes; ++pass) {
    Launch l{};
    l.func = p.os.func;
    l.grid = os_grid;
    l.threads = p.os.threads;
    l.smem = p.os.smem;
    l.pdl = true;
    l.kind = 2;
    OnesweepArgs& a = l.args.os;
    a.keys_in = b.k_src[pass];
    a.keys_out = b.k_dst[pass];
    a.vals_in = p.vb ? b.v_src[pass] : nullptr;
    a.vals_out = p.vb ? b.v_dst[pass] : nullptr;
    a.n = p.n;
    a.tw_c = p.tw_c;
    a.tw_f = p.tw_f;
    a.shift = (uint32_t)p.begin + pass * kRadixBits;
    a.mask = (pass + 1 == p.passes) ? p.last_mask : 0xffu;
    a.pass = pass;
    a.num_tiles = (uint32_t)p.tiles;
    a.desc = desc;
    a.g_hist_pass = g_hist + (size_t)pass * kRadix * p.offb;
    a.tile_counter = counters + pass;
    a.status = status;
    a.spin_limit_ns = g_ts.wait_limit_ns;
    a.skip_tile = g_ts.skip_tile;
    const size_t tile_k = (size_t)p.os.tile * p.kb, tile_v = (size_t)p.os.tile * p.vb;
    a.tma_keys = ((reinterpret_cast<uintptr_t>(a.keys_in) & 15) == 0 && (tile_k & 15) == 0) ? 1u : 0u;
    a.tma_vals = (p.vb == 0 || ((reinterpret_cast<uintptr_t>(a.vals_in) & 15) == 0 && (tile_v & 15) == 0)) ? 1u : 0u;
    out->push_back(l);
  }
  return cudaSuccess;
}

static cudaError_t launch_direct(const std::vector<Launch>& ls, cudaStream_t stream) {
  g_ts.recorded = 0;
  for (const Launch& l : ls) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)l.grid);
    cfg.blockDim = dim3((unsigned)l.threads);
    cfg.dynamicSmemBytes = l.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if (l.pdl && !g_ts.timing) {
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
    }
    void* args[1] = {const_cast<void*>(static_cast<const void*>(&l.args))};
    timing_begin(stream, l.kind);
    CUSORT_TRY(cudaLaunchKernelExC(&cfg, l.func, args));
    timing_end(stream);
  }
  return cudaSuccess;
}

static cudaKernelNodeParams node_params(const Launch& l, void** argv) {
  cudaKernelNodeParams kp = {};
  kp.func = const_cast<void*>(l.func);
  kp.gridDim = dim3((unsigned)l.grid);
  kp.blockDim = dim3((unsigned)l.threads);
  kp.sharedMemBytes = (unsigned)l.smem;
  argv[0] = const_cast<void*>(static_cast<const void*>(&l.args));
  kp.kernelParams = argv;
  kp.extra = nullptr;
  return kp;
}

// Graph mode: one graph per (device, kernels, passes, grids) and host thread,
// built once with programmatic edges, then replayed after updating every
// kernel node's arguments (reference GraphCache, libcusort.cuh:2693-2834).
static cudaError_t launch_graph(const std::vector<Launch>& ls, cudaStream_t stream) {
  int dev = 0;
  CUSORT_TRY(cudaGetDevice(&dev));
  const GraphKey key{dev, ls[1].func, ls.back().func, (uint32_t)ls.size(), ls[0].grid, ls[1].grid, ls.back().grid};
  auto it = g_ts.graphs.find(key);
  if (it == g_ts.graphs.end()) {
    GraphEntry ge;
    CUSORT_TRY(cudaGraphCreate(&ge.graph, 0));
    cudaGraphNode_t prev = nullptr;
    for (const Launch& l : ls) {
      void* argv[1];
      cudaKernelNodeParams kp = node_params(l, argv);
      cudaGraphNode_t node;
      cudaError_t e = cudaGraphAddKernelNode(&node, ge.graph, nullptr, 0, &kp);
      if (e == cudaSuccess && prev) {
        cudaGraphEdgeData ed = {};
        ed.from_port = l.pdl ? cudaGraphKernelNodePortProgrammatic : cudaGraphKernelNodePortDefault;
        ed.type = l.pdl ? cudaGraphDependencyTypeProgrammatic : cudaGraphDependencyTypeDefault;
        e = cudaGraphAddDependencies_v2(ge.graph, &prev, &node, &ed, 1);
      }
      if (e != cudaSuccess) {
        cudaGraphDestroy(ge.graph);
        return e;
      }
      ge.nodes.push_back(node);
      prev = node;
    }
    cudaError_t e = cudaGraphInstantiate(&ge.exec, ge.graph, 0);
    if (e != cudaSuccess) {
      cudaGraphDestroy(ge.graph);
      return e;
    }
    it = g_ts.graphs.emplace(key, std::move(ge)).first;
  }
  GraphEntry& ge = it->second;
  for (size_t i = 0; i < ls.size(); ++i) {
    void* argv[1];
    cudaKernelNodeParams kp = node_params(ls[i], argv);
    CUSORT_TRY(cudaGraphExecKernelNodeSetParams(ge.exec, ge.nodes[i], &kp));
  }
  return cudaGraphLaunch(ge.exec, stream);
}

// ---------------------------------------------------------------------------
// DispatchSort equivalent
// ---------------------------------------------------------------------------
struct SortCall {
  void* d_temp;
  size_t* temp_bytes;
  int kt;
  size_t vb;  // 0 = keys only
  bool desc;
  bool raw;
  // raw form
  const void* k_in;
  void* k_out;
  const void* v_in;
  void* v_out;
  // DoubleBuffer form
  cusort_double_buffer* kdb;
  cusort_double_buffer* vdb;
  int64_t n;
  int begin, end;
  cudaStream_t stream;
  bool force_direct;  // never build/replay a graph (no-allocation entry point)
};

static cudaError_t sort_impl(const SortCall& c) {
  const int kb = key_bytes_of(c.kt);
  if (kb == 0 || c.temp_bytes == nullptr) return cudaErrorInvalidValue;
  if (c.vb != 0 && !value_bytes_ok(c.vb)) return cudaErrorInvalidValue;
  if (c.begin < 0 || c.end < 0 || c.begin > c.end || c.end > 8 * kb) return cudaErrorInvalidValue;
  if (!c.raw && (c.kdb == nullptr || (c.vb && c.vdb == nullptr))) return cudaErrorInvalidValue;

  // Trivial calls (libcusort.cuh:2914-2931).
  if (c.n <= 1 || c.begin == c.end) {
    if (c.d_temp == nullptr) {
      *c.temp_bytes = (c.raw && c.n > 0) ? 1 : 0;
    } else if (c.raw && c.n > 0) {
      CUSORT_TRY(cudaMemcpyAsync(c.k_out, c.k_in, (size_t)c.n * kb, cudaMemcpyDeviceToDevice, c.stream));
      if (c.vb) CUSORT_TRY(cudaMemcpyAsync(c.v_out, c.v_in, (size_t)c.n * c.vb, cudaMemcpyDeviceToDevice, c.stream));
    }
    return cudaSuccess;
  }

  Plan p;
  if (!make_plan(c.kt, c.vb, c.desc, (uint64_t)c.n, c.begin, c.end, c.raw, &p)) return cudaErrorInvalidValue;
  if (c.d_temp == nullptr) {
    *c.temp_bytes = p.total;
    return cudaSuccess;
  }
  if (*c.temp_bytes < p.total) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(c.d_temp) & 15) != 0) return cudaErrorInvalidValue;

  PassBuffers b = {};
  if (c.raw) {
    // pass p writes `out` when (P-1-p) is even, the staging buffer otherwise,
    // so the last pass lands in `out` and `in` is never written.
    uint8_t* t = static_cast<uint8_t*>(c.d_temp);
    void* sk = t + p.off_stage_k;
    void* sv = t + p.off_stage_v;
    const void* ks = c.k_in;
    const void* vs = c.v_in;
    for (uint32_t i = 0; i < p.passes; ++i) {
      const bool to_out = ((p.passes - 1 - i) & 1u) == 0;
      b.k_src[i] = ks;
      b.k_dst[i] = to_out ? c.k_out : sk;
      b.v_src[i] = vs;
      b.v_dst[i] = to_out ? c.v_out : sv;
      ks = b.k_dst[i];
      vs = b.v_dst[i];
    }
  } else {
    int ksel = c.kdb->selector & 1, vsel = c.vb ? (c.vdb->selector & 1) : 0;
    for (uint32_t i = 0; i < p.passes; ++i) {
      b.k_src[i] = c.kdb->d_buffers[ksel];
      b.k_dst[i] = c.kdb->d_buffers[ksel ^ 1];
      if (c.vb) {
        b.v_src[i] = c.vdb->d_buffers[vsel];
        b.v_dst[i] = c.vdb->d_buffers[vsel ^ 1];
      }
      ksel ^= 1;
      vsel ^= 1;
    }
  }

  std::vector<Launch> ls;
  CUSORT_TRY(build_launches(p, c.d_temp, b, &ls));
  if (g_ts.launch_mode == 1 && !g_ts.timing && !c.force_direct)
    CUSORT_TRY(launch_graph(ls, c.stream));
  else
    CUSORT_TRY(launch_direct(ls, c.stream));

  if (!c.raw) {
    c.kdb->selector ^= (int)(p.passes & 1u);
    if (c.vb) c.vdb->selector ^= (int)(p.passes & 1u);
  }
  return cudaSuccess;
}

// Counts of one digit (bits [begin_bit, end_bit), at most 8 bits) of the
// twiddled keys into d_counts[256] (u64), using the all-pass histogram kernel
// with a single pass.  Used by the multi-GPU sort to plan the exchange.
cudaError_t digit_counts_u64(int kt, bool desc, const void* keys, int64_t n, int begin_bit, int end_bit,
                             unsigned long long* d_counts, cudaStream_t stream) {
  const int kb = key_bytes_of(kt);
  if (kb == 0 || begin_bit < 0 || end_bit <= begin_bit || end_bit - begin_bit > 8 || end_bit > 8 * kb)
    return cudaErrorInvalidValue;
  CUSORT_TRY(cudaMemsetAsync(d_counts, 0, kRadix * sizeof(unsigned long long), stream));
  if (n <= 0) return cudaSuccess;
  Plan p;
  // Any n >= 2^30 selects 64-bit counters; the onesweep kernel of this plan is unused.
  if (!make_plan(kt, 0, desc, std::max<uint64_t>((uint64_t)n, 1ull << 30), begin_bit, end_bit, false, &p))
    return cudaErrorInvalidValue;
  int dev = 0, sms = 0, occ_h = 0;
  CUSORT_TRY(cudaGetDevice(&dev));
  CUSORT_TRY(get_sm_count(dev, &sms));
  CUSORT_TRY(get_occupancy(dev, p.hist, &occ_h));
  HistArgs h = {};
  h.keys = keys;
  h.n = (uint64_t)n;
  h.tw_c = p.tw_c;
  h.tw_f = p.tw_f;
  h.begin_bit = (uint32_t)begin_bit;
  h.num_passes = 1;
  h.last_mask = p.last_mask;
  h.g_hist = d_counts;
  const uint64_t vec = (uint64_t)n * kb / 16 + 1;
  const uint64_t want = (vec + p.hist.tile - 1) / p.hist.tile;
  const int grid = (int)std::max<uint64_t>(1, std::min<uint64_t>((uint64_t)sms * occ_h, want));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3((unsigned)p.hist.threads);
  cfg.dynamicSmemBytes = p.hist.smem;
  cfg.stream = stream;
  void* args[1] = {&h};
  return cudaLaunchKernelExC(&cfg, p.hist.func, args);
}

cudaError_t routed_partition(int kt, size_t vb, bool desc, const void* keys, const void* vals, int64_t n,
                             int begin_bit, int end_bit, bool wide_offsets, const RouteTable* d_route, void* d_temp,
                             size_t* temp_bytes, cudaStream_t stream, bool keep_status) {
  const int kb = key_bytes_of(kt);
  if (kb == 0 || temp_bytes == nullptr || n < 0) return cudaErrorInvalidValue;
  if (vb != 0 && !value_bytes_ok(vb)) return cudaErrorInvalidValue;
  if (begin_bit < 0 || end_bit <= begin_bit || end_bit - begin_bit > kRadixBits || end_bit > 8 * kb)
    return cudaErrorInvalidValue;
  const int offb = (wide_offsets || (uint64_t)n >= (1ull << 30)) ? 8 : 4;
  const bool fk = (kt == CUSORT_KEY_F32 || kt == CUSORT_KEY_F64);
  KernelInfo os;
  bool ok = false;
  switch (kb) {
    case 1: case 2: ok = get_routed_k12(kb, (int)vb, offb, fk, &os); break;
    case 4: ok = get_routed_k4((int)vb, offb, fk, &os); break;
    case 8: ok = get_routed_k8((int)vb, offb, fk, &os); break;
    default: ok = false;
  }
  if (!ok) return cudaErrorInvalidValue;
  const uint64_t tiles = ((uint64_t)n + os.tile - 1) / os.tile;
  const size_t need = kCtrlBytes + align256((size_t)std::max<uint64_t>(tiles, 1) * kRadix * offb);
  if (d_temp == nullptr) {
    *temp_bytes = need;
    return cudaSuccess;
  }
  if (*temp_bytes < need || d_route == nullptr || (reinterpret_cast<uintptr_t>(d_temp) & 15) != 0)
    return cudaErrorInvalidValue;
  if (n == 0) return cudaSuccess;

  int dev = 0, sms = 0, occ = 0;
  CUSORT_TRY(cudaGetDevice(&dev));
  CUSORT_TRY(get_sm_count(dev, &sms));
  CUSORT_TRY(get_occupancy(dev, os, &occ));
  uint8_t* t = static_cast<uint8_t*>(d_temp);
  std::vector<Launch> ls(2);
  Launch& li = ls[0];
  li = Launch{};
  li.func = get_init_kernel();
  // keep_status: the status word (first 16 bytes) keeps the bits of earlier
  // passes that used this temp storage
  const uint64_t skip16 = keep_status ? 1 : 0;
  const uint64_t n16 = need / 16 - skip16;
  li.grid = (int)std::min<uint64_t>((uint64_t)sms * 4, std::max<uint64_t>(1, (n16 + 511) / 512));
  li.threads = 512;
  li.pdl = false;
  li.kind = 0;
  li.args.init.ptr = t + 16 * skip16;
  li.args.init.n16 = n16;
  Launch& l = ls[1];
  l = Launch{};
  l.func = os.func;
  l.grid = (int)std::max<uint64_t>(1, std::min<uint64_t>((uint64_t)sms * occ, tiles));
  l.threads = os.threads;
  l.smem = os.smem;
  l.pdl = true;
  l.kind = 2;
  OnesweepArgs& a = l.args.os;
  uint64_t tw_c = 0, tw_f = 0;
  twiddle_constants(kt, kb, desc, &tw_c, &tw_f);
  a.keys_in = keys;
  a.vals_in = vb ? vals : nullptr;
  a.n = (uint64_t)n;
  a.tw_c = tw_c;
  a.tw_f = tw_f;
  a.shift = (uint32_t)begin_bit;
  a.mask = (1u << (end_bit - begin_bit)) - 1u;
  a.pass = 0;
  a.num_tiles = (uint32_t)tiles;
  a.desc = t + kCtrlBytes;
  a.tile_counter = reinterpret_cast<uint32_t*>(t + 64);
  a.status = reinterpret_cast<uint32_t*>(t);
  a.spin_limit_ns = g_ts.wait_limit_ns;
  a.skip_tile = g_ts.skip_tile;
  const size_t tile_k = (size_t)os.tile * kb, tile_v = (size_t)os.tile * vb;
  a.tma_keys = ((reinterpret_cast<uintptr_t>(keys) & 15) == 0 && (tile_k & 15) == 0) ? 1u : 0u;
  a.tma_vals = (vb == 0 || ((reinterpret_cast<uintptr_t>(vals) & 15) == 0 && (tile_v & 15) == 0)) ? 1u : 0u;
  a.g_hist_pass = d_route;  // routed kernels read their RouteTable here
  return launch_direct(ls, stream);
}

void twiddle_constants_of(int kt, bool desc, uint64_t* c, uint64_t* f) {
  twiddle_constants(kt, key_bytes_of(kt), desc, c, f);
}

uint64_t wait_limit_ns() { return g_ts.wait_limit_ns; }

cudaError_t occupancy_of(const KernelInfo& k, int* sms, int* ctas_per_sm) {
  int dev = 0;
  CUSORT_TRY(cudaGetDevice(&dev));
  CUSORT_TRY(get_sm_count(dev, sms));
  return get_occupancy(dev, k, ctas_per_sm);
}

// DoubleBuffer sort whose temp storage is a caller-provided scratch region
// of `scratch_bytes` (used by the no-allocation entry point): rejects calls
// whose temp storage would not fit, and always launches directly.
cudaError_t sort_db_in_scratch(void* scratch, size_t scratch_bytes, int kt, size_t vb, bool desc,
                               cusort_double_buffer* k, cusort_double_buffer* v, int64_t n, int begin, int end,
                               cudaStream_t stream) {
  SortCall c = {};
  c.temp_bytes = nullptr;
  c.kt = kt;
  c.vb = vb;
  c.desc = desc;
  c.raw = false;
  c.kdb = k;
  c.vdb = v;
  c.n = n;
  c.begin = begin;
  c.end = end;
  c.stream = stream;
  c.force_direct = true;
  size_t need = 0;
  c.d_temp = nullptr;
  c.temp_bytes = &need;
  CUSORT_TRY(sort_impl(c));
  if (need > scratch_bytes) return cudaErrorInvalidValue;
  size_t have = scratch_bytes;
  c.d_temp = scratch;
  c.temp_bytes = &have;
  return sort_impl(c);
}

}  // namespace cusort_b200

using namespace cusort_b200;

namespace cusort_b200 {
cudaError_t sort_pairs_direct(void* t, size_t* tb, int kt, const void* ki, void* ko, size_t vb, const void* vi,
                              void* vo, int64_t n, int b, int e, bool desc, cudaStream_t s) {
  SortCall c = {};
  c.d_temp = t;
  c.temp_bytes = tb;
  c.kt = (int)kt;
  c.vb = vb;
  c.desc = desc;
  c.raw = true;
  c.k_in = ki;
  c.k_out = ko;
  c.v_in = vi;
  c.v_out = vo;
  c.n = n;
  c.begin = b;
  c.end = e;
  c.stream = s;
  return sort_impl(c);
}
}  // namespace cusort_b200

// In/out-pointer SortPairs of 8-byte keys with 16-byte values over 6 or more
// digit passes moves the keys with their 32-bit input positions through the
// passes and gathers the values once at the end (CUSORT_INDEX_PATH=1, the
// default): 12 instead of 24 bytes per item and pass, against one random
// 16-byte gather.  The result is the same: both are the stable sort.
// Measured on B200 at 2^26 (ms, direct -> index path): f64 keys + 16-byte
// values 7.03 -> 6.20; and not taken where it lost: u64 + 8-byte values 4.84
// -> 5.59, u32 + 16 bytes 2.92 -> 3.43, u16 + 16 bytes 1.46 -> 2.60 (random
// 8- and 16-byte reads of the gather run far below the streaming rate).
#ifndef CUSORT_INDEX_PATH
#define CUSORT_INDEX_PATH 1
#endif
static bool index_path_pays(int kt, size_t vb, int64_t n, int b, int e) {
  if (!CUSORT_INDEX_PATH || n < (int64_t)(1 << 20) || (uint64_t)n > 0xFFFFFFFFull || b < 0 || e <= b) return false;
  return vb == 16 && key_bytes_of(kt) == 8 && (e - b + 7) / 8 >= 6;
}

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
extern "C" {

static cudaError_t sort_db(void* t, size_t* tb, cusort_key_type kt, cusort_double_buffer* k, size_t vb,
                           cusort_double_buffer* v, int64_t n, int b, int e, bool desc, cudaStream_t s) {
  SortCall c = {};
  c.d_temp = t;
  c.temp_bytes = tb;
  c.kt = (int)kt;
  c.vb = vb;
  c.desc = desc;
  c.raw = false;
  c.kdb = k;
  c.vdb = v;
  c.n = n;
  c.begin = b;
  c.end = e;
  c.stream = s;
  return sort_impl(c);
}

static cudaError_t sort_raw(void* t, size_t* tb, cusort_key_type kt, const void* ki, void* ko, size_t vb,
                            const void* vi, void* vo, int64_t n, int b, int e, bool desc, cudaStream_t s) {
  SortCall c = {};
  c.d_temp = t;
  c.temp_bytes = tb;
  c.kt = (int)kt;
  c.vb = vb;
  c.desc = desc;
  c.raw = true;
  c.k_in = ki;
  c.k_out = ko;
  c.v_in = vi;
  c.v_out = vo;
  c.n = n;
  c.begin = b;
  c.end = e;
  c.stream = s;
  return sort_impl(c);
}

cudaError_t cusort_sort_keys_db(void* t, size_t* tb, cusort_key_type kt, cusort_double_buffer* k, int64_t n, int b,
                                int e, cudaStream_t s) {
  return sort_db(t, tb, kt, k, 0, nullptr, n, b, e, false, s);
}
cudaError_t cusort_sort_keys_descending_db(void* t, size_t* tb, cusort_key_type kt, cusort_double_buffer* k,
                                           int64_t n, int b, int e, cudaStream_t s) {
  return sort_db(t, tb, kt, k, 0, nullptr, n, b, e, true, s);
}
cudaError_t cusort_sort_pairs_db(void* t, size_t* tb, cusort_key_type kt, cusort_double_buffer* k, size_t vb,
                                 cusort_double_buffer* v, int64_t n, int b, int e, cudaStream_t s) {
  if (vb == 0) return cudaErrorInvalidValue;
  return sort_db(t, tb, kt, k, vb, v, n, b, e, false, s);
}
cudaError_t cusort_sort_pairs_descending_db(void* t, size_t* tb, cusort_key_type kt, cusort_double_buffer* k,
                                            size_t vb, cusort_double_buffer* v, int64_t n, int b, int e,
                                            cudaStream_t s) {
  if (vb == 0) return cudaErrorInvalidValue;
  return sort_db(t, tb, kt, k, vb, v, n, b, e, true, s);
}
cudaError_t cusort_sort_keys(void* t, size_t* tb, cusort_key_type kt, const void* ki, void* ko, int64_t n, int b,
                             int e, cudaStream_t s) {
  return sort_raw(t, tb, kt, ki, ko, 0, nullptr, nullptr, n, b, e, false, s);
}
cudaError_t cusort_sort_keys_descending(void* t, size_t* tb, cusort_key_type kt, const void* ki, void* ko,
                                        int64_t n, int b, int e, cudaStream_t s) {
  return sort_raw(t, tb, kt, ki, ko, 0, nullptr, nullptr, n, b, e, true, s);
}
cudaError_t cusort_sort_pairs(void* t, size_t* tb, cusort_key_type kt, const void* ki, void* ko, size_t vb,
                              const void* vi, void* vo, int64_t n, int b, int e, cudaStream_t s) {
  if (vb == 0) return cudaErrorInvalidValue;
  if (index_path_pays((int)kt, vb, n, b, e))
    return sort_pairs_by_index(t, tb, (int)kt, ki, ko, vb, vi, vo, n, b, e, 0, s);
  return sort_raw(t, tb, kt, ki, ko, vb, vi, vo, n, b, e, false, s);
}
cudaError_t cusort_sort_pairs_descending(void* t, size_t* tb, cusort_key_type kt, const void* ki, void* ko,
                                         size_t vb, const void* vi, void* vo, int64_t n, int b, int e,
                                         cudaStream_t s) {
  if (vb == 0) return cudaErrorInvalidValue;
  if (index_path_pays((int)kt, vb, n, b, e))
    return sort_pairs_by_index(t, tb, (int)kt, ki, ko, vb, vi, vo, n, b, e, 1, s);
  return sort_raw(t, tb, kt, ki, ko, vb, vi, vo, n, b, e, true, s);
}

const char* cusort_version(void) { return "1.0.1-b200.1"; }

int cusort_set_launch_mode(int mode) {
  const int prev = g_ts.launch_mode;
  if (mode == 0 || mode == 1) g_ts.launch_mode = mode;
  return prev;
}

cudaError_t cusort_read_device_status(const void* d_temp_storage, uint32_t* status, cudaStream_t stream) {
  if (d_temp_storage == nullptr || status == nullptr) return cudaErrorInvalidValue;
  CUSORT_TRY(cudaMemcpyAsync(status, d_temp_storage, sizeof(uint32_t), cudaMemcpyDeviceToHost, stream));
  return cudaStreamSynchronize(stream);
}

uint64_t cusort_set_wait_limit_ns(uint64_t ns) {
  const uint64_t prev = g_ts.wait_limit_ns;
  if (ns > 0) g_ts.wait_limit_ns = ns;
  return prev;
}

int64_t cusort_debug_set_skip_tile(int64_t tile) {
  const int64_t prev = g_ts.skip_tile;
  g_ts.skip_tile = tile;
  return prev;
}

int cusort_set_kernel_timing(int enable) {
  const int prev = g_ts.timing;
  g_ts.timing = enable ? 1 : 0;
  return prev;
}

int cusort_get_kernel_times(float* ms, int* kinds, int capacity) {
  const int n = g_ts.recorded;
  if (n == 0) return 0;
  if (cudaEventSynchronize(g_ts.events[2 * n - 1]) != cudaSuccess) return -1;
  const int m = std::min(n, capacity);
  for (int i = 0; i < m; ++i) {
    float v = 0.f;
    cudaEventElapsedTime(&v, g_ts.events[2 * i], g_ts.events[2 * i + 1]);
    if (ms) ms[i] = v;
    if (kinds) kinds[i] = g_ts.kinds[i];
  }
  return m;
}

cudaError_t cusort_query_plan(cusort_key_type kt, size_t vb, int64_t n, int begin, int end, int* passes,
                              int* tile_items, int* onesweep_grid, int* histogram_grid, int* offset_bytes) {
  const int kb = key_bytes_of((int)kt);
  if (kb == 0 || (vb != 0 && !value_bytes_ok(vb)) || n < 2 || begin < 0 || begin >= end || end > 8 * kb)
    return cudaErrorInvalidValue;
  Plan p;
  if (!make_plan((int)kt, vb, false, (uint64_t)n, begin, end, false, &p)) return cudaErrorInvalidValue;
  if (passes) *passes = (int)p.passes;
  if (tile_items) *tile_items = p.os.tile;
  if (offset_bytes) *offset_bytes = p.offb;
  if (onesweep_grid || histogram_grid) {
    int dev = 0, sms = 0, occ_os = 0, occ_h = 0;
    CUSORT_TRY(cudaGetDevice(&dev));
    CUSORT_TRY(get_sm_count(dev, &sms));
    CUSORT_TRY(get_occupancy(dev, p.os, &occ_os));
    CUSORT_TRY(get_occupancy(dev, p.hist, &occ_h));
    if (onesweep_grid) *onesweep_grid = (int)std::min<uint64_t>((uint64_t)sms * occ_os, p.tiles);
    if (histogram_grid) *histogram_grid = sms * occ_h;
  }
  return cudaSuccess;
}

}  // extern "C"

// cusort_device.cuh -- device-side building blocks for the B200 radix sort.
//
// PTX wrappers (relaxed GPU-scope loads/stores, globaltimer, mbarrier, 1-D TMA
// bulk copy, programmatic-dependent-launch controls), the key bit-twiddle and
// the warp ranking primitive.  Everything here is sm_100a-only.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "cusort_types.h"

namespace cusort_b200 {
namespace dev {

template <int B> struct UIntOf;
template <> struct UIntOf<1> { using T = uint8_t; };
template <> struct UIntOf<2> { using T = uint16_t; };
template <> struct UIntOf<4> { using T = uint32_t; };
template <> struct UIntOf<8> { using T = unsigned long long; };
template <> struct UIntOf<16> { using T = uint4; };

// ---------------------------------------------------------------------------
// Key bit-twiddle.  Reference semantics: traits::RadixTraits::Twiddle
// (libcusort.cuh:398-429).  Here the per-type xor table is folded into two
// launch-uniform constants so every key type of one width shares one kernel:
//     t = x ^ C ^ (sext(msb(x)) & F)
//   unsigned      : C = 0,   F = 0         (descending: C = ~0)
//   signed        : C = SB,  F = 0         (descending: C = ~SB)
//   float/double  : C = SB,  F = ~SB       (descending: C = ~SB)
// (SB = sign bit).  For floats a set sign bit flips every bit, a clear one
// flips only the sign bit; descending inverts the result.
// ---------------------------------------------------------------------------
template <typename U>
__device__ __forceinline__ U twiddle(U x, U c, U f) {
  constexpr int NB = sizeof(U) * 8;
  U s;
  if constexpr (NB == 64) {
    s = (U)((long long)x >> 63);
  } else {
    // Sign-extend the key's own MSB to the full width of U.
    s = (U)((int32_t)((uint32_t)x << (32 - NB)) >> 31);
  }
  return (U)(x ^ c ^ (s & f));
}

template <typename U>
__device__ __forceinline__ uint32_t digit_of(U x, U c, U f, uint32_t shift, uint32_t mask) {
  return (uint32_t)(twiddle<U>(x, c, f) >> shift) & mask;
}

// Twiddle of one key type class: integer keys only need the xor constant
// (F == 0), floating-point keys the sign-dependent term as well.
template <bool FLOAT_KEY, typename U>
__device__ __forceinline__ U twiddle_k(U x, U c, U f) {
  if constexpr (FLOAT_KEY) return twiddle<U>(x, c, f);
  else return (U)(x ^ c);
}
template <bool FLOAT_KEY, typename U>
__device__ __forceinline__ uint32_t digit_k(U x, U c, U f, uint32_t shift, uint32_t mask) {
  return (uint32_t)(twiddle_k<FLOAT_KEY, U>(x, c, f) >> shift) & mask;
}

// The same value through an opaque register move: the compiler cannot merge
// computations on the result with computations on the original (used to keep
// it from holding derived values live across long stretches of code).
__device__ __forceinline__ uint8_t opaque(uint8_t x) {
  uint32_t t = x;
  asm volatile("mov.b32 %0, %0;" : "+r"(t));
  return (uint8_t)t;
}
__device__ __forceinline__ uint16_t opaque(uint16_t x) {
  uint32_t t = x;
  asm volatile("mov.b32 %0, %0;" : "+r"(t));
  return (uint16_t)t;
}
__device__ __forceinline__ uint32_t opaque(uint32_t x) {
  asm volatile("mov.b32 %0, %0;" : "+r"(x));
  return x;
}
__device__ __forceinline__ unsigned long long opaque(unsigned long long x) {
  asm volatile("mov.b64 %0, %0;" : "+l"(x));
  return x;
}

// Streaming (evict-first) global loads of one element.
__device__ __forceinline__ uint8_t ld_cs(const uint8_t* p) {
  uint16_t v;
  asm volatile("ld.global.cs.u8 %0, [%1];" : "=h"(v) : "l"(p));
  return (uint8_t)v;
}
__device__ __forceinline__ uint16_t ld_cs(const uint16_t* p) {
  uint16_t v;
  asm volatile("ld.global.cs.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ld_cs(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.global.cs.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ unsigned long long ld_cs(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.global.cs.u64 %0, [%1];" : "=l"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ uint4 ld_cs(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.cs.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// ---------------------------------------------------------------------------
// PTX helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t r;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t ld_relaxed(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long ld_relaxed(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Programmatic dependent launch (sm_90+): wait for the prerequisite grid's
// completion + memory flush / allow the dependent grid to start launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// Orders this thread's generic-proxy shared-memory accesses before later
// async-proxy (TMA) accesses to the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// 1-D bulk copy global -> shared (TMA engine), completion counted on `bar`.
// dst, src and bytes must all be multiples of 16.  No multicast.
__device__ __forceinline__ void tma_load_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Streaming 16-byte global load that does not allocate in L1.
__device__ __forceinline__ uint4 ld_stream_v4(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// ---------------------------------------------------------------------------
// Bounded wait bookkeeping.  Every spin in this library gives up after
// `limit_ns` of wall time (or as soon as another thread has raised an error),
// records a status bit and lets the kernel run to completion.
// ---------------------------------------------------------------------------
// `status` may be null: a wait on this thread's own bulk copy must not give up
// because of another CTA's error (the copy would still be in flight).
struct SpinGuard {
  uint64_t t0 = 0;
  __device__ __forceinline__ bool expired(const uint32_t* status, uint64_t limit_ns) {
    if (status != nullptr && *(volatile const uint32_t*)status != 0) return true;
    uint64_t now = globaltimer_ns();
    if (t0 == 0) {
      t0 = now;
      return false;
    }
    return now - t0 > limit_ns;
  }
};

// ---------------------------------------------------------------------------
// Warp ranking.  For one "slot" (one key per lane, lane order = input order)
// returns the number of earlier lanes holding the same digit plus the running
// count of that digit in earlier slots of this warp, and advances the count.
//
// The peer set is found with one shared-memory atomicOr of the lane bit into a
// per-warp, per-digit 64-bit word [count:32 | lane mask:32]; after a warp
// barrier every lane reads its digit's word, and the highest peer lane writes
// back (count + peers, mask 0), which both advances the count and clears the
// mask for the next slot.  On B200 this is ~2x the throughput of an 8-ballot
// match and ~4x the hardware match.any for uniformly random 8-bit digits.
// Reference counterpart (different method, same result): ballot-based
// match_any_sync + leader atomic in the onesweep kernel (libcusort.cuh:1032-1109,
// 2126-2152).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t warp_rank_slot(unsigned long long* wtab, uint32_t digit, uint32_t lane,
                                                   uint32_t lt) {
  atomicOr(reinterpret_cast<unsigned int*>(wtab + digit), 1u << lane);
  __syncwarp();
  const unsigned long long w = wtab[digit];
  __syncwarp();
  const uint32_t peers = (uint32_t)w;
  const uint32_t base = (uint32_t)(w >> 32);
  const uint32_t below = __popc(peers & lt);
  if ((peers >> lane) == 1u) wtab[digit] = (unsigned long long)(base + below + 1u) << 32;
  __syncwarp();
  return base + below;
}

// Ballot-based alternative (kept for measurement; selected at compile time).
template <int BITS>
__device__ __forceinline__ uint32_t match_digit_ballot(uint32_t d) {
  uint32_t m = 0xffffffffu;
#pragma unroll
  for (int b = 0; b < BITS; ++b) {
    const uint32_t bit = (d >> b) & 1u;
    const uint32_t v = __ballot_sync(0xffffffffu, bit);
    m &= ~(v ^ (0u - bit));
  }
  return m;
}

// Predicated shared-memory atomic add (no branch): when `pred` is false the
// instruction is skipped and the previous content of `old` is returned.
__device__ __forceinline__ uint32_t atom_add_shared_if(uint32_t pred, uint32_t* addr, uint32_t v, uint32_t old) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.u32 p, %1, 0;\n @p atom.shared.add.u32 %0, [%2], %3;\n}\n"
      : "+r"(old)
      : "r"(pred), "r"(smem_u32(addr)), "r"(v)
      : "memory");
  return old;
}

// Inclusive warp scan (shfl_up) of 32-bit values.
template <typename T>
__device__ __forceinline__ T warp_inclusive_scan(T v, uint32_t lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    T t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= (uint32_t)o) v += t;
  }
  return v;
}

}  // namespace dev
}  // namespace cusort_b200

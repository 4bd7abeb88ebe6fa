// nsq_common.cuh -- shared device helpers for libnsq (sm_100a only).
//
// Block formats (GGUF/ggml byte layouts), exact fp16 scale decoding,
// mbarrier / bulk-copy PTX wrappers and the bounded-wait policy.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/nsq.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libnsq is built for sm_100a only"
#endif

namespace nsq {

// ---------------------------------------------------------------------------
// Device status word: kernels whose bounded waits give up write an NSQ_ERR_*
// code here (first writer wins) and return; the host reads it through
// nsq_device_status().
extern __device__ int g_device_status;

__device__ __forceinline__ void report_status(int code) { atomicCAS(&g_device_status, 0, code); }

// Bounded waits: give up after this many nanoseconds of %globaltimer.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// Format traits
template <int T>
struct Fmt;
template <>
struct Fmt<NSQ_TYPE_Q4_0> {
  static constexpr int QK = 32, BB = 18, UW = 32;  // UW = weights per GEMV unit
};
template <>
struct Fmt<NSQ_TYPE_Q8_0> {
  static constexpr int QK = 32, BB = 34, UW = 32;
};
template <>
struct Fmt<NSQ_TYPE_Q4_K> {
  static constexpr int QK = 256, BB = 144, UW = 64;
};
template <>
struct Fmt<NSQ_TYPE_Q5_K> {
  static constexpr int QK = 256, BB = 176, UW = 64;
};
template <>
struct Fmt<NSQ_TYPE_Q6_K> {
  static constexpr int QK = 256, BB = 210, UW = 64;
};

// Exact IEEE fp16 -> f32 (subnormals included), the reference's half_to_f32
// (crates/nodestor-inference/src/dequant/mod.rs:234-260).
__device__ __forceinline__ float h2f(uint16_t bits) { return __half2float(__ushort_as_half(bits)); }
// Bits 0..3 of nib to bit 0 of bytes 0..3 (the four products land on
// disjoint bit ranges, so no carries).
__device__ __forceinline__ uint32_t spread4(uint32_t nib) { return (nib * 0x00204081u) & 0x01010101u; }

// ---------------------------------------------------------------------------
// Byte access helpers.  Blocks of Q4_0 / Q8_0 / Q6_K are only 2-byte aligned,
// so runs of bytes are assembled from aligned 32-bit words.
__device__ __forceinline__ uint32_t ld_u8(const uint8_t* p) { return *p; }
__device__ __forceinline__ uint32_t ld_u16(const uint8_t* p) {  // p 2-aligned
  return *reinterpret_cast<const uint16_t*>(p);
}
// NW consecutive little-endian 32-bit words starting at any byte address of
// shared memory (reads NW+1 aligned words).
template <int NW>
__device__ __forceinline__ void ld_words_unaligned(const uint8_t* p, uint32_t (&w)[NW]) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* base = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  const uint32_t sh = (uint32_t)(a & 3) * 8;
  uint32_t r[NW + 1];
#pragma unroll
  for (int i = 0; i < NW + 1; ++i) r[i] = base[i];
#pragma unroll
  for (int i = 0; i < NW; ++i) w[i] = __funnelshift_r(r[i], r[i + 1], sh);
}

// ---------------------------------------------------------------------------
// mbarrier + bulk async copy (TMA, non-multicast) wrappers.
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait with a suspend-time hint: the thread sleeps until the phase
// completes or `hint_ns` passes, instead of spinning on issue slots.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
// Bounded wait on a phase parity: returns false (and records NSQ_ERR_TIMEOUT)
// if the phase has not completed within kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait_sleep(bar, parity, 1000000u)) {
    if (globaltimer() - t0 > kWaitLimitNs) {
      report_status(NSQ_ERR_TIMEOUT);
      return false;
    }
  }
  return true;
}
// 1-D bulk copy global -> shared, completion counted on `bar` (bytes).
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// L2 eviction policies (createpolicy).  Weights are read once per launch:
// copied with evict_first they do not push activations and other reused
// lines out of the L2; activations are read with evict_last.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// bulk_g2s with an L2 cache policy
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
// read-only 16-byte load with an L2 cache policy
__device__ __forceinline__ float4 ldg_f4_hint(const float4* p, uint64_t policy) {
  float4 v;
  asm volatile("ld.global.nc.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p), "l"(policy));
  return v;
}

// dp4a variants: sum of 4 byte products added to c.
__device__ __forceinline__ int dp4a_us(uint32_t a_u8x4, uint32_t b_s8x4, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a_u8x4), "r"(b_s8x4), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_uu(uint32_t a_u8x4, uint32_t b_u8x4, int c) {
  int d;
  asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a_u8x4), "r"(b_u8x4), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a_s8x4, uint32_t b_s8x4, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a_s8x4), "r"(b_s8x4), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_su(uint32_t a_s8x4, uint32_t b_u8x4, int c) {
  int d;
  asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a_s8x4), "r"(b_u8x4), "r"(c));
  return d;
}

// ---------------------------------------------------------------------------
// Prepared activation record: one per (token m, group of 32 activations g).
// x[m, 32g + i] ~= sx * (hi[i] * 256 + lo[i]), |hi*256+lo| <= 32767, and
// s16[h] = sum_{i in 16h..16h+15} (hi[i]*256 + lo[i]).
struct __align__(16) XGroup {
  int8_t hi[32];
  uint8_t lo[32];
  float sx;
  int32_t s16[2];
  int32_t pad;
};
static_assert(sizeof(XGroup) == 80, "XGroup must be 80 bytes");


// ---------------------------------------------------------------------------
// Cross-GPU exchange (peer memory through CUDA IPC mappings).  The first
// kXchgCtlBytes of every exchange buffer hold the control words: flag[r]
// (written by rank r over NVLink: the sequence number of r's latest
// exchange), then this rank's own exchange count and CTA counter.
constexpr int kXchgCtlBytes = 256;
constexpr int kXchgSeq = 16;   // u32 index of the local exchange count
constexpr int kXchgDone = 32;  // u32 index of the local finished-CTA counter

// Host-side description of one exchange launch (filled from an nsq_comm).
struct XchgDesc {
  int P = 1, rank = 0;
  bool wait = true;  // the GEMV waits for the previous exchange itself
  uint8_t* buf[NSQ_MAX_RANKS] = {};  // exchange buffer of each rank, mapped here
  int64_t row0[NSQ_MAX_SEGMENTS] = {}, nfull[NSQ_MAX_SEGMENTS] = {}, off[NSQ_MAX_SEGMENTS] = {};
};

// Release/acquire fence at GPU scope.  The CTAs of an exchange grid order
// their stores (peer stores included) before a counter with it; only the
// grid's last CTA talks to other GPUs, through release stores at system
// scope, and happens-before is transitive across the two scopes.
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Waits until *p - want >= 0 (wrapping); false (and NSQ_ERR_TIMEOUT) after
// kWaitLimitNs.
__device__ __forceinline__ bool wait_geq_bounded(const uint32_t* p, uint32_t want) {
  if ((int32_t)(ld_acquire_sys(p) - want) >= 0) return true;
  const uint64_t t0 = globaltimer();
  for (;;) {
    __nanosleep(128);
    if ((int32_t)(ld_acquire_sys(p) - want) >= 0) return true;
    if (globaltimer() - t0 > kWaitLimitNs) {
      report_status(NSQ_ERR_TIMEOUT);
      return false;
    }
  }
}

// Launch-planning switches: the NSQ_* environment variables below, read
// once, when the library plans its first launch (nsq_reload_tuning reads
// them again).  tune(id, dflt) gives the variable's integer value, or dflt
// when it is unset or empty.  The defaults the planners pass are the
// measured choices; the switches exist for tests and tuning runs.
enum TuneId : int {
  kTuneRowsR, kTuneRowsPPSM, kTuneRowsStages, kTuneRowsPre, kTuneRowsL2Hint, kTuneRowsCPS, kTuneRowsC,
  kTuneRowsBal, kTuneRowsCarve, kTuneMmaMinM, kTuneMmaPPS, kTuneMmaStages, kTuneGemvGeneral, kTuneGemmSplit,
  kTuneGemmTok, kTuneTcMinM, kTuneTcA, kTuneCount
};
int tune(TuneId id, int dflt);
// Counts one kernel launch (nsq_kernel_launches).
void note_launch();

}  // namespace nsq

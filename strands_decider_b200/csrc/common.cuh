// Shared device helpers for the strands-decider B200 backend (sm_100a only).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <utility>

#include "strands_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "this library targets sm_100a (B200) only"
#endif

namespace sdb {

// ----------------------------------------------------------------------------- faults
// A device-side fault word. Every bounded wait that gives up ORs its site code in here and
// the kernel carries on to a clean exit; the host reads and clears it with b200_read_fault.
extern __device__ unsigned int g_fault;

enum FaultSite : unsigned int {
  FAULT_GEMM_WAIT_EMPTY = 1u << 0,
  FAULT_GEMM_WAIT_FULL_A = 1u << 1,
  FAULT_GEMM_WAIT_FULL_B = 1u << 2,
  FAULT_GEMM_WAIT_ACCUM = 1u << 3,
  FAULT_GEMM_WAIT_FULL_W = 1u << 4,
  FAULT_GDN_WAIT_STAGE = 1u << 5,
  FAULT_BAD_INDEX = 1u << 8,
};

__device__ __forceinline__ void raise_fault(unsigned int site) { atomicOr(&g_fault, site); }

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Spin limit for every mbarrier wait: a legitimate wait inside one kernel is microseconds.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// ----------------------------------------------------------------------------- bf16

__device__ __forceinline__ float bf16_to_f32(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }

__device__ __forceinline__ uint16_t f32_to_bf16_rn(float x) {
  __nv_bfloat16 h = __float2bfloat16_rn(x);
  return *reinterpret_cast<uint16_t*>(&h);
}

// {bf16_rn(lo), bf16_rn(hi)} in one conversion (lo in the low half)
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// the two halves of a packed pair h = pack_bf16x2(a, b) as floats: bf16_rn(a), bf16_rn(b)
__device__ __forceinline__ float bf16x2_lo(uint32_t h) { return __uint_as_float(h << 16); }
__device__ __forceinline__ float bf16x2_hi(uint32_t h) { return __uint_as_float(h & 0xffff0000u); }
// the low plane of a pair packed as h = pack_bf16x2(a, b): {bf16_rn(a - hi(a)), bf16_rn(b - hi(b))}
__device__ __forceinline__ uint32_t lo_pair(float a, float b, uint32_t h) {
  return pack_bf16x2(a - bf16x2_lo(h), b - bf16x2_hi(h));
}

// ----------------------------------------------------------------------------- e4m3 low plane
// With B200_LO_E4M3 the low activation plane lo = x - bf16(x) is stored as
// e4m3(lo * 2^B200_LO8_X_SHIFT): one byte per element, at the same element index as the hi
// plane (so a row of ldx elements is ldx bytes). Conversions round to nearest even and
// saturate at +-448.
__device__ __forceinline__ uint16_t f32x2_to_e4m3x2(float a, float b) {  // a -> low byte
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(b), "f"(a));
  return r;
}
__device__ __forceinline__ uint32_t e4m3x4(float a, float b, float c, float d) {
  return uint32_t(f32x2_to_e4m3x2(a, b)) | (uint32_t(f32x2_to_e4m3x2(c, d)) << 16);
}
// The stored low-plane byte of x given its hi plane value h (bf16 bits).
__device__ __forceinline__ float lo8_value(float x, uint16_t h) {
  return (x - bf16_to_f32(h)) * float(1 << B200_LO8_X_SHIFT);
}

// Four consecutive activations at element e (e % 4 == 0) of a hi/lo plane pair: the hi
// plane bf16_rn(v) at out[e]; the lo plane at out + lo_offset as bf16_rn(v - hi), or as its
// e4m3 byte with lo8; no lo plane when lo_offset is 0.
__device__ __forceinline__ void store_planes4(uint16_t* out, long long lo_offset, bool lo8, size_t e, float a,
                                              float b, float c, float d) {
  const uint32_t h01 = pack_bf16x2(a, b), h23 = pack_bf16x2(c, d);
  *reinterpret_cast<uint2*>(out + e) = make_uint2(h01, h23);
  if (!lo_offset) return;
  if (lo8) {
    constexpr float S = float(1 << B200_LO8_X_SHIFT);
    *reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(out + lo_offset) + e) =
        e4m3x4((a - bf16x2_lo(h01)) * S, (b - bf16x2_hi(h01)) * S, (c - bf16x2_lo(h23)) * S,
               (d - bf16x2_hi(h23)) * S);
  } else {
    *reinterpret_cast<uint2*>(out + lo_offset + e) = make_uint2(lo_pair(a, b, h01), lo_pair(c, d, h23));
  }
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }
__device__ __forceinline__ float sigmoid(float x) { return 1.0f / (1.0f + __expf(-x)); }
// sigmoid with the approximate division (2 ulp; 0 for very negative x)
__device__ __forceinline__ float sigmoid_approx(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }
// silu with the approximate division (__fdividef, 2 ulp; x / inf = 0 for very negative x):
// for instruction-bound elementwise loops
__device__ __forceinline__ float silu_approx(float x) { return __fdividef(x, 1.0f + __expf(-x)); }
__device__ __forceinline__ float softplus(float x) { return x > 20.0f ? x : log1pf(__expf(x)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ----------------------------------------------------------------------------- smem / mbarrier

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete, giving up after kWaitLimitNs.
// Returns false (and records `site`) on give-up; the caller then proceeds as if complete.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int site) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t it = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++it & 1023u) == 0) {
      // once any wait on this device has given up, every other wait gives up at once,
      // so a systematic failure ends each launch quickly instead of 2 s per stage
      if (*reinterpret_cast<volatile unsigned int*>(&g_fault) != 0) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        raise_fault(site);
        return false;
      }
    }
  }
}

// mbar_wait for waiters off the critical path (a warp that idles until a late phase): after
// each failed test the thread sleeps, so that it takes no issue slots from the warps that
// produce the phase.
__device__ __forceinline__ bool mbar_wait_idle(uint64_t* bar, uint32_t parity, unsigned int site) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t it = 0;
  while (true) {
    __nanosleep(256);
    if (mbar_try_wait(bar, parity)) return true;
    if ((++it & 63u) == 0) {
      if (*reinterpret_cast<volatile unsigned int*>(&g_fault) != 0) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        raise_fault(site);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ----------------------------------------------------------------------------- TMA

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y)
      : "memory");
}

// 3-D / 4-D tiled loads (coordinates innermost first); the innermost coordinate x times the
// element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z,
                                            int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

// 1-D bulk copy global -> shared (16-byte aligned addresses, size a multiple of 16).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}

// Programmatic dependent launch: a kernel launched with programmatic stream serialization
// may start while the previous kernel in the stream finishes; it must call pdl_wait() before
// touching any memory that kernel reads or writes. pdl_trigger() lets the next such kernel
// be scheduled once every CTA of this one has issued it. Both are no-ops without PDL.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Prefetch [src, src + bytes) into L2 (16-byte aligned address, size a multiple of 16).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ----------------------------------------------------------------------------- tcgen05

// Shared-memory matrix descriptor for a K-major operand tile stored in the 128-byte swizzle
// layout (rows of 128 bytes, 8-row groups of 1024 bytes): start address >> 4 in bits 0-13,
// leading byte offset (unused by swizzled K-major; 1) in 16-29, stride byte offset
// 1024 >> 4 in 32-45, descriptor version 1 in 46-47, layout SWIZZLE_128B (2) in 61-63.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  return uint64_t((saddr >> 4) & 0x3FFFu) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// Shared-memory descriptor for an MN-major operand stored as 128-byte-swizzled tiles of 64
// MN-elements (bf16) x K rows, 128 bytes per K row (what a TMA box of 64 elements x rows writes):
// the 8-row K groups are `sbo` bytes apart and the 64-element MN atoms `lbo` bytes apart.
__device__ __forceinline__ uint64_t umma_desc_sw128_mn(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return uint64_t((saddr >> 4) & 0x3FFFu) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
         (uint64_t((sbo >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// Same for a K-major tile of 64-byte rows written by TMA with 64-byte swizzle (an e4m3
// tile 64 k wide): 8-row core groups 512 bytes apart.
__device__ __forceinline__ uint64_t umma_desc_sw64(uint32_t saddr) {
  return uint64_t((saddr >> 4) & 0x3FFFu) | (uint64_t(1) << 16) | (uint64_t(512 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(4) << 61);
}

// Instruction descriptor, kind::f8f6f4: D fp32, A and B e4m3 (format code 0), both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_e4m3(int M, int N) {
  return (1u << 4) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

// Instruction descriptor, kind::f16: D fp32, A and B bf16, both K-major, M x N.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D (+)= A * B with A read from tensor memory (128 lanes = A's rows, two bf16 of K per 32-bit
// column, lower k in the low half) and B from shared memory.
__device__ __forceinline__ void umma_bf16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D (+)= A * B for e4m3 A and B, K = 32 per instruction, fp32 accumulate in TMEM.
__device__ __forceinline__ void umma_e4m3(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// ---- CTA pairs (clusters of 2) for tcgen05 .cta_group::2
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address in the cluster window of the same shared variable in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(saddr), "r"(rank));
  return d;
}
// All threads of both CTAs (release / acquire at cluster scope).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx_cluster(uint32_t cluster_addr, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cluster.shared::cluster.b64 _, [%0], %1;" ::"r"(cluster_addr),
               "r"(bytes)
               : "memory");
}
// L2 policy for data re-read by many CTAs over a kernel's life (GEMM weight tiles): kept in
// L2 ahead of streamed activations.
__device__ __forceinline__ uint64_t l2_evict_last_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%3, "
      "%4}], [%2], %5;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
// 2-D TMA load into this CTA's shared memory whose completion (complete_tx) is signalled
// on an mbarrier that may sit in the pair's other CTA (cluster-window address). No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tma_load_2d_pair_hint(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int x,
                                                      int y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
      "[%1, {%3, %4}], [%2], %5;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
// M = 256 MMAs over the pair: rows 0..127 of A (and columns 0..N/2-1 of B) from this CTA's
// shared memory, the rest from the other CTA's at the same offsets; D rows split likewise.
__device__ __forceinline__ void umma_pair_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_pair_e4m3(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on an mbarrier (cluster-window address, either CTA of the pair) once every
// pair MMA issued so far by this thread has completed.
__device__ __forceinline__ void umma_pair_commit(uint32_t bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
               : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// 32 lanes x 32 columns of 32-bit accumulators: this thread gets its lane's 32 columns.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// This thread's 16 words into 16 consecutive columns of its lane (the warp's 32-lane quarter).
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint4 (&v)[4]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0].x), "r"(v[0].y), "r"(v[0].z), "r"(v[0].w), "r"(v[1].x), "r"(v[1].y), "r"(v[1].z), "r"(v[1].w),
      "r"(v[2].x), "r"(v[2].y), "r"(v[2].z), "r"(v[2].w), "r"(v[3].x), "r"(v[3].y), "r"(v[3].z), "r"(v[3].w)
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

}  // namespace sdb

// ----------------------------------------------------------------------------- host helpers
#define SDB_CUDA(call)                                   \
  do {                                                   \
    cudaError_t e_ = (call);                             \
    if (e_ != cudaSuccess) {                             \
      sdb_set_last_error(cudaGetErrorString(e_));        \
      return B200_ERR_CUDA;                              \
    }                                                    \
  } while (0)

#define SDB_LAUNCH_CHECK()                                         \
  do {                                                             \
    cudaError_t e_ = cudaGetLastError();                           \
    if (e_ != cudaSuccess) {                                       \
      sdb_set_last_error(cudaGetErrorString(e_));                  \
      return B200_ERR_CUDA;                                        \
    }                                                              \
  } while (0)

namespace sdb {
// Launch `k` with programmatic stream serialization: it may be scheduled once the kernel
// before it in the stream has issued pdl_trigger() in every CTA, and it must pdl_wait()
// before its first access to memory that kernel touches. Returns the launch status.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, std::forward<Args>(args)...);
}
}  // namespace sdb

void sdb_set_last_error(const char* msg);
int sdb_fail(int status, const char* msg);
// Rewrites the calling thread's last error message when it starts with `from` so that it
// starts with `to` instead (an entry point that wraps another reports under its own name).
void sdb_rename_error(const char* from, const char* to);

namespace sdb {
// Device ids this library keeps per-device state for.
constexpr int kMaxDevices = 64;

// A bf16 TMA tensor map with 128-byte swizzle: `rank` dims (innermost first, the innermost
// box 64 elements), byte strides of dims 1..rank-1, the box per dim; out-of-range elements
// read as zero. Defined in gemm.cu.
int encode_bf16_sw128(CUtensorMap* map, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
                      const uint32_t* box);

// Kernel attributes (such as the dynamic shared-memory limit) are per device, and one process
// may drive several GPUs from several host threads. A DeviceOnce runs a set-up step once per
// device, under its lock, with that device current; the step returns a B200 status and is
// retried on the next call if it failed.
struct DeviceOnce {
  std::mutex mu;
  uint64_t done = 0;
};

template <typename F>
inline int once_per_device(DeviceOnce& once, F&& setup) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return sdb_fail(B200_ERR_CUDA, "cannot determine the current CUDA device (or its id is >= 64)");
  std::lock_guard<std::mutex> lk(once.mu);
  if ((once.done >> dev) & 1) return B200_OK;
  const int r = setup(dev);
  if (r == B200_OK) once.done |= uint64_t(1) << dev;
  return r;
}

// Streaming multiprocessors of the current device (looked up once per device; 148 when the
// runtime cannot say).
int sm_count();
}  // namespace sdb

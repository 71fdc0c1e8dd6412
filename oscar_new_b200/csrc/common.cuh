// Shared device helpers for the OSCAR B200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "../../include/oscar_b200.h"

#define OSCAR_DEVINL __device__ __forceinline__

namespace oscar {

constexpr int kDim = 256;           // head_dim D
constexpr int kDataBytes = 64;      // packed codes of one vector
constexpr int kKernelBlock = 128;   // page-table granularity

// ----------------------------------------------------------------------------
// scalar conversions (IEEE round-to-nearest-even, no fast-math anywhere)
// ----------------------------------------------------------------------------
OSCAR_DEVINL float bf16_bits_to_float(uint32_t bits16) { return __uint_as_float(bits16 << 16); }

OSCAR_DEVINL uint16_t float_to_bf16_bits(float x) {
  __nv_bfloat16 b = __float2bfloat16_rn(x);
  return *reinterpret_cast<uint16_t *>(&b);
}

OSCAR_DEVINL uint16_t float_to_half_bits(float x) {
  __half h = __float2half_rn(x);
  return *reinterpret_cast<uint16_t *>(&h);
}

OSCAR_DEVINL float half_bits_to_float(uint16_t bits) {
  __half h = *reinterpret_cast<__half *>(&bits);
  return __half2float(h);
}

// Two fp32 -> packed f16x2 (lo in bits 0..15), round to nearest even.
OSCAR_DEVINL uint32_t pack_half2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

OSCAR_DEVINL uint32_t pack_bf162(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

OSCAR_DEVINL float round_bf16(float x) { return bf16_bits_to_float(float_to_bf16_bits(x)); }

OSCAR_DEVINL uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

OSCAR_DEVINL float ex2(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// ----------------------------------------------------------------------------
// warp-level MMA (legacy HMMA path; used where the tile has only 8 query rows)
// ----------------------------------------------------------------------------
OSCAR_DEVINL void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

OSCAR_DEVINL void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                 uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Transpose an 8x8 b16 matrix held one 32-bit pair per lane (row = lane/4).
OSCAR_DEVINL uint32_t movmatrix_trans(uint32_t x) {
  uint32_t r;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(r) : "r"(x));
  return r;
}

OSCAR_DEVINL void ldmatrix_x4(uint32_t (&r)[4], uint32_t smem_addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr));
}

OSCAR_DEVINL void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t smem_addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr));
}

OSCAR_DEVINL uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ----------------------------------------------------------------------------
// async copies and mbarriers (bounded waits only)
// ----------------------------------------------------------------------------
OSCAR_DEVINL void cp_async_16(uint32_t smem_addr, const void *gptr) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr), "l"(gptr));
}
OSCAR_DEVINL void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
OSCAR_DEVINL void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N));
}

OSCAR_DEVINL void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

OSCAR_DEVINL void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

OSCAR_DEVINL void mbar_arrive(uint64_t *bar) {
  asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(smem_u32(bar))
               : "memory");
}

OSCAR_DEVINL void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile(
      "{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

OSCAR_DEVINL bool mbar_try_wait(uint64_t *bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, "
      "p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}

// As mbar_try_wait, but the thread may stay suspended for up to `hint_ns` nanoseconds
// while the phase is incomplete (it resumes as soon as the phase completes): a waiting
// warp sleeps instead of spinning and leaves its issue slots to the working warps.
OSCAR_DEVINL bool mbar_try_wait_sleep(uint64_t *bar, uint32_t phase, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, "
      "p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Non-blocking probe: has the phase with this parity completed?
OSCAR_DEVINL bool mbar_test(uint64_t *bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, "
      "p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}

// Spin on an mbarrier phase with an iteration limit.  Returns false on timeout; the
// caller records the error and stops consuming (never an unbounded hang).
constexpr uint32_t kWaitLimit = 1u << 20;
OSCAR_DEVINL bool mbar_wait_bounded(uint64_t *bar, uint32_t phase, uint32_t limit = kWaitLimit) {
  if (limit == 0) limit = kWaitLimit;
  for (uint32_t i = 0; i < limit; ++i) {
    if (mbar_try_wait(bar, phase)) return true;
  }
  return false;
}

// 1-D bulk copy global -> shared (no multicast), completion via mbarrier tx count.
OSCAR_DEVINL void bulk_copy_g2s(uint32_t smem_dst, const void *gsrc, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_dst),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ----------------------------------------------------------------------------
// paged-cache geometry helpers (reference layout.py:46-73)
// ----------------------------------------------------------------------------
OSCAR_DEVINL int64_t slot_byte_offset(int64_t slot, int head, const oscar_geometry &g) {
  return (slot / g.block_tokens) * g.page_bytes +
         ((slot % g.block_tokens) * g.kv_heads + head) * (int64_t)g.slot_bytes;
}

// Element offset (bf16 units) of window token index `idx`, kv 0/1, head.
OSCAR_DEVINL int64_t window_elem_offset(int64_t owner, int idx, int kv, int head,
                                        const oscar_geometry &g) {
  return owner * (g.page_bytes / 2) + ((int64_t)(idx * 2 + kv) * g.kv_heads + head) * kDim;
}

OSCAR_DEVINL int window_index(int pos, const oscar_geometry &g) {
  return pos < g.sink ? pos : g.sink + pos % g.ring;
}

}  // namespace oscar

// Opt kernel `Kernel` into `bytes` of dynamic shared memory on the current device.  The
// attribute is per (kernel, device), so the grant is remembered per device; concurrent
// first calls may both set it, which is harmless.
template <auto Kernel>
inline bool ensure_dynamic_smem(size_t bytes) {
  static std::atomic<size_t> granted[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  if (granted[dev].load(std::memory_order_relaxed) >= bytes) return true;
  if (cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) != cudaSuccess)
    return false;
  size_t cur = granted[dev].load(std::memory_order_relaxed);
  while (cur < bytes && !granted[dev].compare_exchange_weak(cur, bytes)) {
  }
  return true;
}

#define OSCAR_CHECK_LAUNCH()                                  \
  do {                                                        \
    if (cudaPeekAtLastError() != cudaSuccess) {               \
      cudaGetLastError();                                     \
      return OSCAR_ERR_LAUNCH;                                \
    }                                                         \
  } while (0)

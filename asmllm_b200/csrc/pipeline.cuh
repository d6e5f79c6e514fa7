// asmllm_b200/csrc/pipeline.cuh -- shared-memory ring primitives of the
// bulk-copy kernels (tma_matvec.cu, decode_persistent.cu): mbarriers with
// bounded waits, the bulk global->shared copy, and the named barriers the
// consumer warps use (1: all consumers, 2 / 3: one warpgroup each).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace asmllm {

constexpr long long kWaitCycles = 2000000000LL;  // ~1 s at the B200 SM clock

static __device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

static __device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

static __device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

static __device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar),
      "r"(bytes)
      : "memory");
}

static __device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar)
      : "memory");
}

static __device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity; false after kWaitCycles.
static __device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitCycles) return false;
  }
  return true;
}

static __device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

static __device__ __forceinline__ void consumer_bar_sync(int nthreads) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

// Barrier over the 256 threads of warpgroup wg (named barrier 2 + wg) that
// also ORs a flag across them: every warp gets the same answer.
static __device__ __forceinline__ bool wg_bar_or(int wg, bool v) {
  unsigned r;
  if (wg == 0)
    asm volatile(
        "{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\t"
        "bar.red.or.pred po, 2, 256, pi;\n\tselp.u32 %0, 1, 0, po;\n\t}"
        : "=r"(r)
        : "r"((unsigned)v)
        : "memory");
  else
    asm volatile(
        "{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\t"
        "bar.red.or.pred po, 3, 256, pi;\n\tselp.u32 %0, 1, 0, po;\n\t}"
        : "=r"(r)
        : "r"((unsigned)v)
        : "memory");
  return r != 0;
}

// Barrier over the nthreads threads (whole warps) that use named barrier id,
// ORing a flag across them: every warp gets the same answer.
static __device__ __forceinline__ bool group_bar_or(int id, int nthreads, bool v) {
  unsigned r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.or.pred po, %2, %3, pi;\n\tselp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(r)
      : "r"((unsigned)v), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

// Orderable 64-bit key of (value, row): larger value first, then lower row
// (numpy.argmax returns the first maximum).  Zero is below every key.
static __device__ __forceinline__ unsigned long long argmax_key(float v, int row) {
  unsigned u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)row);
}

// Row of a key (0 for the empty key).
static __device__ __forceinline__ int argmax_row(unsigned long long key) {
  return key ? (int)(0xFFFFFFFFu - (unsigned)(key & 0xFFFFFFFFull)) : 0;
}

}  // namespace asmllm

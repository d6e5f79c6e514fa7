// asmllm_b200/csrc/common.cuh -- device helpers shared by the sm_100a kernels.
//
// The activation quantize here is the bit-exact restatement of the reference
// NEON kernel src/kernels/arm64/matmul_q4_neon.S:57-143 (THRISHAL12345/asmllm):
//   amax = FMAXV(|x|)           NaN-propagating max          (:69-86)
//   d    = amax / 127           IEEE division, stored fp32   (:89-92)
//   inv  = amax == 0 ? 0 : 127/amax                          (:94-101)
//   q    = SQXTN(SQXTN(FCVTNS(x * inv)))  RNE, NaN->0, saturate to int8 (:104-135)
// CUDA's __fdiv_rn / __fmul_rn are IEEE round-to-nearest; __float2int_rn is
// round-half-even.  Clamping to [-128, 127] before rounding gives the same
// int8 as rounding then saturating (both are monotone), and NaN is mapped to
// 0 first, as FCVTNS does.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace asmllm {

constexpr int QK = 32;                 // elements per Q4_0 / Q8_0 block
constexpr unsigned kFull = 0xffffffffu;

// ARM FMAX: a NaN operand gives NaN.  Inputs are |x| (never -0).
__device__ __forceinline__ float arm_fmax(float a, float b) {
  return (a != a) ? a : ((b != b) ? b : fmaxf(a, b));
}

// Quantizes the 32-element block held one element per lane (lane i holds
// element i of the block).  Returns this lane's int8 value; every lane gets
// the block scale d and the sum of the block's 32 int8 values.
__device__ __forceinline__ int quantize_block_lane(float v, float& d, int& qsum) {
  float a = fabsf(v);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a = arm_fmax(a, __shfl_xor_sync(kFull, a, o));
  d = __fdiv_rn(a, 127.0f);
  const float inv = (a == 0.0f) ? 0.0f : __fdiv_rn(127.0f, a);
  const float t = __fmul_rn(v, inv);
  const int q = (t != t) ? 0 : __float2int_rn(fminf(fmaxf(t, -128.0f), 127.0f));
  int s = q;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(kFull, s, o);
  qsum = s;
  return q;
}

// Quantizes one 32-element block held by a single thread (xb: 16-byte aligned
// global pointer).  Same formulas as quantize_block_lane; writes the 32 int8
// values packed little-endian into q[8], returns d and the block's q-sum.
__device__ __forceinline__ void quantize_block_thread(const float* __restrict__ xb, unsigned q[8],
                                                      float& d, int& qsum) {
  float v[32];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 t = reinterpret_cast<const float4*>(xb)[i];
    v[4 * i] = t.x;
    v[4 * i + 1] = t.y;
    v[4 * i + 2] = t.z;
    v[4 * i + 3] = t.w;
  }
  float a = fabsf(v[0]);
#pragma unroll
  for (int i = 1; i < 32; ++i) a = arm_fmax(a, fabsf(v[i]));
  d = __fdiv_rn(a, 127.0f);
  const float inv = (a == 0.0f) ? 0.0f : __fdiv_rn(127.0f, a);
  int s = 0;
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    int b[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float t = __fmul_rn(v[4 * w + j], inv);
      b[j] = (t != t) ? 0 : __float2int_rn(fminf(fmaxf(t, -128.0f), 127.0f));
      s += b[j];
    }
    q[w] = __byte_perm(__byte_perm((unsigned)b[0], (unsigned)b[1], 0x0040u),
                       __byte_perm((unsigned)b[2], (unsigned)b[3], 0x0040u), 0x5410u);
  }
  qsum = s;
}

// Quantizes one 32-element block spread over 8 consecutive lanes (lane group
// of 8 aligned in the warp; this lane holds elements 4j..4j+3, j = lane & 7).
// All 32 lanes of the warp must call it.  Same formulas as above; returns the
// 4 int8 values packed little-endian, and d and the block q-sum to all 8 lanes.
__device__ __forceinline__ unsigned quantize_quad(float4 v, float& d, int& qsum) {
  float a = arm_fmax(arm_fmax(fabsf(v.x), fabsf(v.y)), arm_fmax(fabsf(v.z), fabsf(v.w)));
  a = arm_fmax(a, __shfl_xor_sync(kFull, a, 1));
  a = arm_fmax(a, __shfl_xor_sync(kFull, a, 2));
  a = arm_fmax(a, __shfl_xor_sync(kFull, a, 4));
  d = __fdiv_rn(a, 127.0f);
  const float inv = (a == 0.0f) ? 0.0f : __fdiv_rn(127.0f, a);
  int q[4];
  const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float t = __fmul_rn(e[j], inv);
    q[j] = (t != t) ? 0 : __float2int_rn(fminf(fmaxf(t, -128.0f), 127.0f));
  }
  int s = q[0] + q[1] + q[2] + q[3];
  s += __shfl_xor_sync(kFull, s, 1);
  s += __shfl_xor_sync(kFull, s, 2);
  s += __shfl_xor_sync(kFull, s, 4);
  qsum = s;
  return __byte_perm(__byte_perm((unsigned)q[0], (unsigned)q[1], 0x0040u),
                     __byte_perm((unsigned)q[2], (unsigned)q[3], 0x0040u), 0x5410u);
}

// Quantizes one 32-element block spread over 4 consecutive lanes (lane group
// of 4 aligned in the warp; this lane holds elements 8j..8j+7, j = lane & 3,
// in v0 = 8j..8j+3 and v1 = 8j+4..8j+7).  All 32 lanes of the warp must call
// it.  Same formulas as quantize_quad; returns this lane's 8 int8 values
// packed little-endian in q0 (first four) and q1, and d and the block q-sum to
// all 4 lanes.
__device__ __forceinline__ void quantize_oct(float4 v0, float4 v1, float& d, int& qsum, unsigned& q0, unsigned& q1) {
  float a = arm_fmax(arm_fmax(arm_fmax(fabsf(v0.x), fabsf(v0.y)), arm_fmax(fabsf(v0.z), fabsf(v0.w))),
                     arm_fmax(arm_fmax(fabsf(v1.x), fabsf(v1.y)), arm_fmax(fabsf(v1.z), fabsf(v1.w))));
  a = arm_fmax(a, __shfl_xor_sync(kFull, a, 1));
  a = arm_fmax(a, __shfl_xor_sync(kFull, a, 2));
  d = __fdiv_rn(a, 127.0f);
  const float inv = (a == 0.0f) ? 0.0f : __fdiv_rn(127.0f, a);
  const float e[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
  int q[8];
  int s = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float t = __fmul_rn(e[j], inv);
    q[j] = (t != t) ? 0 : __float2int_rn(fminf(fmaxf(t, -128.0f), 127.0f));
    s += q[j];
  }
  s += __shfl_xor_sync(kFull, s, 1);
  s += __shfl_xor_sync(kFull, s, 2);
  qsum = s;
  q0 = __byte_perm(__byte_perm((unsigned)q[0], (unsigned)q[1], 0x0040u),
                   __byte_perm((unsigned)q[2], (unsigned)q[3], 0x0040u), 0x5410u);
  q1 = __byte_perm(__byte_perm((unsigned)q[4], (unsigned)q[5], 0x0040u),
                   __byte_perm((unsigned)q[6], (unsigned)q[7], 0x0040u), 0x5410u);
}

// Bulk prefetch of [p, p + bytes) into L2 (sm_90+ bulk-copy unit).  Fire and
// forget: nothing waits on it; p 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// 16-byte asynchronous global -> shared copy (Ampere-style cp.async; the
// wait below is a hardware wait on the copies this thread issued, no spin).
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Programmatic dependent launch (sm_90+): `pdl_trigger` lets the next kernel
// in the stream start launching; `pdl_wait` blocks until the previous kernel
// has completed and its writes are visible.  Both are no-ops for a kernel
// launched without the programmatic-serialization attribute.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// dp4a with unsigned bytes in `a` and signed bytes in `b`.
__device__ __forceinline__ int dp4a_us(unsigned a, int b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ int dp4a_ss(int a, int b, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Streaming 16-byte load of weights read exactly once per call: not kept in
// L1, L2 fetches in 256-byte units.
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p));
  return r;
}

__device__ __forceinline__ unsigned short ld_stream_u16(const void* p) {
  unsigned short r;
  asm("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(r) : "l"(p));
  return r;
}

__device__ __forceinline__ float ld_stream_f32(const void* p) {
  float r;
  asm("ld.global.nc.L1::no_allocate.f32 %0, [%1];" : "=f"(r) : "l"(p));
  return r;
}

__device__ __forceinline__ float half_bits_to_float(unsigned short h) {
  float f;
  asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(h));
  return f;
}

// Scale loaders: fp32 or fp16 storage, fp32 value.
template <bool F16> struct ScaleLoad;
template <> struct ScaleLoad<false> {
  using T = float;
  static __device__ __forceinline__ float load(const void* base, size_t i) {
    return ld_stream_f32(static_cast<const float*>(base) + i);
  }
};
template <> struct ScaleLoad<true> {
  using T = unsigned short;
  static __device__ __forceinline__ float load(const void* base, size_t i) {
    return half_bits_to_float(ld_stream_u16(static_cast<const unsigned short*>(base) + i));
  }
};

// Exact int8 -> fp32 of byte j of w, with w's bytes biased by +128
// (w = raw ^ 0x80808080): 0x4B0000bb is 2^23 + bb, minus 2^23 + 128.
__device__ __forceinline__ float s8_biased_to_f32(unsigned wb, int j) {
  return __int_as_float(__byte_perm(wb, 0x4B000000u, 0x7540u | j)) - 8388736.0f;
}

// Exact (nibble - 8) -> fp32 for byte j of w holding 0..15.
__device__ __forceinline__ float u4_to_f32_minus8(unsigned wb, int j) {
  return __int_as_float(__byte_perm(wb, 0x4B000000u, 0x7540u | j)) - 8388616.0f;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

}  // namespace asmllm

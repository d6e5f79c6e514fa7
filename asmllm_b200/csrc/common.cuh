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

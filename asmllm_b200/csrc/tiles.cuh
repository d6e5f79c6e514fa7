// asmllm_b200/csrc/tiles.cuh -- the "activation tiles": Q8_0-quantized
// activation rows laid out as the fp16 B operand of the tensor-core batched
// product (prefill_gemm.cu), so that the product copies each block's tile
// into shared memory with one bulk copy and feeds it to tcgen05.mma as is.
//
// For N tokens (rows) of K = 32 nb values, with np = act_tiles_tokens(N)
// (N rounded up to the product's token tile) the buffer holds
//   plane B:  nb * np * 64 bytes; block b, token n, position k in 0..31 at
//             b*np*64 + (n/8)*512 + (k/8)*128 + (n%8)*16 + (k%8)*2,
//             the fp16 value of the int8 quant of element 32b + perm(k),
//             perm(8c + j) = 4c + {0, 2, 1, 3, 16, 18, 17, 19}[j];
//   plane D:  nb * np fp32 at byte nb*np*64: the block scale d of (b, n).
// Tokens n >= N hold zeros.  The int8 quants and d are exactly those of the
// Q8_0 quantize (bit-exact with the reference, matmul_q4_neon.S:57-143); fp16
// holds every int8 exactly.  Any np-token range starting at a multiple of 8
// is one contiguous run of each plane, whatever tile width reads it.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace asmllm {

__host__ __device__ inline int act_tiles_tokens(int64_t N) {
  return N <= 16 ? 16 : N <= 32 ? 32 : N <= 64 ? 64 : (int)((N + 127) / 128 * 128);
}

__host__ __device__ inline size_t act_tiles_bytes(int64_t N, int64_t K) {
  return (size_t)(K / 32) * (size_t)act_tiles_tokens(N) * 68;
}

__device__ __forceinline__ uint32_t tiles_hsub2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Chunk c (positions 8c .. 8c+7) of an int8 block from its words c
// (elements 4c..4c+3) and c+4 (elements 4c+16..4c+19): (q ^ 0x80) is placed
// in the low byte of fp16 1024.0 (0x64xx = 1024 + byte, exact) and 1152 is
// subtracted, which gives q exactly.
__device__ __forceinline__ uint4 tiles_i8_chunk(uint32_t lo, uint32_t hi) {
  constexpr uint32_t kSub128 = 0x64806480u;  // 1152.0 in both halves
  lo ^= 0x80808080u;
  hi ^= 0x80808080u;
  uint4 r;
  r.x = tiles_hsub2(__byte_perm(lo, 0x64646464u, 0x4240), kSub128);  // elements 4c, 4c+2
  r.y = tiles_hsub2(__byte_perm(lo, 0x64646464u, 0x4341), kSub128);  // 4c+1, 4c+3
  r.z = tiles_hsub2(__byte_perm(hi, 0x64646464u, 0x4240), kSub128);  // 4c+16, 4c+18
  r.w = tiles_hsub2(__byte_perm(hi, 0x64646464u, 0x4341), kSub128);  // 4c+17, 4c+19
  return r;
}

__device__ __forceinline__ size_t tiles_chunk_offset(int np, int n, int b, int c) {
  return (size_t)b * np * 64 + (size_t)(n >> 3) * 512 + (size_t)c * 128 + (size_t)(n & 7) * 16;
}

// Stores one quantized block from an 8-lane group (lane8 = 0..7 holding the
// packed int8 of elements 4*lane8 .. 4*lane8+3, as quantize_quad returns
// them).  Every lane of the warp must call it (a shuffle); `valid` = false
// groups store nothing.
__device__ __forceinline__ void tiles_store_quad(unsigned char* tiles, int np, int nb, int n, int b, int lane8,
                                                 uint32_t q, float d, bool valid) {
  const uint32_t hi = __shfl_down_sync(0xffffffffu, q, 4, 8);
  if (!valid) return;
  if (lane8 < 4) *reinterpret_cast<uint4*>(tiles + tiles_chunk_offset(np, n, b, lane8)) = tiles_i8_chunk(q, hi);
  if (lane8 == 0) reinterpret_cast<float*>(tiles + (size_t)nb * np * 64)[(size_t)b * np + n] = d;
}

}  // namespace asmllm

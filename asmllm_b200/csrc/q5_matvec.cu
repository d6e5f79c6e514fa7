// asmllm_b200/csrc/q5_matvec.cu -- Q5_0 x fp32 matvec (asm_matmul_q5).
//
// Reference: THRISHAL12345/asmllm src/kernels/x86_64/matmul_q5_avx2.asm
// (layout tests/reference/ops.py:67-99).  Q5_0 block of 32 weights: ql
// [16 bytes] holds weight j's low 4 bits in the low nibble of byte j (j < 16)
// or the high nibble of byte j - 16; qh [4 bytes] holds weight j's fifth bit
// as bit j % 8 of byte j / 8; value = (nibble | bit << 4) - 16, times the
// block scale.  The activation stays fp32 (the reference's Q5 kernels take
// fp32 x on both ISAs); y[r] = sum_b scale[r][b] * sum_j w[r][b][j] * x[32b+j].
//
// One warp per two rows, one lane per 32-block; x staged once per CTA in
// shared memory (36 floats per block: conflict-free 16-byte reads).  The 5-bit
// values become floats through an exact byte-permute trick: the float with
// bit pattern 0x4B0000nn is 2^23 + nn.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "matvec.cuh"

namespace asmllm {

namespace {

constexpr int kQ5Threads = 256;
constexpr int kQ5Rows = 2;

// Four 5-bit values: byte i of `lo4` holds a low nibble, bits 4i..4i+3 of
// `bits` (0..15) the four fifth bits.  Returns the float of value i - 16.
__device__ __forceinline__ float q5_value(unsigned v, int i) {
  return __int_as_float((int)__byte_perm(v, 0x4B000000u, 0x7650u | (unsigned)i)) - 8388624.0f;
}

__device__ __forceinline__ unsigned q5_bytes(unsigned lo4, unsigned bits4) {
  // spread bit k of bits4 to bit 4 of byte k (bit k lands at 8k, then << 4)
  return lo4 | (((bits4 * 0x00204081u) & 0x01010101u) << 4);
}

__global__ void __launch_bounds__(kQ5Threads) q5_f32_matvec_kernel(const uint8_t* __restrict__ ql,
                                                                   const uint8_t* __restrict__ qh,
                                                                   const float* __restrict__ scales,
                                                                   const float* __restrict__ x,
                                                                   float* __restrict__ y, int M, int nb) {
  extern __shared__ __align__(16) float sx[];  // [nb][36]
  const int lane = threadIdx.x & 31;
  pdl_trigger();
  pdl_wait();
  for (int i = threadIdx.x; i < nb * QK; i += kQ5Threads) sx[(i >> 5) * 36 + (i & 31)] = x[i];
  __syncthreads();

  const int ngroups = (M + kQ5Rows - 1) / kQ5Rows;
  const int nwarps = gridDim.x * (kQ5Threads / 32);
  for (int g = blockIdx.x * (kQ5Threads / 32) + (threadIdx.x >> 5); g < ngroups; g += nwarps) {
    float acc[kQ5Rows] = {0.0f, 0.0f};
#pragma unroll 2
    for (int b = lane; b < nb; b += 32) {
      const float4* xp = reinterpret_cast<const float4*>(sx + b * 36);
#pragma unroll
      for (int r = 0; r < kQ5Rows; ++r) {
        const int row = g * kQ5Rows + r;
        if (row >= M) break;
        const size_t blk = (size_t)row * nb + b;
        const uint4 q = ld_stream_v4(ql + blk * 16);
        const unsigned h = *reinterpret_cast<const unsigned*>(qh + blk * 4);
        const float sc = scales[blk];
        const unsigned qw[4] = {q.x, q.y, q.z, q.w};
        float s = 0.0f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          // weights 4k..4k+3 (low nibbles of bytes 4k..) and 16+4k.. (high nibbles)
          const unsigned lo = q5_bytes(qw[k] & 0x0F0F0F0Fu, (h >> (4 * k)) & 0xFu);
          const unsigned hi = q5_bytes((qw[k] >> 4) & 0x0F0F0F0Fu, (h >> (16 + 4 * k)) & 0xFu);
          const float4 xl = xp[k], xh = xp[4 + k];
          s = __fmaf_rn(q5_value(lo, 0), xl.x, s);
          s = __fmaf_rn(q5_value(lo, 1), xl.y, s);
          s = __fmaf_rn(q5_value(lo, 2), xl.z, s);
          s = __fmaf_rn(q5_value(lo, 3), xl.w, s);
          s = __fmaf_rn(q5_value(hi, 0), xh.x, s);
          s = __fmaf_rn(q5_value(hi, 1), xh.y, s);
          s = __fmaf_rn(q5_value(hi, 2), xh.z, s);
          s = __fmaf_rn(q5_value(hi, 3), xh.w, s);
        }
        acc[r] = __fmaf_rn(s, sc, acc[r]);
      }
    }
#pragma unroll
    for (int r = 0; r < kQ5Rows; ++r) {
      const float v = warp_sum(acc[r]);
      const int row = g * kQ5Rows + r;
      if (lane == r && row < M) y[row] = v;
    }
  }
}

}  // namespace

size_t q5_smem_bytes(int64_t K) { return (size_t)(K / QK) * 36 * sizeof(float); }

cudaError_t launch_q5_matvec(const uint8_t* ql, const uint8_t* qh, const float* scales, const float* x, float* y,
                             int64_t M, int64_t K, cudaStream_t stream) {
  const int nb = (int)(K / QK);
  if (nb == 0) return cudaMemsetAsync(y, 0, (size_t)M * sizeof(float), stream);
  int dev = 0, sms = 0, optin = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  const size_t smem = q5_smem_bytes(K);
  if (smem > (size_t)optin) return cudaErrorInvalidValue;
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(q5_f32_matvec_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  const long long ngroups = (M + kQ5Rows - 1) / kQ5Rows;
  long long grid = (ngroups + (kQ5Threads / 32) - 1) / (kQ5Threads / 32);
  if (grid > (long long)sms * 4) grid = (long long)sms * 4;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kQ5Threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_opt_pdl.load() ? 1 : 0;
  int Mi = (int)M;
  return cudaLaunchKernelEx(&cfg, q5_f32_matvec_kernel, ql, qh, scales, x, y, Mi, nb);
}

}  // namespace asmllm

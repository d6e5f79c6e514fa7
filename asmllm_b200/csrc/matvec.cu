// asmllm_b200/csrc/matvec.cu -- batch-1 quantized matvec kernels for sm_100a.
//
// Four kernel families, one per semantics of the reference library
// (THRISHAL12345/asmllm):
//   q4q8   Q4_0 weights x Q8_0 activations   src/kernels/arm64/matmul_q4_neon.S:38-317
//   q8q8   Q8_0 weights x Q8_0 activations   (composed: same quantize/combine, s8 dot)
//   q4f32  Q4_0 weights x fp32 activations   src/kernels/x86_64/matmul_q4_avx2.asm:100-262
//   q8f32  Q8_0 weights x fp32 activations   src/kernels/x86_64/matmul_q8_avx2.asm:93-169
//
// Design (all four are HBM-bound streams over the weights):
//   * One CTA = 8 warps; the grid is persistent (at most the resident CTAs of
//     all SMs) and the row groups are split evenly and contiguously over all
//     warps.  A warp owns ROWS rows at a time and walks their blocks with its
//     32 lanes; every weight byte is loaded once with 16-byte streaming loads
//     (ld.global.nc.L1::no_allocate.L2::256B), ROWS*U of them in flight per
//     lane.
//   * The activation is staged in shared memory once per CTA.  For the Q8_0
//     families each CTA quantizes x itself in its prologue (bit-exact with the
//     reference, see common.cuh), so a matvec is one launch and needs no
//     scratch memory.  The first weight tile is issued before the prologue so
//     the quantize overlaps the HBM latency.
//   * Shared layouts are padded per family so each lane's 16-byte reads of
//     its block fall in distinct banks (48 B per Q8_0 block, 144 B per fp32
//     block, 80 B per fp32 half block).
//   * Q4 x Q8 block dot: isum = dp4a(lo_nibbles, xq[0:16]) + dp4a(hi_nibbles*16,
//     xq[16:32])/16 - 8*sum(xq), exactly the reference's sum of (n-8)*q.
//   * Combine per block: acc = fma(float(isum), wd*xd, acc) as the reference
//     (matmul_q4_neon.S:241-243); the per-lane partial sums are then added
//     with a warp butterfly, so y differs from the reference only by fp32
//     summation order.
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"
#include "matvec.cuh"

namespace asmllm {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

// Shared-memory bytes per block of K for each family.
constexpr int kQ4Q8SmemPerBlock = 48 + 8;   // padded xq + (xd, qsum)
constexpr int kQ8Q8SmemPerBlock = 32 + 4;   // xq + xd
constexpr int kQ4F32SmemPerBlock = 36 * 4;  // 32 floats + 4 pad
constexpr int kQ8F32SmemPerBlock = 2 * 20 * 4;  // two half blocks of 16 floats + 4 pad

__device__ __forceinline__ void group_range(int ngroups, int& g0, int& g1) {
  const int gw = blockIdx.x * kWarps + (threadIdx.x >> 5);
  const long long nw = (long long)gridDim.x * kWarps;
  g0 = (int)(((long long)ngroups * gw) / nw);
  g1 = (int)(((long long)ngroups * (gw + 1)) / nw);
}

// --------------------------------------------------------------------------
// Q4_0 x Q8_0
// --------------------------------------------------------------------------
template <int ROWS, int U, bool F16S, bool DBG>
__global__ void __launch_bounds__(kThreads)
q4q8_matvec_kernel(const uint8_t* __restrict__ qs, const void* __restrict__ scales,
                   const float* __restrict__ x, float* __restrict__ y, int M, int nb,
                   int32_t* __restrict__ isums) {
  extern __shared__ __align__(16) unsigned char smem[];
  unsigned char* sxq = smem;                                    // nb * 48
  float2* sdq = reinterpret_cast<float2*>(smem + (size_t)nb * 48);  // nb * 8
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int ngroups = (M + ROWS - 1) / ROWS;
  int g0, g1;
  group_range(ngroups, g0, g1);
  constexpr int CH = 32 * U;  // blocks per chunk
  const int nchunks = (nb + CH - 1) / CH;

  uint4 w[ROWS][U];
  float sc[ROWS][U];

  auto load_tile = [&](int g, int c) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int b = c * CH + u * 32 + lane;
#pragma unroll
      for (int r = 0; r < ROWS; ++r) {
        const int row = g * ROWS + r;
        if (b < nb && row < M) {
          const size_t blk = (size_t)row * nb + b;
          w[r][u] = ld_stream_v4(qs + blk * 16);
          sc[r][u] = ScaleLoad<F16S>::load(scales, blk);
        } else {
          w[r][u] = make_uint4(0u, 0u, 0u, 0u);
          sc[r][u] = 0.0f;
        }
      }
    }
  };

  if (g0 < g1) load_tile(g0, 0);

  // Prologue: quantize x (fp32[K]) into shared memory, one warp per block.
  for (int b = warp; b < nb; b += kWarps) {
    float d;
    int qsum;
    const int q = quantize_block_lane(x[(size_t)b * QK + lane], d, qsum);
    sxq[b * 48 + lane] = (unsigned char)(q & 0xff);
    if (lane == 0) sdq[b] = make_float2(d, __int_as_float(qsum));
  }
  __syncthreads();

  for (int g = g0; g < g1; ++g) {
    float acc[ROWS];
#pragma unroll
    for (int r = 0; r < ROWS; ++r) acc[r] = 0.0f;
    for (int c = 0; c < nchunks; ++c) {
      if (g != g0 || c != 0) load_tile(g, c);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int b = c * CH + u * 32 + lane;
        if (b < nb) {
          const uint4* xp = reinterpret_cast<const uint4*>(sxq + b * 48);
          const uint4 xa = xp[0];  // xq[0..15]  (pairs with low nibbles)
          const uint4 xb = xp[1];  // xq[16..31] (pairs with high nibbles)
          const float2 dq = sdq[b];
          const int qsum8 = __float_as_int(dq.y) * 8;
#pragma unroll
          for (int r = 0; r < ROWS; ++r) {
            const uint4 q = w[r][u];
            int lo = 0, hi = 0;
            lo = dp4a_us(q.x & 0x0F0F0F0Fu, (int)xa.x, lo);
            hi = dp4a_us(q.x & 0xF0F0F0F0u, (int)xb.x, hi);
            lo = dp4a_us(q.y & 0x0F0F0F0Fu, (int)xa.y, lo);
            hi = dp4a_us(q.y & 0xF0F0F0F0u, (int)xb.y, hi);
            lo = dp4a_us(q.z & 0x0F0F0F0Fu, (int)xa.z, lo);
            hi = dp4a_us(q.z & 0xF0F0F0F0u, (int)xb.z, hi);
            lo = dp4a_us(q.w & 0x0F0F0F0Fu, (int)xa.w, lo);
            hi = dp4a_us(q.w & 0xF0F0F0F0u, (int)xb.w, hi);
            const int isum = lo + (hi >> 4) - qsum8;
            if (DBG) {
              const int row = g * ROWS + r;
              if (row < M) isums[(size_t)row * nb + b] = isum;
            }
            acc[r] = __fmaf_rn(__int2float_rn(isum), __fmul_rn(sc[r][u], dq.x), acc[r]);
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      const float v = warp_sum(acc[r]);
      const int row = g * ROWS + r;
      if (lane == r && row < M) y[row] = v;
    }
  }
}

// --------------------------------------------------------------------------
// Q8_0 x Q8_0 (lane pairs share a block: each lane loads one 16-byte half)
// --------------------------------------------------------------------------
template <int ROWS, int U, bool F16S, bool DBG>
__global__ void __launch_bounds__(kThreads)
q8q8_matvec_kernel(const int8_t* __restrict__ qw, const void* __restrict__ scales,
                   const float* __restrict__ x, float* __restrict__ y, int M, int nb,
                   int32_t* __restrict__ isums) {
  extern __shared__ __align__(16) unsigned char smem[];
  unsigned char* sxq = smem;                                  // nb * 32
  float* sd = reinterpret_cast<float*>(smem + (size_t)nb * 32);  // nb * 4
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int ngroups = (M + ROWS - 1) / ROWS;
  int g0, g1;
  group_range(ngroups, g0, g1);
  const int nhb = 2 * nb;
  constexpr int CH = 32 * U;  // half blocks per chunk
  const int nchunks = (nhb + CH - 1) / CH;

  uint4 w[ROWS][U];
  float sc[ROWS][U];

  auto load_tile = [&](int g, int c) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int hb = c * CH + u * 32 + lane;
#pragma unroll
      for (int r = 0; r < ROWS; ++r) {
        const int row = g * ROWS + r;
        if (hb < nhb && row < M) {
          w[r][u] = ld_stream_v4(qw + ((size_t)row * nb * 32 + (size_t)hb * 16));
          sc[r][u] = ScaleLoad<F16S>::load(scales, (size_t)row * nb + (hb >> 1));
        } else {
          w[r][u] = make_uint4(0u, 0u, 0u, 0u);
          sc[r][u] = 0.0f;
        }
      }
    }
  };

  if (g0 < g1) load_tile(g0, 0);

  for (int b = warp; b < nb; b += kWarps) {
    float d;
    int qsum;
    const int q = quantize_block_lane(x[(size_t)b * QK + lane], d, qsum);
    sxq[b * 32 + lane] = (unsigned char)(q & 0xff);
    if (lane == 0) sd[b] = d;
  }
  __syncthreads();

  for (int g = g0; g < g1; ++g) {
    float acc[ROWS];
#pragma unroll
    for (int r = 0; r < ROWS; ++r) acc[r] = 0.0f;
    for (int c = 0; c < nchunks; ++c) {
      if (g != g0 || c != 0) load_tile(g, c);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int hb = c * CH + u * 32 + lane;
        const bool valid = hb < nhb;  // same for both lanes of a pair
        uint4 xa = make_uint4(0u, 0u, 0u, 0u);
        float xd = 0.0f;
        if (valid) {
          xa = reinterpret_cast<const uint4*>(sxq)[hb];
          xd = sd[hb >> 1];
        }
#pragma unroll
        for (int r = 0; r < ROWS; ++r) {
          const uint4 q = w[r][u];
          int part = 0;
          part = dp4a_ss((int)q.x, (int)xa.x, part);
          part = dp4a_ss((int)q.y, (int)xa.y, part);
          part = dp4a_ss((int)q.z, (int)xa.z, part);
          part = dp4a_ss((int)q.w, (int)xa.w, part);
          const int isum = part + __shfl_xor_sync(kFull, part, 1);
          if (valid && !(lane & 1)) {
            if (DBG) {
              const int row = g * ROWS + r;
              if (row < M) isums[(size_t)row * nb + (hb >> 1)] = isum;
            }
            acc[r] = __fmaf_rn(__int2float_rn(isum), __fmul_rn(sc[r][u], xd), acc[r]);
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      const float v = warp_sum(acc[r]);
      const int row = g * ROWS + r;
      if (lane == r && row < M) y[row] = v;
    }
  }
}

// --------------------------------------------------------------------------
// Q4_0 x fp32 (x86 semantics)
// --------------------------------------------------------------------------
template <int ROWS, int U, bool F16S>
__global__ void __launch_bounds__(kThreads)
q4f32_matvec_kernel(const uint8_t* __restrict__ qs, const void* __restrict__ scales,
                    const float* __restrict__ x, float* __restrict__ y, int M, int nb) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* sx = reinterpret_cast<float*>(smem);  // nb * 36 floats
  const int lane = threadIdx.x & 31;
  const int ngroups = (M + ROWS - 1) / ROWS;
  int g0, g1;
  group_range(ngroups, g0, g1);
  constexpr int CH = 32 * U;
  const int nchunks = (nb + CH - 1) / CH;

  uint4 w[ROWS][U];
  float sc[ROWS][U];

  auto load_tile = [&](int g, int c) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int b = c * CH + u * 32 + lane;
#pragma unroll
      for (int r = 0; r < ROWS; ++r) {
        const int row = g * ROWS + r;
        if (b < nb && row < M) {
          const size_t blk = (size_t)row * nb + b;
          w[r][u] = ld_stream_v4(qs + blk * 16);
          sc[r][u] = ScaleLoad<F16S>::load(scales, blk);
        } else {
          w[r][u] = make_uint4(0u, 0u, 0u, 0u);
          sc[r][u] = 0.0f;
        }
      }
    }
  };

  if (g0 < g1) load_tile(g0, 0);

  const int K = nb * QK;
  for (int i = threadIdx.x; i < K; i += kThreads) sx[(i >> 5) * 36 + (i & 31)] = x[i];
  __syncthreads();

  for (int g = g0; g < g1; ++g) {
    float acc[ROWS];
#pragma unroll
    for (int r = 0; r < ROWS; ++r) acc[r] = 0.0f;
    for (int c = 0; c < nchunks; ++c) {
      if (g != g0 || c != 0) load_tile(g, c);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int b = c * CH + u * 32 + lane;
        if (b < nb) {
          const float4* xp = reinterpret_cast<const float4*>(sx + b * 36);
          float blk[ROWS];
#pragma unroll
          for (int r = 0; r < ROWS; ++r) blk[r] = 0.0f;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float4 xl = xp[k];      // elements 4k .. 4k+3
            const float4 xh = xp[4 + k];  // elements 16+4k .. 16+4k+3
#pragma unroll
            for (int r = 0; r < ROWS; ++r) {
              const unsigned word = k == 0 ? w[r][u].x : k == 1 ? w[r][u].y : k == 2 ? w[r][u].z : w[r][u].w;
              const unsigned lo = word & 0x0F0F0F0Fu;
              const unsigned hi = (word >> 4) & 0x0F0F0F0Fu;
              float t = blk[r];
              t = __fmaf_rn(u4_to_f32_minus8(lo, 0), xl.x, t);
              t = __fmaf_rn(u4_to_f32_minus8(lo, 1), xl.y, t);
              t = __fmaf_rn(u4_to_f32_minus8(lo, 2), xl.z, t);
              t = __fmaf_rn(u4_to_f32_minus8(lo, 3), xl.w, t);
              t = __fmaf_rn(u4_to_f32_minus8(hi, 0), xh.x, t);
              t = __fmaf_rn(u4_to_f32_minus8(hi, 1), xh.y, t);
              t = __fmaf_rn(u4_to_f32_minus8(hi, 2), xh.z, t);
              t = __fmaf_rn(u4_to_f32_minus8(hi, 3), xh.w, t);
              blk[r] = t;
            }
          }
#pragma unroll
          for (int r = 0; r < ROWS; ++r) acc[r] = __fmaf_rn(blk[r], sc[r][u], acc[r]);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      const float v = warp_sum(acc[r]);
      const int row = g * ROWS + r;
      if (lane == r && row < M) y[row] = v;
    }
  }
}

// --------------------------------------------------------------------------
// Q8_0 x fp32 (x86 semantics); each lane takes one 16-element half block
// --------------------------------------------------------------------------
template <int ROWS, int U, bool F16S>
__global__ void __launch_bounds__(kThreads)
q8f32_matvec_kernel(const int8_t* __restrict__ qw, const void* __restrict__ scales,
                    const float* __restrict__ x, float* __restrict__ y, int M, int nb) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* sx = reinterpret_cast<float*>(smem);  // 2*nb half blocks * 20 floats
  const int lane = threadIdx.x & 31;
  const int ngroups = (M + ROWS - 1) / ROWS;
  int g0, g1;
  group_range(ngroups, g0, g1);
  const int nhb = 2 * nb;
  constexpr int CH = 32 * U;
  const int nchunks = (nhb + CH - 1) / CH;

  uint4 w[ROWS][U];
  float sc[ROWS][U];

  auto load_tile = [&](int g, int c) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int hb = c * CH + u * 32 + lane;
#pragma unroll
      for (int r = 0; r < ROWS; ++r) {
        const int row = g * ROWS + r;
        if (hb < nhb && row < M) {
          w[r][u] = ld_stream_v4(qw + ((size_t)row * nb * 32 + (size_t)hb * 16));
          sc[r][u] = ScaleLoad<F16S>::load(scales, (size_t)row * nb + (hb >> 1));
        } else {
          w[r][u] = make_uint4(0u, 0u, 0u, 0u);
          sc[r][u] = 0.0f;
        }
      }
    }
  };

  if (g0 < g1) load_tile(g0, 0);

  const int K = nb * QK;
  for (int i = threadIdx.x; i < K; i += kThreads) sx[(i >> 4) * 20 + (i & 15)] = x[i];
  __syncthreads();

  for (int g = g0; g < g1; ++g) {
    float acc[ROWS];
#pragma unroll
    for (int r = 0; r < ROWS; ++r) acc[r] = 0.0f;
    for (int c = 0; c < nchunks; ++c) {
      if (g != g0 || c != 0) load_tile(g, c);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int hb = c * CH + u * 32 + lane;
        if (hb < nhb) {
          const float4* xp = reinterpret_cast<const float4*>(sx + hb * 20);
          float blk[ROWS];
#pragma unroll
          for (int r = 0; r < ROWS; ++r) blk[r] = 0.0f;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float4 xv = xp[k];
#pragma unroll
            for (int r = 0; r < ROWS; ++r) {
              const unsigned word = (k == 0 ? w[r][u].x : k == 1 ? w[r][u].y : k == 2 ? w[r][u].z : w[r][u].w) ^ 0x80808080u;
              float t = blk[r];
              t = __fmaf_rn(s8_biased_to_f32(word, 0), xv.x, t);
              t = __fmaf_rn(s8_biased_to_f32(word, 1), xv.y, t);
              t = __fmaf_rn(s8_biased_to_f32(word, 2), xv.z, t);
              t = __fmaf_rn(s8_biased_to_f32(word, 3), xv.w, t);
              blk[r] = t;
            }
          }
#pragma unroll
          for (int r = 0; r < ROWS; ++r) acc[r] = __fmaf_rn(blk[r], sc[r][u], acc[r]);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      const float v = warp_sum(acc[r]);
      const int row = g * ROWS + r;
      if (lane == r && row < M) y[row] = v;
    }
  }
}

// --------------------------------------------------------------------------
// Standalone / batched activation quantize: one warp per 32-block.
// --------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads)
quantize_q8_0_kernel(const float* __restrict__ x, int8_t* __restrict__ xq,
                     float* __restrict__ xd, long long nblocks) {
  const int lane = threadIdx.x & 31;
  const long long nw = (long long)gridDim.x * kWarps;
  for (long long b = (long long)blockIdx.x * kWarps + (threadIdx.x >> 5); b < nblocks; b += nw) {
    float d;
    int qsum;
    const int q = quantize_block_lane(x[b * QK + lane], d, qsum);
    xq[b * QK + lane] = (int8_t)q;
    if (lane == 0) xd[b] = d;
  }
}

// --------------------------------------------------------------------------
// GGUF block split: 18-byte Q4_0 / 34-byte Q8_0 blocks -> qs plane + scales.
// --------------------------------------------------------------------------
template <int QBYTES>
__global__ void gguf_split_kernel(const uint8_t* __restrict__ raw, uint8_t* __restrict__ qs,
                                  void* __restrict__ scales, int f16, long long nblocks) {
  constexpr int BB = QBYTES + 2;  // block bytes: fp16 d + quants
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nblocks; i += stride) {
    const uint8_t* src = raw + i * BB;  // 2-byte aligned
    const unsigned short* s16 = reinterpret_cast<const unsigned short*>(src);
    const unsigned short dbits = s16[0];
    unsigned* dst = reinterpret_cast<unsigned*>(qs + i * QBYTES);
#pragma unroll
    for (int k = 0; k < QBYTES / 4; ++k)
      dst[k] = (unsigned)s16[1 + 2 * k] | ((unsigned)s16[2 + 2 * k] << 16);
    if (f16) {
      static_cast<unsigned short*>(scales)[i] = dbits;
    } else {
      static_cast<float*>(scales)[i] = half_bits_to_float(dbits);
    }
  }
}

// ==========================================================================
// Host-side launchers
// ==========================================================================

namespace {

struct DevInfo {
  int sms = 0;
  int smem_optin = 0;
  bool init = false;
};
DevInfo g_dev[64];

std::mutex g_dev_mu;

const DevInfo& dev_info(int dev) {
  DevInfo& d = g_dev[dev & 63];
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (!d.init) {
    cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    d.init = true;
  }
  return d;
}

// Occupancy of each (kernel, shared bytes, device), computed once: later
// launches (including ones recorded into a CUDA graph) only do the launch.
std::mutex g_occ_mu;
std::map<std::tuple<const void*, size_t, int>, int> g_occ;

template <typename KernelT>
cudaError_t launch_persistent(KernelT kernel, int ngroups, size_t smem, cudaStream_t stream,
                              int dev, void** args) {
  const DevInfo& di = dev_info(dev);
  const auto key = std::make_tuple((const void*)kernel, smem, dev);
  int per_sm = 0;
  {
    std::lock_guard<std::mutex> lk(g_occ_mu);
    auto it = g_occ.find(key);
    if (it != g_occ.end()) per_sm = it->second;
  }
  if (per_sm == 0) {
    if (smem > 48 * 1024) {  // opt in to > 48 KB of dynamic shared memory
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, di.smem_optin);
      if (e != cudaSuccess) return e;
    }
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) per_sm = 1;
    std::lock_guard<std::mutex> lk(g_occ_mu);
    g_occ[key] = per_sm;
  }
  const long long needed = ((long long)ngroups + kWarps - 1) / kWarps;
  long long grid = (long long)per_sm * di.sms;
  if (needed < grid) grid = needed;
  if (grid < 1) grid = 1;
  return cudaLaunchKernel((const void*)kernel, dim3((unsigned)grid), dim3(kThreads), args, smem, stream);
}

}  // namespace

int64_t max_k(int fmt, bool fp32_act, int dev) {
  const DevInfo& di = dev_info(dev);
  const int per_block = fmt == kFmtQ4_0 ? (fp32_act ? kQ4F32SmemPerBlock : kQ4Q8SmemPerBlock)
                                        : (fp32_act ? kQ8F32SmemPerBlock : kQ8Q8SmemPerBlock);
  const int64_t nb = di.smem_optin / per_block;
  int64_t k = nb * QK;
  if (k > (int64_t)1 << 30) k = (int64_t)1 << 30;
  return k;
}

// Kernel configuration: rows per warp x 32-block iterations per load batch.
// Chosen from the shape; ASMLLM_MATVEC_CFG=<rows>x<u> forces one for sweeps.
struct Cfg { int rows, u; };

static Cfg pick_cfg(int M, int nb, int sms) {
  (void)nb;
  // Two rows per warp keeps 8 x 16-byte loads in flight per lane at K=4096;
  // small M drops to one row so every SM gets several warps.
  if ((long long)M < (long long)sms * kWarps * 4) return {1, 4};
  return {2, 4};
}

static Cfg cfg_override(Cfg c) {
  static int forced_rows = -1, forced_u = -1;
  if (forced_rows < 0) {
    forced_rows = 0;
    const char* s = getenv("ASMLLM_MATVEC_CFG");
    int r = 0, u = 0;
    if (s && sscanf(s, "%dx%d", &r, &u) == 2) { forced_rows = r; forced_u = u; }
  }
  if (forced_rows > 0) return {forced_rows, forced_u};
  return c;
}

#define ASMLLM_DISPATCH_RU(ROWS_, U_, CALL)                                    \
  if (c.rows == ROWS_ && c.u == U_) { CALL(ROWS_, U_); }

cudaError_t launch_matvec(const MatvecArgs& a, cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (a.M <= 0) return cudaSuccess;
  const int M = (int)a.M;
  const int nb = (int)(a.K / QK);
  if (nb == 0) return cudaMemsetAsync(a.y, 0, (size_t)a.M * sizeof(float), stream);
  const DevInfo& di = dev_info(dev);
  Cfg c = cfg_override(pick_cfg(M, nb, di.sms));
  if (!((c.rows == 1 || c.rows == 2 || c.rows == 4) && (c.u == 2 || c.u == 4))) c = {2, 4};

  const void* w = a.w;
  const void* s = a.scales;
  const float* x = a.x;
  float* y = a.y;
  int32_t* isums = a.isums;
  int Mi = M, nbi = nb;
  void* args7[] = {(void*)&w, (void*)&s, (void*)&x, (void*)&y, (void*)&Mi, (void*)&nbi, (void*)&isums};
  void* args6[] = {(void*)&w, (void*)&s, (void*)&x, (void*)&y, (void*)&Mi, (void*)&nbi};

  if (!a.fp32_act) {
    const bool q4 = a.fmt == kFmtQ4_0;
    const int rows_for_groups = c.rows;
    const int ngroups = (M + rows_for_groups - 1) / rows_for_groups;
    const size_t smem = (size_t)nb * (q4 ? kQ4Q8SmemPerBlock : kQ8Q8SmemPerBlock);
    if (smem > (size_t)di.smem_optin) return cudaErrorInvalidValue;
#define CALL_Q8ACT(R, U)                                                                      \
  {                                                                                           \
    if (q4) {                                                                                 \
      if (a.isums) {                                                                          \
        return a.scales_f16 ? launch_persistent(q4q8_matvec_kernel<R, U, true, true>, ngroups, smem, stream, dev, args7)   \
                            : launch_persistent(q4q8_matvec_kernel<R, U, false, true>, ngroups, smem, stream, dev, args7); \
      }                                                                                       \
      return a.scales_f16 ? launch_persistent(q4q8_matvec_kernel<R, U, true, false>, ngroups, smem, stream, dev, args7)    \
                          : launch_persistent(q4q8_matvec_kernel<R, U, false, false>, ngroups, smem, stream, dev, args7);  \
    }                                                                                         \
    if (a.isums) {                                                                            \
      return a.scales_f16 ? launch_persistent(q8q8_matvec_kernel<R, U, true, true>, ngroups, smem, stream, dev, args7)     \
                          : launch_persistent(q8q8_matvec_kernel<R, U, false, true>, ngroups, smem, stream, dev, args7);   \
    }                                                                                         \
    return a.scales_f16 ? launch_persistent(q8q8_matvec_kernel<R, U, true, false>, ngroups, smem, stream, dev, args7)      \
                        : launch_persistent(q8q8_matvec_kernel<R, U, false, false>, ngroups, smem, stream, dev, args7);    \
  }
    ASMLLM_DISPATCH_RU(1, 4, CALL_Q8ACT)
    ASMLLM_DISPATCH_RU(2, 4, CALL_Q8ACT)
    ASMLLM_DISPATCH_RU(4, 4, CALL_Q8ACT)
    ASMLLM_DISPATCH_RU(1, 2, CALL_Q8ACT)
    ASMLLM_DISPATCH_RU(2, 2, CALL_Q8ACT)
    ASMLLM_DISPATCH_RU(4, 2, CALL_Q8ACT)
#undef CALL_Q8ACT
    return cudaErrorInvalidValue;
  }

  // fp32 activations: four rows per warp share each lane's x reads.
  const bool q4 = a.fmt == kFmtQ4_0;
  constexpr int R = 4, U = 2;
  const int ngroups = (M + R - 1) / R;
  const size_t smem = (size_t)nb * (q4 ? kQ4F32SmemPerBlock : kQ8F32SmemPerBlock);
  if (smem > (size_t)di.smem_optin) return cudaErrorInvalidValue;
  if (q4) {
    return a.scales_f16 ? launch_persistent(q4f32_matvec_kernel<R, U, true>, ngroups, smem, stream, dev, args6)
                        : launch_persistent(q4f32_matvec_kernel<R, U, false>, ngroups, smem, stream, dev, args6);
  }
  return a.scales_f16 ? launch_persistent(q8f32_matvec_kernel<R, U, true>, ngroups, smem, stream, dev, args6)
                      : launch_persistent(q8f32_matvec_kernel<R, U, false>, ngroups, smem, stream, dev, args6);
}

cudaError_t launch_quantize(const float* x, int8_t* xq, float* xd, long long nblocks,
                            cudaStream_t stream) {
  if (nblocks <= 0) return cudaSuccess;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const DevInfo& di = dev_info(dev);
  long long grid = (nblocks + kWarps - 1) / kWarps;
  const long long cap = (long long)di.sms * 8;
  if (grid > cap) grid = cap;
  quantize_q8_0_kernel<<<(unsigned)grid, kThreads, 0, stream>>>(x, xq, xd, nblocks);
  return cudaGetLastError();
}

cudaError_t launch_gguf_split(int fmt, const uint8_t* raw, uint8_t* qs, void* scales, int f16,
                              long long nblocks, cudaStream_t stream) {
  if (nblocks <= 0) return cudaSuccess;
  long long grid = (nblocks + 255) / 256;
  if (grid > 65535LL * 8) grid = 65535LL * 8;
  if (fmt == kFmtQ4_0)
    gguf_split_kernel<16><<<(unsigned)grid, 256, 0, stream>>>(raw, qs, scales, f16, nblocks);
  else
    gguf_split_kernel<32><<<(unsigned)grid, 256, 0, stream>>>(raw, qs, scales, f16, nblocks);
  return cudaGetLastError();
}

}  // namespace asmllm

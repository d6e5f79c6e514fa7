// asmllm_b200/csrc/matvec.cu -- batch-1 quantized matvec kernels for sm_100a.
//
// Semantics (reference THRISHAL12345/asmllm):
//   Q4_0 x Q8_0   src/kernels/arm64/matmul_q4_neon.S:38-317   (asm_matmul_q4)
//   Q8_0 x Q8_0   the same quantize and combine around an s8 dot (no reference kernel)
//   Q4_0 x fp32   src/kernels/x86_64/matmul_q4_avx2.asm:100-262 (asm_matmul_q4_avx512 / _f32)
//   Q8_0 x fp32   src/kernels/x86_64/matmul_q8_avx2.asm:93-169  (asm_matmul_q8)
//
// Design.  Every kernel here is an HBM-bound stream over the weights.
//   * Unit of work: 16 weight bytes per lane -- one Q4_0 block (32 nibbles) or
//     one half of a Q8_0 block.  A row is NU = K/32 (Q4) or K/16 (Q8) units at
//     16-byte stride, so both formats share the addressing
//     w + (row*NU + unit)*16 and every load is a coalesced 16-byte
//     ld.global.nc.L1::no_allocate.L2::256B (each weight byte is read once).
//   * A warp owns ROWS rows at a time; a "tile" is U units per lane for those
//     rows.  Tiles are double-buffered in registers: the next tile's loads are
//     in flight while the current one is consumed, so each warp keeps up to
//     2*ROWS*U 16-byte loads outstanding.
//   * The grid is persistent (at most the co-resident CTAs of all SMs) and the
//     row groups are split evenly and contiguously over all warps.
//   * The activation sits in shared memory, in a layout padded so each lane's
//     16-byte reads hit distinct banks.  For the Q8_0 families it is the
//     "activation image": per 32-block a 48-byte slot (32 int8 + 16 pad) and
//     then (d, qsum) pairs -- written either by act_image_kernel (a pre-pass,
//     once per x, shareable by several matvecs) or by the matvec's own
//     prologue (FUSED: one launch, no scratch).  Both use quantize_quad, the
//     bit-exact restatement of matmul_q4_neon.S:57-143.
//   * Programmatic dependent launch: each kernel issues its first weight tile,
//     lets the next kernel launch, then waits for the previous kernel before
//     touching x / the image or writing y.  Consecutive matvecs overlap their
//     ramp-up and tail; stream semantics are unchanged.
//   * Q4 x Q8 block dot: isum = dp4a(lo nibbles, xq[0:16]) + dp4a(hi nibbles*16,
//     xq[16:32])/16 - 8*sum(xq) == sum((n-8)*q), exact.  Combine per block:
//     acc = fma(float(isum), wd*xd, acc) as the reference (matmul_q4_neon.S:241-243);
//     lane partials are then added by a warp butterfly, so y differs from the
//     reference only in fp32 summation order.
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <cstdio>
#include <cstdlib>
#include <atomic>
#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"
#include "matvec.cuh"

namespace asmllm {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kImgSlot = 48;  // bytes per 32-block of int8 in the activation image

// Shared-memory bytes per 32-block of K for the fp32-activation families.
constexpr int kQ4F32SmemPerBlock = 36 * 4;      // 32 floats + 4 pad
constexpr int kQ8F32SmemPerBlock = 2 * 20 * 4;  // two half blocks of 16 floats + 4 pad

__device__ __forceinline__ void group_range(int ngroups, int& g0, int& g1) {
  const int gw = blockIdx.x * kWarps + (threadIdx.x >> 5);
  const long long nw = (long long)gridDim.x * kWarps;
  g0 = (int)(((long long)ngroups * gw) / nw);
  g1 = (int)(((long long)ngroups * (gw + 1)) / nw);
}

template <int ROWS, int U>
struct Tile {
  uint4 w[ROWS][U];
  float sc[ROWS][U];
};

// Loads tile (group g, chunk c): units c*32*U + k*32 + lane, rows g*ROWS + r.
template <int FMT, int ROWS, int U, bool F16S>
__device__ __forceinline__ void load_tile(Tile<ROWS, U>& t, const uint8_t* __restrict__ w,
                                          const void* __restrict__ scales, int M, int NU, int nb,
                                          int g, int c, int lane) {
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const int u = c * 32 * U + k * 32 + lane;
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      const int row = g * ROWS + r;
      if (u < NU && row < M) {
        t.w[r][k] = ld_stream_v4(w + ((size_t)row * NU + u) * 16);
        const int b = FMT == kFmtQ4_0 ? u : (u >> 1);
        t.sc[r][k] = ScaleLoad<F16S>::load(scales, (size_t)row * nb + b);
      } else {
        t.w[r][k] = make_uint4(0u, 0u, 0u, 0u);
        t.sc[r][k] = 0.0f;
      }
    }
  }
}

// Bulk-prefetches the weight rows (and, when 16-byte aligned, the scales) of
// row group g into L2; lanes 0..ROWS-1 each issue one row.
template <int ROWS, bool F16S>
__device__ __forceinline__ void prefetch_group(const uint8_t* __restrict__ w, const void* __restrict__ scales,
                                               int M, int NU, int nb, int g, int lane) {
  const int row = g * ROWS + lane;
  if (lane < ROWS && row < M) {
    prefetch_l2_bulk(w + (size_t)row * NU * 16, (unsigned)NU * 16u);
    const size_t sb = (size_t)nb * (F16S ? 2 : 4);
    if (sb % 16 == 0) prefetch_l2_bulk(static_cast<const unsigned char*>(scales) + (size_t)row * sb, (unsigned)sb);
  }
}

// Sums each row's lane partials and stores y (lane r stores row r).
template <int ROWS>
__device__ __forceinline__ void finalize_rows(float (&acc)[ROWS], float* __restrict__ y, int g,
                                              int M, int lane) {
#pragma unroll
  for (int r = 0; r < ROWS; ++r) {
    const float v = warp_sum(acc[r]);
    const int row = g * ROWS + r;
    if (lane == r && row < M) y[row] = v;
    acc[r] = 0.0f;
  }
}

// --------------------------------------------------------------------------
// Activation image pre-pass: x fp32 [nrows][K] -> image [nrows][img_bytes(nb)]
// --------------------------------------------------------------------------
// Before waiting for the previous kernel it bulk-prefetches into L2 the first
// pf_bytes of the weights (and scales) of the matvec that will read this
// image: this small kernel becomes resident while the previous kernel drains,
// so HBM keeps streaming across the quantize -> matvec dependency chain.
__device__ __forceinline__ void prefetch_range(const unsigned char* p, unsigned long long bytes) {
  if (!p || bytes < 16) return;
  const unsigned long long nthr = (unsigned long long)gridDim.x * blockDim.x;
  const unsigned long long t = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x;
  unsigned long long chunk = ((bytes + nthr - 1) / nthr + 4095) & ~4095ull;  // >= 4 KB per request
  const unsigned long long beg = t * chunk;
  if (beg >= bytes) return;
  unsigned long long n = bytes - beg < chunk ? bytes - beg : chunk;
  n &= ~15ull;
  if (n) prefetch_l2_bulk(p + beg, (unsigned)n);
}

__global__ void __launch_bounds__(kThreads)
act_image_kernel(const float* __restrict__ x, unsigned char* __restrict__ img, int nb,
                 long long nrows, long long row_stride, const unsigned char* __restrict__ pf_w,
                 unsigned long long pf_w_bytes, const unsigned char* __restrict__ pf_s,
                 unsigned long long pf_s_bytes) {
  pdl_trigger();
  prefetch_range(pf_w, pf_w_bytes);
  prefetch_range(pf_s, pf_s_bytes);
  pdl_wait();  // x may come from the previous kernel; the image may still be read by it
  const int lane8 = threadIdx.x & 7;
  const long long total = nrows * nb;
  const long long nw = (long long)gridDim.x * kWarps;
  for (long long wb = (long long)blockIdx.x * kWarps + (threadIdx.x >> 5); wb * 4 < total; wb += nw) {
    const long long gb = wb * 4 + ((threadIdx.x & 31) >> 3);  // warp-uniform loop, 4 blocks per warp
    const bool valid = gb < total;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (valid) v = reinterpret_cast<const float4*>(x + gb * QK)[lane8];
    float d;
    int qsum;
    const unsigned q = quantize_quad(v, d, qsum);
    if (valid) {
      const long long n = gb / nb, b = gb - n * nb;
      unsigned char* row = img + n * row_stride;
      reinterpret_cast<unsigned*>(row + b * kImgSlot)[lane8] = q;
      if (lane8 == 0) reinterpret_cast<float2*>(row + (size_t)nb * kImgSlot)[b] = make_float2(d, __int_as_float(qsum));
    }
  }
}

// --------------------------------------------------------------------------
// Q8_0-activation matvec: Q4_0 (FMT 2) or Q8_0 (FMT 8) weights
// --------------------------------------------------------------------------
template <int FMT, int ROWS, int U, bool F16S, bool DBG, bool FUSED>
__global__ void __launch_bounds__(kThreads, 2)
q8act_matvec_kernel(const uint8_t* __restrict__ w, const void* __restrict__ scales,
                    const void* __restrict__ act, float* __restrict__ y, int M, int nb,
                    int32_t* __restrict__ isums, int pf, int pre) {
  extern __shared__ __align__(16) unsigned char smem[];
  const float2* sdq = reinterpret_cast<const float2*>(smem + (size_t)nb * kImgSlot);
  const int lane = threadIdx.x & 31;
  constexpr int UPB = FMT == kFmtQ4_0 ? 1 : 2;  // units per block
  const int NU = nb * UPB;
  const int ngroups = (M + ROWS - 1) / ROWS;
  int g0, g1;
  group_range(ngroups, g0, g1);
  constexpr int CH = 32 * U;
  const int nchunks = (NU + CH - 1) / CH;
  const int T = (g1 - g0) * nchunks;

  // Weights are read before waiting for the previous kernel only when the
  // caller declared them static (pre != 0); L2 prefetches are always safe
  // (L2 is coherent, a prefetch never returns data to the SM).
  Tile<ROWS, U> A, B;
  if (pre && T > 0) load_tile<FMT, ROWS, U, F16S>(A, w, scales, M, NU, nb, g0, 0, lane);
  for (int gp = g0 + 1; gp < g1 && gp <= g0 + pf; ++gp) prefetch_group<ROWS, F16S>(w, scales, M, NU, nb, gp, lane);
  pdl_trigger();
  pdl_wait();
  if (!pre && T > 0) load_tile<FMT, ROWS, U, F16S>(A, w, scales, M, NU, nb, g0, 0, lane);

  if (FUSED) {
    // Quantize x into the shared image: 8 lanes per block, 32 blocks per pass.
    const float* x = static_cast<const float*>(act);
    const int lane8 = threadIdx.x & 7;
#pragma unroll 2
    for (int base = 0; base < nb; base += kThreads / 8) {
      const int b = base + (threadIdx.x >> 3);
      const bool valid = b < nb;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (valid) v = reinterpret_cast<const float4*>(x + (size_t)b * QK)[lane8];
      float d;
      int qsum;
      const unsigned q = quantize_quad(v, d, qsum);
      if (valid) {
        reinterpret_cast<unsigned*>(smem + b * kImgSlot)[lane8] = q;
        if (lane8 == 0) reinterpret_cast<float2*>(smem + (size_t)nb * kImgSlot)[b] = make_float2(d, __int_as_float(qsum));
      }
    }
  } else {
    const unsigned char* img = static_cast<const unsigned char*>(act);
    const int n16 = (int)(act_image_bytes(nb) / 16);
    for (int i = threadIdx.x; i < n16; i += kThreads) cp_async16(smem + 16 * i, img + 16 * i);
    cp_async_wait_all();
  }
  __syncthreads();

  float acc[ROWS];
#pragma unroll
  for (int r = 0; r < ROWS; ++r) acc[r] = 0.0f;

  auto compute = [&](const Tile<ROWS, U>& t, int g, int c) {
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const int u = c * CH + k * 32 + lane;
      if (FMT == kFmtQ4_0) {
        if (u < NU) {
          const uint4* xp = reinterpret_cast<const uint4*>(smem + u * kImgSlot);
          const uint4 xa = xp[0];  // xq[0..15]  with the low nibbles
          const uint4 xb = xp[1];  // xq[16..31] with the high nibbles
          const float2 dq = sdq[u];
          const int qsum8 = __float_as_int(dq.y) * 8;
#pragma unroll
          for (int r = 0; r < ROWS; ++r) {
            const uint4 q = t.w[r][k];
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
              if (row < M) isums[(size_t)row * nb + u] = isum;
            }
            acc[r] = __fmaf_rn(__int2float_rn(isum), __fmul_rn(t.sc[r][k], dq.x), acc[r]);
          }
        }
      } else {
        const bool valid = u < NU;  // same for both lanes of a pair (NU even, chunks of 32)
        const int b = u >> 1;
        uint4 xa = make_uint4(0u, 0u, 0u, 0u);
        float xd = 0.0f;
        if (valid) {
          xa = *reinterpret_cast<const uint4*>(smem + b * kImgSlot + (u & 1) * 16);
          xd = sdq[b].x;
        }
#pragma unroll
        for (int r = 0; r < ROWS; ++r) {
          const uint4 q = t.w[r][k];
          int part = 0;
          part = dp4a_ss((int)q.x, (int)xa.x, part);
          part = dp4a_ss((int)q.y, (int)xa.y, part);
          part = dp4a_ss((int)q.z, (int)xa.z, part);
          part = dp4a_ss((int)q.w, (int)xa.w, part);
          const int isum = part + __shfl_xor_sync(kFull, part, 1);
          if (valid && !(lane & 1)) {
            if (DBG) {
              const int row = g * ROWS + r;
              if (row < M) isums[(size_t)row * nb + b] = isum;
            }
            acc[r] = __fmaf_rn(__int2float_rn(isum), __fmul_rn(t.sc[r][k], xd), acc[r]);
          }
        }
      }
    }
    if (c == nchunks - 1) {
      finalize_rows<ROWS>(acc, y, g, M, lane);
      if (pf > 0 && g + pf + 1 < g1) prefetch_group<ROWS, F16S>(w, scales, M, NU, nb, g + pf + 1, lane);
    }
  };

  int g = g0, c = 0;
  for (int t = 0; t < T; t += 2) {
    int gb = g, cb = c + 1;
    if (cb == nchunks) { cb = 0; ++gb; }
    if (t + 1 < T) load_tile<FMT, ROWS, U, F16S>(B, w, scales, M, NU, nb, gb, cb, lane);
    compute(A, g, c);
    int ga = gb, ca = cb + 1;
    if (ca == nchunks) { ca = 0; ++ga; }
    if (t + 2 < T) load_tile<FMT, ROWS, U, F16S>(A, w, scales, M, NU, nb, ga, ca, lane);
    if (t + 1 < T) compute(B, gb, cb);
    g = ga;
    c = ca;
  }
}

// --------------------------------------------------------------------------
// fp32-activation matvec (x86 semantics): Q4_0 (FMT 2) or Q8_0 (FMT 8)
// --------------------------------------------------------------------------
template <int FMT, int ROWS, int U, bool F16S>
__global__ void __launch_bounds__(kThreads, 2)
f32act_matvec_kernel(const uint8_t* __restrict__ w, const void* __restrict__ scales,
                     const float* __restrict__ x, float* __restrict__ y, int M, int nb, int pf, int pre) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* sx = reinterpret_cast<float*>(smem);
  const int lane = threadIdx.x & 31;
  constexpr int UPB = FMT == kFmtQ4_0 ? 1 : 2;
  const int NU = nb * UPB;
  const int ngroups = (M + ROWS - 1) / ROWS;
  int g0, g1;
  group_range(ngroups, g0, g1);
  constexpr int CH = 32 * U;
  const int nchunks = (NU + CH - 1) / CH;
  const int T = (g1 - g0) * nchunks;

  // Weights are read before waiting for the previous kernel only when the
  // caller declared them static (pre != 0); L2 prefetches are always safe
  // (L2 is coherent, a prefetch never returns data to the SM).
  Tile<ROWS, U> A, B;
  if (pre && T > 0) load_tile<FMT, ROWS, U, F16S>(A, w, scales, M, NU, nb, g0, 0, lane);
  for (int gp = g0 + 1; gp < g1 && gp <= g0 + pf; ++gp) prefetch_group<ROWS, F16S>(w, scales, M, NU, nb, gp, lane);
  pdl_trigger();
  pdl_wait();
  if (!pre && T > 0) load_tile<FMT, ROWS, U, F16S>(A, w, scales, M, NU, nb, g0, 0, lane);

  const int K = nb * QK;
  if (FMT == kFmtQ4_0) {
    for (int i = threadIdx.x; i < K; i += kThreads) sx[(i >> 5) * 36 + (i & 31)] = x[i];
  } else {
    for (int i = threadIdx.x; i < K; i += kThreads) sx[(i >> 4) * 20 + (i & 15)] = x[i];
  }
  __syncthreads();

  float acc[ROWS];
#pragma unroll
  for (int r = 0; r < ROWS; ++r) acc[r] = 0.0f;

  auto compute = [&](const Tile<ROWS, U>& t, int g, int c) {
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const int u = c * CH + k * 32 + lane;
      if (u < NU) {
        float blk[ROWS];
#pragma unroll
        for (int r = 0; r < ROWS; ++r) blk[r] = 0.0f;
        if (FMT == kFmtQ4_0) {
          const float4* xp = reinterpret_cast<const float4*>(sx + u * 36);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float4 xl = xp[j];      // elements 4j .. 4j+3 (low nibbles of bytes 4j..)
            const float4 xh = xp[4 + j];  // elements 16+4j .. (high nibbles)
#pragma unroll
            for (int r = 0; r < ROWS; ++r) {
              const unsigned word = j == 0 ? t.w[r][k].x : j == 1 ? t.w[r][k].y : j == 2 ? t.w[r][k].z : t.w[r][k].w;
              const unsigned lo = word & 0x0F0F0F0Fu;
              const unsigned hi = (word >> 4) & 0x0F0F0F0Fu;
              float s = blk[r];
              s = __fmaf_rn(u4_to_f32_minus8(lo, 0), xl.x, s);
              s = __fmaf_rn(u4_to_f32_minus8(lo, 1), xl.y, s);
              s = __fmaf_rn(u4_to_f32_minus8(lo, 2), xl.z, s);
              s = __fmaf_rn(u4_to_f32_minus8(lo, 3), xl.w, s);
              s = __fmaf_rn(u4_to_f32_minus8(hi, 0), xh.x, s);
              s = __fmaf_rn(u4_to_f32_minus8(hi, 1), xh.y, s);
              s = __fmaf_rn(u4_to_f32_minus8(hi, 2), xh.z, s);
              s = __fmaf_rn(u4_to_f32_minus8(hi, 3), xh.w, s);
              blk[r] = s;
            }
          }
        } else {
          const float4* xp = reinterpret_cast<const float4*>(sx + u * 20);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float4 xv = xp[j];
#pragma unroll
            for (int r = 0; r < ROWS; ++r) {
              const unsigned word = (j == 0 ? t.w[r][k].x : j == 1 ? t.w[r][k].y : j == 2 ? t.w[r][k].z : t.w[r][k].w) ^ 0x80808080u;
              float s = blk[r];
              s = __fmaf_rn(s8_biased_to_f32(word, 0), xv.x, s);
              s = __fmaf_rn(s8_biased_to_f32(word, 1), xv.y, s);
              s = __fmaf_rn(s8_biased_to_f32(word, 2), xv.z, s);
              s = __fmaf_rn(s8_biased_to_f32(word, 3), xv.w, s);
              blk[r] = s;
            }
          }
        }
#pragma unroll
        for (int r = 0; r < ROWS; ++r) acc[r] = __fmaf_rn(blk[r], t.sc[r][k], acc[r]);
      }
    }
    if (c == nchunks - 1) {
      finalize_rows<ROWS>(acc, y, g, M, lane);
      if (pf > 0 && g + pf + 1 < g1) prefetch_group<ROWS, F16S>(w, scales, M, NU, nb, g + pf + 1, lane);
    }
  };

  int g = g0, c = 0;
  for (int t = 0; t < T; t += 2) {
    int gb = g, cb = c + 1;
    if (cb == nchunks) { cb = 0; ++gb; }
    if (t + 1 < T) load_tile<FMT, ROWS, U, F16S>(B, w, scales, M, NU, nb, gb, cb, lane);
    compute(A, g, c);
    int ga = gb, ca = cb + 1;
    if (ca == nchunks) { ca = 0; ++ga; }
    if (t + 2 < T) load_tile<FMT, ROWS, U, F16S>(A, w, scales, M, NU, nb, ga, ca, lane);
    if (t + 1 < T) compute(B, gb, cb);
    g = ga;
    c = ca;
  }
}

// --------------------------------------------------------------------------
// Standalone / batched activation quantize to separate xq / xd arrays.
// --------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads)
quantize_q8_0_kernel(const float* __restrict__ x, int8_t* __restrict__ xq,
                     float* __restrict__ xd, long long nblocks) {
  pdl_trigger();
  pdl_wait();
  const int lane8 = threadIdx.x & 7;
  const long long nw = (long long)gridDim.x * kWarps;
  for (long long wb = (long long)blockIdx.x * kWarps + (threadIdx.x >> 5); wb * 4 < nblocks; wb += nw) {
    const long long gb = wb * 4 + ((threadIdx.x & 31) >> 3);
    const bool valid = gb < nblocks;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (valid) v = reinterpret_cast<const float4*>(x + gb * QK)[lane8];
    float d;
    int qsum;
    const unsigned q = quantize_quad(v, d, qsum);
    if (valid) {
      reinterpret_cast<unsigned*>(xq + gb * QK)[lane8] = q;
      if (lane8 == 0) xd[gb] = d;
    }
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

}  // namespace

std::atomic<int> g_opt_pdl{1};

// Stream-ordered scratch (activation images and tiles the library makes for
// one call).  Outside stream capture it comes from a per-device pool that
// keeps its memory across synchronizations: the device's default pool
// returns freed memory to the driver at every synchronize, and mapping it
// again cost ~0.5 ms per call when the caller synchronized between calls.
// Inside capture it is a graph allocation (cudaMallocAsync).
namespace {
std::mutex g_pool_mu;
cudaMemPool_t g_pool[64] = {};
}  // namespace

cudaError_t scratch_alloc_async(void** p, size_t bytes, cudaStream_t stream) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess) {
    cudaGetLastError();
    cs = cudaStreamCaptureStatusActive;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (cs != cudaStreamCaptureStatusNone || dev < 0 || dev >= 64) return cudaMallocAsync(p, bytes, stream);
  cudaMemPool_t pool = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_pool_mu);
    if (!g_pool[dev]) {
      cudaMemPoolProps props = {};
      props.allocType = cudaMemAllocationTypePinned;
      props.handleTypes = cudaMemHandleTypeNone;
      props.location.type = cudaMemLocationTypeDevice;
      props.location.id = dev;
      e = cudaMemPoolCreate(&g_pool[dev], &props);
      if (e != cudaSuccess) {
        g_pool[dev] = nullptr;
        return e;
      }
      unsigned long long keep = ~0ull;
      cudaMemPoolSetAttribute(g_pool[dev], cudaMemPoolAttrReleaseThreshold, &keep);
    }
    pool = g_pool[dev];
  }
  return cudaMallocFromPoolAsync(p, bytes, pool, stream);
}

cudaError_t scratch_free_async(void* p, cudaStream_t stream) { return cudaFreeAsync(p, stream); }

void scratch_trim() {
  std::lock_guard<std::mutex> lk(g_pool_mu);
  for (auto& pool : g_pool)
    if (pool) cudaMemPoolTrimTo(pool, 0);
}

// Runtime switches (asm_set_option): bulk-copy pipeline kernel for the Q8_0
// families (else the register-streaming kernels) and programmatic dependent
// launch (g_opt_pdl above); both on by default.
std::atomic<int> g_opt_tma{1};

// L2 prefetch of the following matvec's weights by the activation pre-pass,
// at most this many MB (asm_set_option "image_prefetch_mb"; 0 = off, the
// default: no gain measured with the bulk-copy matvecs).
std::atomic<int> g_opt_image_prefetch_mb{0};

// Matvecs with K at or above this quantize x in a pre-pass kernel instead of
// in every CTA's prologue (0: never).
std::atomic<int> g_opt_image_min_k{0};

namespace {

// Occupancy of each (kernel, shared bytes, device), computed once: later
// launches (including ones recorded into a CUDA graph) only do the launch.
std::mutex g_occ_mu;
std::map<std::tuple<const void*, size_t, int>, int> g_occ;

cudaError_t launch_pdl(const void* kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       void** args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_opt_pdl.load() ? 1 : 0;
  return cudaLaunchKernelExC(&cfg, kernel, args);
}

// L2 prefetch window of each warp of the register-streaming kernels (measured best).
constexpr int kPfBudgetKb = 24;

template <typename KernelT>
cudaError_t launch_persistent(KernelT kernel, int ngroups, size_t smem, cudaStream_t stream,
                              int dev, void** args, int* pf_arg = nullptr, size_t group_bytes = 0) {
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
  // All co-resident CTAs.
  const int cap = per_sm;
  const long long needed = ((long long)ngroups + kWarps - 1) / kWarps;
  long long grid = (long long)cap * di.sms;
  if (needed < grid) grid = needed;
  if (grid < 1) grid = 1;
  if (pf_arg) {
    const long long groups_per_warp = ((long long)ngroups + grid * kWarps - 1) / (grid * kWarps);
    long long pf = group_bytes ? ((long long)kPfBudgetKb * 1024) / (long long)group_bytes : 0;
    if (pf > groups_per_warp) pf = groups_per_warp;
    *pf_arg = (int)pf;
  }
  return launch_pdl((const void*)kernel, dim3((unsigned)grid), dim3(kThreads), smem, stream, args);
}

// Kernel configuration: rows per warp x units per lane per tile.
struct Cfg {
  int rows, u;
};

Cfg pick_cfg(int M, int NU, int sms, bool fp32_act) {
  (void)NU;
  if (fp32_act) return {2, 2};
  if ((long long)M < (long long)sms * kWarps * 4) return {1, 4};
  return {2, 2};
}

template <int FMT, int R, int U>
cudaError_t launch_q8act_cfg(const MatvecArgs& a, int ngroups, size_t smem, cudaStream_t stream, int dev,
                             void** args) {
  const bool fused = a.image == nullptr;
  int* pf = static_cast<int*>(args[7]);
  const size_t gb = (size_t)R * (size_t)(a.K / QK) * ((FMT == kFmtQ4_0 ? 16 : 32) + (a.scales_f16 ? 2 : 4));
  if (a.isums) {
    if (fused)
      return launch_persistent(q8act_matvec_kernel<FMT, R, U, false, true, true>, ngroups, smem, stream, dev, args, pf, gb);
    return launch_persistent(q8act_matvec_kernel<FMT, R, U, false, true, false>, ngroups, smem, stream, dev, args, pf, gb);
  }
  if (a.scales_f16) {
    if (fused)
      return launch_persistent(q8act_matvec_kernel<FMT, R, U, true, false, true>, ngroups, smem, stream, dev, args, pf, gb);
    return launch_persistent(q8act_matvec_kernel<FMT, R, U, true, false, false>, ngroups, smem, stream, dev, args, pf, gb);
  }
  if (fused)
    return launch_persistent(q8act_matvec_kernel<FMT, R, U, false, false, true>, ngroups, smem, stream, dev, args, pf, gb);
  return launch_persistent(q8act_matvec_kernel<FMT, R, U, false, false, false>, ngroups, smem, stream, dev, args, pf, gb);
}

template <int FMT>
cudaError_t launch_q8act(const MatvecArgs& a, Cfg c, int M, int nb, cudaStream_t stream, int dev, void** args) {
  const int ngroups = (M + c.rows - 1) / c.rows;
  const size_t smem = act_image_bytes(nb);
  if (c.rows == 1 && c.u == 2) return launch_q8act_cfg<FMT, 1, 2>(a, ngroups, smem, stream, dev, args);
  if (c.rows == 1 && c.u == 4) return launch_q8act_cfg<FMT, 1, 4>(a, ngroups, smem, stream, dev, args);
  if (c.rows == 2 && c.u == 4) return launch_q8act_cfg<FMT, 2, 4>(a, ngroups, smem, stream, dev, args);
  const int ng2 = (M + 1) / 2;
  return launch_q8act_cfg<FMT, 2, 2>(a, ng2, smem, stream, dev, args);
}

}  // namespace

int64_t max_k(int fmt, bool fp32_act, int dev) {
  const DevInfo& di = dev_info(dev);
  const int per_block = fp32_act ? (fmt == kFmtQ4_0 ? kQ4F32SmemPerBlock : kQ8F32SmemPerBlock) : (kImgSlot + 8);
  const int64_t nb = (di.smem_optin - 16) / per_block;
  return nb * QK;
}

cudaError_t launch_matvec(const MatvecArgs& a, cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (a.M <= 0) return cudaSuccess;
  const int M = (int)a.M;
  const int nb = (int)(a.K / QK);
  if (nb == 0) return cudaMemsetAsync(a.y, 0, (size_t)a.M * sizeof(float), stream);
  const DevInfo& di = dev_info(dev);
  const int NU = a.fmt == kFmtQ4_0 ? nb : 2 * nb;
  const Cfg c = pick_cfg(M, NU, di.sms, a.fp32_act);

  const void* w = a.w;
  const void* s = a.scales;
  const void* act = a.image ? a.image : (const void*)a.x;
  float* y = a.y;
  int32_t* isums = a.isums;
  int Mi = M, nbi = nb;

  int pf = 0;
  int pre = a.weights_static ? 1 : 0;
  if (matvec_is_fused(a)) {  // the decode fusions live in the bulk-copy kernel only
    if (a.fp32_act || !tma_matvec_supported(a, di.smem_optin)) return cudaErrorNotSupported;
    return launch_tma_matvec(a, di.sms, di.smem_optin, stream, g_opt_pdl.load() != 0);
  }
  // Packed rows are read by the bulk-copy kernel only.
  if (a.packed && (a.fp32_act || !g_opt_tma.load() || !tma_matvec_supported(a, di.smem_optin)))
    return cudaErrorNotSupported;
  if (!a.fp32_act && g_opt_tma.load() && !a.isums_force_ldg && tma_matvec_supported(a, di.smem_optin)) {
    // Long rows: quantizing x once in a pre-pass (which also starts pulling the
    // weights into L2) beats every CTA quantizing all of x in its prologue
    // (measured at K = 11008: 8.1 vs 10.7 us; at K = 4096 the fused prologue
    // is as fast).  The image lives in stream-ordered scratch.
    const int min_k = g_opt_image_min_k.load();
    // (An independent launch quantizes in its own prologue: a pre-pass would
    // have to wait for the previous kernel.)
    if (a.image == nullptr && a.isums == nullptr && !a.act_independent && min_k > 0 && a.K >= min_k) {
      void* img = nullptr;
      e = scratch_alloc_async(&img, act_image_bytes(nb), stream);
      if (e != cudaSuccess) return e;
      const size_t wbytes = (size_t)a.M * nb * ((a.fmt == kFmtQ4_0 ? 16 : 32) + (a.packed ? 2 : 0));
      const size_t sbytes = a.packed ? 0 : (size_t)a.M * nb * (a.scales_f16 ? 2 : 4);
      e = launch_act_image(a.x, img, 1, a.K, stream, a.w, wbytes, a.packed ? nullptr : a.scales, sbytes);
      if (e == cudaSuccess) {
        MatvecArgs b = a;
        b.image = img;
        e = launch_tma_matvec(b, di.sms, di.smem_optin, stream, g_opt_pdl.load() != 0);
      }
      const cudaError_t f = scratch_free_async(img, stream);
      return e != cudaSuccess ? e : f;
    }
    return launch_tma_matvec(a, di.sms, di.smem_optin, stream, g_opt_pdl.load() != 0);
  }
  if (!a.fp32_act) {
    if (act_image_bytes(nb) > (size_t)di.smem_optin) return cudaErrorInvalidValue;
    void* args[] = {(void*)&w, (void*)&s, (void*)&act, (void*)&y, (void*)&Mi, (void*)&nbi, (void*)&isums, (void*)&pf, (void*)&pre};
    return a.fmt == kFmtQ4_0 ? launch_q8act<kFmtQ4_0>(a, c, M, nb, stream, dev, args)
                             : launch_q8act<kFmtQ8_0>(a, c, M, nb, stream, dev, args);
  }
  void* args[] = {(void*)&w, (void*)&s, (void*)&act, (void*)&y, (void*)&Mi, (void*)&nbi, (void*)&pf, (void*)&pre};
  const bool q4 = a.fmt == kFmtQ4_0;
  const size_t smem = (size_t)nb * (q4 ? kQ4F32SmemPerBlock : kQ8F32SmemPerBlock);
  if (smem > (size_t)di.smem_optin) return cudaErrorInvalidValue;
  constexpr int R = 2, U = 2;
  const int ngroups = (M + R - 1) / R;
  const size_t gb = (size_t)R * nb * ((q4 ? 16 : 32) + (a.scales_f16 ? 2 : 4));
  if (q4) {
    return a.scales_f16 ? launch_persistent(f32act_matvec_kernel<kFmtQ4_0, R, U, true>, ngroups, smem, stream, dev, args, &pf, gb)
                        : launch_persistent(f32act_matvec_kernel<kFmtQ4_0, R, U, false>, ngroups, smem, stream, dev, args, &pf, gb);
  }
  return a.scales_f16 ? launch_persistent(f32act_matvec_kernel<kFmtQ8_0, R, U, true>, ngroups, smem, stream, dev, args, &pf, gb)
                      : launch_persistent(f32act_matvec_kernel<kFmtQ8_0, R, U, false>, ngroups, smem, stream, dev, args, &pf, gb);
}

cudaError_t launch_act_image(const float* x, void* image, long long nrows, int64_t K, cudaStream_t stream,
                             const void* pf_w, size_t pf_w_bytes, const void* pf_s, size_t pf_s_bytes) {
  if (nrows <= 0 || K <= 0) return cudaSuccess;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const DevInfo& di = dev_info(dev);
  int nb = (int)(K / QK);
  const long long total = nrows * nb;
  long long grid = (total + 4 * kWarps - 1) / (4 * kWarps);
  const long long cap = (long long)di.sms * 8;
  if (grid > cap) grid = cap;
  unsigned char* img = static_cast<unsigned char*>(image);
  long long stride = (long long)act_image_bytes(nb);
  // Prefetch at most "image_prefetch_mb" MB of the following matvec's weights,
  // in proportion between the weight and scale planes; 16-byte aligned starts only.
  const size_t pf_cap = (size_t)g_opt_image_prefetch_mb.load() << 20;
  const size_t tot = pf_w_bytes + pf_s_bytes;
  if (tot > pf_cap && tot > 0) {
    pf_w_bytes = (size_t)((double)pf_w_bytes * pf_cap / tot);
    pf_s_bytes = (size_t)((double)pf_s_bytes * pf_cap / tot);
  }
  const unsigned char* pw = ((uintptr_t)pf_w % 16 == 0) ? static_cast<const unsigned char*>(pf_w) : nullptr;
  const unsigned char* ps = ((uintptr_t)pf_s % 16 == 0) ? static_cast<const unsigned char*>(pf_s) : nullptr;
  unsigned long long bw = pw ? pf_w_bytes : 0, bs = ps ? pf_s_bytes : 0;
  void* args[] = {(void*)&x, (void*)&img, (void*)&nb, (void*)&nrows, (void*)&stride,
                  (void*)&pw, (void*)&bw, (void*)&ps, (void*)&bs};
  return launch_pdl((const void*)act_image_kernel, dim3((unsigned)grid), dim3(kThreads), 0, stream, args);
}

cudaError_t launch_quantize(const float* x, int8_t* xq, float* xd, long long nblocks,
                            cudaStream_t stream) {
  if (nblocks <= 0) return cudaSuccess;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const DevInfo& di = dev_info(dev);
  long long grid = (nblocks + 4 * kWarps - 1) / (4 * kWarps);
  const long long cap = (long long)di.sms * 8;
  if (grid > cap) grid = cap;
  void* args[] = {(void*)&x, (void*)&xq, (void*)&xd, (void*)&nblocks};
  return launch_pdl((const void*)quantize_q8_0_kernel, dim3((unsigned)grid), dim3(kThreads), 0, stream, args);
}

// Launch-dependency floor: a chain of kernels that do nothing but the
// programmatic-dependent-launch protocol the matvecs use (trigger at entry,
// then wait for the previous grid when `wait` is set), one CTA per SM.
__global__ void floor_kernel(int wait) {
  pdl_trigger();
  if (wait) pdl_wait();
}

cudaError_t launch_floor_chain(int n, bool pdl, bool wait, cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const DevInfo& di = dev_info(dev);
  const int wt = wait ? 1 : 0;
  for (int i = 0; i < n; ++i) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)di.sms);
    cfg.blockDim = dim3(kThreads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    e = cudaLaunchKernelEx(&cfg, floor_kernel, wt);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// Packed rows: row r = its qs bytes (wq16 16-byte units), then its fp16
// scales (ws16 units).  One thread per 16-byte unit of the output.
__global__ void pack_rows_kernel(const uint4* __restrict__ qs, const uint4* __restrict__ sc, uint4* __restrict__ out,
                                 long long M, int wq16, int ws16) {
  const long long per = wq16 + ws16, total = M * per;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / per;
    const int j = (int)(i - r * per);
    out[i] = j < wq16 ? qs[r * wq16 + j] : sc[r * ws16 + (j - wq16)];
  }
}

cudaError_t launch_pack_rows(int fmt, const void* qs, const void* scales_f16, void* out, int64_t M, int64_t K,
                             cudaStream_t stream) {
  const int64_t nb = K / QK;
  if (M <= 0 || nb <= 0 || nb % 8 != 0) return cudaErrorInvalidValue;
  const int wq16 = (int)(nb * (fmt == kFmtQ4_0 ? 16 : 32) / 16), ws16 = (int)(nb * 2 / 16);
  long long blocks = (M * (wq16 + ws16) + 255) / 256;
  if (blocks > 148LL * 32) blocks = 148LL * 32;
  pack_rows_kernel<<<(unsigned)blocks, 256, 0, stream>>>(static_cast<const uint4*>(qs),
                                                         static_cast<const uint4*>(scales_f16),
                                                         static_cast<uint4*>(out), (long long)M, wq16, ws16);
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

// asmllm_b200/csrc/attention.cuh -- one query head of batch-1 decode
// attention, shared by the standalone kernel (decode.cu, 256 threads) and the
// persistent decode kernel (decode_persistent.cu, its 512 consumer threads).
//
// Reference: THRISHAL12345/asmllm src/runtime/generate.py:281-296 with the
// RoPE of tests/reference/ops.py:119-141 and the softmax of ops.py:144-153:
//   q, k <- RoPE(q, k) on interleaved pairs (x0*c - x1*s, x0*s + x1*c)
//   cache[pos] <- (k, v)            (fp16 here)
//   p <- softmax(q . K[0..pos]^T / sqrt(hd));  out <- p . V[0..pos]
// then the head's 128 outputs are quantized to 4 Q8_0 blocks of the o-proj's
// activation image.
//
// Data another kernel (or another CTA) wrote -- qkv, cache rows -- is read
// with ld.global.cg (L2, the coherence point), never from an SM's L1.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "common.cuh"
#include "tiles.cuh"

namespace asmllm {

constexpr int kAttnHd = 128;  // head dimension the attention code is built for

// Shared-memory scratch of one head: p [ctx], q/k/v [128], acc [NT/16][128], red [NT/32].
struct AttnSmem {
  float* p;
  float* q;
  float* k;
  float* v;
  float* acc;
  float* red;
};

template <int NT>
__host__ __device__ constexpr size_t attn_smem_bytes_fixed() {
  return (size_t)(3 * kAttnHd + (NT / 16) * kAttnHd + NT / 32) * sizeof(float);
}

// Carves the scratch out of a 16-byte aligned buffer: fixed arrays first, p last.
template <int NT>
__device__ __forceinline__ AttnSmem attn_smem_carve(unsigned char* base) {
  AttnSmem s;
  float* f = reinterpret_cast<float*>(base);
  s.q = f;
  s.k = f + kAttnHd;
  s.v = f + 2 * kAttnHd;
  s.acc = f + 3 * kAttnHd;
  s.red = s.acc + (NT / 16) * kAttnHd;
  s.p = s.red + ((NT / 32 + 3) & ~3);
  return s;
}

// L2 prefetch of one 128-byte line (a hint).
__device__ __forceinline__ void prefetch_line_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// Brings K/V rows [0, n) of KV head j towards L2 (2 lines of K and 2 of V per
// position; every address inside the cache when n <= ctx).
template <int NT>
__device__ __forceinline__ void attn_prefetch_rows(const __half* kc, const __half* vc, int n, int j, int n_kv,
                                                   int tid) {
  const size_t row_stride = (size_t)n_kv * kAttnHd;
  for (int i = tid; i < 4 * n; i += NT) {
    const int t = i >> 2, part = i & 3;
    prefetch_line_l2((part < 2 ? kc : vc) + (size_t)t * row_stride + (size_t)j * kAttnHd + (part & 1) * 64);
  }
}

template <int NT, class Sync>
__device__ __forceinline__ float attn_block_reduce(float v, float* red, bool is_max, int tid, Sync sync) {
  const int warp = tid >> 5, lane = tid & 31;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float t = __shfl_xor_sync(kFull, v, o);
    v = is_max ? fmaxf(v, t) : v + t;
  }
  sync();  // red may still be read from a previous reduction
  if (lane == 0 && tid < NT) red[warp] = v;
  sync();
  float r = red[0];
#pragma unroll
  for (int i = 1; i < NT / 32; ++i) r = is_max ? fmaxf(r, red[i]) : r + red[i];
  return r;
}

// Attention of query head h at position pos (0 <= pos < ctx, checked by the
// caller), computed by threads tid 0..NT-1; a caller with more threads runs
// them through every sync() too (they do no work), so the arithmetic -- and
// the result -- does not depend on the caller's block size.  The
// first CTA of a KV group (h % group == 0) appends k, v at pos; every CTA of
// the group keeps its own fp16-rounded copy for position pos (the append is
// not visible to the group's other CTAs yet).
template <int NT, class Sync>
__device__ void attention_head(const float* qkv, __half* kc, __half* vc, const float2* rope_cs, int pos, int h,
                               int n_heads, int n_kv, float sqrt_hd, unsigned char* image, const AttnSmem& sm,
                               int tid, Sync sync, int n_rep = 1, size_t rep_stride = 0,
                               unsigned char* tiles = nullptr, int np = 0, int tile_row = 0) {
  static_assert(NT == 256, "attention is laid out for 256 working threads");
  constexpr int kSlices = NT / 16;  // position slices of P.V (16 groups of 8 dims each)
  const int warp = tid >> 5, lane = tid & 31;
  const int group = n_heads / n_kv, j = h / group;
  const size_t row_stride = (size_t)n_kv * kAttnHd;  // halves between consecutive positions
  const bool writer = (h % group) == 0;
  if (tid < 128) {  // 0..63: q pairs, 64..127: k pairs
    const int i = tid & 63;
    const float* src = tid < 64 ? qkv + (size_t)h * kAttnHd : qkv + (size_t)(n_heads + j) * kAttnHd;
    const float2 x = __ldcg(reinterpret_cast<const float2*>(src) + i);
    const float2 cs = rope_cs[(size_t)pos * (kAttnHd / 2) + i];
    const float o0 = __fsub_rn(__fmul_rn(x.x, cs.x), __fmul_rn(x.y, cs.y));
    const float o1 = __fadd_rn(__fmul_rn(x.x, cs.y), __fmul_rn(x.y, cs.x));
    if (tid < 64) {
      sm.q[2 * i] = o0;
      sm.q[2 * i + 1] = o1;
    } else {
      const __half2 k2 = __floats2half2_rn(o0, o1);
      sm.k[2 * i] = __low2float(k2);
      sm.k[2 * i + 1] = __high2float(k2);
      if (writer) reinterpret_cast<__half2*>(kc + (size_t)pos * row_stride + (size_t)j * kAttnHd)[i] = k2;
    }
  } else if (tid < 256) {
    const int d = tid - 128;
    const __half vh = __float2half_rn(__ldcg(qkv + (size_t)(n_heads + n_kv + j) * kAttnHd + d));
    sm.v[d] = __half2float(vh);
    if (writer) vc[(size_t)pos * row_stride + (size_t)j * kAttnHd + d] = vh;
  }
  sync();

  // Scores: one thread per position, the whole 128-dim dot (16 loads of 8
  // halves in flight per thread).
  const int n = pos + 1;
  const bool act = tid < NT;
  for (int t = tid; act && t < n; t += NT) {
    float dot = 0.0f;
    if (t < pos) {
      const uint4* kr = reinterpret_cast<const uint4*>(kc + (size_t)t * row_stride + (size_t)j * kAttnHd);
      uint4 raw[kAttnHd / 8];
#pragma unroll
      for (int c = 0; c < kAttnHd / 8; ++c) raw[c] = __ldcg(kr + c);
#pragma unroll
      for (int c = 0; c < kAttnHd / 8; ++c) {
        const __half2* hp = reinterpret_cast<const __half2*>(&raw[c]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 kf = __half22float2(hp[e]);
          dot = __fmaf_rn(sm.q[c * 8 + 2 * e], kf.x, dot);
          dot = __fmaf_rn(sm.q[c * 8 + 2 * e + 1], kf.y, dot);
        }
      }
    } else {
#pragma unroll 16
      for (int d = 0; d < kAttnHd; ++d) dot = __fmaf_rn(sm.q[d], sm.k[d], dot);
    }
    sm.p[t] = __fdiv_rn(dot, sqrt_hd);
  }
  sync();

  // Softmax as the reference: exp(s - max(s)) / sum.
  float m = -INFINITY;
  for (int t = tid; act && t < n; t += NT) m = fmaxf(m, sm.p[t]);
  m = attn_block_reduce<NT>(m, sm.red, true, tid, sync);
  float sum = 0.0f;
  for (int t = tid; act && t < n; t += NT) {
    const float e = expf(__fsub_rn(sm.p[t], m));
    sm.p[t] = e;
    sum += e;
  }
  sum = attn_block_reduce<NT>(sum, sm.red, false, tid, sync);
  for (int t = tid; act && t < n; t += NT) sm.p[t] = __fdiv_rn(sm.p[t], sum);
  sync();

  // out[d] = sum_t p[t] v[t][d]: thread (slice, group) takes 8 dims and the
  // positions slice, slice + kSlices, ...; the slices are summed in order.
  if (act) {
    const int g = tid & 15, sl = tid >> 4;
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
#pragma unroll 4
    for (int t = sl; t < n; t += kSlices) {
      const float p = sm.p[t];
      if (t < pos) {
        const uint4 raw = __ldcg(reinterpret_cast<const uint4*>(vc + (size_t)t * row_stride + (size_t)j * kAttnHd) + g);
        const __half2* hp = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 vf = __half22float2(hp[e]);
          acc[2 * e] = __fmaf_rn(p, vf.x, acc[2 * e]);
          acc[2 * e + 1] = __fmaf_rn(p, vf.y, acc[2 * e + 1]);
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = __fmaf_rn(p, sm.v[g * 8 + e], acc[e]);
      }
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) sm.acc[sl * kAttnHd + g * 8 + e] = acc[e];
  }
  sync();
  if (tid < kAttnHd) {
    float o = sm.acc[tid];
#pragma unroll
    for (int i = 1; i < kSlices; ++i) o += sm.acc[i * kAttnHd + tid];
    sm.q[tid] = o;  // the head's output (q is no longer needed)
  }
  sync();

  // Quantize the head's 128 outputs (4 Q8_0 blocks, 8 lanes per block) into
  // the image slots of blocks 4h .. 4h+3 (or into row tile_row of the tiles).
  if (warp == 0) {
    const int b = lane >> 3, l8 = lane & 7;
    const float4 o = reinterpret_cast<const float4*>(sm.q)[b * 8 + l8];
    float d;
    int qsum;
    const unsigned q = quantize_quad(o, d, qsum);
    const int nb = n_heads * (kAttnHd / QK);
    const int blk = h * (kAttnHd / QK) + b;
    if (tiles) {
      tiles_store_quad(tiles, np, nb, tile_row, blk, l8, q, d, true);
      return;
    }
    for (int r = 0; r < n_rep; ++r) {  // identical replicas (see the persistent decode kernel)
      unsigned char* im = image + (size_t)r * rep_stride;
      reinterpret_cast<unsigned*>(im + (size_t)blk * 48)[l8] = q;
      if (l8 == 0) reinterpret_cast<float2*>(im + (size_t)nb * 48)[blk] = make_float2(d, __int_as_float(qsum));
    }
  }
}

}  // namespace asmllm

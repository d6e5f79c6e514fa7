// asmllm_b200/csrc/decode.cu -- attention for one batch-1 decode position.
//
// The decode step of the reference (THRISHAL12345/asmllm
// src/runtime/generate.py:255-326, AsmEngineForward.forward_token) does, per
// layer: RMSNorm -> q/k/v matvecs -> RoPE on q and k -> append k, v to the
// cache -> per head softmax(q.K^T / sqrt(hd)) . V -> o matvec -> residual ->
// RMSNorm -> gate/up matvecs -> silu(gate)*up -> down matvec -> residual.
// The matvecs and their RMSNorm / residual / SwiGLU / argmax fusions are the
// bulk-copy matvec's prologue and epilogue modes (tma_matvec.cu); this file
// holds the rest of the layer: RoPE, the fp16 KV append, the attention and
// the Q8_0 quantization of its output (one kernel, one CTA per query head).
//
// Layouts (device):
//   qkv      fp32 [n_heads + 2 n_kv][hd]: q heads, then k heads, then v heads
//   k/v cache fp16 [ctx][n_kv][hd] for this layer
//   rope_cs  fp32 pairs [ctx][hd/2] = (cos, sin) of pos * theta^(-2i/hd)
//   image    Q8_0 activation image of the attention output, n_heads*hd/32 blocks
// Every Q8_0 block (32 values) lies inside one head (hd = 128 = 4 blocks), so
// each CTA quantizes its own head's output.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "matvec.cuh"

namespace asmllm {

namespace {

constexpr int kHd = 128;      // head dimension this kernel is built for
constexpr int kThreads = 256;  // 8 warps

__device__ __forceinline__ float block_reduce(float v, float* red, bool is_max) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float t = __shfl_xor_sync(kFull, v, o);
    v = is_max ? fmaxf(v, t) : v + t;
  }
  __syncthreads();  // red may still be read from a previous reduction
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int i = 1; i < kThreads / 32; ++i) r = is_max ? fmaxf(r, red[i]) : r + red[i];
  return r;
}

__global__ void __launch_bounds__(kThreads) attention_decode_kernel(
    const float* __restrict__ qkv, __half* __restrict__ kc, __half* __restrict__ vc,
    const float2* __restrict__ rope_cs, const int32_t* __restrict__ pos_p, unsigned char* __restrict__ image,
    int n_heads, int n_kv, int ctx, float sqrt_hd, unsigned* __restrict__ err) {
  extern __shared__ float s_p[];  // [ctx] scores, then probabilities
  __shared__ float s_q[kHd], s_k[kHd], s_v[kHd], s_out[2][kHd], s_red[kThreads / 32];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = blockIdx.x, group = n_heads / n_kv, j = h / group;
  pdl_trigger();
  pdl_wait();  // qkv comes from the previous kernel
  const int pos = *pos_p;
  if (pos < 0 || pos >= ctx) {
    if (tid == 0) atomicOr(err, kErrDecodeRange);
    return;
  }
  // RoPE on interleaved pairs (x0, x1) = (x[2i], x[2i+1]), as the reference
  // ref_rope (tests/reference/ops.py:119-141): x0*c - x1*s, x0*s + x1*c, each
  // product rounded (no contraction).  The first CTA of a KV group appends the
  // new k, v (fp16) to the cache; every CTA of the group keeps its own copy of
  // the fp16-rounded values for position pos.
  const bool writer = (h % group) == 0;
  if (tid < 128) {  // 0..63: q pairs, 64..127: k pairs
    const int i = tid & 63;
    const float* src = tid < 64 ? qkv + (size_t)h * kHd : qkv + (size_t)(n_heads + j) * kHd;
    const float2 x = reinterpret_cast<const float2*>(src)[i];
    const float2 cs = rope_cs[(size_t)pos * (kHd / 2) + i];
    const float o0 = __fsub_rn(__fmul_rn(x.x, cs.x), __fmul_rn(x.y, cs.y));
    const float o1 = __fadd_rn(__fmul_rn(x.x, cs.y), __fmul_rn(x.y, cs.x));
    if (tid < 64) {
      s_q[2 * i] = o0;
      s_q[2 * i + 1] = o1;
    } else {
      const __half2 k2 = __floats2half2_rn(o0, o1);
      s_k[2 * i] = __low2float(k2);
      s_k[2 * i + 1] = __high2float(k2);
      if (writer) reinterpret_cast<__half2*>(kc + ((size_t)pos * n_kv + j) * kHd)[i] = k2;
    }
  } else {
    const int d = tid - 128;
    const __half vh = __float2half_rn(qkv[(size_t)(n_heads + n_kv + j) * kHd + d]);
    s_v[d] = __half2float(vh);
    if (writer) vc[((size_t)pos * n_kv + j) * kHd + d] = vh;
  }
  __syncthreads();

  // Scores: one warp per position, 4 dims per lane; the position being
  // appended comes from shared memory (the cache write above may not be
  // visible to the other CTAs of the group yet).
  const int n = pos + 1;
  const float4 q4 = reinterpret_cast<const float4*>(s_q)[lane];
  for (int t0 = warp; t0 < n; t0 += 4 * (kThreads / 32)) {
    float dot[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int t = t0 + u * (kThreads / 32);
      float4 k4 = make_float4(0.f, 0.f, 0.f, 0.f);
      if (t < pos) {
        const uint2 raw = reinterpret_cast<const uint2*>(kc + ((size_t)t * n_kv + j) * kHd)[lane];
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
        k4 = make_float4(a.x, a.y, b.x, b.y);
      } else if (t == pos) {
        k4 = reinterpret_cast<const float4*>(s_k)[lane];
      }
      dot[u] = __fmaf_rn(q4.w, k4.w, __fmaf_rn(q4.z, k4.z, __fmaf_rn(q4.y, k4.y, __fmul_rn(q4.x, k4.x))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
      for (int u = 0; u < 4; ++u) dot[u] += __shfl_xor_sync(kFull, dot[u], o);
    }
    if (lane == 0) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int t = t0 + u * (kThreads / 32);
        if (t < n) s_p[t] = __fdiv_rn(dot[u], sqrt_hd);
      }
    }
  }
  __syncthreads();

  // Softmax as the reference: exp(s - max(s)) / sum.
  float m = -INFINITY;
  for (int t = tid; t < n; t += kThreads) m = fmaxf(m, s_p[t]);
  m = block_reduce(m, s_red, true);
  float sum = 0.0f;
  for (int t = tid; t < n; t += kThreads) {
    const float e = expf(__fsub_rn(s_p[t], m));
    s_p[t] = e;
    sum += e;
  }
  sum = block_reduce(sum, s_red, false);
  for (int t = tid; t < n; t += kThreads) s_p[t] = __fdiv_rn(s_p[t], sum);
  __syncthreads();

  // out[d] = sum_t p[t] v[t][d]: two halves of the positions, then combined.
  {
    const int d = tid & (kHd - 1), half = tid >> 7;
    float acc = 0.0f;
#pragma unroll 8
    for (int t = half; t < pos; t += 2)
      acc = __fmaf_rn(s_p[t], __half2float(vc[((size_t)t * n_kv + j) * kHd + d]), acc);
    if (((pos - half) & 1) == 0) acc = __fmaf_rn(s_p[pos], s_v[d], acc);
    s_out[half][d] = acc;
  }
  __syncthreads();

  // Quantize the head's 128 outputs (4 Q8_0 blocks, 8 lanes per block) into
  // the image slots of blocks 4h .. 4h+3.
  if (warp == 0) {
    const int b = lane >> 3, l8 = lane & 7;
    float4 o;
    o.x = s_out[0][b * 32 + l8 * 4 + 0] + s_out[1][b * 32 + l8 * 4 + 0];
    o.y = s_out[0][b * 32 + l8 * 4 + 1] + s_out[1][b * 32 + l8 * 4 + 1];
    o.z = s_out[0][b * 32 + l8 * 4 + 2] + s_out[1][b * 32 + l8 * 4 + 2];
    o.w = s_out[0][b * 32 + l8 * 4 + 3] + s_out[1][b * 32 + l8 * 4 + 3];
    float d;
    int qsum;
    const unsigned q = quantize_quad(o, d, qsum);
    const int nb = n_heads * (kHd / QK);
    const int blk = h * (kHd / QK) + b;
    reinterpret_cast<unsigned*>(image + (size_t)blk * 48)[l8] = q;
    if (l8 == 0) reinterpret_cast<float2*>(image + (size_t)nb * 48)[blk] = make_float2(d, __int_as_float(qsum));
  }
}

}  // namespace

cudaError_t launch_attention_decode(const float* qkv, void* k_cache, void* v_cache, const float* rope_cs,
                                    const int32_t* pos, void* image, int n_heads, int n_kv, int head_dim, int ctx,
                                    float sqrt_hd, cudaStream_t stream, bool pdl) {
  if (head_dim != kHd || n_heads <= 0 || n_kv <= 0 || n_heads % n_kv != 0 || ctx <= 0)
    return cudaErrorNotSupported;
  const size_t smem = (size_t)ctx * sizeof(float);
  int dev = 0, optin = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (smem + 6 * kHd * sizeof(float) + 64 > (size_t)optin) return cudaErrorNotSupported;
  if (smem > 48 * 1024) {
    const cudaError_t e =
        cudaFuncSetAttribute(attention_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)n_heads);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  __half* kc = static_cast<__half*>(k_cache);
  __half* vc = static_cast<__half*>(v_cache);
  const float2* cs = reinterpret_cast<const float2*>(rope_cs);
  unsigned char* img = static_cast<unsigned char*>(image);
  unsigned* err = device_error_word();
  if (!err) return cudaErrorUnknown;
  return cudaLaunchKernelEx(&cfg, attention_decode_kernel, qkv, kc, vc, cs, pos, img, n_heads, n_kv, ctx, sqrt_hd,
                            err);
}

}  // namespace asmllm

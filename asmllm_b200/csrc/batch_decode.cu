// asmllm_b200/csrc/batch_decode.cu -- the glue of a batched decode step
// (B sequences in lockstep at one position), around the tensor-core batched
// product of prefill_gemm.cu.
//
// The reference decodes one sequence at a time (THRISHAL12345/asmllm
// src/runtime/generate.py:255-326, AsmEngineForward.forward_token); a batch
// of B sequences is B such steps whose seven matvecs per layer become one
// batched product each (weights streamed once for all B rows).  The glue per
// row is the same arithmetic as the batch-1 path:
//   rows_norm_tiles   x <- embed[token] | x + delta | x, then RMSNorm
//                     (x / sqrt(mean(x^2) + eps)) * w (tests/reference/ops.py:
//                     103-116) and the Q8_0 quantize of the result, stored as
//                     the row's activation tiles (tiles.cuh) the next product reads;
//   rows_swiglu_tiles h = (g / (1 + exp(-g))) * u (generate.py:370) from the
//                     interleaved gate/up product rows, quantized;
//   attention_batch   RoPE, fp16 KV append and attention per (head, row)
//                     (generate.py:281-296), the per-head code of attention.cuh;
//   rows_argmax       the first maximum of each row's logits as an orderable
//                     64-bit key (value, index), so that tensor-parallel ranks
//                     combine their vocabulary slices with one max all-reduce;
//   rows_advance      token[row][pos + 1] = argmax (after the prompt), pos += 1.
// Data written by other kernels is read through L2 (ld.global.cg).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "attention.cuh"
#include "common.cuh"
#include "matvec.cuh"
#include "pipeline.cuh"
#include "tiles.cuh"

namespace asmllm {

namespace {

constexpr int kRowThreads = 256;  // 8 warps

struct CtaSync {
  __device__ __forceinline__ void operator()() const { __syncthreads(); }
};

// Quantizes nb blocks of fp32 values in shared memory into token row n of
// the activation tiles (passes of 32 blocks, 8 lanes per block; every lane
// takes part in every pass, so the shuffles see whole warps).
__device__ __forceinline__ void quantize_row_tiles(const float* v, int nb, unsigned char* tiles, int np, int n) {
  const int lane8 = threadIdx.x & 7;
  for (int base = 0; base < nb; base += kRowThreads / 8) {
    const int b = base + (threadIdx.x >> 3);
    const bool valid = b < nb;
    const float4 x = valid ? reinterpret_cast<const float4*>(v + (size_t)b * QK)[lane8] : make_float4(0.f, 0.f, 0.f, 0.f);
    float d;
    int qsum;
    const unsigned q = quantize_quad(x, d, qsum);
    tiles_store_quad(tiles, np, nb, n, b, lane8, q, d, valid);
  }
}

__global__ void __launch_bounds__(kRowThreads) rows_norm_tiles_kernel(const RowsArgs a, unsigned* __restrict__ err) {
  extern __shared__ __align__(16) float srow[];  // [dim]
  __shared__ float part[kRowThreads / 32];
  const int r = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int dim = a.dim, n4 = dim / 4;
  pdl_trigger();
  pdl_wait();  // x, delta, tokens and pos come from earlier kernels
  float* x = a.x + (size_t)r * dim;
  const float4* src = reinterpret_cast<const float4*>(x);
  if (a.embed) {
    const int p = __ldcg(a.pos);
    int tok = (p >= 0 && p < a.max_tokens) ? __ldcg(a.tokens + (size_t)r * a.max_tokens + p) : -1;
    if (tok < 0 || tok >= a.vocab) {
      if (tid == 0) atomicOr(err, kErrDecodeRange);
      tok = 0;
    }
    src = reinterpret_cast<const float4*>(a.embed + (size_t)tok * dim);
  }
  const float4* dl = a.delta ? reinterpret_cast<const float4*>(a.delta + (size_t)r * dim) : nullptr;
  float ss = 0.0f;
  for (int i = tid; i < n4; i += kRowThreads) {
    float4 v = __ldcg(src + i);
    if (dl) {
      const float4 d = __ldcg(dl + i);
      v = make_float4(__fadd_rn(v.x, d.x), __fadd_rn(v.y, d.y), __fadd_rn(v.z, d.z), __fadd_rn(v.w, d.w));
    }
    if (a.embed || dl) __stcg(reinterpret_cast<float4*>(x) + i, v);
    reinterpret_cast<float4*>(srow)[i] = v;
    ss = __fadd_rn(ss, __fadd_rn(__fadd_rn(__fmul_rn(v.x, v.x), __fmul_rn(v.y, v.y)),
                                 __fadd_rn(__fmul_rn(v.z, v.z), __fmul_rn(v.w, v.w))));
  }
  if (a.norm_w) {
    ss = warp_sum(ss);
    if (lane == 0) part[warp] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int i = 0; i < kRowThreads / 32; ++i) tot = __fadd_rn(tot, part[i]);
    const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)dim), a.eps));
    for (int i = tid; i < n4; i += kRowThreads) {  // (x / rms) * w, as the reference RMSNorm
      const float4 v = reinterpret_cast<const float4*>(srow)[i];
      const float4 w = reinterpret_cast<const float4*>(a.norm_w)[i];
      reinterpret_cast<float4*>(srow)[i] =
          make_float4(__fmul_rn(__fdiv_rn(v.x, rms), w.x), __fmul_rn(__fdiv_rn(v.y, rms), w.y),
                      __fmul_rn(__fdiv_rn(v.z, rms), w.z), __fmul_rn(__fdiv_rn(v.w, rms), w.w));
    }
  }
  __syncthreads();
  quantize_row_tiles(srow, dim / QK, static_cast<unsigned char*>(a.tiles), a.np, r);
}

__global__ void __launch_bounds__(kRowThreads) rows_swiglu_tiles_kernel(const float* __restrict__ gu, int ffn,
                                                                        unsigned char* __restrict__ tiles, int np) {
  extern __shared__ __align__(16) float srow[];  // [ffn]
  const int r = blockIdx.x, tid = threadIdx.x;
  pdl_trigger();
  pdl_wait();  // the gate/up product rows come from the previous kernel
  const float2* g2 = reinterpret_cast<const float2*>(gu + (size_t)r * 2 * ffn);  // (gate_i, up_i)
  for (int i = tid; i < ffn; i += kRowThreads) {
    const float2 v = __ldcg(g2 + i);
    srow[i] = __fmul_rn(__fdiv_rn(v.x, __fadd_rn(1.0f, expf(-v.x))), v.y);
  }
  __syncthreads();
  quantize_row_tiles(srow, ffn / QK, tiles, np, r);
}

__global__ void __launch_bounds__(kRowThreads) attention_batch_kernel(
    const float* __restrict__ qkv, size_t qkv_stride, __half* __restrict__ kc, __half* __restrict__ vc,
    size_t cache_stride, const float2* __restrict__ rope_cs, const int32_t* __restrict__ pos_p,
    unsigned char* __restrict__ tiles, int np, int n_heads, int n_kv, int ctx, float sqrt_hd,
    unsigned* __restrict__ err) {
  extern __shared__ __align__(16) unsigned char smem[];
  const AttnSmem sm = attn_smem_carve<kRowThreads>(smem);
  const int tid = threadIdx.x, h = blockIdx.x, r = blockIdx.y;
  const int j = h / (n_heads / n_kv);
  __half* k = kc + (size_t)r * cache_stride;
  __half* v = vc + (size_t)r * cache_stride;
  pdl_trigger();
  {  // cached rows towards L2 while the previous kernel finishes (a hint, clamped to the cache)
    int hint = __ldcg(pos_p) + 1;
    hint = hint < 0 ? 0 : (hint > ctx ? ctx : hint);
    attn_prefetch_rows<kRowThreads>(k, v, hint, j, n_kv, tid);
  }
  pdl_wait();
  const int pos = __ldcg(pos_p);
  if (pos < 0 || pos >= ctx) {
    if (tid == 0) atomicOr(err, kErrDecodeRange);
    return;
  }
  attention_head<kRowThreads>(qkv + (size_t)r * qkv_stride, k, v, rope_cs, pos, h, n_heads, n_kv, sqrt_hd, nullptr,
                              sm, tid, CtaSync{}, 1, 0, tiles, np, r);
}

// Orderable key as a signed 64-bit value (top bit flipped): the max over int64
// of the keys is the max of the unsigned keys, so ranks may combine keys with
// a signed max all-reduce.
__device__ __forceinline__ long long signed_key(unsigned long long k) {
  return (long long)(k ^ 0x8000000000000000ull);
}

__global__ void __launch_bounds__(kRowThreads) rows_argmax_kernel(const float* __restrict__ logits, int n,
                                                                  size_t stride, int offset,
                                                                  long long* __restrict__ keys) {
  __shared__ unsigned long long part[kRowThreads / 32];
  const int r = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  pdl_trigger();
  pdl_wait();
  const float* row = logits + (size_t)r * stride;
  unsigned long long best = 0;  // below every key
  for (int i = tid; i < n; i += kRowThreads) {
    const float v = __ldcg(row + i);
    if (v == v) {
      const unsigned long long k = argmax_key(v, i + offset);
      best = k > best ? k : best;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(kFull, best, o);
    best = t > best ? t : best;
  }
  if (lane == 0) part[warp] = best;
  __syncthreads();
  if (tid == 0) {
    unsigned long long b = part[0];
    for (int i = 1; i < kRowThreads / 32; ++i) b = part[i] > b ? part[i] : b;
    keys[r] = signed_key(b);
  }
}

__global__ void rows_advance_kernel(const long long* __restrict__ keys, int rows, int32_t* __restrict__ tokens,
                                    int max_tokens, int32_t* __restrict__ pos_p, int n_prompt) {
  pdl_trigger();
  pdl_wait();
  const int p = __ldcg(pos_p);
  for (int r = threadIdx.x; r < rows; r += blockDim.x) {
    if (p + 1 >= n_prompt && p + 1 < max_tokens) {
      const unsigned long long k = (unsigned long long)__ldcg(keys + r) ^ 0x8000000000000000ull;
      tokens[(size_t)r * max_tokens + p + 1] = argmax_row(k);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) *pos_p = p + 1;
}

cudaLaunchConfig_t row_config(unsigned gx, unsigned gy, unsigned threads, size_t smem, cudaStream_t stream,
                              cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(gx, gy);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_opt_pdl.load() ? 1 : 0;
  return cfg;
}

template <class K>
cudaError_t allow_smem(K kernel, size_t smem) {
  if (smem <= 48 * 1024) return cudaSuccess;
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}

}  // namespace

cudaError_t launch_rows_norm_tiles(const RowsArgs& a, cudaStream_t stream) {
  const size_t smem = (size_t)a.dim * sizeof(float);
  cudaError_t e = allow_smem(rows_norm_tiles_kernel, smem);
  if (e != cudaSuccess) return e;
  unsigned* err = device_error_word();
  if (!err) return cudaErrorUnknown;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = row_config((unsigned)a.rows, 1, kRowThreads, smem, stream, attr);
  return cudaLaunchKernelEx(&cfg, rows_norm_tiles_kernel, a, err);
}

cudaError_t launch_rows_swiglu_tiles(const float* gu, int rows, int ffn, void* tiles, int np, cudaStream_t stream) {
  const size_t smem = (size_t)ffn * sizeof(float);
  cudaError_t e = allow_smem(rows_swiglu_tiles_kernel, smem);
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = row_config((unsigned)rows, 1, kRowThreads, smem, stream, attr);
  return cudaLaunchKernelEx(&cfg, rows_swiglu_tiles_kernel, gu, ffn, static_cast<unsigned char*>(tiles), np);
}

cudaError_t launch_attention_batch(const float* qkv, size_t qkv_stride, void* k_cache, void* v_cache,
                                   size_t cache_stride, const float* rope_cs, const int32_t* pos, void* tiles, int np,
                                   int rows, int n_heads, int n_kv, int head_dim, int ctx, float sqrt_hd,
                                   cudaStream_t stream) {
  if (head_dim != kAttnHd || n_heads <= 0 || n_kv <= 0 || n_heads % n_kv != 0 || ctx <= 0 || rows <= 0)
    return cudaErrorNotSupported;
  const size_t smem = attn_smem_bytes_fixed<kRowThreads>() + 16 + (size_t)ctx * sizeof(float);
  int dev = 0, optin = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (smem > (size_t)optin) return cudaErrorNotSupported;
  cudaError_t e = allow_smem(attention_batch_kernel, smem);
  if (e != cudaSuccess) return e;
  unsigned* err = device_error_word();
  if (!err) return cudaErrorUnknown;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = row_config((unsigned)n_heads, (unsigned)rows, kRowThreads, smem, stream, attr);
  return cudaLaunchKernelEx(&cfg, attention_batch_kernel, qkv, qkv_stride, static_cast<__half*>(k_cache),
                            static_cast<__half*>(v_cache), cache_stride, reinterpret_cast<const float2*>(rope_cs),
                            pos, static_cast<unsigned char*>(tiles), np, n_heads, n_kv, ctx, sqrt_hd, err);
}

cudaError_t launch_rows_argmax(const float* logits, int rows, int n, size_t stride, int offset, long long* keys,
                               cudaStream_t stream) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = row_config((unsigned)rows, 1, kRowThreads, 0, stream, attr);
  return cudaLaunchKernelEx(&cfg, rows_argmax_kernel, logits, n, stride, offset, keys);
}

cudaError_t launch_rows_advance(const long long* keys, int rows, int32_t* tokens, int max_tokens, int32_t* pos,
                                int n_prompt, cudaStream_t stream) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = row_config(1, 1, 256, 0, stream, attr);
  return cudaLaunchKernelEx(&cfg, rows_advance_kernel, keys, rows, tokens, max_tokens, pos, n_prompt);
}

}  // namespace asmllm

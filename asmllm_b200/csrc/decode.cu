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

#include "attention.cuh"
#include "common.cuh"
#include "matvec.cuh"

namespace asmllm {

namespace {

constexpr int kThreads = 256;  // 8 warps

struct CtaSync {
  __device__ __forceinline__ void operator()() const { __syncthreads(); }
};

__global__ void __launch_bounds__(kThreads) attention_decode_kernel(
    const float* __restrict__ qkv, __half* __restrict__ kc, __half* __restrict__ vc,
    const float2* __restrict__ rope_cs, const int32_t* __restrict__ pos_p, unsigned char* __restrict__ image,
    int n_heads, int n_kv, int ctx, float sqrt_hd, unsigned* __restrict__ err) {
  extern __shared__ __align__(16) unsigned char smem[];  // fixed scratch, then p [ctx]
  const AttnSmem sm = attn_smem_carve<kThreads>(smem);
  const int tid = threadIdx.x;
  const int h = blockIdx.x, j = h / (n_heads / n_kv);
  pdl_trigger();
  // Before the wait: bring this head's cached K/V rows towards L2.  They were
  // written steps ago; the position read here may be one step stale (the
  // previous step's last kernel may still be running), so it only bounds the
  // hint, clamped to the cache.  Every address stays inside the cache.
  {
    int hint = __ldcg(pos_p) + 1;
    hint = hint < 0 ? 0 : (hint > ctx ? ctx : hint);
    attn_prefetch_rows<kThreads>(kc, vc, hint, j, n_kv, tid);
  }
  pdl_wait();  // qkv comes from the previous kernel
  const int pos = __ldcg(pos_p);
  if (pos < 0 || pos >= ctx) {
    if (tid == 0) atomicOr(err, kErrDecodeRange);
    return;
  }
  attention_head<kThreads>(qkv, kc, vc, rope_cs, pos, h, n_heads, n_kv, sqrt_hd, image, sm, tid, CtaSync{});
}

}  // namespace

cudaError_t launch_attention_decode(const float* qkv, void* k_cache, void* v_cache, const float* rope_cs,
                                    const int32_t* pos, void* image, int n_heads, int n_kv, int head_dim, int ctx,
                                    float sqrt_hd, cudaStream_t stream, bool pdl) {
  if (head_dim != kAttnHd || n_heads <= 0 || n_kv <= 0 || n_heads % n_kv != 0 || ctx <= 0)
    return cudaErrorNotSupported;
  const size_t smem = attn_smem_bytes_fixed<kThreads>() + 16 + (size_t)ctx * sizeof(float);
  int dev = 0, optin = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (smem > (size_t)optin) return cudaErrorNotSupported;
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

// asmllm_b200/csrc/decode_persistent.cuh -- program of the persistent decode
// kernel (decode_persistent.cu): the operations of one decode step, in order.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

namespace asmllm {

constexpr int kOpMatvec = 0;
constexpr int kOpAttention = 1;

struct PersistOp {
  int kind = kOpMatvec;
  int pro = 0, epi = 0;       // matvec: kPro* / kEpi* of matvec.cuh
  int M = 0, nb = 0, R = 0;   // rows, 32-blocks per row, rows per ring stage (2, 4 or 8)
  int from_embed = 0;         // prologue source = embedding row of the step's token
  int first_of_step = 0;      // attention: the step's first (bookkeeping of the token)
  const uint8_t* w = nullptr;
  const __half* s = nullptr;
  const float* x = nullptr;             // prologue source (kProQuant / kProNorm)
  const unsigned char* image = nullptr; // prologue source (kProImage), replica 0
  size_t image_stride = 0;              // bytes between its replicas
  const float* norm_w = nullptr;
  float* y = nullptr;                   // kEpiStore / kEpiResidual / kEpiArgmax output
  __half* kc = nullptr;                 // attention: this layer's caches [ctx][n_kv][128]
  __half* vc = nullptr;
};

struct PersistArgs {
  const PersistOp* ops = nullptr;  // device array, n_ops per step
  int n_ops = 0;
  int n_steps = 0;
  float eps = 0.0f, sqrt_hd = 0.0f;
  const float* embed = nullptr;
  int vocab = 0;
  const float2* rope = nullptr;
  int ctx = 0, n_heads = 0, n_kv = 0;
  // Activations every CTA reads after a barrier (the residual stream x and
  // the two activation images) are kept in xr identical replicas, CTA b
  // reading replica b % xr: the same few cache lines read by every SM at once
  // would otherwise queue at a handful of L2 slices.
  int xr = 1;
  size_t x_stride = 0;         // floats between replicas of x
  size_t img_attn_stride = 0;  // bytes between replicas of img_attn
  size_t img_h_stride = 0;     // bytes between replicas of img_h
  float* x = nullptr;  // residual stream [xr][dim]
  float* qkv = nullptr;
  unsigned char* img_attn = nullptr;  // [xr][image bytes]
  float* h = nullptr;
  unsigned char* img_h = nullptr;  // [xr][image bytes]
  unsigned* counters = nullptr;
  unsigned long long* best = nullptr;  // [2], zero between runs
  int32_t* tokens = nullptr;
  int32_t* pos = nullptr;
  int max_tokens = 0, n_prompt = 0;
  unsigned* sync = nullptr;   // grid barrier counter, zero at launch
  unsigned* abort = nullptr;  // nonzero: some CTA gave up; zero at launch
  unsigned* err = nullptr;    // device error word
  int NS = 0, slot_bytes = 0, scratch_bytes = 0;
};

size_t persist_attn_scratch_bytes(int ctx);
bool persist_plan(PersistArgs& a, const std::vector<PersistOp>& ops, int fmt, int smem_optin, int* per_sm,
                  size_t* smem);
cudaError_t launch_decode_persistent(const PersistArgs& a, int fmt, size_t smem, int sms, int per_sm,
                                     cudaStream_t stream);

}  // namespace asmllm

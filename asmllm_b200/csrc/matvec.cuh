// asmllm_b200/csrc/matvec.cuh -- host-side interface of the matvec kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace asmllm {

// GGUF tensor type ids of the two weight formats.
constexpr int kFmtQ4_0 = 2;
constexpr int kFmtQ8_0 = 8;

struct MatvecArgs {
  int fmt = kFmtQ4_0;       // kFmtQ4_0 or kFmtQ8_0
  bool fp32_act = false;    // false: Q8_0 activations (NEON semantics); true: fp32 x (x86)
  bool scales_f16 = false;  // scale plane dtype
  const void* w = nullptr;  // device: Q4_0 [M][K/32][16] or Q8_0 [M][K/32][32]
  const void* scales = nullptr;
  const float* x = nullptr;
  float* y = nullptr;
  int32_t* isums = nullptr;  // optional: per-(row, block) int32 sums (Q8_0 activations only)
  int64_t M = 0, K = 0;
};

cudaError_t launch_matvec(const MatvecArgs& a, cudaStream_t stream);
cudaError_t launch_quantize(const float* x, int8_t* xq, float* xd, long long nblocks,
                            cudaStream_t stream);
cudaError_t launch_gguf_split(int fmt, const uint8_t* raw, uint8_t* qs, void* scales, int f16,
                              long long nblocks, cudaStream_t stream);
int64_t max_k(int fmt, bool fp32_act, int dev);

}  // namespace asmllm

// asmllm_b200/csrc/glue.cu -- the reference's decode-glue kernels on the GPU:
// RMSNorm, RoPE, softmax, single-head attention and SiLU * up, behind the
// reference's own entry points (asm_rmsnorm, asm_rope, asm_softmax,
// asm_attention, asm_silu_hadamard; THRISHAL12345/asmllm build_kernel.py:89-93,
// bound by src/runtime/generate.py:221-250 and tests/correctness/test_runner.py:376-467).
//
// Arithmetic follows the reference's numpy definitions (tests/reference/ops.py:
// 103-170, generate.py:370) operation by operation in fp32, without fused
// multiply-adds:
//   * every sum over a vector (mean(x^2) of RMSNorm, the softmax denominator)
//     is numpy's pairwise summation, restated below, so RMSNorm is bit-exact
//     against numpy;
//   * exp, sin, cos and pow are evaluated in double precision and rounded
//     once to fp32 -- the way the reference's x86 kernels use the x87 unit
//     (rope_avx2.asm:98, softmax_avx2.asm:75-87).  numpy's own fp32 SIMD
//     versions are not correctly rounded (they differ from the rounded
//     double value by one unit in the last place on a large share of inputs),
//     so RoPE, softmax and SiLU agree with numpy to about one ulp, as the
//     reference's kernels do;
//   * attention's dot products and P.V sums run in index order with fused
//     multiply-adds (numpy's matmul order is its BLAS's).
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "common.cuh"
#include "matvec.cuh"

namespace asmllm {

namespace {

constexpr int kGlueThreads = 256;
constexpr int kPwLeaf = 128;  // numpy PW_BLOCKSIZE

// numpy's pairwise summation of n values (numpy/_core/src/umath/loops_utils.h.src,
// pairwise_sum): n < 8 -> a running sum from 0; n <= 128 -> eight running
// sums over i = j mod 8, combined as ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)), then
// the n % 8 tail added in order; else the two halves at n2 = n/2 rounded down
// to a multiple of 8, summed recursively and added.  Checked against np.sum on
// fp32 vectors of every size class (tests/test_glue_gpu.py).

// Sum of one leaf (n <= 128) of values v(s) .. v(s + n - 1).
template <class V>
__device__ float pw_leaf(int s, int n, V v) {
  if (n < 8) {
    float r = 0.0f;
    for (int i = 0; i < n; ++i) r = __fadd_rn(r, v(s + i));
    return r;
  }
  float r[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) r[j] = v(s + j);
  int i = 8;
  for (; i < n - (n % 8); i += 8) {
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = __fadd_rn(r[j], v(s + i + j));
  }
  float res = __fadd_rn(__fadd_rn(__fadd_rn(r[0], r[1]), __fadd_rn(r[2], r[3])),
                        __fadd_rn(__fadd_rn(r[4], r[5]), __fadd_rn(r[6], r[7])));
  for (; i < n; ++i) res = __fadd_rn(res, v(s + i));
  return res;
}

// Leaves of the split tree of [0, n), left to right: starts and lengths.
// Returns the number of leaves (at most cap; the host sizes cap).
__device__ int pw_leaves(int n, int* start, int* len, int cap) {
  int st_s[40], st_n[40];
  int sp = 1, nl = 0;
  st_s[0] = 0;
  st_n[0] = n;
  while (sp > 0) {
    --sp;
    const int s = st_s[sp], m = st_n[sp];
    if (m <= kPwLeaf) {
      if (nl < cap) {
        start[nl] = s;
        len[nl] = m;
      }
      ++nl;
      continue;
    }
    int m2 = m / 2;
    m2 -= m2 % 8;
    st_s[sp] = s + m2;  // right half below the left so the left pops first
    st_n[sp] = m - m2;
    ++sp;
    st_s[sp] = s;
    st_n[sp] = m2;
    ++sp;
  }
  return nl;
}

// The tree's total from its leaf sums (post-order, left before right).
__device__ float pw_combine(int n, const float* leaf) {
  int fn[40], fs[40];
  float fl[40];
  int sp = 1, li = 0;
  float ret = 0.0f;
  fn[0] = n;
  fs[0] = 0;
  while (sp > 0) {
    const int t = sp - 1;
    const int m = fn[t];
    if (m <= kPwLeaf) {
      ret = leaf[li++];
      --sp;
      continue;
    }
    int m2 = m / 2;
    m2 -= m2 % 8;
    if (fs[t] == 0) {
      fs[t] = 1;
      fn[sp] = m2;
      fs[sp] = 0;
      ++sp;
    } else if (fs[t] == 1) {
      fl[t] = ret;
      fs[t] = 2;
      fn[sp] = m - m2;
      fs[sp] = 0;
      ++sp;
    } else {
      ret = __fadd_rn(fl[t], ret);
      --sp;
    }
  }
  return ret;
}

// Pairwise sum of v(0) .. v(n - 1) by the whole CTA: leaves in parallel, the
// tree by thread 0.  Shared scratch: 3 * cap words.  Every thread returns it.
template <class V>
__device__ float cta_pairwise_sum(int n, V v, int* s_start, int* s_len, float* s_leaf, int cap, float* s_out) {
  __shared__ int s_nl;
  if (threadIdx.x == 0) s_nl = pw_leaves(n, s_start, s_len, cap);
  __syncthreads();
  const int nl = s_nl;
  for (int i = threadIdx.x; i < nl; i += blockDim.x) s_leaf[i] = pw_leaf(s_start[i], s_len[i], v);
  __syncthreads();
  if (threadIdx.x == 0) *s_out = pw_combine(n, s_leaf);
  __syncthreads();
  return *s_out;
}

// NaN-propagating maximum (numpy.max returns NaN if any element is NaN).
__device__ __forceinline__ float nan_max(float a, float b) {
  return (a != a) ? a : ((b != b) ? b : fmaxf(a, b));
}

__device__ __forceinline__ float cta_max(float v, float* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = nan_max(v, __shfl_xor_sync(kFull, v, o));
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float m = red[0];
  for (int i = 1; i < (int)(blockDim.x >> 5); ++i) m = nan_max(m, red[i]);
  return m;
}

// fp32 exp, sin, cos, pow of fp32 arguments, each rounded once from double.
__device__ __forceinline__ float exp_r(float x) { return (float)exp((double)x); }

// ---------------------------------------------------------------- kernels

// y = (x / sqrt(mean(x^2) + eps)) * w  (ops.py:103-116).
__global__ void __launch_bounds__(kGlueThreads) rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                               float* __restrict__ y, int n, float eps, int cap) {
  extern __shared__ int glue_smem[];
  int* s_start = glue_smem;
  int* s_len = s_start + cap;
  float* s_leaf = reinterpret_cast<float*>(s_len + cap);
  __shared__ float s_sum;
  const float tot = cta_pairwise_sum(
      n, [&](int i) { const float t = x[i]; return __fmul_rn(t, t); }, s_start, s_len, s_leaf, cap, &s_sum);
  const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)n), eps));
  for (int i = threadIdx.x; i < n; i += blockDim.x) y[i] = __fmul_rn(__fdiv_rn(x[i], rms), w[i]);
}

// y = exp(x - max(x)) / sum(exp(x - max(x)))  (ops.py:144-153).
__device__ void softmax_row(const float* __restrict__ x, float* __restrict__ y, int n, int* s_start, int* s_len,
                            float* s_leaf, int cap, float* red, float* s_sum) {
  float m = -INFINITY;
  bool any_nan = false;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float t = x[i];
    any_nan |= t != t;
    m = nan_max(m, t);
  }
  if (any_nan) m = __int_as_float(0x7fc00000);
  m = cta_max(m, red);
  for (int i = threadIdx.x; i < n; i += blockDim.x) y[i] = exp_r(__fsub_rn(x[i], m));
  __syncthreads();
  const float tot = cta_pairwise_sum(n, [&](int i) { return y[i]; }, s_start, s_len, s_leaf, cap, s_sum);
  for (int i = threadIdx.x; i < n; i += blockDim.x) y[i] = __fdiv_rn(y[i], tot);
}

__global__ void __launch_bounds__(kGlueThreads) softmax_kernel(const float* __restrict__ x, float* __restrict__ y,
                                                               int n, int cap) {
  extern __shared__ int glue_smem[];
  __shared__ float red[kGlueThreads / 32];
  __shared__ float s_sum;
  softmax_row(x, y, n, glue_smem, glue_smem + cap, reinterpret_cast<float*>(glue_smem + 2 * cap), cap, red, &s_sum);
}

// RoPE on interleaved pairs (ops.py:119-141), q and k in place:
//   freq_i = 1 / theta^(2i / hd), angle = pos * freq_i,
//   (x0, x1) <- (x0 c - x1 s, x0 s + x1 c).
__global__ void rope_kernel(float* __restrict__ q, float* __restrict__ k, int hd, float pos_f, float theta) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= hd / 2) return;
  const float e = __fdiv_rn((float)(2 * i), (float)hd);
  const float p = (float)pow((double)theta, (double)e);
  const float f = __fdiv_rn(1.0f, p);
  const float ang = __fmul_rn(pos_f, f);
  const float c = (float)cos((double)ang), s = (float)sin((double)ang);
  float* vs[2] = {q, k};
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    float* v = vs[t];
    const float x0 = v[2 * i], x1 = v[2 * i + 1];
    v[2 * i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    v[2 * i + 1] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
  }
}

// gate <- (gate / (1 + exp(-gate))) * up  (generate.py:370; swiglu_avx2.asm:7-17).
__global__ void silu_hadamard_kernel(float* __restrict__ gate, const float* __restrict__ up, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float g = gate[i];
    gate[i] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, exp_r(-g))), up[i]);
  }
}

// One query row per CTA (attention_avx2.asm:59-200): scores[j] = (q_i . k_j) *
// scale for every key (no mask, as ops.py:156-170), softmax, y_i = p . V.
__global__ void __launch_bounds__(kGlueThreads) attention_kernel(const float* __restrict__ q,
                                                                 const float* __restrict__ k,
                                                                 const float* __restrict__ v, float* __restrict__ y,
                                                                 int seq, int hd, float scale, int cap) {
  extern __shared__ int glue_smem[];
  __shared__ float red[kGlueThreads / 32];
  __shared__ float s_sum;
  float* sc = reinterpret_cast<float*>(glue_smem + 3 * cap);  // [seq] scores, then probabilities
  float* pr = sc + seq;
  const int i = blockIdx.x;
  const float* qi = q + (size_t)i * hd;
  for (int j = threadIdx.x; j < seq; j += blockDim.x) {
    const float* kj = k + (size_t)j * hd;
    float d = 0.0f;
    for (int t = 0; t < hd; ++t) d = __fmaf_rn(qi[t], kj[t], d);
    sc[j] = __fmul_rn(d, scale);
  }
  __syncthreads();
  softmax_row(sc, pr, seq, glue_smem, glue_smem + cap, reinterpret_cast<float*>(glue_smem + 2 * cap), cap, red,
              &s_sum);
  __syncthreads();
  for (int t = threadIdx.x; t < hd; t += blockDim.x) {
    float a = 0.0f;
    for (int j = 0; j < seq; ++j) a = __fmaf_rn(pr[j], v[(size_t)j * hd + t], a);
    y[(size_t)i * hd + t] = a;
  }
}

// Leaves of numpy's split tree of n values (host copy of pw_leaves' count).
int pw_leaf_count(long long n) {
  if (n <= kPwLeaf) return 1;
  long long m2 = n / 2;
  m2 -= m2 % 8;
  return pw_leaf_count(m2) + pw_leaf_count(n - m2);
}

cudaError_t set_smem(const void* kernel, size_t bytes) {
  if (bytes <= 48 * 1024) return cudaSuccess;
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

}  // namespace

int64_t glue_max_len() { return 1 << 20; }

cudaError_t launch_rmsnorm(const float* x, const float* w, float* y, int64_t n, float eps, cudaStream_t stream) {
  if (n <= 0 || n > glue_max_len()) return cudaErrorInvalidValue;
  const int cap = pw_leaf_count(n);
  const size_t smem = (size_t)cap * 12;
  cudaError_t e = set_smem((const void*)rmsnorm_kernel, smem);
  if (e != cudaSuccess) return e;
  rmsnorm_kernel<<<1, kGlueThreads, smem, stream>>>(x, w, y, (int)n, eps, cap);
  return cudaGetLastError();
}

cudaError_t launch_softmax(const float* x, float* y, int64_t n, cudaStream_t stream) {
  if (n <= 0 || n > glue_max_len()) return cudaErrorInvalidValue;
  const int cap = pw_leaf_count(n);
  const size_t smem = (size_t)cap * 12;
  cudaError_t e = set_smem((const void*)softmax_kernel, smem);
  if (e != cudaSuccess) return e;
  softmax_kernel<<<1, kGlueThreads, smem, stream>>>(x, y, (int)n, cap);
  return cudaGetLastError();
}

cudaError_t launch_rope(float* q, float* k, int64_t hd, int64_t pos, float theta, cudaStream_t stream) {
  if (hd <= 0 || hd % 2 || hd > glue_max_len()) return cudaErrorInvalidValue;
  const int half = (int)(hd / 2);
  const int threads = 128;
  rope_kernel<<<(half + threads - 1) / threads, threads, 0, stream>>>(q, k, (int)hd, (float)pos, theta);
  return cudaGetLastError();
}

cudaError_t launch_silu_hadamard(float* gate, const float* up, int64_t n, cudaStream_t stream) {
  if (n <= 0) return cudaErrorInvalidValue;
  long long blocks = (n + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  silu_hadamard_kernel<<<(unsigned)blocks, 256, 0, stream>>>(gate, up, (long long)n);
  return cudaGetLastError();
}

size_t attention_smem(int64_t seq) { return (size_t)pw_leaf_count(seq) * 12 + (size_t)seq * 8; }

cudaError_t launch_attention(const float* q, const float* k, const float* v, float* y, int64_t seq, int64_t hd,
                             float scale, cudaStream_t stream) {
  if (seq <= 0 || hd <= 0 || seq > 0x7fffffffLL || hd > 0x7fffffffLL) return cudaErrorInvalidValue;
  int dev = 0, optin = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  const size_t smem = attention_smem(seq);
  if (smem > (size_t)optin) return cudaErrorNotSupported;
  cudaError_t e = set_smem((const void*)attention_kernel, smem);
  if (e != cudaSuccess) return e;
  const int cap = pw_leaf_count(seq);
  attention_kernel<<<(unsigned)seq, kGlueThreads, smem, stream>>>(q, k, v, y, (int)seq, (int)hd, scale, cap);
  return cudaGetLastError();
}

}  // namespace asmllm

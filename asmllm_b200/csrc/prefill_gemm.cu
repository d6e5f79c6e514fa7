// asmllm_b200/csrc/prefill_gemm.cu -- batched (prefill) Q4_0/Q8_0 x Q8_0
// matrix product on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// Y[n][m] = sum_b (wd[m][b] * xd[n][b]) * isum_b[m][n],
// isum_b[m][n] = sum_{i<32} w[m][32b+i] * xq[n][32b+i]   (int32, exact)
// for N activation rows already quantized to Q8_0 (the activation image of
// asm_act_image_q8_0_async, one row per token).  Per row and token this is
// exactly the reference's NEON combine (THRISHAL12345/asmllm
// src/kernels/arm64/matmul_q4_neon.S:239-255): s = wd * xd (fp32 multiply),
// acc = fma(float(isum), s, acc), blocks in order -- so every output equals
// the single-token Q4_0 x Q8_0 result of the reference semantics bit for bit.
//
// The per-32-block scales differ for every (row, token, block), so they
// cannot live inside the MMA: each block is one tcgen05.mma (kind::i8, M=128
// rows, N=64 tokens, K=32) into a fresh int32 accumulator in tensor memory,
// and the 128 epilogue threads (one per row) read it back (tcgen05.ld) and
// apply the scales in fp32.  Two accumulators alternate so the tensor core
// works on block b+2 while the threads scale block b.  Q4_0 weights are
// expanded to int8 (nibble - 8) in shared memory (the "in-SMEM dequantised
// tiles"); activations are copied as they are.
//
// Pipelining: chunks of kKB blocks are staged into two shared-memory buffers;
// while the tensor core and the epilogue work on chunk c, every thread holds
// its global loads for chunk c+1 in registers and stores them (expanding the
// nibbles) into the other buffer afterwards.  The epilogue uses the packed
// fp32x2 multiply and fma (two IEEE fp32 operations per instruction, the
// same rounding as the scalar ones).
//
// Shared-memory operand layout (no swizzle, K-major "core matrices" of 8
// rows x 16 bytes): element (row, k) of block b at
//   b * tile + (row / 8) * 256 + (k / 16) * 128 + (row % 8) * 16 + k % 16
// so the descriptor's leading byte offset (between the two 16-byte K halves)
// is 128 and its stride byte offset (between 8-row groups) is 256.
//
// Waits are bounded (the mbarrier of each MMA commit); on timeout the kernel
// sets bit 0 of the device error word and stops issuing, then releases its
// tensor memory.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "matvec.cuh"
#include "pipeline.cuh"

namespace asmllm {

namespace {

constexpr int kGM = 128;       // rows per CTA (MMA M)
constexpr int kGN = 64;        // tokens per CTA (MMA N)
constexpr int kKB = 8;         // 32-blocks per staged chunk
constexpr int kGThreads = 128;  // 4 warps: one row each thread
constexpr int kTmemCols = 2 * kGN;  // two int32 accumulators of kGN columns
constexpr int kATile = kGM * 32;    // bytes of one block of A (int8)
constexpr int kBTile = kGN * 32;    // bytes of one block of B

__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
  // start address >> 4 | LBO 128 B >> 4 | SBO 256 B >> 4 | version 1 (sm_100) | no swizzle
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(256 >> 4) << 32) |
         ((uint64_t)1 << 46);
}

// kind::i8: D s32 (c_format 2), A and B signed 8-bit, both K-major, N, M.
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kGN >> 3) << 17) |
                            ((uint32_t)(kGM >> 4) << 24);

__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 64 consecutive int32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,"
      "%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Expands 16 bytes of Q4_0 nibbles into the block's 32 int8 weights (nibble - 8):
// lo = elements 0..15 (low nibbles), hi = elements 16..31 (high nibbles).
__device__ __forceinline__ void q4_to_i8(uint4 q, uint4& lo, uint4& hi) {
  auto ex = [](unsigned w, unsigned& l, unsigned& h) {  // per-byte n - 8, wrapping: the int8 value
    l = __vsub4(w & 0x0F0F0F0Fu, 0x08080808u);
    h = __vsub4((w >> 4) & 0x0F0F0F0Fu, 0x08080808u);
  };
  ex(q.x, lo.x, hi.x);
  ex(q.y, lo.y, hi.y);
  ex(q.z, lo.z, hi.z);
  ex(q.w, lo.w, hi.w);
}

__device__ __forceinline__ unsigned long long pack2(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}

__device__ __forceinline__ void unpack2(unsigned long long v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}

// acc += float(d) * (wd * xd) for two tokens at once, each element rounded as
// the scalar fmul / fma.
__device__ __forceinline__ unsigned long long scale_acc2(unsigned long long acc, int d0, int d1, float wd,
                                                         unsigned long long xd2) {
  unsigned long long s, dv, r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(s) : "l"(pack2(wd, wd)), "l"(xd2));
  dv = pack2(__int2float_rn(d0), __int2float_rn(d1));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(dv), "l"(s), "l"(acc));
  return r;
}

// Staging registers of one chunk for one thread: its row's kKB weight blocks
// (and scales) and its share of the activation blocks.
struct ChunkRegs {
  uint4 a[kKB][2];
  float wd[kKB];
  uint4 bv[kKB * kGN * 2 / kGThreads];
  float bxd[kKB * kGN * 2 / kGThreads];
};

template <int FMT>
__device__ __forceinline__ void load_chunk(ChunkRegs& R, const uint8_t* __restrict__ w,
                                           const __half* __restrict__ scales, const unsigned char* __restrict__ images,
                                           size_t img_stride, int row, int M, int N, int nb, int n0, int c0, int kb,
                                           int tid) {
  constexpr int UB = FMT == kFmtQ4_0 ? 16 : 32;
#pragma unroll
  for (int b = 0; b < kKB; ++b) {
    R.a[b][0] = R.a[b][1] = make_uint4(0u, 0u, 0u, 0u);
    R.wd[b] = 0.0f;
    if (b < kb && row < M) {
      const uint8_t* src = w + ((size_t)row * nb + c0 + b) * UB;
      R.a[b][0] = *reinterpret_cast<const uint4*>(src);
      if (FMT != kFmtQ4_0) R.a[b][1] = *reinterpret_cast<const uint4*>(src + 16);
      R.wd[b] = __half2float(scales[(size_t)row * nb + c0 + b]);
    }
  }
#pragma unroll
  for (int j = 0; j < kKB * kGN * 2 / kGThreads; ++j) {
    const int i = tid + j * kGThreads;
    const int half = i & 1, tb = i >> 1, n = tb % kGN, b = tb / kGN;
    R.bv[j] = make_uint4(0u, 0u, 0u, 0u);
    R.bxd[j] = 0.0f;
    if (b < kb && n0 + n < N) {
      const unsigned char* im = images + (size_t)(n0 + n) * img_stride;
      R.bv[j] = __ldcg(reinterpret_cast<const uint4*>(im + (size_t)(c0 + b) * 48) + half);
      if (half == 0) R.bxd[j] = __ldcg(reinterpret_cast<const float2*>(im + (size_t)nb * 48) + c0 + b).x;
    }
  }
}

template <int FMT>
__device__ __forceinline__ void store_chunk(const ChunkRegs& R, unsigned char* sA, unsigned char* sB, float* sWd,
                                            float* sXd, int tid) {
  const int g = tid >> 3, r = tid & 7;
#pragma unroll
  for (int b = 0; b < kKB; ++b) {
    uint4 lo = R.a[b][0], hi = R.a[b][1];
    if (FMT == kFmtQ4_0) q4_to_i8(R.a[b][0], lo, hi);
    unsigned char* t = sA + b * kATile + g * 256 + r * 16;
    *reinterpret_cast<uint4*>(t) = lo;
    *reinterpret_cast<uint4*>(t + 128) = hi;
    sWd[b * kGM + tid] = R.wd[b];
  }
#pragma unroll
  for (int j = 0; j < kKB * kGN * 2 / kGThreads; ++j) {
    const int i = tid + j * kGThreads;
    const int half = i & 1, tb = i >> 1, n = tb % kGN, b = tb / kGN;
    *reinterpret_cast<uint4*>(sB + b * kBTile + (n >> 3) * 256 + half * 128 + (n & 7) * 16) = R.bv[j];
    if (half == 0) sXd[b * kGN + n] = R.bxd[j];
  }
}

template <int FMT>
__global__ void __launch_bounds__(kGThreads, 1)
q8act_gemm_kernel(const uint8_t* __restrict__ w, const __half* __restrict__ scales,
                  const unsigned char* __restrict__ images, size_t img_stride, float* __restrict__ y, int M,
                  int N, int nb, unsigned* __restrict__ err) {
  extern __shared__ __align__(1024) unsigned char smem[];
  constexpr size_t kBuf = (size_t)kKB * (kATile + kBTile) + (size_t)kKB * (kGM + kGN) * sizeof(float);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(smem + 2 * kBuf);  // [2]
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(mbar + 2);
  auto bufA = [&](int s) { return smem + s * kBuf; };
  auto bufB = [&](int s) { return smem + s * kBuf + kKB * kATile; };
  auto bufWd = [&](int s) { return reinterpret_cast<float*>(smem + s * kBuf + kKB * (kATile + kBTile)); };
  auto bufXd = [&](int s) { return bufWd(s) + kKB * kGM; };

  const int tid = threadIdx.x, warp = tid >> 5;
  const int m0 = blockIdx.x * kGM, n0 = blockIdx.y * kGN;
  const int row = m0 + tid;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(s_tmem)),
                 "r"((uint32_t)kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    mbar_init(smem_u32(&mbar[0]), 1);
    mbar_init(smem_u32(&mbar[1]), 1);
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  pdl_trigger();
  pdl_wait();  // the activation images may come from the previous kernel

  unsigned long long acc[kGN / 2];  // token pairs
#pragma unroll
  for (int n = 0; n < kGN / 2; ++n) acc[n] = 0ull;  // (+0.0f, +0.0f)
  uint32_t phase[2] = {0u, 0u};
  bool ok = true;
  const int nchunks = (nb + kKB - 1) / kKB;

  ChunkRegs R;
  load_chunk<FMT>(R, w, scales, images, img_stride, row, M, N, nb, n0, 0, min(kKB, nb), tid);
  store_chunk<FMT>(R, bufA(0), bufB(0), bufWd(0), bufXd(0), tid);
  fence_proxy_async();  // the generic-proxy writes become visible to the tensor core
  __syncthreads();

  for (int c = 0; c < nchunks && ok; ++c) {
    const int sb = c & 1, c0 = c * kKB, kb = min(kKB, nb - c0);
    unsigned char* sA = bufA(sb);
    unsigned char* sB = bufB(sb);
    const float* sWd = bufWd(sb);
    const float* sXd = bufXd(sb);
    auto issue = [&](int b) {
      if (tid == 0) {
        tc_fence_after();
        umma_i8(tmem + (uint32_t)((b & 1) * kGN), umma_desc(smem_u32(sA + b * kATile)),
                umma_desc(smem_u32(sB + b * kBTile)));
        umma_commit(smem_u32(&mbar[b & 1]));
      }
    };
    issue(0);
    if (kb > 1) issue(1);
    const bool more = c + 1 < nchunks;
    if (more)  // next chunk's loads in flight during this chunk's blocks
      load_chunk<FMT>(R, w, scales, images, img_stride, row, M, N, nb, n0, c0 + kKB, min(kKB, nb - c0 - kKB), tid);
    for (int b = 0; b < kb; ++b) {
      const int buf = b & 1;
      const bool done = mbar_wait_bounded(smem_u32(&mbar[buf]), phase[buf]);
      phase[buf] ^= 1u;
      if (__syncthreads_or(!done)) {  // one decision for the CTA
        if (tid == 0) atomicOr(err, kErrRingTimeout);
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t d[kGN];
      tmem_ld64(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(buf * kGN), d);
      const float wd = sWd[b * kGM + tid];
      const unsigned long long* xd2 = reinterpret_cast<const unsigned long long*>(sXd + b * kGN);
#pragma unroll
      for (int n = 0; n < kGN / 2; ++n) acc[n] = scale_acc2(acc[n], (int)d[2 * n], (int)d[2 * n + 1], wd, xd2[n]);
      tc_fence_before();
      __syncthreads();  // every thread has read accumulator buf: it may be overwritten
      if (b + 2 < kb) issue(b + 2);
    }
    if (more && ok) {  // chunk c-1's buffer is free (its MMAs completed): fill it with chunk c+1
      store_chunk<FMT>(R, bufA(sb ^ 1), bufB(sb ^ 1), bufWd(sb ^ 1), bufXd(sb ^ 1), tid);
      fence_proxy_async();
    }
    __syncthreads();
  }

  if (row < M) {
#pragma unroll
    for (int n = 0; n < kGN / 2; ++n) {
      float a0, a1;
      unpack2(acc[n], a0, a1);
      if (n0 + 2 * n < N) y[(size_t)(n0 + 2 * n) * M + row] = a0;
      if (n0 + 2 * n + 1 < N) y[(size_t)(n0 + 2 * n + 1) * M + row] = a1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)kTmemCols)
                 : "memory");
}

}  // namespace

size_t gemm_smem_bytes() {
  return 2 * ((size_t)kKB * (kATile + kBTile) + (size_t)kKB * (kGM + kGN) * sizeof(float)) + 2 * sizeof(uint64_t) + 16;
}

cudaError_t launch_q8act_gemm(int fmt, const void* w, const void* scales_f16, const void* images, size_t img_stride,
                              float* y, int64_t M, int64_t N, int64_t K, cudaStream_t stream) {
  const int nb = (int)(K / QK);
  const size_t smem = gemm_smem_bytes();
  auto kernel = fmt == kFmtQ4_0 ? q8act_gemm_kernel<kFmtQ4_0> : q8act_gemm_kernel<kFmtQ8_0>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((M + kGM - 1) / kGM), (unsigned)((N + kGN - 1) / kGN));
  cfg.blockDim = dim3(kGThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_opt_pdl.load() ? 1 : 0;
  const uint8_t* wp = static_cast<const uint8_t*>(w);
  const __half* sp = static_cast<const __half*>(scales_f16);
  const unsigned char* ip = static_cast<const unsigned char*>(images);
  int Mi = (int)M, Ni = (int)N;
  unsigned* err = device_error_word();
  if (!err) return cudaErrorUnknown;
  return cudaLaunchKernelEx(&cfg, kernel, wp, sp, ip, img_stride, y, Mi, Ni, nb, err);
}

}  // namespace asmllm

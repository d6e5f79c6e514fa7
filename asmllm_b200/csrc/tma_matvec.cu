// asmllm_b200/csrc/tma_matvec.cu -- Q4_0/Q8_0 x Q8_0 matvec streamed by the
// bulk-copy (TMA) engine through shared-memory rings (sm_100a).
//
// Same semantics as q8act_matvec_kernel in matvec.cu (reference
// THRISHAL12345/asmllm src/kernels/arm64/matmul_q4_neon.S:38-317): the
// activation is quantized to Q8_0 bit-exactly, each (row, block) int32 dot is
// exact, and y[r] = sum_b fma(float(isum), wd*xd) differs from the reference
// only in fp32 summation order.
//
// Structure (one CTA per SM, 8 warps, at most ~110 KB of shared memory):
//   * The matrix is cut into row groups of RS consecutive rows; a stage is
//     RS rows x one chunk of their blocks (the whole row unless a row is too
//     long for the ring), i.e. one bulk copy per plane when whole rows, else
//     one per row and plane.  CTA c takes groups c, c + grid, ... (all CTAs
//     stream one contiguous span at a time), or one contiguous range for the
//     epilogues that need it (SwiGLU pairs, the tensor-parallel exchange).
//   * Every warp streams its own ring of NSW slots: lane 0 issues its next
//     stages' copies (cp.async.bulk, completion on the slot's mbarrier), the
//     warp consumes a slot and lane 0 refills it with the stage NSW ahead.
//     There is no producer warp and no barrier between warps in the stage
//     loop.  Weights the caller declared static are requested before
//     griddepcontrol.wait, so under programmatic dependent launch a matvec's
//     rings fill while the previous kernel still runs; at ~110 KB per CTA the
//     next launch's CTA fits beside this one on every SM.
//   * The CTA builds the Q8_0 activation image in shared memory (quantizing
//     x, 8 lanes per block, or copying a prepared image).  For rows of at
//     most 128 blocks each lane then keeps its blocks (lane + 32 j) in
//     registers; longer rows read them from shared memory once per stage for
//     all RS rows.  Lane partials are reduced across the warp in a fixed
//     order, so y is deterministic.
//   * Every mbarrier wait is bounded (about a second of clock cycles); on
//     timeout the kernel sets bit 0 of g_device_error, lets the copies it
//     issued land, and returns.
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"
#include "matvec.cuh"
#include "pipeline.cuh"

namespace asmllm {

__device__ unsigned int g_device_error;
// Optional mapped pinned host word that also receives the error bits (set by
// the synchronous entries: they test it after their stream synchronize
// instead of copying g_device_error back).  A plain store: concurrent
// reporters may overwrite each other's bits there, g_device_error keeps them all.
__device__ unsigned int* g_error_mirror;

__device__ __forceinline__ void raise_device_error(unsigned bits) {
  atomicOr(&g_device_error, bits);
  unsigned int* m = g_error_mirror;
  if (m) *reinterpret_cast<volatile unsigned int*>(m) = bits;
}

namespace {

constexpr int kNcw = 8;          // warps per CTA, each streaming its own ring
constexpr int kMaxNsw = 6;       // ring slots per warp (cap)
constexpr int kBarBytes = 512;   // kNcw x kMaxNsw full mbarriers
constexpr int kPartBytes = 256;  // per-warp partials (RMSNorm sums, argmax keys)
static_assert(kNcw * kMaxNsw * 8 <= kBarBytes, "barrier area");

}  // namespace

// Tuning of the bulk-copy matvec (asm_set_option "mv_rows", "mv_slots",
// "mv_smem_kb", "mv_ctas"): 0 = automatic.
std::atomic<int> g_opt_mv_rows{0};
std::atomic<int> g_opt_mv_slots{0};
std::atomic<int> g_opt_mv_smem_kb{110};
std::atomic<int> g_opt_mv_ctas{1};


// ---- tensor-parallel exchange words: (sequence << 32) | payload bits ------
__device__ __forceinline__ void st_volatile_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_volatile_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// The payload of the exchange word at p once it carries sequence seq; bounded
// (a peer that never writes sets the error bit and yields 0; after one
// timeout, `ok` makes the caller's later waits return at once).
__device__ __forceinline__ unsigned xchg_wait(const unsigned long long* p, unsigned seq, bool& ok) {
  unsigned long long v = ld_volatile_u64(p);
  if ((unsigned)(v >> 32) == seq) return (unsigned)v;
  if (!ok) return 0u;
  const long long t0 = clock64();
  do {
    v = ld_volatile_u64(p);
    if (clock64() - t0 > kWaitCycles) {
      ok = false;
      raise_device_error(kErrXchgTimeout);
      return 0u;
    }
  } while ((unsigned)(v >> 32) != seq);
  return (unsigned)v;
}

// Word of (parity, source rank, row) in the exchange buffer `buf`.
__device__ __forceinline__ unsigned long long* xchg_word(const MvFuse& fz, unsigned long long* buf, unsigned seq,
                                                         int src, int row) {
  return buf + ((size_t)(seq & 1u) * fz.tp + src) * fz.xchg_rows + row;
}

// Called once per CTA (thread 0) after its rows' keys are folded into
// fz.best: the last CTA to arrive turns the maximum into the next token,
// advances the position and leaves best / done zero for the next launch.
// With tensor parallelism the ranks' maxima are exchanged first (keys carry
// global rows, so every rank picks the same token).
__device__ void argmax_arrive(const MvFuse& fz, unsigned nctas, unsigned seq) {
  __threadfence();
  if (atomicAdd(fz.done, 1u) != nctas - 1) return;
  __threadfence();
  unsigned long long b = atomicExch(fz.best, 0ull);
  if (fz.tp > 1) {
    const unsigned long long tag = (unsigned long long)seq << 32;
    for (int r = 0; r < fz.tp; ++r) {
      st_volatile_u64(xchg_word(fz, fz.xchg[r], seq, fz.tp_rank, 0), tag | (b >> 32));
      st_volatile_u64(xchg_word(fz, fz.xchg[r], seq, fz.tp_rank, 1), tag | (b & 0xFFFFFFFFull));
    }
    bool ok = true;
    unsigned long long m = 0;
    for (int r = 0; r < fz.tp; ++r) {
      const unsigned long long hi = xchg_wait(xchg_word(fz, fz.xchg[fz.tp_rank], seq, r, 0), seq, ok);
      const unsigned long long lo = xchg_wait(xchg_word(fz, fz.xchg[fz.tp_rank], seq, r, 1), seq, ok);
      const unsigned long long k = (hi << 32) | lo;
      m = k > m ? k : m;
    }
    b = m;
    *fz.ar_seq = seq;
  }
  const int idx = argmax_row(b);
  volatile int32_t* pos = fz.pos;
  const int p = *pos;
  if (p >= 0 && p + 1 < fz.max_tokens) {
    if (p + 1 >= fz.n_prompt) fz.tokens[p + 1] = idx;  // prompt positions keep their ids
  } else {
    raise_device_error(kErrDecodeRange);
  }
  *pos = p + 1;
  atomicExch(fz.done, 0u);
}

// Source row of a quantizing prologue: x, or the embedding row of the token
// at the current position (out-of-range ids read row 0 and set an error bit).
__device__ __forceinline__ const float* prologue_source(const MvFuse& fz, const void* act, int K) {
  if (fz.embed == nullptr) return static_cast<const float*>(act);
  const int p = __ldcg(fz.pos);
  int tok = (p >= 0 && p < fz.max_tokens) ? __ldcg(fz.tokens + p) : -1;
  if (tok < 0 || tok >= fz.vocab) {
    if (threadIdx.x == 0) raise_device_error(kErrDecodeRange);
    tok = 0;
  }
  return fz.embed + (size_t)tok * K;
}

// Rows of a stage reduced across the warp: acc[r] is this lane's partial of
// row r.  log2(RS) halving steps leave each lane one row's partial (lanes
// whose bit o is set keep the upper half of the rows), then the remaining
// offsets sum within groups of 32/RS lanes.  Lane l ends with the total of
// row l / (32/RS) when l % (32/RS) == 0.  The order of the additions is
// fixed, so the result is the same every run.
template <int RS>
__device__ __forceinline__ float rows_reduce(const float (&acc)[RS], int lane) {
  float v[RS];
#pragma unroll
  for (int i = 0; i < RS; ++i) v[i] = acc[i];
#pragma unroll
  for (int n = RS, o = 16; n > 1; n >>= 1, o >>= 1) {
    const bool up = lane & o;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float keep = up ? v[n / 2 + i] : v[i];
      const float give = up ? v[i] : v[n / 2 + i];
      v[i] = keep + __shfl_xor_sync(kFull, give, o);
    }
  }
#pragma unroll
  for (int o = 16 / RS; o > 0; o >>= 1) v[0] += __shfl_xor_sync(kFull, v[0], o);
  return v[0];
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Q4_0 block dot of 16 nibble bytes q with the block's 32 int8 activations
// (xa = elements 0..15, xb = 16..31): sum (n - 8) * x, exact.  Byte j holds
// element j in its low nibble and element 16 + j in its high nibble;
// dp4a(q & 0xF0.., xb) is 16x the high-nibble sum, and qsum8 = 8 * sum(x).
__device__ __forceinline__ int q4_block_dot(const uint4 q, const uint4 xa, const uint4 xb, int qsum8) {
  int lo = 0, hi = 0;
  lo = dp4a_us(q.x & 0x0F0F0F0Fu, (int)xa.x, lo);
  hi = dp4a_us(q.x & 0xF0F0F0F0u, (int)xb.x, hi);
  lo = dp4a_us(q.y & 0x0F0F0F0Fu, (int)xa.y, lo);
  hi = dp4a_us(q.y & 0xF0F0F0F0u, (int)xb.y, hi);
  lo = dp4a_us(q.z & 0x0F0F0F0Fu, (int)xa.z, lo);
  hi = dp4a_us(q.z & 0xF0F0F0F0u, (int)xb.z, hi);
  lo = dp4a_us(q.w & 0x0F0F0F0Fu, (int)xa.w, lo);
  hi = dp4a_us(q.w & 0xF0F0F0F0u, (int)xb.w, hi);
  return lo + (hi >> 4) - qsum8;
}

// Q8_0 block dot of 32 int8 weights (q0 = 0..15, q1 = 16..31) with the
// block's int8 activations.
__device__ __forceinline__ int q8_block_dot(const uint4 q0, const uint4 q1, const uint4 xa, const uint4 xb) {
  int p = 0, t = 0;
  p = dp4a_ss((int)q0.x, (int)xa.x, p);
  t = dp4a_ss((int)q1.x, (int)xb.x, t);
  p = dp4a_ss((int)q0.y, (int)xa.y, p);
  t = dp4a_ss((int)q1.y, (int)xb.y, t);
  p = dp4a_ss((int)q0.z, (int)xa.z, p);
  t = dp4a_ss((int)q1.z, (int)xb.z, t);
  p = dp4a_ss((int)q0.w, (int)xa.w, p);
  t = dp4a_ss((int)q1.w, (int)xb.w, t);
  return p + t;
}

template <bool F16S>
__device__ __forceinline__ float smem_scale(const unsigned char* p) {
  if (F16S) return __half2float(*reinterpret_cast<const __half*>(p));
  return *reinterpret_cast<const float*>(p);
}

// One launch's work split (host-computed, see tma_plan).
struct MvShape {
  int M, nb;
  int C, cb;       // chunks per row and blocks per chunk (the last chunk may be shorter)
  int NSW;         // ring slots per consumer warp
  int slot_bytes;  // RS rows x cb blocks of weights, then their scales
  int flags;       // kMvPre | kMvIndep
};
constexpr int kMvPre = 1;    // weights static: issue copies before the grid-dependency wait
constexpr int kMvIndep = 2;  // x and y independent of the previous kernel: no wait before the prologue

// Bytes of the activation image as the kernel keeps it in shared memory:
// x32 [nb][32] int8 values, then dq [nb] (d fp32, q-sum int32), rounded to 128.
__host__ __device__ inline size_t smem_image_bytes(int64_t nb) { return ((size_t)nb * 40 + 127) & ~(size_t)127; }

template <int FMT, bool F16S, bool DBG, int PRO, int EPI, int RS, int XR, int P>
__global__ void __launch_bounds__(kNcw * 32, 2)
tma_matvec_kernel(const uint8_t* __restrict__ w, const void* __restrict__ scales, const void* __restrict__ act,
                  float* __restrict__ y, int32_t* __restrict__ isums, const MvShape sh, const MvFuse fz) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int UB = FMT == kFmtQ4_0 ? 16 : 32;  // weight bytes per block
  constexpr int SS = F16S ? 2 : 4;               // scale bytes per block
  constexpr int NCT = kNcw * 32;
  static_assert(EPI != kEpiSwiglu || RS % 2 == 0, "SwiGLU pairs need an even number of rows per stage");
  const int M = sh.M, nb = sh.nb, C = sh.C, cb = sh.cb, NSW = sh.NSW;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);  // full[warp][slot]
  float* part = reinterpret_cast<float*>(smem + kBarBytes);
  unsigned char* x32 = smem + kBarBytes + kPartBytes;
  const float2* sdq = reinterpret_cast<const float2*>(x32 + (size_t)nb * 32);
  unsigned char* ring = x32 + smem_image_bytes(nb);
  const size_t row_w = (size_t)nb * UB, row_s = (size_t)nb * SS;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Row groups of RS rows.  Epilogues whose rows are independent (store,
  // argmax, the one-GPU residual add) take groups grid-strided: group q of
  // this CTA = group q * grid + cta, so at any moment the CTAs stream one
  // contiguous span.  SwiGLU (pairs and per-CTA block counters) and the
  // tensor-parallel residual exchange take one contiguous range per CTA.
  const int n_g = (M + RS - 1) / RS;
  const int G = (int)gridDim.x, cta = (int)blockIdx.x;
  const bool stride = EPI == kEpiStore || EPI == kEpiArgmax || (EPI == kEpiResidual && fz.tp <= 1);
  const int g0 = (int)((long long)n_g * cta / G), g1 = (int)((long long)n_g * (cta + 1) / G);
  const int nq = stride ? (cta < n_g ? (n_g - 1 - cta) / G + 1 : 0) : g1 - g0;
  const int r0 = g0 * RS, r1 = min(M, g1 * RS);  // the contiguous range (SwiGLU, exchange)
  auto group_of = [&](int q) { return stride ? cta + q * G : g0 + q; };
  const bool pre = (sh.flags & kMvPre) != 0, indep = (sh.flags & kMvIndep) != 0;

  pdl_trigger();
  if (nq == 0) {
    if ((EPI == kEpiArgmax || (EPI == kEpiResidual && fz.tp > 1)) && threadIdx.x == 0) {
      pdl_wait();
      const unsigned seq0 = fz.tp > 1 ? __ldcg(fz.ar_seq) + 1u : 0u;
      if (EPI == kEpiArgmax) {
        argmax_arrive(fz, gridDim.x, seq0);
      } else if (atomicAdd(fz.ar_done, 1u) == gridDim.x - 1) {
        *fz.ar_seq = seq0;
        atomicExch(fz.ar_done, 0u);
      }
    }
    if (indep && threadIdx.x == 0) pdl_wait();
    return;
  }

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNcw * NSW; ++i) mbar_init(smem_u32(&bars[i]), 1);
    fence_mbar_init();
  }
  __syncthreads();

  // This warp's stages: its groups q = warp, warp + kNcw, ..., C chunk stages
  // each, in ring slots warp * NSW + k % NSW.  The warp streams its own ring:
  // lane 0 issues a stage's bulk copies (one per row and plane, or one per
  // plane when a stage is whole rows), the warp consumes it, and lane 0 then
  // reuses the slot for stage k + NSW.  No warp waits for another.
  const int nqw = warp < nq ? (nq - 1 - warp) / kNcw + 1 : 0;
  const int nk = nqw * C;
  auto issue = [&](int k) {
    const int m = k / C, c = k - m * C;
    const int row0 = group_of(warp + m * kNcw) * RS, nrows = min(RS, M - row0);
    const int cbn = min(cb, nb - c * cb);
    const int slot = warp * NSW + k % NSW;
    const uint32_t full = smem_u32(&bars[slot]);
    const uint32_t sw = smem_u32(ring + (size_t)slot * sh.slot_bytes);
    const uint32_t ss = sw + (uint32_t)(RS * cb * UB);
    const unsigned char* gs = static_cast<const unsigned char*>(scales);
    mbar_arrive_expect_tx(full, (uint32_t)(nrows * cbn * (UB + SS)));
    if (C == 1) {
      bulk_g2s(sw, w + (size_t)row0 * row_w, (uint32_t)(nrows * row_w), full);
      bulk_g2s(ss, gs + (size_t)row0 * row_s, (uint32_t)(nrows * row_s), full);
    } else {
      for (int r = 0; r < nrows; ++r) {
        bulk_g2s(sw + (uint32_t)(r * cb * UB), w + (size_t)(row0 + r) * row_w + (size_t)c * cb * UB,
                 (uint32_t)(cbn * UB), full);
        bulk_g2s(ss + (uint32_t)(r * cb * SS), gs + (size_t)(row0 + r) * row_s + (size_t)c * cb * SS,
                 (uint32_t)(cbn * SS), full);
      }
    }
  };
  const int n_first = min(NSW, nk);
  // Weights do not depend on the previous kernel when the caller declared
  // them static: under programmatic dependent launch the rings fill while the
  // previous kernel still runs.
  if (pre && lane == 0)
    for (int k = 0; k < n_first; ++k) issue(k);
  if (!indep) pdl_wait();  // x / the image may come from the previous kernel; y may still be in use
  if (!pre && lane == 0)
    for (int k = 0; k < n_first; ++k) issue(k);

  // Tensor-parallel call number (the previous exchange's last CTA stored it).
  const unsigned seq = (fz.tp > 1 && (EPI == kEpiResidual || EPI == kEpiArgmax)) ? __ldcg(fz.ar_seq) + 1u : 0u;

  // ---------------------------------------------------------- activation image
  if (PRO != kProImage) {
    const float* x = prologue_source(fz, act, nb * QK);
    const bool copy = fz.x_copy != nullptr && blockIdx.x == 0;
    const int lane8 = threadIdx.x & 7;
    constexpr int BPP = NCT / 8;  // blocks per pass
    float rms = 1.0f;
    if (PRO == kProNorm) {
      // rms = sqrt(mean(x^2) + eps), one fixed-order sum shared by every thread.
      float ssum = 0.0f;
      for (int i = threadIdx.x; i < nb * 8; i += NCT) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(x) + i);
        ssum = __fadd_rn(ssum, __fadd_rn(__fadd_rn(__fmul_rn(v.x, v.x), __fmul_rn(v.y, v.y)),
                                         __fadd_rn(__fmul_rn(v.z, v.z), __fmul_rn(v.w, v.w))));
        if (copy) reinterpret_cast<float4*>(fz.x_copy)[i] = v;
      }
      ssum = warp_sum(ssum);
      if (lane == 0) part[warp] = ssum;
      __syncthreads();
      float tot = 0.0f;
#pragma unroll
      for (int i = 0; i < kNcw; ++i) tot = __fadd_rn(tot, part[i]);
      rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)(nb * QK)), fz.eps));
    } else if (copy) {
      for (int i = threadIdx.x; i < nb * 8; i += NCT)
        reinterpret_cast<float4*>(fz.x_copy)[i] = __ldcg(reinterpret_cast<const float4*>(x) + i);
    }
    for (int base = 0; base < nb; base += 4 * BPP) {
      float4 v[4];
#pragma unroll
      for (int p = 0; p < 4; ++p) {  // the loads of 4 passes before any use
        const int b = base + p * BPP + (threadIdx.x >> 3);
        v[p] = b < nb ? __ldcg(reinterpret_cast<const float4*>(x + (size_t)b * QK) + lane8)
                      : make_float4(0.f, 0.f, 0.f, 0.f);
        if (PRO == kProNorm && b < nb) {  // (x / rms) * w, as the reference RMSNorm
          const float4 nw = reinterpret_cast<const float4*>(fz.norm_w + (size_t)b * QK)[lane8];
          v[p] = make_float4(__fmul_rn(__fdiv_rn(v[p].x, rms), nw.x), __fmul_rn(__fdiv_rn(v[p].y, rms), nw.y),
                             __fmul_rn(__fdiv_rn(v[p].z, rms), nw.z), __fmul_rn(__fdiv_rn(v[p].w, rms), nw.w));
        }
      }
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const int b = base + p * BPP + (threadIdx.x >> 3);
        if (base + p * BPP >= nb) break;  // uniform across the CTA
        float d;
        int qsum;
        const unsigned q = quantize_quad(v[p], d, qsum);
        if (b < nb) {
          reinterpret_cast<unsigned*>(x32 + (size_t)b * 32)[lane8] = q;
          if (lane8 == 0) const_cast<float2*>(sdq)[b] = make_float2(d, __int_as_float(qsum));
        }
      }
    }
  } else {
    // A prepared image (48-byte slots, then the (d, q-sum) pairs): the two
    // 16-byte halves of each slot, then the pairs.
    const unsigned char* src = static_cast<const unsigned char*>(act);
    for (int i = threadIdx.x; i < 2 * nb; i += NCT) cp_async16(x32 + 16 * i, src + (size_t)(i >> 1) * 48 + (i & 1) * 16);
    const int npair = (nb * 8 + 15) / 16;
    for (int i = threadIdx.x; i < npair; i += NCT)
      cp_async16(x32 + (size_t)nb * 32 + 16 * i, src + (size_t)nb * 48 + 16 * i);
    cp_async_wait_all();
  }
  __syncthreads();

  // Short rows (nb <= 32 * XR): this lane's activation blocks lane + 32 j stay in registers.
  uint4 rxa[XR > 0 ? XR : 1], rxb[XR > 0 ? XR : 1];
  float rxd[XR > 0 ? XR : 1];
  int rqs8[XR > 0 ? XR : 1];
#pragma unroll
  for (int j = 0; j < XR; ++j) {
    const int b = lane + 32 * j;
    if (b < nb) {
      rxa[j] = *reinterpret_cast<const uint4*>(x32 + (size_t)b * 32);
      rxb[j] = *reinterpret_cast<const uint4*>(x32 + (size_t)b * 32 + 16);
      const float2 dq = sdq[b];
      rxd[j] = dq.x;
      rqs8[j] = __float_as_int(dq.y) * 8;
    } else {
      rxa[j] = rxb[j] = make_uint4(0u, 0u, 0u, 0u);
      rxd[j] = 0.0f;
      rqs8[j] = 0;
    }
  }

  // ---------------------------------------------------------- stages
  // An iteration consumes P consecutive stages of this warp (P > 1 only for
  // whole-row plans): their RS rows each are reduced together, so the warp
  // has P times the independent work between waits.
  constexpr int PR = P * RS;  // rows reduced per iteration
  unsigned long long best_local = 0;  // kEpiArgmax: this lane's best (value, row)
  float acc[PR];
#pragma unroll
  for (int r = 0; r < PR; ++r) acc[r] = 0.0f;
  bool ok = true;
  int k = 0;
  for (; k < nk; k += P) {
    const int np = min(P, nk - k);  // stages in this iteration (warp-uniform)
    bool got = true;
#pragma unroll
    for (int p = 0; p < P; ++p)
      if (p < np) got = mbar_wait_bounded(smem_u32(&bars[warp * NSW + (k + p) % NSW]), (unsigned)((k + p) / NSW) & 1u) && got;
    if (__any_sync(kFull, !got)) {  // every lane stops together
      ok = false;
      if (lane == 0) raise_device_error(kErrRingTimeout);
      break;
    }
    const int c = k % C;  // chunk of these stages (P == 1 whenever C > 1)
#pragma unroll
    for (int p = 0; p < P; ++p) {
      if (p >= np) break;
      const int row0 = group_of(warp + ((k + p) / C) * kNcw) * RS, nr = min(RS, M - row0);
      const unsigned char* sw = ring + (size_t)(warp * NSW + (k + p) % NSW) * sh.slot_bytes;
      const unsigned char* ss = sw + (size_t)RS * cb * UB;
      if (XR > 0) {  // whole rows (C == 1), activation in registers
#pragma unroll
        for (int r = 0; r < RS; ++r) {
          if (r < nr) {  // uniform across the warp
#pragma unroll
            for (int j = 0; j < XR; ++j) {
              const int b = lane + 32 * j;
              if (b < nb) {
                const float sc = smem_scale<F16S>(ss + ((size_t)r * cb + b) * SS);
                int isum;
                if (FMT == kFmtQ4_0) {
                  const uint4 q = *reinterpret_cast<const uint4*>(sw + (size_t)r * cb * UB + (size_t)b * 16);
                  isum = q4_block_dot(q, rxa[j], rxb[j], rqs8[j]);
                } else {
                  const unsigned char* qp = sw + (size_t)r * cb * UB + (size_t)b * 32;
                  isum = q8_block_dot(*reinterpret_cast<const uint4*>(qp), *reinterpret_cast<const uint4*>(qp + 16),
                                      rxa[j], rxb[j]);
                }
                if (DBG) isums[(size_t)(row0 + r) * nb + b] = isum;
                acc[p * RS + r] = __fmaf_rn(__int2float_rn(isum), __fmul_rn(sc, rxd[j]), acc[p * RS + r]);
              }
            }
          }
        }
      } else {
        const int cbn = min(cb, nb - c * cb);
#pragma unroll 2
        for (int bl = lane; bl < cbn; bl += 32) {
          const int b = c * cb + bl;
          const uint4 xa = *reinterpret_cast<const uint4*>(x32 + (size_t)b * 32);
          const uint4 xb = *reinterpret_cast<const uint4*>(x32 + (size_t)b * 32 + 16);
          const float2 dq = sdq[b];
#pragma unroll
          for (int r = 0; r < RS; ++r) {
            if (r < nr) {  // uniform across the warp
              const float sc = smem_scale<F16S>(ss + ((size_t)r * cb + bl) * SS);
              int isum;
              if (FMT == kFmtQ4_0) {
                const uint4 q = *reinterpret_cast<const uint4*>(sw + (size_t)r * cb * UB + (size_t)bl * 16);
                isum = q4_block_dot(q, xa, xb, __float_as_int(dq.y) * 8);
              } else {
                const unsigned char* qp = sw + (size_t)r * cb * UB + (size_t)bl * 32;
                isum = q8_block_dot(*reinterpret_cast<const uint4*>(qp), *reinterpret_cast<const uint4*>(qp + 16), xa,
                                    xb);
              }
              if (DBG) isums[(size_t)(row0 + r) * nb + b] = isum;
              acc[p * RS + r] = __fmaf_rn(__int2float_rn(isum), __fmul_rn(sc, dq.x), acc[p * RS + r]);
            }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) {  // the slots are free again: stage t + NSW goes into the slot of stage t
      fence_proxy_async_smem();
      for (int p = 0; p < np; ++p)
        if (k + p + NSW < nk) issue(k + p + NSW);
    }
    if (c == C - 1) {
      const float v = rows_reduce<PR>(acc, lane);
      constexpr int HOP = 32 / PR;  // lanes between the holders of consecutive rows
      const int rr = lane / HOP;    // row (of the PR) this lane's v totals, holders only
      const int p = rr / RS, r = rr - p * RS;
      const int row0 = group_of(warp + ((k + p) / C) * kNcw) * RS;
      const int nr = p < np ? min(RS, M - row0) : 0;
      const bool holder = (lane % HOP) == 0 && r < nr;
      if (EPI == kEpiSwiglu) {
        // Rows (2i, 2i + 1) = (gate_i, up_i), in one stage (RS is even): h_i =
        // silu(gate) * up, as the reference's (gate / (1 + exp(-gate))) * up.
        const float u = __shfl_down_sync(kFull, v, HOP);
        if (holder && (r & 1) == 0 && r + 1 < nr) {
          const float g = v;
          __stcg(fz.h + ((row0 + r) >> 1), __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u));
        }
      } else if (holder) {
        const int row = row0 + r;
        if (EPI == kEpiResidual) {
          if (fz.tp > 1) {  // this rank's partial: to every rank's exchange buffer
            const unsigned long long wv = ((unsigned long long)seq << 32) | __float_as_uint(v);
            for (int t = 0; t < fz.tp; ++t) st_volatile_u64(xchg_word(fz, fz.xchg[t], seq, fz.tp_rank, row), wv);
          } else {
            y[row] = __fadd_rn(__ldcg(y + row), v);
          }
        } else {
          y[row] = v;
          if (EPI == kEpiArgmax && v == v) {
            const unsigned long long key = argmax_key(v, row + fz.vocab_offset);
            best_local = key > best_local ? key : best_local;
          }
        }
      }
#pragma unroll
      for (int r2 = 0; r2 < PR; ++r2) acc[r2] = 0.0f;
    }
  }
  if (!ok && lane == 0) {
    // A wait gave up: let the copies this warp issued land before the CTA exits.
    for (int t = k; t < nk && t < k + NSW; ++t)
      mbar_wait_bounded(smem_u32(&bars[warp * NSW + t % NSW]), (unsigned)(t / NSW) & 1u);
  }
  __syncwarp();

  if (EPI == kEpiArgmax) {
    // CTA maximum (warp shuffles, then the warps' values in shared memory),
    // one atomicMax per CTA, then the last CTA to arrive picks the token.
    unsigned long long b = best_local;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long t = __shfl_xor_sync(kFull, b, o);
      b = t > b ? t : b;
    }
    unsigned long long* wbest = reinterpret_cast<unsigned long long*>(part);
    __syncthreads();  // every warp is done with part
    if (lane == 0) wbest[warp] = b;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long mx = 0;
      for (int i = 0; i < kNcw; ++i) mx = wbest[i] > mx ? wbest[i] : mx;
      if (mx) atomicMax(fz.best, mx);
      argmax_arrive(fz, gridDim.x, seq);
    }
  }
  if (EPI == kEpiResidual && fz.tp > 1) {
    // Sum the tp partials of this CTA's rows in rank order (the same sum on
    // every rank) into the residual stream; the last CTA records the sequence.
    __syncthreads();
    bool xok = true;
    for (int row = r0 + (int)threadIdx.x; row < r1; row += NCT) {
      float sum = 0.0f;
      for (int t = 0; t < fz.tp; ++t)
        sum = __fadd_rn(sum, __uint_as_float(xchg_wait(xchg_word(fz, fz.xchg[fz.tp_rank], seq, t, row), seq, xok)));
      y[row] = __fadd_rn(__ldcg(y + row), sum);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      if (atomicAdd(fz.ar_done, 1u) == gridDim.x - 1) {
        *fz.ar_seq = seq;
        atomicExch(fz.ar_done, 0u);
      }
    }
  }
  if (EPI == kEpiSwiglu) {
    // This CTA's pairs [p0, p1) are in fz.h.  One release per CTA, then one
    // arrival per Q8_0 block it touched (adding its pair count); the CTA whose
    // arrival completes a block's 32 values quantizes that block.
    const int p0 = r0 >> 1, p1 = r1 >> 1;
    constexpr int kChunk = 64;
    __shared__ int s_last[kChunk];
    const int b0 = p0 >> 5, nblk = ((p1 + 31) >> 5) - b0;  // blocks touched
    __syncthreads();
    for (int c0 = 0; c0 < nblk; c0 += kChunk) {
      const int nc = min(kChunk, nblk - c0);
      if (threadIdx.x == 0) {
        __threadfence();
        for (int i = 0; i < nc; ++i) {
          const int blk = b0 + c0 + i;
          const int n = min(p1, (blk + 1) * 32) - max(p0, blk * 32);
          s_last[i] = atomicAdd(fz.counters + blk, (unsigned)n) + (unsigned)n == 32u;
        }
        __threadfence();
      }
      __syncthreads();
      for (int i = warp; i < nc; i += kNcw) {  // a warp quantizes each block this CTA completed
        if (!s_last[i]) continue;
        const int blk = b0 + c0 + i;
        const float4 hv4 = __ldcg(reinterpret_cast<const float4*>(fz.h + (size_t)blk * QK) + (lane & 7));
        float d;
        int qsum;
        const unsigned q = quantize_quad(hv4, d, qsum);
        if (lane < 8) reinterpret_cast<unsigned*>(fz.image_out + (size_t)blk * 48)[lane] = q;
        if (lane == 0) {
          reinterpret_cast<float2*>(fz.image_out + (size_t)(M >> 6) * 48)[blk] = make_float2(d, __int_as_float(qsum));
          fz.counters[blk] = 0u;
        }
      }
      __syncthreads();  // s_last is reused by the next chunk
    }
  }
  // An independent launch did not wait for the previous kernel before its
  // work; it does so before it ends, so that its completion still implies
  // the completion of everything before it in the stream.
  if (indep && threadIdx.x == 0) pdl_wait();
}

// ==========================================================================
// Host side
// ==========================================================================
namespace {

std::mutex g_tma_mu;
std::map<std::tuple<const void*, int>, bool> g_tma_attr;  // (kernel, device) -> smem opt-in done

// Work split of one launch.
struct TmaPlan {
  int RS = 0, XR = 0, C = 1, cb = 0, NSW = 0, slot_bytes = 0;
  size_t smem = 0;
  int per_sm = 1;
};

// Chooses rows per stage RS, chunks per row C (blocks per chunk cb) and ring
// slots per warp NSW so that one CTA fits the shared-memory budget: by
// default 110 KB, which leaves room on every SM for one CTA of the kernel
// launched next (under programmatic dependent launch it starts streaming its
// own weights while this one finishes).  Rows with nb <= 128 blocks keep the
// activation in registers (XR = 4) and stream one row per stage, consumed two
// stages per loop iteration (P = 2; SwiGLU pairs: two-row stages); longer rows
// read it from shared memory once per stage for RS = 4 rows (2 for SwiGLU
// pairs), cut into chunks when a stage would not fit twice per warp.  Chunk
// boundaries fall on multiples of 32 blocks, so every copy is 16-byte aligned
// and every plan adds a row's products in the same order.  When even the smallest plan does not fit the
// budget (a very long activation image), the CTA takes the whole opt-in
// shared memory and runs alone on its SM.
bool tma_plan(int fmt, bool f16s, int64_t nb, int epi, int smem_optin, TmaPlan* p) {
  const int ub = fmt == kFmtQ4_0 ? 16 : 32, ss = f16s ? 2 : 4;
  const int align = f16s ? 8 : 4;
  if (nb <= 0 || nb % align != 0) return false;  // 16-byte aligned scale rows
  const size_t fixed = (size_t)kBarBytes + kPartBytes + smem_image_bytes(nb);
  const bool swiglu = epi == kEpiSwiglu;
  const int xr = nb <= 128 ? 4 : 0;
  const int forced_rs = g_opt_mv_rows.load();
  int rs_pref = swiglu ? 2 : (xr ? 1 : 4);
  if (forced_rs == 1 || forced_rs == 2 || forced_rs == 4) rs_pref = (swiglu && forced_rs == 1) ? 2 : forced_rs;
  if (xr && rs_pref > 2) rs_pref = 2;  // register-activation kernels take 1 or 2 rows per stage
  const int nsw_cap = std::max(2, std::min(kMaxNsw, g_opt_mv_slots.load() > 0 ? g_opt_mv_slots.load() : kMaxNsw));
  auto try_budget = [&](size_t budget, TmaPlan* out) -> bool {
    if (budget <= fixed) return false;
    const size_t ring = budget - fixed;
    for (int rs = rs_pref; rs >= (swiglu ? 2 : 1); rs /= 2) {
      for (int C = 1; C <= 64; ++C) {
        if (xr && C > 1) break;  // activation registers cover whole rows only
        // Chunks of a multiple of 32 blocks: lane l then always takes the
        // blocks b = l (mod 32) in ascending order, whatever the plan, so y
        // does not depend on it (bit for bit).
        const int64_t cb = C == 1 ? nb : ((nb + C - 1) / C + 31) / 32 * 32;
        if (C > 1 && (int64_t)(C - 1) * cb >= nb) continue;  // no empty last chunk
        const size_t slot = ((size_t)rs * cb * (ub + ss) + 127) & ~(size_t)127;
        int nsw = (int)(ring / ((size_t)kNcw * slot));
        if (nsw < 2) continue;
        if (nsw > nsw_cap) nsw = nsw_cap;
        out->RS = rs;
        out->XR = xr;
        out->C = C;
        out->cb = (int)cb;
        out->NSW = nsw;
        out->slot_bytes = (int)slot;
        out->smem = fixed + (size_t)kNcw * nsw * slot;
        return true;
      }
      if (rs == 1) break;
    }
    return false;
  };
  size_t budget = (size_t)g_opt_mv_smem_kb.load() * 1024;
  if (budget > (size_t)smem_optin) budget = smem_optin;
  if (try_budget(budget, p)) return true;
  return try_budget((size_t)smem_optin - 1024, p);  // room for the static shared memory
}

template <int FMT, bool F16S, bool DBG, int PRO, int EPI, int RS, int XR, int P>
cudaError_t launch_tma_t(const MatvecArgs& a, const TmaPlan& p, int sms, cudaStream_t stream, bool pdl) {
  auto kernel = tma_matvec_kernel<FMT, F16S, DBG, PRO, EPI, RS, XR, P>;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(g_tma_mu);
    auto key = std::make_tuple((const void*)kernel, dev);
    if (!g_tma_attr[key]) {
      int optin = 0;
      cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
      cudaFuncAttributes fa;
      cudaError_t e = cudaFuncGetAttributes(&fa, kernel);
      if (e != cudaSuccess) return e;
      // dynamic + static shared memory must fit the opt-in limit
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)fa.sharedSizeBytes);
      if (e != cudaSuccess) return e;
      // Full shared-memory carveout: room for the next kernel's CTA beside this one.
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
      if (e != cudaSuccess) return e;
      g_tma_attr[key] = true;
    }
  }
  const void* w = a.w;
  const void* s = a.scales;
  const void* act = a.image ? a.image : (const void*)a.x;
  float* y = a.y;
  int32_t* isums = a.isums;
  MvShape sh;
  sh.M = (int)a.M;
  sh.nb = (int)(a.K / QK);
  sh.C = p.C;
  sh.cb = p.cb;
  sh.NSW = p.NSW;
  sh.slot_bytes = p.slot_bytes;
  sh.flags = (a.weights_static ? kMvPre : 0) | (a.act_independent ? kMvIndep : 0);
  MvFuse fz = a.fuse ? *a.fuse : MvFuse{};
  void* args[] = {(void*)&w, (void*)&s, (void*)&act, (void*)&y, (void*)&isums, (void*)&sh, (void*)&fz};
  int per_sm = g_opt_mv_ctas.load();
  if (per_sm < 1) per_sm = 1;
  long long grid = (long long)sms * per_sm;
  const long long groups = (a.M + RS - 1) / RS;
  if (grid > groups) grid = groups;
  if (grid < 1) grid = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kNcw * 32);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelExC(&cfg, (const void*)kernel, args);
}

int prologue_of(const MatvecArgs& a) {
  if (a.image) return kProImage;
  return (a.fuse && a.fuse->norm_w) ? kProNorm : kProQuant;
}

bool is_fused(const MatvecArgs& a) {
  return a.epi != kEpiStore || prologue_of(a) == kProNorm || (a.fuse && (a.fuse->embed || a.fuse->x_copy));
}

// Decode fusions: fp16 scales, no per-block sums; the combinations a decode
// step uses (RMSNorm -> q/k/v, gate/up or lm_head; image or x -> residual).
template <int FMT, int RS, int XR, int P>
cudaError_t launch_tma_fused(const MatvecArgs& a, const TmaPlan& p, int sms, cudaStream_t stream, bool pdl) {
  const int pro = prologue_of(a);
  switch (a.epi) {
    case kEpiStore:
      if (pro == kProNorm) return launch_tma_t<FMT, true, false, kProNorm, kEpiStore, RS, XR, P>(a, p, sms, stream, pdl);
      break;
    case kEpiResidual:
      if (pro == kProImage) return launch_tma_t<FMT, true, false, kProImage, kEpiResidual, RS, XR, P>(a, p, sms, stream, pdl);
      if (pro == kProQuant) return launch_tma_t<FMT, true, false, kProQuant, kEpiResidual, RS, XR, P>(a, p, sms, stream, pdl);
      break;
    case kEpiSwiglu:
      if constexpr (RS % 2 == 0) {
        if (pro == kProNorm) return launch_tma_t<FMT, true, false, kProNorm, kEpiSwiglu, RS, XR, P>(a, p, sms, stream, pdl);
      }
      break;
    case kEpiArgmax:
      if (pro == kProNorm) return launch_tma_t<FMT, true, false, kProNorm, kEpiArgmax, RS, XR, P>(a, p, sms, stream, pdl);
      break;
    default:
      break;
  }
  return cudaErrorNotSupported;
}

template <int FMT, int RS, int XR, int P>
cudaError_t launch_tma_r(const MatvecArgs& a, const TmaPlan& p, int sms, cudaStream_t stream, bool pdl) {
  if (is_fused(a)) return launch_tma_fused<FMT, RS, XR, P>(a, p, sms, stream, pdl);
  const bool fused = a.image == nullptr;
  if (a.isums) {
    return fused ? launch_tma_t<FMT, false, true, kProQuant, kEpiStore, RS, XR, P>(a, p, sms, stream, pdl)
                 : launch_tma_t<FMT, false, true, kProImage, kEpiStore, RS, XR, P>(a, p, sms, stream, pdl);
  }
  if (a.scales_f16) {
    return fused ? launch_tma_t<FMT, true, false, kProQuant, kEpiStore, RS, XR, P>(a, p, sms, stream, pdl)
                 : launch_tma_t<FMT, true, false, kProImage, kEpiStore, RS, XR, P>(a, p, sms, stream, pdl);
  }
  return fused ? launch_tma_t<FMT, false, false, kProQuant, kEpiStore, RS, XR, P>(a, p, sms, stream, pdl)
               : launch_tma_t<FMT, false, false, kProImage, kEpiStore, RS, XR, P>(a, p, sms, stream, pdl);
}

template <int FMT>
cudaError_t launch_tma_fmt(const MatvecArgs& a, const TmaPlan& p, int sms, cudaStream_t stream, bool pdl) {
  if (p.XR) {
    if (p.RS == 2) return launch_tma_r<FMT, 2, 4, 1>(a, p, sms, stream, pdl);
    return launch_tma_r<FMT, 1, 4, 2>(a, p, sms, stream, pdl);
  }
  switch (p.RS) {
    case 4: return launch_tma_r<FMT, 4, 0, 1>(a, p, sms, stream, pdl);
    case 2: return launch_tma_r<FMT, 2, 0, 1>(a, p, sms, stream, pdl);
    default: return launch_tma_r<FMT, 1, 0, 1>(a, p, sms, stream, pdl);
  }
}

}  // namespace

bool tma_matvec_supported(const MatvecArgs& a, int smem_optin) {
  if (a.fp32_act || a.M <= 0 || a.K <= 0 || a.M > 0x7fffffffLL) return false;
  // Bulk copies read from 16-byte aligned global addresses only (row starts
  // are multiples of 16 by the plan; the planes' bases must be too).
  if ((uintptr_t)a.w % 16 != 0 || (uintptr_t)a.scales % 16 != 0) return false;
  if (a.image && (uintptr_t)a.image % 16 != 0) return false;
  TmaPlan p;
  if (!tma_plan(a.fmt, a.isums ? false : a.scales_f16, a.K / QK, a.epi, smem_optin, &p)) return false;
  if (is_fused(a)) {
    if (!a.scales_f16 || a.isums || a.act_independent) return false;
    if (a.epi == kEpiSwiglu && a.M % 64 != 0) return false;
  }
  return true;
}

bool matvec_is_fused(const MatvecArgs& a) { return is_fused(a); }

cudaError_t launch_tma_matvec(const MatvecArgs& a, int sms, int smem_optin, cudaStream_t stream, bool pdl) {
  TmaPlan p;
  if (!tma_plan(a.fmt, a.isums ? false : a.scales_f16, a.K / QK, a.epi, smem_optin, &p)) return cudaErrorInvalidValue;
  if (a.fmt == kFmtQ4_0) return launch_tma_fmt<kFmtQ4_0>(a, p, sms, stream, pdl);
  return launch_tma_fmt<kFmtQ8_0>(a, p, sms, stream, pdl);
}

cudaError_t set_device_error_mirror(unsigned* host_mapped) {
  unsigned* dptr = nullptr;
  if (host_mapped) {
    cudaError_t e = cudaHostGetDevicePointer(reinterpret_cast<void**>(&dptr), host_mapped, 0);
    if (e != cudaSuccess) return e;
  }
  return cudaMemcpyToSymbol(g_error_mirror, &dptr, sizeof(dptr));
}

unsigned* device_error_word() {
  static std::mutex mu;
  static std::map<int, unsigned*> addr;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  auto it = addr.find(dev);
  if (it != addr.end()) return it->second;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
  addr[dev] = static_cast<unsigned*>(p);
  return static_cast<unsigned*>(p);
}

cudaError_t read_device_error(unsigned* out, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_device_error, sizeof(unsigned));
  if (e == cudaSuccess && clear && *out) {
    const unsigned zero = 0;
    e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(unsigned));
  }
  return e;
}

}  // namespace asmllm

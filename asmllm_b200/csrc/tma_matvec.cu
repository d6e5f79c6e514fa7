// asmllm_b200/csrc/tma_matvec.cu -- Q4_0/Q8_0 x Q8_0 matvec streamed by the
// bulk-copy (TMA) engine through a shared-memory ring (sm_100a).
//
// Same semantics as q8act_matvec_kernel in matvec.cu (reference
// THRISHAL12345/asmllm src/kernels/arm64/matmul_q4_neon.S:38-317): the
// activation is quantized to Q8_0 bit-exactly, each (row, block) int32 dot is
// exact, and y[r] = sum_b fma(float(isum), wd*xd) differs from the reference
// only in fp32 summation order.
//
// Structure of one CTA (persistent: two per SM by default, ~100 KB of shared
// memory each):
//   * The matrix is cut into stages of R whole rows (R in {8,4,2,1}, ~16 KB
//     of weights); rows are contiguous in memory, so a stage is exactly two
//     cp.async.bulk copies: the R rows' weights and their scales.  CTA c
//     takes stages c, c + grid, ... (all CTAs stream one contiguous span at
//     a time), or a contiguous range of rows for the epilogues that need one
//     (SwiGLU pairs, the tensor-parallel exchange).
//   * 1 producer warp: one lane issues the stages into per-warpgroup rings of
//     shared-memory slots (full/empty mbarriers, expect_tx).  Weights do not
//     depend on the previous kernel, so when the caller declares them static
//     the producer starts before griddepcontrol.wait: under programmatic
//     dependent launch the rings fill while the previous matvec still runs.
//   * NWG warpgroups of 8 consumer warps own alternate stages.  After
//     griddepcontrol.wait they build the Q8_0 activation image in shared
//     memory (quantizing x, 8 lanes per block, or copying a prepared image).
//     Per stage, 8/R warps share a row: each takes a strided subset of its
//     16-byte units, reduces across lanes, and (when R < 8) the row's partials
//     are summed in fixed order through shared memory -- y is deterministic.
//   * Every mbarrier wait is bounded (about a second of clock cycles); on
//     timeout the kernel sets bit 0 of g_device_error, stops, lets the copies
//     it issued land, and returns.
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

#ifndef ASMLLM_TMA_GROUPBAR
#define ASMLLM_TMA_GROUPBAR 1  // per-row-group barrier per stage (sweep and decode +1 % measured)
#endif
#ifndef ASMLLM_TMA_STRIDE
#define ASMLLM_TMA_STRIDE 1  // grid-strided stages for plain stores (sweep +1.3 % measured)
#endif

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

constexpr int kBarBytes = 256;                   // room for 2 x 15 mbarriers + abort flag
constexpr int kPartBytes = 2 * 2 * 8 * 2 * 4;    // row partials [2 parities][2 warpgroups][8 warps][2 rows]

}  // namespace


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

template <int FMT, bool F16S, bool DBG, int PRO, int EPI, int NWG, int R, int RW>
__global__ void __launch_bounds__((NWG * 8 + 1) * 32, 2)
tma_matvec_kernel(const uint8_t* __restrict__ w, const void* __restrict__ scales,
                  const void* __restrict__ act, float* __restrict__ y, int M, int nb,
                  int32_t* __restrict__ isums, int NS, int pre, int pf_stages, const MvFuse fz) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int UB = FMT == kFmtQ4_0 ? 16 : 32;  // weight bytes per block
  constexpr int SS = F16S ? 2 : 4;               // scale bytes per block
  constexpr int UPB = FMT == kFmtQ4_0 ? 1 : 2;   // 16-byte units per block
  constexpr int NCW = NWG * 8;                   // consumer warps
  constexpr int NCT = NCW * 32;                  // consumer threads

  // Shared layout: [barriers + abort flag | row partials | activation image | ring]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);  // full[0..NS), empty[NS..2NS)
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + kBarBytes - 4);
  float* part = reinterpret_cast<float*>(smem + kBarBytes);  // [2][NWG][8][2] partial row sums
  unsigned char* img = smem + kBarBytes + kPartBytes;
  const size_t img_bytes = (act_image_bytes(nb) + 127) & ~(size_t)127;
  unsigned char* stages = img + img_bytes;
  const size_t row_w = (size_t)nb * UB, row_s = (size_t)nb * SS;
  const size_t stage_bytes = (size_t)R * (row_w + row_s);  // R whole rows, then their scales
  constexpr int NRG = R / RW;                              // row groups per stage (RW rows each)
  constexpr int WPG = 8 / NRG;                             // warps sharing a row group (unit slices)
  const int NU = nb * UPB;                                 // units per row
  const int NSW = NS / NWG;                                // ring slots per warpgroup

  // SwiGLU pairs (gate, up) must not straddle CTAs or row groups.
  static_assert(EPI != kEpiSwiglu || (RW == 2 && WPG > 1), "SwiGLU epilogue needs two-row groups");
  constexpr int G = EPI == kEpiSwiglu ? 2 : 1;  // row granularity of the CTA split

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = G * (int)((long long)(M / G) * blockIdx.x / gridDim.x);
  const int r1 = G * (int)((long long)(M / G) * (blockIdx.x + 1) / gridDim.x);
  // Epilogues whose rows are independent (store, argmax, the one-GPU residual
  // add) take their stages grid-strided: stage s of this CTA = stage
  // s * grid + cta of the matrix, so at any moment the CTAs stream one
  // contiguous span.  SwiGLU (pairs and per-CTA block counters) and the
  // tensor-parallel residual exchange need a contiguous row range per CTA.
  const bool stride = ASMLLM_TMA_STRIDE && (EPI == kEpiStore || EPI == kEpiArgmax ||
                                            (EPI == kEpiResidual && fz.tp <= 1));
  const int n_st = (M + R - 1) / R;
  const int S = stride ? ((int)blockIdx.x < n_st ? (n_st - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0)
                       : (r1 - r0 + R - 1) / R;  // stages; stage s owned by warpgroup s % NWG
  auto stage_row0 = [&](int t) { return stride ? (t * (int)gridDim.x + (int)blockIdx.x) * R : r0 + t * R; };
  const int r_end = stride ? M : r1;

  pdl_trigger();
  if (S == 0) {
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
    return;
  }

  if (threadIdx.x == 0) {
    for (int i = 0; i < NSW * NWG; ++i) {
      mbar_init(smem_u32(&bars[i]), 1);       // full: producer arrive + tx bytes
      mbar_init(smem_u32(&bars[NS + i]), 8);  // empty: the 8 warps of the owning warpgroup
    }
    *s_abort = 0;
    fence_mbar_init();
  }
  __syncthreads();

  // ------------------------------------------------------------ producer
  if (warp == NCW) {
    if (lane == 0) {
      if (!pre) pdl_wait();  // weights may be written by the previous kernel
      // Stages beyond the ring go to L2 ahead of time (bulk prefetch: no shared
      // memory, nothing waits on it), keeping HBM busy while the consumers wait
      // for the previous kernel and quantize x.
      int pf_next = NS;
      const int pf_end = min(S, NS + pf_stages);
      auto prefetch_stage = [&](int t) {
        const int row0 = stage_row0(t);
        const int nrows = min(R, r_end - row0);
        prefetch_l2_bulk(w + (size_t)row0 * row_w, (unsigned)((size_t)nrows * row_w));
        prefetch_l2_bulk(static_cast<const unsigned char*>(scales) + (size_t)row0 * row_s,
                         (unsigned)((size_t)nrows * row_s));
      };
      int s = 0;
      for (; s < S && !*s_abort; ++s) {
        if (s == 1)
          for (; pf_next < pf_end; ++pf_next) prefetch_stage(pf_next);
        else if (s > 1 && pf_next < S && pf_next < s + NS + pf_stages)
          prefetch_stage(pf_next++);  // keep the window pf_stages ahead of the ring
        const int g = s % NWG, k = s / NWG;  // k-th stage of warpgroup g
        const int slot = g * NSW + k % NSW, round = k / NSW;
        if (round > 0 && !mbar_wait_bounded(smem_u32(&bars[NS + slot]), (round - 1) & 1)) {
          raise_device_error(kErrRingTimeout);
          *s_abort = 1;
          break;
        }
        const int row0 = stage_row0(s);
        const int nrows = min(R, r_end - row0);
        const uint32_t full = smem_u32(&bars[slot]);
        mbar_arrive_expect_tx(full, (uint32_t)((size_t)nrows * (row_w + row_s)));
        const uint32_t st = smem_u32(stages + (size_t)slot * stage_bytes);
        bulk_g2s(st, w + (size_t)row0 * row_w, (uint32_t)((size_t)nrows * row_w), full);
        bulk_g2s(st + (uint32_t)((size_t)R * row_w), static_cast<const unsigned char*>(scales) + (size_t)row0 * row_s,
                 (uint32_t)((size_t)nrows * row_s), full);
      }
      if (*s_abort) {  // let the copies already issued land before the CTA exits
        for (int t = (s > NS ? s - NS : 0); t < s; ++t) {
          const int g = t % NWG, k = t / NWG;
          mbar_wait_bounded(smem_u32(&bars[g * NSW + k % NSW]), (k / NSW) & 1);
        }
      }
    }
    return;
  }

  // ------------------------------------------------------------ consumers
  const int wg = warp >> 3, wi = warp & 7;
  const int rg = wi / WPG, sg = wi - rg * WPG;  // this warp's row group in a stage and its unit slice
  pdl_wait();  // x / the image may come from the previous kernel; y may still be in use
  // Tensor-parallel call number (the previous exchange's last CTA stored it).
  const unsigned seq = (fz.tp > 1 && (EPI == kEpiResidual || EPI == kEpiArgmax)) ? __ldcg(fz.ar_seq) + 1u : 0u;
  if (PRO != kProImage) {
    const float* x = prologue_source(fz, act, nb * QK);
    const bool copy = fz.x_copy != nullptr && blockIdx.x == 0;
    const int lane8 = threadIdx.x & 7;
    constexpr int BPP = NCT / 8;  // blocks per pass
    float rms = 1.0f;
    if (PRO == kProNorm) {
      // rms = sqrt(mean(x^2) + eps), one fixed-order sum shared by every thread.
      float ss = 0.0f;
      for (int i = threadIdx.x; i < nb * 8; i += NCT) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(x) + i);
        ss = __fadd_rn(ss, __fadd_rn(__fadd_rn(__fmul_rn(v.x, v.x), __fmul_rn(v.y, v.y)),
                                     __fadd_rn(__fmul_rn(v.z, v.z), __fmul_rn(v.w, v.w))));
        if (copy) reinterpret_cast<float4*>(fz.x_copy)[i] = v;
      }
      ss = warp_sum(ss);
      if (lane == 0) part[warp] = ss;
      consumer_bar_sync(NCT);
      float tot = 0.0f;
#pragma unroll
      for (int i = 0; i < NCW; ++i) tot = __fadd_rn(tot, part[i]);
      rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)(nb * QK)), fz.eps));
    } else if (copy) {
      for (int i = threadIdx.x; i < nb * 8; i += NCT)
        reinterpret_cast<float4*>(fz.x_copy)[i] = __ldcg(reinterpret_cast<const float4*>(x) + i);
    }

    for (int base = 0; base < nb; base += 4 * BPP) {
      float4 v[4];
#pragma unroll
      for (int p = 0; p < 4; ++p) {  // issue the loads of 4 passes before any use
        const int b = base + p * BPP + (threadIdx.x >> 3);
        v[p] = b < nb ? __ldcg(reinterpret_cast<const float4*>(x + (size_t)b * QK) + lane8) : make_float4(0.f, 0.f, 0.f, 0.f);
        if (PRO == kProNorm && b < nb) {  // (x / rms) * w, as the reference RMSNorm
          const float4 nw = reinterpret_cast<const float4*>(fz.norm_w + (size_t)b * QK)[lane8];
          v[p] = make_float4(__fmul_rn(__fdiv_rn(v[p].x, rms), nw.x), __fmul_rn(__fdiv_rn(v[p].y, rms), nw.y),
                             __fmul_rn(__fdiv_rn(v[p].z, rms), nw.z), __fmul_rn(__fdiv_rn(v[p].w, rms), nw.w));
        }
      }
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const int b = base + p * BPP + (threadIdx.x >> 3);
        if (base + p * BPP >= nb) break;  // uniform across the consumers
        float d;
        int qsum;
        const unsigned q = quantize_quad(v[p], d, qsum);
        if (b < nb) {
          reinterpret_cast<unsigned*>(img + b * 48)[lane8] = q;
          if (lane8 == 0) reinterpret_cast<float2*>(img + (size_t)nb * 48)[b] = make_float2(d, __int_as_float(qsum));
        }
      }
    }
  } else {
    const unsigned char* src = static_cast<const unsigned char*>(act);
    const int n16 = (int)(act_image_bytes(nb) / 16);
    for (int i = threadIdx.x; i < n16; i += NCT) cp_async16(img + 16 * i, src + 16 * i);
    cp_async_wait_all();
  }
  consumer_bar_sync(NCT);

  const float2* sdq = reinterpret_cast<const float2*>(img + (size_t)nb * 48);
  unsigned long long best_local = 0;  // kEpiArgmax: this lane's best (value, row)
  auto emit = [&](int row, float t) {
    if (EPI == kEpiResidual) {
      if (fz.tp > 1) {  // this rank's partial: to every rank's exchange buffer
        const unsigned long long wv = ((unsigned long long)seq << 32) | __float_as_uint(t);
        for (int r = 0; r < fz.tp; ++r) st_volatile_u64(xchg_word(fz, fz.xchg[r], seq, fz.tp_rank, row), wv);
      } else {
        y[row] = __fadd_rn(__ldcg(y + row), t);
      }
    } else {
      y[row] = t;
      if (EPI == kEpiArgmax && t == t) {
        const unsigned long long key = argmax_key(t, row + fz.vocab_offset);
        best_local = key > best_local ? key : best_local;
      }
    }
  };
  // Rows (row, row + 1) = (gate_i, up_i): h_i = silu(gate) * up, as the
  // reference's (gate / (1 + exp(-gate))) * up; stored to fz.h as the rows
  // finish.  The Q8_0 blocks of h are made after the stage loop.
  auto swiglu_emit = [&](int row, const float* pr) {
    if (lane == 0) {
      float g = pr[0], u = pr[1];
      for (int j = 1; j < WPG; ++j) {
        g += pr[j * 2];
        u += pr[j * 2 + 1];
      }
      __stcg(fz.h + (row >> 1), __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u));
    }
  };
  for (int s = wg, k = 0; s < S; s += NWG, ++k) {
    const int slot = wg * NSW + k % NSW;
    const bool ok = mbar_wait_bounded(smem_u32(&bars[slot]), (k / NSW) & 1);
    if (!ok) raise_device_error(kErrRingTimeout);
    const int row0 = stage_row0(s);
    const int nrows = min(R, r_end - row0);
    const unsigned char* st = stages + (size_t)slot * stage_bytes;
    // Rows rbase .. rbase+RW-1 of the stage; this warp takes units
    // sg*32 + lane + 32*WPG*j and reads each activation block once for its RW rows.
    const int rbase = rg * RW;
    const int nr = nrows - rbase;  // rows of this group present (<= 0: none)
    float acc[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) acc[r] = 0.0f;
    if (ok && nr > 0) {
      const unsigned char* w0 = st + (size_t)rbase * row_w;
      const unsigned char* s0 = st + (size_t)R * row_w + (size_t)rbase * row_s;
      if (FMT == kFmtQ4_0) {
#pragma unroll 4
        for (int b = sg * 32 + lane; b < nb; b += 32 * WPG) {
          const uint4* xp = reinterpret_cast<const uint4*>(img + b * 48);
          const uint4 xa = xp[0], xb = xp[1];
          const float2 dq = sdq[b];
          const int qsum8 = __float_as_int(dq.y) * 8;
#pragma unroll
          for (int r = 0; r < RW; ++r) {
            if (r < nr) {  // uniform across the warp
              const uint4 q = *reinterpret_cast<const uint4*>(w0 + r * row_w + b * 16);
              const float sc = F16S ? __half2float(*reinterpret_cast<const __half*>(s0 + r * row_s + b * 2))
                                    : *reinterpret_cast<const float*>(s0 + r * row_s + b * 4);
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
              if (DBG) isums[(size_t)(row0 + rbase + r) * nb + b] = isum;
              acc[r] = __fmaf_rn(__int2float_rn(isum), __fmul_rn(sc, dq.x), acc[r]);
            }
          }
        }
      } else {
#pragma unroll 4
        for (int u0 = sg * 32; u0 < NU; u0 += 32 * WPG) {
          const int u = u0 + lane;
          const bool valid = u < NU;  // same for both lanes of a pair
          const int b = u >> 1;
          uint4 xa = make_uint4(0u, 0u, 0u, 0u);
          float xd = 0.0f;
          if (valid) {
            xa = *reinterpret_cast<const uint4*>(img + b * 48 + (u & 1) * 16);
            xd = sdq[b].x;
          }
#pragma unroll
          for (int r = 0; r < RW; ++r) {
            if (r < nr) {  // uniform across the warp
              uint4 q = make_uint4(0u, 0u, 0u, 0u);
              float sc = 0.0f;
              if (valid) {
                q = *reinterpret_cast<const uint4*>(w0 + r * row_w + u * 16);
                sc = F16S ? __half2float(*reinterpret_cast<const __half*>(s0 + r * row_s + b * 2))
                          : *reinterpret_cast<const float*>(s0 + r * row_s + b * 4);
              }
              int p = 0;
              p = dp4a_ss((int)q.x, (int)xa.x, p);
              p = dp4a_ss((int)q.y, (int)xa.y, p);
              p = dp4a_ss((int)q.z, (int)xa.z, p);
              p = dp4a_ss((int)q.w, (int)xa.w, p);
              const int isum = p + __shfl_xor_sync(kFull, p, 1);
              if (valid && !(lane & 1)) {
                if (DBG) isums[(size_t)(row0 + rbase + r) * nb + b] = isum;
                acc[r] = __fmaf_rn(__int2float_rn(isum), __fmul_rn(sc, xd), acc[r]);
              }
            }
          }
        }
      }
    }
    // Lane sums: RW == 1 -> lane 0 holds the row; RW == 2 -> a butterfly that
    // first trades rows between half-warps (lane 0 ends with row 0, lane 16 row 1).
    float v;
    if (RW == 1) {
      v = warp_sum(acc[0]);
    } else {
      const bool upper = lane & 16;
      v = upper ? acc[RW - 1] : acc[0];
      v += __shfl_xor_sync(kFull, upper ? acc[0] : acc[RW - 1], 16);
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&bars[NS + slot]));  // this warp is done with the slot
    const int my_row = RW == 1 ? 0 : (lane >> 4);            // row (within the group) this lane's v covers
    const bool holder = (lane & 15) == 0 && (RW == 2 || lane == 0);
    // Row groups split over WPG warps: partials through shared memory, summed
    // in slice order (deterministic); double-buffered by stage parity.
    float* pb = part + ((k & 1) * NWG + wg) * 16;  // [8 warps][2 rows]
    if (WPG == 1) {
      if (ok && holder && my_row < nr) emit(row0 + rbase + my_row, v);
    } else if (holder) {
      pb[wi * 2 + my_row] = v;
    }
    // One decision per group of warps that share rows (their partials meet
    // here; named barriers 4..11), or per warpgroup: stop together if any
    // warp timed out or the producer gave up (no warp can be left waiting at
    // this barrier; a group that stops leaves the ring's empty barriers
    // short, so the producer's bounded wait raises the abort for the rest).
    const bool stop = (ASMLLM_TMA_GROUPBAR && WPG < 8)
                          ? group_bar_or(4 + wg * NRG + rg, 32 * WPG, !ok || *s_abort)
                          : wg_bar_or(wg, !ok || *s_abort);
    if (stop) {
      *s_abort = 1;
      break;
    }
    if (WPG > 1 && sg == 0) {
      if (EPI == kEpiSwiglu) {
        if (nr >= 2) swiglu_emit(row0 + rbase, pb + rg * WPG * 2);  // whole warp
      } else if (lane < RW && lane < nr) {  // lane r finishes row rbase + r
        float t = pb[(rg * WPG) * 2 + lane];
        for (int j = 1; j < WPG; ++j) t += pb[(rg * WPG + j) * 2 + lane];
        emit(row0 + rbase + lane, t);
      }
    }
  }
  if (EPI == kEpiArgmax) {
    // CTA maximum (warp shuffles, then the warps' values in shared memory),
    // one atomicMax per CTA, then the last CTA to arrive picks the token.
    unsigned long long b = best_local;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long t = __shfl_xor_sync(kFull, b, o);
      b = t > b ? t : b;
    }
    consumer_bar_sync(NCT);  // every warp is done with the row partials
    unsigned long long* wbest = reinterpret_cast<unsigned long long*>(part);
    if (lane == 0) wbest[warp] = b;
    consumer_bar_sync(NCT);
    if (threadIdx.x == 0) {
      unsigned long long m = 0;
      for (int i = 0; i < NCW; ++i) m = wbest[i] > m ? wbest[i] : m;
      if (m) atomicMax(fz.best, m);
      argmax_arrive(fz, gridDim.x, seq);
    }
  }
  if (EPI == kEpiResidual && fz.tp > 1) {
    // Sum the tp partials of this CTA's rows in rank order (the same sum on
    // every rank) into the residual stream; the last CTA records the sequence.
    bool ok = true;
    for (int row = r0 + (int)threadIdx.x; row < r1; row += NCT) {
      float sum = 0.0f;
      for (int r = 0; r < fz.tp; ++r)
        sum = __fadd_rn(sum, __uint_as_float(xchg_wait(xchg_word(fz, fz.xchg[fz.tp_rank], seq, r, row), seq, ok)));
      y[row] = __fadd_rn(__ldcg(y + row), sum);
    }
    consumer_bar_sync(NCT);
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
    consumer_bar_sync(NCT);
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
      consumer_bar_sync(NCT);
      for (int i = warp; i < nc; i += NCW) {  // a warp quantizes each block this CTA completed
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
      consumer_bar_sync(NCT);  // s_last is reused by the next chunk
    }
  }
}

// ==========================================================================
// Host side
// ==========================================================================
namespace {

std::mutex g_tma_mu;
std::map<std::tuple<const void*, int>, bool> g_tma_attr;  // (kernel, device) -> smem opt-in done

int env_int2(const char* name, int dflt) {
  const char* e = getenv(name);
  return e ? atoi(e) : dflt;
}
// Defaults from measurement on B200 (2 CTAs per SM with ~100 KB each streamed
// best; deeper single-CTA rings and L2 prefetch windows did not help).
const int g_tma_ctas = env_int2("ASMLLM_TMA_CTAS_PER_SM", 2);
const int g_tma_smem_kb = env_int2("ASMLLM_TMA_SMEM_KB", 100);
constexpr int g_tma_nwg = 2;  // consumer warpgroups
#ifndef ASMLLM_TMA_RW
#define ASMLLM_TMA_RW 2
#endif
constexpr int kTmaRowsPerWarp = ASMLLM_TMA_RW;  // rows each consumer warp takes in a stage
// One row per warp with 8-row stages (each warp alone on its rows) failed the
// graph-replay determinism test when tried; only two rows per warp is validated.
static_assert(kTmaRowsPerWarp == 2, "only ASMLLM_TMA_RW=2 is validated");
const int g_tma_carveout = env_int2("ASMLLM_TMA_CARVEOUT", 100);  // percent of the unified L1/shared
const int g_tma_pf_kb = env_int2("ASMLLM_TMA_PF_KB", 0);          // L2 prefetch window per CTA (off)
const int g_tma_stage_kb = env_int2("ASMLLM_TMA_STAGE_KB", 16);    // weight bytes per stage (target)
const int g_tma_max_slots = env_int2("ASMLLM_TMA_MAX_SLOTS", 8);   // ring slots per CTA (cap)

struct TmaPlan {
  int R = 0, NS = 0;
  size_t smem = 0;
};

// Stage = R whole consecutive rows (contiguous in memory: one bulk copy for
// their weights and one for their scales), R in {8, 4, 2, 1}, the largest
// whose weights fit in the stage target (16 KB); rows above 24 KB are left
// to the register-streaming kernel.
bool tma_plan(int fmt, bool f16s, int64_t nb, int smem_optin, TmaPlan* p) {
  const int ub = fmt == kFmtQ4_0 ? 16 : 32, ss = f16s ? 2 : 4;
  if (nb % (f16s ? 8 : 4) != 0) return false;  // 16-byte aligned scale rows
  const size_t row_w = (size_t)nb * ub, row_s = (size_t)nb * ss;
  if (row_w > 24 * 1024) return false;
  int R = 8;
  while (R > 1 && (size_t)R * row_w > (size_t)g_tma_stage_kb * 1024) R /= 2;
  const size_t stage = (size_t)R * (row_w + row_s);
  const size_t img = (act_image_bytes(nb) + 127) & ~(size_t)127;
  size_t budget = (size_t)g_tma_smem_kb * 1024;
  if (budget > (size_t)smem_optin) budget = smem_optin;
  const size_t fixed = kBarBytes + kPartBytes + img;
  const size_t nwg = g_tma_nwg == 1 ? 1 : 2;
  auto slots = [&](size_t b) -> size_t {
    if (b < fixed) return 0;
    size_t n = (b - fixed) / stage;
    // the barrier area holds 2 x 15 mbarriers beside the abort flag
    const size_t cap = g_tma_max_slots < 2 ? 2 : g_tma_max_slots > 14 ? 14 : (size_t)g_tma_max_slots;
    if (n > cap) n = cap;
    return n - n % nwg;  // equal rings per warpgroup
  };
  size_t ns = slots(budget);
  // Long rows (a large activation image plus big stages): take the whole
  // opt-in shared memory, one CTA per SM.
  if (ns < 2 * nwg) ns = slots(budget = (size_t)smem_optin - 1024);  // room for static shared memory
  if (ns < 2 * nwg) return false;
  p->R = R;
  p->NS = (int)ns;
  p->smem = fixed + ns * stage;
  return true;
}

template <int FMT, bool F16S, bool DBG, int PRO, int EPI, int NWG, int R>
cudaError_t launch_tma_t(const MatvecArgs& a, const TmaPlan& p, int sms, cudaStream_t stream, bool pdl) {
  constexpr int RW = R >= 2 ? kTmaRowsPerWarp : 1;
  auto kernel = tma_matvec_kernel<FMT, F16S, DBG, PRO, EPI, NWG, R, RW>;
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
      // Full shared-memory carveout: room for the next matvec's CTA beside this one.
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, g_tma_carveout);
      if (e != cudaSuccess) return e;
      g_tma_attr[key] = true;
    }
  }
  const void* w = a.w;
  const void* s = a.scales;
  const void* act = a.image ? a.image : (const void*)a.x;
  float* y = a.y;
  int M = (int)a.M, nb = (int)(a.K / QK);
  int32_t* isums = a.isums;
  int NS = p.NS, pre = a.weights_static ? 1 : 0;
  const size_t stage_b = (size_t)R * (size_t)nb * ((FMT == kFmtQ4_0 ? 16 : 32) + (F16S ? 2 : 4));
  int pf = (int)(((size_t)g_tma_pf_kb * 1024) / stage_b);
  MvFuse fz = a.fuse ? *a.fuse : MvFuse{};
  void* args[] = {(void*)&w,     (void*)&s,  (void*)&act, (void*)&y,  (void*)&M,  (void*)&nb,
                  (void*)&isums, (void*)&NS, (void*)&pre, (void*)&pf, (void*)&fz};
  // Persistent grid: as many CTAs per SM as fit beside each other (the
  // default 2 at ~100 KB; 1 for the long-row plans that take more).
  int smem_sm = 0;
  cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
  int per_sm = g_tma_ctas > 0 ? g_tma_ctas : 1;
  const int fit = smem_sm > 0 ? (int)((size_t)smem_sm / (p.smem + 1024)) : per_sm;
  if (per_sm > fit) per_sm = fit > 0 ? fit : 1;
  long long grid = (long long)sms * per_sm;
  const long long groups = (M + R - 1) / R;
  if (grid > groups) grid = groups;
  if (grid < 1) grid = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3((NWG * 8 + 1) * 32);
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
template <int FMT, int NWG, int R>
cudaError_t launch_tma_fused(const MatvecArgs& a, const TmaPlan& p, int sms, cudaStream_t stream, bool pdl) {
  const int pro = prologue_of(a);
  switch (a.epi) {
    case kEpiStore:
      if (pro == kProNorm) return launch_tma_t<FMT, true, false, kProNorm, kEpiStore, NWG, R>(a, p, sms, stream, pdl);
      break;
    case kEpiResidual:
      if (pro == kProImage) return launch_tma_t<FMT, true, false, kProImage, kEpiResidual, NWG, R>(a, p, sms, stream, pdl);
      if (pro == kProQuant) return launch_tma_t<FMT, true, false, kProQuant, kEpiResidual, NWG, R>(a, p, sms, stream, pdl);
      break;
    case kEpiSwiglu:
      if constexpr (R >= 2) {
        if (pro == kProNorm) return launch_tma_t<FMT, true, false, kProNorm, kEpiSwiglu, NWG, R>(a, p, sms, stream, pdl);
      }
      break;
    case kEpiArgmax:
      if (pro == kProNorm) return launch_tma_t<FMT, true, false, kProNorm, kEpiArgmax, NWG, R>(a, p, sms, stream, pdl);
      break;
    default:
      break;
  }
  return cudaErrorNotSupported;
}

template <int FMT, int NWG, int R>
cudaError_t launch_tma_r(const MatvecArgs& a, const TmaPlan& p, int sms, cudaStream_t stream, bool pdl) {
  if (is_fused(a)) return launch_tma_fused<FMT, NWG, R>(a, p, sms, stream, pdl);
  const bool fused = a.image == nullptr;
  if (a.isums) {
    return fused ? launch_tma_t<FMT, false, true, kProQuant, kEpiStore, NWG, R>(a, p, sms, stream, pdl)
                 : launch_tma_t<FMT, false, true, kProImage, kEpiStore, NWG, R>(a, p, sms, stream, pdl);
  }
  if (a.scales_f16) {
    return fused ? launch_tma_t<FMT, true, false, kProQuant, kEpiStore, NWG, R>(a, p, sms, stream, pdl)
                 : launch_tma_t<FMT, true, false, kProImage, kEpiStore, NWG, R>(a, p, sms, stream, pdl);
  }
  return fused ? launch_tma_t<FMT, false, false, kProQuant, kEpiStore, NWG, R>(a, p, sms, stream, pdl)
               : launch_tma_t<FMT, false, false, kProImage, kEpiStore, NWG, R>(a, p, sms, stream, pdl);
}

template <int FMT, int NWG>
cudaError_t launch_tma_fmt(const MatvecArgs& a, const TmaPlan& p, int sms, cudaStream_t stream, bool pdl) {
  switch (p.R) {
    case 8: return launch_tma_r<FMT, NWG, 8>(a, p, sms, stream, pdl);
    case 4: return launch_tma_r<FMT, NWG, 4>(a, p, sms, stream, pdl);
    case 2: return launch_tma_r<FMT, NWG, 2>(a, p, sms, stream, pdl);
    default: return launch_tma_r<FMT, NWG, 1>(a, p, sms, stream, pdl);
  }
}

}  // namespace

bool tma_matvec_supported(const MatvecArgs& a, int smem_optin) {
  if (a.fp32_act || a.M <= 0 || a.K <= 0) return false;
  TmaPlan p;
  if (!tma_plan(a.fmt, a.isums ? false : a.scales_f16, a.K / QK, smem_optin, &p)) return false;
  if (is_fused(a)) {
    if (!a.scales_f16 || a.isums) return false;
    if (a.epi == kEpiSwiglu && (p.R < 2 || a.M % 64 != 0)) return false;
  }
  return true;
}

bool matvec_is_fused(const MatvecArgs& a) { return is_fused(a); }

cudaError_t launch_tma_matvec(const MatvecArgs& a, int sms, int smem_optin, cudaStream_t stream, bool pdl) {
  TmaPlan p;
  if (!tma_plan(a.fmt, a.isums ? false : a.scales_f16, a.K / QK, smem_optin, &p)) return cudaErrorInvalidValue;
  if (a.fmt == kFmtQ4_0) return launch_tma_fmt<kFmtQ4_0, 2>(a, p, sms, stream, pdl);
  return launch_tma_fmt<kFmtQ8_0, 2>(a, p, sms, stream, pdl);
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

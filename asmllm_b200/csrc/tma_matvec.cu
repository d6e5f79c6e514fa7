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
//
// The fused decode-step matvecs, and plain matvecs with rows of more than 128
// blocks in launches that wait for the previous kernel, are streamed by the
// row-stage kernel of tma_rows.cuh instead (use_rows below): in such chains
// its CTA-wide ~16 KB stages measured 6-40 % faster than per-warp rings.
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
std::atomic<int> g_opt_mv_smem_kb{0};
std::atomic<int> g_opt_mv_ctas{1};
std::atomic<int> g_opt_mv_kernel{0};


// ---- tensor-parallel exchange words: (sequence << 32) | payload bits ------
__device__ __forceinline__ void st_volatile_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_volatile_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Limit of an exchange wait in SM clock cycles (asm_set_option "xchg_wait_us").
__device__ long long g_xchg_wait_cycles = kWaitCycles;

// The payload of the exchange word at p once it carries sequence seq; bounded
// (a peer that never writes sets the error bit and yields 0; after one
// timeout, `ok` makes the caller's later waits return at once).
__device__ __forceinline__ unsigned xchg_wait(const unsigned long long* p, unsigned seq, bool& ok) {
  unsigned long long v = ld_volatile_u64(p);
  if ((unsigned)(v >> 32) == seq) return (unsigned)v;
  if (!ok) return 0u;
  const long long limit = g_xchg_wait_cycles;
  const long long t0 = clock64();
  do {
    __nanosleep(32);  // leave issue slots to the kernels running beside the waiting one
    v = ld_volatile_u64(p);
    if (clock64() - t0 > limit) {
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

// Shared-memory loads at 32-bit shared addresses (volatile: they stay after
// the mbarrier wait that makes the bulk-copied bytes visible).
__device__ __forceinline__ uint4 lds_v4(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}

template <bool F16S>
__device__ __forceinline__ float lds_scale(uint32_t a) {
  if (F16S) {
    unsigned short h;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(h) : "r"(a));
    return half_bits_to_float(h);
  }
  float f;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(f) : "r"(a));
  return f;
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
// Within block b's 32 bytes the two 16-byte halves (elements 0-15 and
// 16-31) swap places when bit 2 of b is set: lanes reading blocks b .. b + 7
// (a quarter warp's 16-byte reads) then hit eight distinct bank quads.
__device__ __forceinline__ int xhalf(int b, int h) { return b * 32 + ((h ^ ((b >> 2) & 1)) << 4); }
__host__ __device__ inline size_t smem_image_bytes(int64_t nb) { return ((size_t)nb * 40 + 127) & ~(size_t)127; }

template <int FMT, bool F16S, bool DBG, int PRO, int EPI, int RS, int XR, int NBQ, bool PK>
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
  // Weight layouts.  Planes (PK false): w = [M][row_w] quants, scales =
  // [M][row_s].  Packed rows (PK true): w = [M][row_w + row_s], each row its
  // quants then its fp16 scales (the GGUF byte count), so R consecutive whole
  // rows are one contiguous copy.  A slot of whole packed rows keeps that
  // layout; any other slot holds [RS][cb] quant blocks then [RS][cb] scales.
  static_assert(!PK || F16S, "packed rows carry fp16 scales");
  const size_t g_wstride = PK ? row_w + row_s : row_w;  // global row stride of the quants
  const size_t g_sstride = PK ? row_w + row_s : row_s;  // and of the scales
  const unsigned char* gsc = PK ? w + row_w : static_cast<const unsigned char*>(scales);
  const bool pk_slot = PK && C == 1;
  const size_t sl_wstride = pk_slot ? row_w + row_s : (size_t)cb * UB;  // in a slot: row stride of the quants,
  const size_t sl_sbase = pk_slot ? row_w : (size_t)RS * cb * UB;        // where the scales start,
  const size_t sl_sstride = pk_slot ? row_w + row_s : (size_t)cb * SS;   // and their row stride

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Row groups of RS rows.  Epilogues whose rows are independent (store,
  // argmax, the one-GPU residual add) take groups grid-strided: group q of
  // this CTA = group q * grid + cta, so at any moment the CTAs stream one
  // contiguous span.  SwiGLU (pairs and per-CTA block counters) and the
  // tensor-parallel residual exchange take one contiguous range per CTA.
  const int n_g = (M + RS - 1) / RS;
  const int G = (int)gridDim.x, cta = (int)blockIdx.x;
  // (The row-split gather keeps contiguous ranges: a CTA's rows then go to a
  // peer as consecutive 64-bit words, so each warp store is one 256-byte burst
  // over NVLink instead of 32 scattered words.)
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

  // Source of a quantizing prologue and its register batches: 4 lanes per
  // block (8 elements each), 64 blocks per pass; the loads of up to PB passes
  // are issued before any use, so x costs one L2 round trip per PB passes
  // (one in all for K <= 12288).
  const float* x = PRO != kProImage ? prologue_source(fz, act, nb * QK) : nullptr;
  const int lane4 = threadIdx.x & 3;
  constexpr int BPP = NCT / 4;  // blocks per pass
  constexpr int PB = 6;         // passes per batch of loads
  float4 v0[PB], v1[PB];
  auto load_batch = [&](int base) {
#pragma unroll
    for (int p = 0; p < PB; ++p) {
      const int b = base + p * BPP + (threadIdx.x >> 2);
      if (b < nb) {
        const float4* src = reinterpret_cast<const float4*>(x + (size_t)b * QK) + 2 * lane4;
        v0[p] = __ldcg(src);
        v1[p] = __ldcg(src + 1);
      } else {
        v0[p] = v1[p] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  };
  // An independent launch's x does not come from the previous kernel: its
  // first batch is requested before the barrier set-up and the ring's first
  // copies, so the L2 round trip overlaps them.
  const bool early = PRO == kProQuant && indep && fz.x_copy == nullptr;
  if (early) load_batch(0);

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
  // Stages are issued in order by lane 0; its cursor (stage index, slot,
  // chunk, row group) advances by one per copy set, without divisions.
  const uint32_t ring_u32 = smem_u32(ring), bars_u32 = smem_u32(bars);
  const int grp_step = stride ? kNcw * G : kNcw;  // row groups between a warp's consecutive groups
  int i_k = 0, i_slot = 0, i_c = 0, i_grp = group_of(warp);
  auto issue_next = [&]() {  // lane 0 only
    if (i_k >= nk) return;
    const int row0 = i_grp * RS, nrows = min(RS, M - row0);
    const int cbn = min(cb, nb - i_c * cb);
    const uint32_t full = bars_u32 + 8u * (uint32_t)(warp * NSW + i_slot);
    const uint32_t sw = ring_u32 + (uint32_t)(warp * NSW + i_slot) * (uint32_t)sh.slot_bytes;
    const uint32_t ss = sw + (uint32_t)sl_sbase;
    mbar_arrive_expect_tx(full, (uint32_t)(nrows * cbn * (UB + SS)));
    if (pk_slot) {  // whole packed rows: one copy
      bulk_g2s(sw, w + (size_t)row0 * g_wstride, (uint32_t)(nrows * g_wstride), full);
    } else if (C == 1) {
      bulk_g2s(sw, w + (size_t)row0 * row_w, (uint32_t)(nrows * row_w), full);
      bulk_g2s(ss, gsc + (size_t)row0 * row_s, (uint32_t)(nrows * row_s), full);
    } else {
      for (int r = 0; r < nrows; ++r) {
        bulk_g2s(sw + (uint32_t)(r * cb * UB), w + (size_t)(row0 + r) * g_wstride + (size_t)i_c * cb * UB,
                 (uint32_t)(cbn * UB), full);
        bulk_g2s(ss + (uint32_t)(r * cb * SS), gsc + (size_t)(row0 + r) * g_sstride + (size_t)i_c * cb * SS,
                 (uint32_t)(cbn * SS), full);
      }
    }
    ++i_k;
    if (++i_slot == NSW) i_slot = 0;
    if (++i_c == C) {
      i_c = 0;
      i_grp += grp_step;
    }
  };
  const int n_first = min(NSW, nk);
  // Weights do not depend on the previous kernel when the caller declared
  // them static: under programmatic dependent launch the rings fill while the
  // previous kernel still runs.
  if (pre && lane == 0)
    for (int t = 0; t < n_first; ++t) issue_next();
  if (!indep) pdl_wait();  // x / the image may come from the previous kernel; y may still be in use
  if (!pre && lane == 0)
    for (int t = 0; t < n_first; ++t) issue_next();

  // Tensor-parallel call number (the previous exchange's last CTA stored it).
  const unsigned seq = (fz.tp > 1 && (EPI == kEpiResidual || EPI == kEpiArgmax)) ? __ldcg(fz.ar_seq) + 1u : 0u;

  // ---------------------------------------------------------- activation image
  if (PRO != kProImage) {
    const bool copy = fz.x_copy != nullptr && blockIdx.x == 0;
    auto sq4 = [](float4 v) {
      return __fadd_rn(__fadd_rn(__fmul_rn(v.x, v.x), __fmul_rn(v.y, v.y)),
                       __fadd_rn(__fmul_rn(v.z, v.z), __fmul_rn(v.w, v.w)));
    };
    const bool held = nb <= PB * BPP;  // all of x in one batch: the norm pass's loads serve the quantize
    float rms = 1.0f;
    if (PRO == kProNorm || copy) {
      // rms = sqrt(mean(x^2) + eps), one fixed-order sum shared by every thread.
      float ssum = 0.0f;
      for (int base = 0; base < nb; base += PB * BPP) {
        if (!(early && base == 0)) load_batch(base);
#pragma unroll
        for (int p = 0; p < PB; ++p) {
          const int b = base + p * BPP + (threadIdx.x >> 2);
          if (b < nb) {
            if (PRO == kProNorm) ssum = __fadd_rn(ssum, __fadd_rn(sq4(v0[p]), sq4(v1[p])));
            if (copy) {
              float4* dst = reinterpret_cast<float4*>(fz.x_copy + (size_t)b * QK) + 2 * lane4;
              dst[0] = v0[p];
              dst[1] = v1[p];
            }
          }
        }
      }
      if (PRO == kProNorm) {
        ssum = warp_sum(ssum);
        if (lane == 0) part[warp] = ssum;
        __syncthreads();
        float tot = 0.0f;
#pragma unroll
        for (int i = 0; i < kNcw; ++i) tot = __fadd_rn(tot, part[i]);
        rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)(nb * QK)), fz.eps));
      }
    }
    for (int base = 0; base < nb; base += PB * BPP) {
      if (!((PRO == kProNorm || copy) && held) && !(early && base == 0)) load_batch(base);
#pragma unroll
      for (int p = 0; p < PB; ++p) {
        if (base + p * BPP >= nb) break;  // uniform across the CTA
        const int b = base + p * BPP + (threadIdx.x >> 2);
        float4 a = v0[p], c4 = v1[p];
        if (PRO == kProNorm && b < nb) {  // (x / rms) * w, as the reference RMSNorm
          const float4* nwp = reinterpret_cast<const float4*>(fz.norm_w + (size_t)b * QK) + 2 * lane4;
          const float4 w0 = nwp[0], w1 = nwp[1];
          a = make_float4(__fmul_rn(__fdiv_rn(a.x, rms), w0.x), __fmul_rn(__fdiv_rn(a.y, rms), w0.y),
                          __fmul_rn(__fdiv_rn(a.z, rms), w0.z), __fmul_rn(__fdiv_rn(a.w, rms), w0.w));
          c4 = make_float4(__fmul_rn(__fdiv_rn(c4.x, rms), w1.x), __fmul_rn(__fdiv_rn(c4.y, rms), w1.y),
                           __fmul_rn(__fdiv_rn(c4.z, rms), w1.z), __fmul_rn(__fdiv_rn(c4.w, rms), w1.w));
        }
        float d;
        int qsum;
        unsigned q0, q1;
        quantize_oct(a, c4, d, qsum, q0, q1);
        if (b < nb) {
          *reinterpret_cast<uint2*>(x32 + xhalf(b, lane4 >> 1) + 8 * (lane4 & 1)) = make_uint2(q0, q1);
          if (lane4 == 0) const_cast<float2*>(sdq)[b] = make_float2(d, __int_as_float(qsum));
        }
      }
    }
  } else {
    // A prepared image (48-byte slots, then the (d, q-sum) pairs): the two
    // 16-byte halves of each slot, then the pairs.
    const unsigned char* src = static_cast<const unsigned char*>(act);
    for (int i = threadIdx.x; i < 2 * nb; i += NCT)
      cp_async16(x32 + xhalf(i >> 1, i & 1), src + (size_t)(i >> 1) * 48 + (i & 1) * 16);
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
      rxa[j] = *reinterpret_cast<const uint4*>(x32 + xhalf(b, 0));
      rxb[j] = *reinterpret_cast<const uint4*>(x32 + xhalf(b, 1));
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
  // Each stage is read out of its slot into registers first (a lane's blocks
  // lane + 32 j of every row, at most NBL of them), the slot goes straight
  // back to the copy engine for stage k + NSW, and only then does the warp
  // compute: a slot is held for the shared-memory reads alone, so nearly the
  // whole ring stays in flight.
  constexpr int PR = RS;                       // rows reduced per iteration
  constexpr int QW = FMT == kFmtQ4_0 ? 1 : 2;  // uint4 of quants per block
  // Blocks a lane holds per row of a stage: the activation registers' count,
  // or the register class NBQ (Q4_0 blocks of one row) divided among the rows
  // and quant words.  The plan keeps every chunk within 32 * NBL blocks.
  constexpr int NBL = XR > 0 ? XR : (NBQ / (QW * RS) > 0 ? NBQ / (QW * RS) : 1);
  unsigned long long best_local = 0;  // kEpiArgmax: this lane's best (value, row)
  float acc[PR];
#pragma unroll
  for (int r = 0; r < PR; ++r) acc[r] = 0.0f;
  bool ok = true;
  int k = 0, slot = 0, c = 0, grp = group_of(warp);
  unsigned phase = 0;
  for (; k < nk; ++k) {
    const int np = 1;
    const uint32_t sbar = bars_u32 + 8u * (uint32_t)(warp * NSW + slot);
    const bool got = mbar_wait_bounded(sbar, phase);
    if (__any_sync(kFull, !got)) {  // every lane stops together
      ok = false;
      if (lane == 0) raise_device_error(kErrRingTimeout);
      break;
    }
    const int row0 = grp * RS, nr = min(RS, M - row0);
    const int cbn = min(cb, nb - c * cb);
    const uint32_t sw = ring_u32 + (uint32_t)(warp * NSW + slot) * (uint32_t)sh.slot_bytes;
    const uint32_t ssc = sw + (uint32_t)sl_sbase;
    const uint32_t lw = sw + (uint32_t)lane * UB, ls = ssc + (uint32_t)lane * SS;  // this lane's first block
    uint4 q[RS][NBL][QW];
    float sc[RS][NBL];
    // Loads are predicated per lane: a block beyond the stage (a short last
    // chunk, a missing last row) reads as zero weights, zero scale and zero
    // activation, whose product adds exactly nothing -- so the block dots run
    // unconditionally, as independent instructions the scheduler can interleave.
#pragma unroll
    for (int r = 0; r < RS; ++r)
#pragma unroll
      for (int j = 0; j < NBL; ++j) {
        const bool in = r < nr && lane + 32 * j < cbn;
        const uint32_t o = (uint32_t)r * (uint32_t)sl_wstride + (uint32_t)(32 * j * UB);
#pragma unroll
        for (int h = 0; h < QW; ++h) q[r][j][h] = in ? lds_v4(lw + o + 16u * h) : make_uint4(0u, 0u, 0u, 0u);
        sc[r][j] = in ? lds_scale<F16S>(ls + (uint32_t)r * (uint32_t)sl_sstride + (uint32_t)(32 * j * SS)) : 0.0f;
      }
    __syncwarp();
    if (lane == 0 && i_k < nk) {  // the slot is free again: the next stage in order goes into it
      fence_proxy_async_smem();
      issue_next();
    }
#pragma unroll
    for (int j = 0; j < NBL; ++j) {
      const int bl = lane + 32 * j;
      const bool in = bl < cbn;
      const int b = c * cb + bl;
      uint4 xa, xb;
      float xd;
      int qs8;
      if (XR > 0) {
        xa = rxa[j < XR ? j : 0];
        xb = rxb[j < XR ? j : 0];
        xd = rxd[j < XR ? j : 0];
        qs8 = rqs8[j < XR ? j : 0];
      } else {
        const uint32_t xs = smem_u32(x32);
        const int bb = in ? b : 0;
        xa = lds_v4(xs + (uint32_t)xhalf(bb, 0));
        xb = lds_v4(xs + (uint32_t)xhalf(bb, 1));
        const float2 dq = sdq[in ? b : 0];
        xd = in ? dq.x : 0.0f;
        qs8 = in ? __float_as_int(dq.y) * 8 : 0;
        if (!in) xa = xb = make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int r = 0; r < RS; ++r) {
        const int isum = FMT == kFmtQ4_0 ? q4_block_dot(q[r][j][0], xa, xb, qs8)
                                         : q8_block_dot(q[r][j][0], q[r][j][QW - 1], xa, xb);
        if (DBG && in && r < nr) isums[(size_t)(row0 + r) * nb + b] = isum;
        acc[r] = __fmaf_rn(__int2float_rn(isum), __fmul_rn(sc[r][j], xd), acc[r]);
      }
    }
    if (c == C - 1) {
      const float v = rows_reduce<PR>(acc, lane);
      constexpr int HOP = 32 / PR;  // lanes between the holders of consecutive rows
      const int rr = lane / HOP;    // row (of the PR) this lane's v totals, holders only
      const int p = rr / RS, r = rr - p * RS;
      const bool holder = (lane % HOP) == 0 && p < np && r < nr;
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
        } else if (EPI == kEpiGather) {
          y[(size_t)fz.tp_rank * M + row] = v;  // this rank's row of the full output (to the peers below)
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
    if (++slot == NSW) {  // the consumer's cursor: next slot, phase, chunk, row group
      slot = 0;
      phase ^= 1u;
    }
    if (++c == C) {
      c = 0;
      grp += grp_step;
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
  if (EPI == kEpiGather && fz.tp > 1) {
    // This CTA's rows go to every other rank's gather buffer only once the
    // previous kernel in the stream has completed.  By induction a rank's
    // stores of step t then follow its wait kernel of step t - 1, which
    // followed every peer's stores of step t - 1, which followed each peer's
    // wait of step t - 2: no rank overwrites a parity a peer still reads.
    // The step number is read after that wait, when the counter is final.
    __syncthreads();  // every warp's rows are in y
    unsigned* s_seq = reinterpret_cast<unsigned*>(part);
    if (threadIdx.x == 0) {
      pdl_wait();
      *s_seq = __ldcg(fz.ar_seq) + 1u;
    }
    __syncthreads();
    const unsigned gseq = *s_seq;
    for (int i = threadIdx.x; i < nq * RS; i += NCT) {
      const int q = i / RS, row = group_of(q) * RS + (i - q * RS);
      if (row >= M) continue;
      const unsigned long long wv =
          ((unsigned long long)gseq << 32) | __float_as_uint(__ldcg(y + (size_t)fz.tp_rank * M + row));
      for (int t = 0; t < fz.tp; ++t)
        if (t != fz.tp_rank) st_volatile_u64(xchg_word(fz, fz.xchg[t], gseq, fz.tp_rank, row), wv);
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
  int RS = 0, XR = 0, NBQ = 4, C = 1, cb = 0, NSW = 0, slot_bytes = 0;
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
bool tma_plan(int fmt, bool f16s, bool packed, int64_t nb, int epi, int smem_optin, int smem_sm, int reserved,
              TmaPlan* p) {
  const int ub = fmt == kFmtQ4_0 ? 16 : 32, ss = f16s ? 2 : 4;
  const int align = f16s ? 8 : 4;
  if (nb <= 0 || nb % align != 0) return false;  // 16-byte aligned scale rows
  if (packed && !f16s) return false;
  const size_t fixed = (size_t)kBarBytes + kPartBytes + smem_image_bytes(nb);
  const bool swiglu = epi == kEpiSwiglu;
  const int xr = nb <= 128 ? 4 : 0;
  const int forced_rs = g_opt_mv_rows.load();
  const int nsw_cap = std::max(2, std::min(kMaxNsw, g_opt_mv_slots.load() > 0 ? g_opt_mv_slots.load() : kMaxNsw));
  // The bulk-copy engine's cost is per copy (each issuing warp gets through
  // about one copy per ~0.6 us whatever its size; measured), so the plan
  // wants the most bytes per copy: whole rows (one copy per plane, a single
  // copy for packed rows) before chunks (one copy per row and plane), then
  // the deepest ring.  Rows with the activation in registers take 1 or 2 rows
  // per stage; SwiGLU stages hold whole (gate, up) pairs.
  auto try_budget = [&](size_t budget, TmaPlan* out) -> bool {
    if (budget <= fixed) return false;
    const size_t ring = budget - fixed;
    double best = -1.0;
    const int qw = fmt == kFmtQ4_0 ? 1 : 2;
    for (int rs : {2, 1})
    for (int nbq : {4, 8, 12}) {
      if (swiglu && rs < 2) continue;
      if (forced_rs > 0 && rs != forced_rs && !(swiglu && forced_rs == 1 && rs == 2)) continue;
      if (xr && fmt == kFmtQ8_0 && rs == 2 && !swiglu && forced_rs != 2) continue;  // Q8_0 registers: one row
      if (xr && nbq != 4) continue;  // the activation-register kernels hold 4 blocks per lane
      if (!xr && rs == 2 && nbq > 8) continue;  // two rows of staged blocks: at most 8 Q4_0 blocks' registers
      // blocks a lane holds per row of a stage (the kernel's NBL)
      const int nbl = xr ? xr : std::max(1, nbq / (qw * rs));
      for (int C = 1; C <= 256; ++C) {
        if (xr && C > 1) break;  // activation registers cover whole rows only
        // Chunks of a multiple of 32 blocks: lane l then always takes the
        // blocks b = l (mod 32) in ascending order, whatever the plan, so y
        // does not depend on it (bit for bit).
        const int64_t cb = C == 1 ? nb : ((nb + C - 1) / C + 31) / 32 * 32;
        if (C > 1 && (int64_t)(C - 1) * cb >= nb) continue;  // no empty last chunk
        if (cb > 32LL * nbl) continue;                       // more blocks than a lane holds
        const size_t bytes = (size_t)rs * cb * (ub + ss);
        const size_t slot = (bytes + 127) & ~(size_t)127;
        int nsw = (int)(ring / ((size_t)kNcw * slot));
        if (nsw < 2) continue;
        if (nsw > nsw_cap) nsw = nsw_cap;
        const int copies = C == 1 ? (packed ? 1 : 2) : 2 * rs;
        // Lanes compute every block slot they hold (missing blocks are zeros),
        // so util = blocks present / block slots computed.  Copies cost per
        // copy up to a few KB (measured), then bytes dominate: score the
        // bytes per copy up to 4 KB, times util; a deeper ring, more rows per
        // stage and a smaller register class break ties.
        const double util = (double)nb / ((double)C * 32.0 * nbl);
        const double per_copy = std::min(4096.0, (double)bytes / copies);
        const double score = per_copy * util + 1e-3 * nsw + 1e-6 * rs - 1e-8 * nbq;
        if (score > best) {
          best = score;
          out->NBQ = xr ? 4 : nbq;
          out->RS = rs;
          out->XR = xr;
          out->C = C;
          out->cb = (int)cb;
          out->NSW = nsw;
          out->slot_bytes = (int)slot;
          out->smem = fixed + (size_t)kNcw * nsw * slot;
        }
        break;  // the first chunk count that fits is the one with the largest copies
      }
    }
    return best >= 0.0;
  };
  // Default budget: the most that still lets two CTAs (this launch's and the
  // next one's) share an SM: half the SM's shared memory less the per-block
  // reservation and the kernel's static shared memory (256 bytes).
  size_t budget = g_opt_mv_smem_kb.load() > 0 ? (size_t)g_opt_mv_smem_kb.load() * 1024
                                               : (size_t)(smem_sm / 2 - reserved - 256);
  if (budget > (size_t)smem_optin) budget = smem_optin;
  if (try_budget(budget, p)) return true;
  return try_budget((size_t)smem_optin - 1024, p);  // room for the static shared memory
}

template <int FMT, bool F16S, bool DBG, int PRO, int EPI, int RS, int XR, int NBQ, bool PK = false>
cudaError_t launch_tma_t(const MatvecArgs& a, const TmaPlan& p, int sms, cudaStream_t stream, bool pdl) {
  auto kernel = tma_matvec_kernel<FMT, F16S, DBG, PRO, EPI, RS, XR, NBQ, PK>;
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
template <int FMT, int RS, int XR, int NBQ>
cudaError_t launch_tma_fused(const MatvecArgs& a, const TmaPlan& p, int sms, cudaStream_t stream, bool pdl) {
  const int pro = prologue_of(a);
  switch (a.epi) {
    case kEpiStore:
      if (pro == kProNorm) return launch_tma_t<FMT, true, false, kProNorm, kEpiStore, RS, XR, NBQ>(a, p, sms, stream, pdl);
      break;
    case kEpiResidual:
      if (pro == kProImage) return launch_tma_t<FMT, true, false, kProImage, kEpiResidual, RS, XR, NBQ>(a, p, sms, stream, pdl);
      if (pro == kProQuant) return launch_tma_t<FMT, true, false, kProQuant, kEpiResidual, RS, XR, NBQ>(a, p, sms, stream, pdl);
      break;
    case kEpiSwiglu:
      if constexpr (RS % 2 == 0) {
        if (pro == kProNorm) return launch_tma_t<FMT, true, false, kProNorm, kEpiSwiglu, RS, XR, NBQ>(a, p, sms, stream, pdl);
      }
      break;
    case kEpiArgmax:
      if (pro == kProNorm) return launch_tma_t<FMT, true, false, kProNorm, kEpiArgmax, RS, XR, NBQ>(a, p, sms, stream, pdl);
      break;
    default:
      break;
  }
  return cudaErrorNotSupported;
}

template <int FMT, int RS, int XR, int NBQ>
cudaError_t launch_tma_r(const MatvecArgs& a, const TmaPlan& p, int sms, cudaStream_t stream, bool pdl) {
  if (a.epi == kEpiGather) {  // row-split: fp32 x, fp16 scales (planes or packed rows)
    if (a.image || prologue_of(a) != kProQuant) return cudaErrorNotSupported;
    return a.packed ? launch_tma_t<FMT, true, false, kProQuant, kEpiGather, RS, XR, NBQ, true>(a, p, sms, stream, pdl)
                    : launch_tma_t<FMT, true, false, kProQuant, kEpiGather, RS, XR, NBQ>(a, p, sms, stream, pdl);
  }
  if (is_fused(a)) return launch_tma_fused<FMT, RS, XR, NBQ>(a, p, sms, stream, pdl);
  const bool fused = a.image == nullptr;
  if (a.packed) {
    return fused ? launch_tma_t<FMT, true, false, kProQuant, kEpiStore, RS, XR, NBQ, true>(a, p, sms, stream, pdl)
                 : launch_tma_t<FMT, true, false, kProImage, kEpiStore, RS, XR, NBQ, true>(a, p, sms, stream, pdl);
  }
  if (a.isums) {
    return fused ? launch_tma_t<FMT, false, true, kProQuant, kEpiStore, RS, XR, NBQ>(a, p, sms, stream, pdl)
                 : launch_tma_t<FMT, false, true, kProImage, kEpiStore, RS, XR, NBQ>(a, p, sms, stream, pdl);
  }
  if (a.scales_f16) {
    return fused ? launch_tma_t<FMT, true, false, kProQuant, kEpiStore, RS, XR, NBQ>(a, p, sms, stream, pdl)
                 : launch_tma_t<FMT, true, false, kProImage, kEpiStore, RS, XR, NBQ>(a, p, sms, stream, pdl);
  }
  return fused ? launch_tma_t<FMT, false, false, kProQuant, kEpiStore, RS, XR, NBQ>(a, p, sms, stream, pdl)
               : launch_tma_t<FMT, false, false, kProImage, kEpiStore, RS, XR, NBQ>(a, p, sms, stream, pdl);
}

template <int FMT>
cudaError_t launch_tma_fmt(const MatvecArgs& a, const TmaPlan& p, int sms, cudaStream_t stream, bool pdl) {
  if (p.XR) {
    if (p.RS == 2) return launch_tma_r<FMT, 2, 4, 4>(a, p, sms, stream, pdl);
    return launch_tma_r<FMT, 1, 4, 4>(a, p, sms, stream, pdl);
  }
  if (p.RS == 2) return p.NBQ == 4 ? launch_tma_r<FMT, 2, 0, 4>(a, p, sms, stream, pdl)
                                   : launch_tma_r<FMT, 2, 0, 8>(a, p, sms, stream, pdl);
  switch (p.NBQ) {
    case 4: return launch_tma_r<FMT, 1, 0, 4>(a, p, sms, stream, pdl);
    case 8: return launch_tma_r<FMT, 1, 0, 8>(a, p, sms, stream, pdl);
    default: return launch_tma_r<FMT, 1, 0, 12>(a, p, sms, stream, pdl);
  }
}

// Shared-memory figures of a device, read once.
struct SmemInfo {
  int sm = 0, reserved = 0;
};
SmemInfo smem_info(int smem_optin) {
  static std::mutex mu;
  static std::map<int, SmemInfo> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  SmemInfo s;
  if (cudaDeviceGetAttribute(&s.sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess) s.sm = smem_optin;
  if (cudaDeviceGetAttribute(&s.reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev) != cudaSuccess) s.reserved = 1024;
  cache[dev] = s;
  return s;
}

bool plan_of(const MatvecArgs& a, int smem_optin, TmaPlan* p) {
  const SmemInfo si = smem_info(smem_optin);
  return tma_plan(a.fmt, a.packed || (a.isums ? false : a.scales_f16), a.packed, a.K / QK, a.epi, smem_optin, si.sm,
                  si.reserved, p);
}

}  // namespace

#include "tma_rows.cuh"
#include "narrow_gemm.cuh"

namespace {

// Which kernel streams a launch: the fused decode-step matvecs and plain
// matvecs with rows longer than 128 blocks whose launch waits for the
// previous kernel go to the row-stage kernel; everything else (plain short
// rows, packed rows, independent launches, the row-split gather) to the
// warp-ring kernel.  Measured: 7B decode 572 -> 606 tokens/s with the fused
// K = 4096 matvecs on row stages, 465 with warp rings everywhere; plain
// dependent K = 4096 chains are a few percent faster on warp rings.
// Option "mv_kernel": 0 = that choice, 1 = warp rings always, 2 = row
// stages wherever they apply.
bool use_rows(const MatvecArgs& a, int smem_optin, RowsPlan* rp) {
  const int mode = g_opt_mv_kernel.load();
  if (mode == 1 || a.packed || a.act_independent || a.epi == kEpiGather) return false;
  if (mode == 0 && a.K / QK <= 128 && !is_fused(a)) return false;
  if (!rows_plan(a.fmt, a.isums ? false : a.scales_f16, a.K / QK, smem_optin, rp)) return false;
  if (a.epi == kEpiSwiglu && rp->R < 2) return false;
  return true;
}

}  // namespace

bool tma_matvec_supported(const MatvecArgs& a, int smem_optin) {
  if (a.fp32_act || a.M <= 0 || a.K <= 0 || a.M > 0x7fffffffLL) return false;
  // Bulk copies read from 16-byte aligned global addresses only (row starts
  // are multiples of 16 by the plan; the planes' bases must be too).
  if ((uintptr_t)a.w % 16 != 0 || (!a.packed && (uintptr_t)a.scales % 16 != 0)) return false;
  if (a.image && (uintptr_t)a.image % 16 != 0) return false;
  if (a.epi == kEpiGather) {  // row-split: fp32 x and fp16 scales only, any chain mode
    if (a.isums || a.image || !(a.packed || a.scales_f16) || prologue_of(a) != kProQuant) return false;
    if (!a.fuse || a.fuse->tp < 1 || a.fuse->tp > kMaxTp || a.fuse->tp_rank < 0 || a.fuse->tp_rank >= a.fuse->tp)
      return false;
    TmaPlan p;
    return plan_of(a, smem_optin, &p);
  }
  if (a.packed && (a.isums || is_fused(a))) return false;
  RowsPlan rp;
  if (use_rows(a, smem_optin, &rp)) {
    if (is_fused(a) && (!a.scales_f16 || a.isums || (a.epi == kEpiSwiglu && a.M % 64 != 0))) return false;
    return true;
  }
  TmaPlan p;
  if (!plan_of(a, smem_optin, &p)) return false;
  if (is_fused(a)) {
    if (!a.scales_f16 || a.isums || a.act_independent) return false;
    if (a.epi == kEpiSwiglu && a.M % 64 != 0) return false;
  }
  return true;
}

bool matvec_is_fused(const MatvecArgs& a) { return is_fused(a); }

cudaError_t launch_tma_matvec(const MatvecArgs& a, int sms, int smem_optin, cudaStream_t stream, bool pdl) {
  RowsPlan rp;
  if (use_rows(a, smem_optin, &rp)) {
    if (a.fmt == kFmtQ4_0) return launch_rows_fmt<kFmtQ4_0>(a, rp, sms, stream, pdl);
    return launch_rows_fmt<kFmtQ8_0>(a, rp, sms, stream, pdl);
  }
  TmaPlan p;
  if (!plan_of(a, smem_optin, &p)) return cudaErrorInvalidValue;
  if (a.fmt == kFmtQ4_0) return launch_tma_fmt<kFmtQ4_0>(a, p, sms, stream, pdl);
  return launch_tma_fmt<kFmtQ8_0>(a, p, sms, stream, pdl);
}

// ---------------------------------------------------------- row-split wait
// One thread per (matvec, peer rank, row) word: spin (bounded) until the word
// carries this step's sequence, store its value into the full output.  The
// last CTA advances the step counter.  The next step's matvecs may start
// (and compute) while this kernel waits; they read the counter and store to
// the peers only after it has completed (see the kEpiGather epilogue).
__global__ void __launch_bounds__(256) rowsplit_wait_kernel(const RowsplitWait w) {
  pdl_trigger();
  pdl_wait();  // this rank's matvecs of the step are done
  const unsigned seq = __ldcg(w.seq) + 1u;
  bool ok = true;
  for (int j = 0; j < w.n; ++j) {
    const long long M = w.M[j];
    const long long total = M * w.tp;  // words of all source ranks (own rows skipped)
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
      const int src = (int)(i / M);
      if (src == w.rank) continue;
      const long long row = i - (long long)src * M;
      const unsigned long long* word = w.own[j] + ((size_t)(seq & 1u) * w.tp + src) * (size_t)M + row;
      w.y_full[j][(size_t)src * M + row] = __uint_as_float(xchg_wait(word, seq, ok));
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(w.done, 1u) == gridDim.x - 1) {
      *w.seq = seq;
      atomicExch(w.done, 0u);
    }
  }
}

cudaError_t launch_rowsplit_wait(const RowsplitWait& w, int sms, cudaStream_t stream) {
  if (w.n < 0 || w.n > 8 || w.tp < 1 || w.tp > kMaxTp || w.rank < 0 || w.rank >= w.tp || !w.seq || !w.done)
    return cudaErrorInvalidValue;
  long long words = 0;
  for (int j = 0; j < w.n; ++j) {
    if (w.M[j] <= 0 || !w.own[j] || !w.y_full[j]) return cudaErrorInvalidValue;
    words += w.M[j] * (w.tp - 1);
  }
  long long grid = (words + 255) / 256;
  if (grid > sms) grid = sms;
  if (grid < 1) grid = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  RowsplitWait a = w;
  void* args[] = {(void*)&a};
  return cudaLaunchKernelExC(&cfg, (const void*)rowsplit_wait_kernel, args);
}

cudaError_t set_xchg_wait_cycles(long long cycles) {
  const long long v = cycles > 0 ? cycles : kWaitCycles;
  return cudaMemcpyToSymbol(g_xchg_wait_cycles, &v, sizeof(v));
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

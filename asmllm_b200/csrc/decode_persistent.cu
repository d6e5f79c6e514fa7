// asmllm_b200/csrc/decode_persistent.cu -- the whole batch-1 decode loop as
// one persistent cooperative kernel (sm_100a).
//
// The multi-launch decode step (decode.cu + the fused matvec modes of
// tma_matvec.cu) pays a dependency boundary per kernel: the next matvec's
// consumers wait for the previous grid to complete and flush, then fetch and
// quantize their activation, while HBM idles.  Here every CTA stays resident
// for all the steps, and the producer warp of each CTA streams weights
// through its shared-memory ring without stopping at operation boundaries --
// the next matrix's first stages are already in shared memory while the
// consumers wait at the grid barrier and build the next activation image.
//
// Program: a list of operations per decode step (per layer: q/k/v matvec with
// RMSNorm prologue, attention, o matvec + residual, gate/up matvec with
// RMSNorm prologue and SwiGLU epilogue, down matvec + residual; then the
// lm_head matvec with RMSNorm prologue and argmax), the same arithmetic as the
// multi-launch path (reference THRISHAL12345/asmllm src/runtime/generate.py:
// 255-326; each row's reduction order is the same, so the two paths agree bit
// for bit).  Operations are separated by a grid barrier: a monotonic arrival
// counter in global memory (release add per CTA; acquire polls by one thread
// per CTA, bounded).  The launch is cooperative, so every CTA is resident and
// the barrier cannot wait for a CTA that never runs.
//
// Position and tokens: step s runs position pos0 + s, where pos0 is *pos at
// launch.  The token of step s is the prompt id tokens[pos] while pos <
// n_prompt (and at s == 0), else the argmax of step s - 1, which every CTA
// decodes from the packed maximum best[(s - 1) & 1] after the barrier.  CTA 0
// records generated ids in tokens[] and leaves *pos = pos0 + n_steps.
//
// Bounded waits everywhere: the ring mbarriers and the grid barrier give up
// after ~1 s of clock cycles, set a bit in the device error word and the
// global abort word (which every poller checks), and the CTA stops.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <vector>

#include "attention.cuh"
#include "common.cuh"
#include "decode_persistent.cuh"
#include "matvec.cuh"
#include "pipeline.cuh"

namespace asmllm {

namespace {

constexpr int kNWG = 2;                  // consumer warpgroups
constexpr int kNCW = kNWG * 8;           // consumer warps
constexpr int kNCT = kNCW * 32;          // consumer threads
constexpr int kThreads = kNCT + 32;      // + 1 producer warp
constexpr int kBarBytesP = 256;          // 2 x 8 ring mbarriers (full, empty) + flags
constexpr int kPartBytesP = 2 * 2 * 8 * 2 * 4;
constexpr int kNormRegs = 2;  // float4s of x per consumer thread held in registers (K <= 4096)

struct ConsumerSync {
  __device__ __forceinline__ void operator()() const { consumer_bar_sync(kNCT); }
};

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Barrier over the consumer threads (named barrier 1) that also ORs a flag:
// every consumer gets the same answer.
__device__ __forceinline__ bool consumers_or(bool v) {
  unsigned r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.or.pred po, 1, %2, pi;\n\tselp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(r)
      : "r"((unsigned)v), "r"(kNCT)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ void red_release_gpu_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Rows [r0, r1) of an operation for this CTA: an even split of M (in units
// of G rows: 2 for the SwiGLU pairs).
__device__ __forceinline__ void op_rows(const PersistOp& op, int& r0, int& r1) {
  const int G = op.epi == kEpiSwiglu ? 2 : 1;
  r0 = G * (int)((long long)(op.M / G) * blockIdx.x / gridDim.x);
  r1 = G * (int)((long long)(op.M / G) * (blockIdx.x + 1) / gridDim.x);
}

template <int FMT>
__global__ void __launch_bounds__(kThreads, 2) decode_persistent_kernel(const PersistArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int UB = FMT == kFmtQ4_0 ? 16 : 32;  // weight bytes per block
  constexpr int UPB = FMT == kFmtQ4_0 ? 1 : 2;   // 16-byte units per block
  constexpr int SS = 2;                          // fp16 scales
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);  // full[0..NS), empty[NS..2NS)
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + kBarBytesP - 4);
  volatile int* s_flag = reinterpret_cast<volatile int*>(smem + kBarBytesP - 12);  // [2] barrier results
  volatile int* s_tok = reinterpret_cast<volatile int*>(smem + kBarBytesP - 16);
  float* part = reinterpret_cast<float*>(smem + kBarBytesP);
  unsigned char* scratch = smem + kBarBytesP + kPartBytesP;  // activation image / attention scratch
  unsigned char* ring = scratch + a.scratch_bytes;
  const int NS = a.NS, NSW = NS / kNWG;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(smem_u32(&bars[i]), 1);       // full: producer arrive + tx bytes
      mbar_init(smem_u32(&bars[NS + i]), 8);  // empty: the 8 warps of the owning warpgroup
    }
    *s_abort = 0;
    fence_mbar_init();
  }
  __syncthreads();

  const int pos0 = __ldcg(a.pos);
  // One decision for every CTA (all read the same pos0): a run that would
  // leave the cache or the token array does nothing but report it.
  if (pos0 < 0 || pos0 + a.n_steps > a.ctx || pos0 + a.n_steps >= a.max_tokens) {
    if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(a.err, kErrDecodeRange);
    return;
  }

  // ------------------------------------------------------------ producer
  if (warp == kNCW) {
    if (lane == 0) {
      int kq[kNWG] = {0, 0};  // stages issued per warpgroup
      int gsb = 0;            // stages of this CTA so far (stage t goes to warpgroup t & 1)
      bool stop = false;
      for (int st = 0; st < a.n_steps && !stop; ++st) {
        for (int oi = 0; oi < a.n_ops && !stop; ++oi) {
          const PersistOp& op = a.ops[oi];
          if (op.kind != kOpMatvec) continue;
          int r0, r1;
          op_rows(op, r0, r1);
          const int R = op.R;
          const size_t row_w = (size_t)op.nb * UB, row_s = (size_t)op.nb * SS;
          const int S = (r1 - r0 + R - 1) / R;
          for (int s = 0; s < S; ++s) {
            if (*s_abort) {
              stop = true;
              break;
            }
            const int g = (gsb + s) & 1, k = kq[g]++;
            const int slot = g * NSW + k % NSW, round = k / NSW;
            if (round > 0 && !mbar_wait_bounded(smem_u32(&bars[NS + slot]), (round - 1) & 1)) {
              atomicOr(a.err, kErrRingTimeout);
              atomicExch(a.abort, 1u);
              *s_abort = 1;
              stop = true;
              break;
            }
            const int row0 = r0 + s * R;
            const int nrows = min(R, r1 - row0);
            const uint32_t full = smem_u32(&bars[slot]);
            mbar_arrive_expect_tx(full, (uint32_t)((size_t)nrows * (row_w + row_s)));
            const uint32_t dst = smem_u32(ring + (size_t)slot * a.slot_bytes);
            bulk_g2s(dst, op.w + (size_t)row0 * row_w, (uint32_t)((size_t)nrows * row_w), full);
            bulk_g2s(dst + (uint32_t)((size_t)R * row_w), reinterpret_cast<const unsigned char*>(op.s) + (size_t)row0 * row_s,
                     (uint32_t)((size_t)nrows * row_s), full);
          }
          gsb += S;
        }
      }
      if (stop) {  // let the copies already issued land before the CTA exits
        for (int g = 0; g < kNWG; ++g)
          for (int k = kq[g] > NSW ? kq[g] - NSW : 0; k < kq[g]; ++k)
            mbar_wait_bounded(smem_u32(&bars[g * NSW + k % NSW]), (k / NSW) & 1);
      }
    }
    return;
  }

  // ------------------------------------------------------------ consumers
  const int tid = threadIdx.x;  // 0 .. kNCT-1
  const int wg = warp >> 3, wi = warp & 7;
  int kg = 0;    // stages consumed by this warp's warpgroup
  int gsb = 0;   // stages of this CTA so far
  unsigned opi = 0;  // operations completed by the whole grid before the current one
  bool dead = false;

  // Grid barrier: all CTAs arrived for `target` operations.  Thread 0 polls
  // (acquire); the answer reaches every consumer through shared memory.
  auto grid_wait = [&](unsigned target) -> bool {
    const int fi = opi & 1;  // alternating flag: a slow reader of the last answer is never overwritten
    if (tid == 0) {
      int ok = 1;
      if (ld_acquire_gpu(a.sync) < target) {
        const long long t0 = clock64();
        while (ld_acquire_gpu(a.sync) < target) {
          if (ld_acquire_gpu(a.abort) || clock64() - t0 > kWaitCycles) {
            ok = 0;
            break;
          }
          __nanosleep(32);
        }
      }
      if (!ok) {
        atomicOr(a.err, kErrRingTimeout);
        atomicExch(a.abort, 1u);
        *s_abort = 1;
      }
      s_flag[fi] = ok;
    }
    consumer_bar_sync(kNCT);
    return s_flag[fi] != 0;
  };
  // Every consumer's writes of this operation are done (the CTA barrier
  // orders them before thread 0's release, and a release is cumulative), one
  // decision for the whole CTA on whether to go on (a warpgroup may have
  // stopped alone), then the arrival.
  auto grid_arrive = [&]() {
    dead = consumers_or(dead || *s_abort);
    if (tid == 0) red_release_gpu_add(a.sync, 1u);
  };

  for (int st = 0; st < a.n_steps && !dead; ++st) {
    const int pos = pos0 + st;
    for (int oi = 0; oi < a.n_ops && !dead; ++oi) {
      const PersistOp& op = a.ops[oi];
      if (op.kind == kOpAttention && (int)blockIdx.x < a.n_heads) {
        // cache rows [0, pos) of this head were written in earlier steps
        attn_prefetch_rows<kNCT>(op.kc, op.vc, pos, (int)blockIdx.x / (a.n_heads / a.n_kv), a.n_kv, tid);
      }
      // RMSNorm weights do not depend on the previous operation: this thread's
      // share (float4 i = tid + kNCT * j) is loaded before the wait.
      const bool norm_regs = op.kind == kOpMatvec && op.pro == kProNorm && op.nb * 8 <= kNormRegs * kNCT;
      float4 nw[kNormRegs];
      if (norm_regs) {
#pragma unroll
        for (int j = 0; j < kNormRegs; ++j) {
          const int i = tid + kNCT * j;
          nw[j] = i < op.nb * 8 ? reinterpret_cast<const float4*>(op.norm_w)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      if (opi > 0 && !grid_wait(opi * gridDim.x)) {
        dead = true;
        break;
      }
      if (op.kind == kOpAttention) {
        if (op.first_of_step && blockIdx.x == 0 && tid == 0 && st > 0) {
          // every CTA has read best[(st-1)&1] (operation 0's prologue): clear it
          // for step st + 1, and record the token step st - 1 produced.
          if (pos >= a.n_prompt) a.tokens[pos] = *s_tok;
          a.best[(st - 1) & 1] = 0ull;
        }
        if ((int)blockIdx.x < a.n_heads) {
          const AttnSmem sm = attn_smem_carve<256>(scratch);
          attention_head<256>(a.qkv, op.kc, op.vc, a.rope, pos, (int)blockIdx.x, a.n_heads, a.n_kv, a.sqrt_hd,
                              a.img_attn, sm, tid, ConsumerSync{}, a.xr, a.img_attn_stride);
        }
        grid_arrive();
        ++opi;
        continue;
      }

      // ---------------------------------------------------------- matvec
      int r0, r1;
      op_rows(op, r0, r1);
      const int R = op.R, nb = op.nb, M = op.M;
      const size_t row_w = (size_t)nb * UB, row_s = (size_t)nb * SS;
      const int S = (r1 - r0 + R - 1) / R;
      const int NRG = R / 2, WPG = 8 / NRG;  // two rows per warp
      const int rg = wi / WPG, sg = wi - rg * WPG;
      unsigned char* img = scratch;

      // Prologue: the Q8_0 image of this operation's activation.
      if (op.pro == kProImage) {
        const int n16 = (int)(act_image_bytes(nb) / 16);
        const unsigned char* src = op.image + (size_t)(blockIdx.x % a.xr) * op.image_stride;
        for (int i = tid; i < n16; i += kNCT) cp_async16(img + 16 * i, src + 16 * i);
        cp_async_wait_all();
      } else {
        const float* x = op.x + (size_t)(blockIdx.x % a.xr) * a.x_stride;
        if (op.from_embed) {
          // this step's token: a prompt id, or the argmax of the previous step
          int tok;
          if (st == 0 || pos < a.n_prompt) {
            tok = __ldcg(a.tokens + pos);
          } else {
            tok = argmax_row(__ldcg(a.best + ((st - 1) & 1)));
          }
          if (tok < 0 || tok >= a.vocab) {
            if (tid == 0) atomicOr(a.err, kErrDecodeRange);
            tok = 0;
          }
          if (tid == 0) *s_tok = tok;
          x = a.embed + (size_t)tok * (nb * QK);
        }
        const bool copy = op.from_embed && blockIdx.x == 0;  // the residual stream starts as the embedding
        const int lane8 = tid & 7;
        constexpr int BPP = kNCT / 8;
        float rms = 1.0f;
        if (norm_regs) {
          // One load of x into registers: float4 i = tid + kNCT * j is lane
          // (tid & 7) of block i / 8, the quantize's own layout.  The same sums
          // in the same order as the two-pass form below.
          float4 v[kNormRegs];
#pragma unroll
          for (int j = 0; j < kNormRegs; ++j) {
            const int i = tid + kNCT * j;
            v[j] = i < nb * 8 ? __ldcg(reinterpret_cast<const float4*>(x) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
          }
          float ss = 0.0f;
#pragma unroll
          for (int j = 0; j < kNormRegs; ++j) {
            const int i = tid + kNCT * j;
            if (i < nb * 8) {
              ss = __fadd_rn(ss, __fadd_rn(__fadd_rn(__fmul_rn(v[j].x, v[j].x), __fmul_rn(v[j].y, v[j].y)),
                                           __fadd_rn(__fmul_rn(v[j].z, v[j].z), __fmul_rn(v[j].w, v[j].w))));
              if (copy)
                for (int r = 0; r < a.xr; ++r) reinterpret_cast<float4*>(a.x + (size_t)r * a.x_stride)[i] = v[j];
            }
          }
          ss = warp_sum(ss);
          if (lane == 0) part[warp] = ss;
          consumer_bar_sync(kNCT);
          float tot = 0.0f;
#pragma unroll
          for (int i = 0; i < kNCW; ++i) tot = __fadd_rn(tot, part[i]);
          rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)(nb * QK)), a.eps));
#pragma unroll
          for (int j = 0; j < kNormRegs; ++j) {
            if (kNCT * j >= nb * 8) break;  // uniform
            const int i = tid + kNCT * j, b = i >> 3;
            const float4 e = make_float4(__fmul_rn(__fdiv_rn(v[j].x, rms), nw[j].x),
                                         __fmul_rn(__fdiv_rn(v[j].y, rms), nw[j].y),
                                         __fmul_rn(__fdiv_rn(v[j].z, rms), nw[j].z),
                                         __fmul_rn(__fdiv_rn(v[j].w, rms), nw[j].w));
            float d;
            int qsum;
            const unsigned q = quantize_quad(e, d, qsum);
            if (b < nb) {
              reinterpret_cast<unsigned*>(img + b * 48)[lane8] = q;
              if (lane8 == 0) reinterpret_cast<float2*>(img + (size_t)nb * 48)[b] = make_float2(d, __int_as_float(qsum));
            }
          }
        } else if (op.pro == kProNorm) {
          float ss = 0.0f;
          for (int i = tid; i < nb * 8; i += kNCT) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(x) + i);
            ss = __fadd_rn(ss, __fadd_rn(__fadd_rn(__fmul_rn(v.x, v.x), __fmul_rn(v.y, v.y)),
                                         __fadd_rn(__fmul_rn(v.z, v.z), __fmul_rn(v.w, v.w))));
            if (copy)
              for (int r = 0; r < a.xr; ++r) reinterpret_cast<float4*>(a.x + (size_t)r * a.x_stride)[i] = v;
          }
          ss = warp_sum(ss);
          if (lane == 0) part[warp] = ss;
          consumer_bar_sync(kNCT);
          float tot = 0.0f;
#pragma unroll
          for (int i = 0; i < kNCW; ++i) tot = __fadd_rn(tot, part[i]);
          rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)(nb * QK)), a.eps));
        } else if (copy) {
          for (int i = tid; i < nb * 8; i += kNCT)
            for (int r = 0; r < a.xr; ++r)
              reinterpret_cast<float4*>(a.x + (size_t)r * a.x_stride)[i] = __ldcg(reinterpret_cast<const float4*>(x) + i);
        }
        for (int base = 0; !norm_regs && base < nb; base += 4 * BPP) {
          float4 v[4];
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const int b = base + p * BPP + (tid >> 3);
            v[p] = b < nb ? __ldcg(reinterpret_cast<const float4*>(x + (size_t)b * QK) + lane8)
                          : make_float4(0.f, 0.f, 0.f, 0.f);
            if (op.pro == kProNorm && b < nb) {
              const float4 nw = reinterpret_cast<const float4*>(op.norm_w + (size_t)b * QK)[lane8];
              v[p] = make_float4(__fmul_rn(__fdiv_rn(v[p].x, rms), nw.x), __fmul_rn(__fdiv_rn(v[p].y, rms), nw.y),
                                 __fmul_rn(__fdiv_rn(v[p].z, rms), nw.z), __fmul_rn(__fdiv_rn(v[p].w, rms), nw.w));
            }
          }
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const int b = base + p * BPP + (tid >> 3);
            if (base + p * BPP >= nb) break;
            float d;
            int qsum;
            const unsigned q = quantize_quad(v[p], d, qsum);
            if (b < nb) {
              reinterpret_cast<unsigned*>(img + b * 48)[lane8] = q;
              if (lane8 == 0) reinterpret_cast<float2*>(img + (size_t)nb * 48)[b] = make_float2(d, __int_as_float(qsum));
            }
          }
        }
      }
      consumer_bar_sync(kNCT);

      // Stages of this warpgroup: global stage index gsb + s owned by (gsb + s) & 1.
      const float2* sdq = reinterpret_cast<const float2*>(img + (size_t)nb * 48);
      unsigned long long best_local = 0;
      for (int s = (wg - gsb) & 1; s < S; s += 2) {
        const int slot = wg * NSW + kg % NSW;
        const int par = (kg / NSW) & 1;
        const int kpar = kg & 1;
        ++kg;
        const bool ok = mbar_wait_bounded(smem_u32(&bars[slot]), par);
        if (!ok) atomicOr(a.err, kErrRingTimeout);
        const int row0 = r0 + s * R;
        const int nrows = min(R, r1 - row0);
        const unsigned char* stg = ring + (size_t)slot * a.slot_bytes;
        const int rbase = rg * 2;
        const int nr = nrows - rbase;
        float acc0 = 0.0f, acc1 = 0.0f;
        if (ok && nr > 0) {
          const unsigned char* w0 = stg + (size_t)rbase * row_w;
          const unsigned char* s0 = stg + (size_t)R * row_w + (size_t)rbase * row_s;
          if (FMT == kFmtQ4_0) {
#pragma unroll 4
            for (int b = sg * 32 + lane; b < nb; b += 32 * WPG) {
              const uint4* xp = reinterpret_cast<const uint4*>(img + b * 48);
              const uint4 xa = xp[0], xb = xp[1];
              const float2 dq = sdq[b];
              const int qsum8 = __float_as_int(dq.y) * 8;
#pragma unroll
              for (int r = 0; r < 2; ++r) {
                if (r < nr) {
                  const uint4 q = *reinterpret_cast<const uint4*>(w0 + r * row_w + b * 16);
                  const float sc = __half2float(*reinterpret_cast<const __half*>(s0 + r * row_s + b * 2));
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
                  const float t = __fmaf_rn(__int2float_rn(isum), __fmul_rn(sc, dq.x), r == 0 ? acc0 : acc1);
                  if (r == 0) acc0 = t; else acc1 = t;
                }
              }
            }
          } else {
            const int NU = nb * UPB;
#pragma unroll 4
            for (int u0 = sg * 32; u0 < NU; u0 += 32 * WPG) {
              const int u = u0 + lane;
              const bool valid = u < NU;
              const int b = u >> 1;
              uint4 xa = make_uint4(0u, 0u, 0u, 0u);
              float xd = 0.0f;
              if (valid) {
                xa = *reinterpret_cast<const uint4*>(img + b * 48 + (u & 1) * 16);
                xd = sdq[b].x;
              }
#pragma unroll
              for (int r = 0; r < 2; ++r) {
                if (r < nr) {
                  uint4 q = make_uint4(0u, 0u, 0u, 0u);
                  float sc = 0.0f;
                  if (valid) {
                    q = *reinterpret_cast<const uint4*>(w0 + r * row_w + u * 16);
                    sc = __half2float(*reinterpret_cast<const __half*>(s0 + r * row_s + b * 2));
                  }
                  int p = 0;
                  p = dp4a_ss((int)q.x, (int)xa.x, p);
                  p = dp4a_ss((int)q.y, (int)xa.y, p);
                  p = dp4a_ss((int)q.z, (int)xa.z, p);
                  p = dp4a_ss((int)q.w, (int)xa.w, p);
                  const int isum = p + __shfl_xor_sync(kFull, p, 1);
                  if (valid && !(lane & 1)) {
                    const float t = __fmaf_rn(__int2float_rn(isum), __fmul_rn(sc, xd), r == 0 ? acc0 : acc1);
                    if (r == 0) acc0 = t; else acc1 = t;
                  }
                }
              }
            }
          }
        }
        // two-row butterfly: lane 0 ends with row 0, lane 16 with row 1
        const bool upper = lane & 16;
        float v = upper ? acc1 : acc0;
        v += __shfl_xor_sync(kFull, upper ? acc0 : acc1, 16);
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&bars[NS + slot]));  // this warp is done with the slot
        float* pb = part + (kpar * kNWG + wg) * 16;                 // [8 warps][2 rows]
        if ((lane & 15) == 0) pb[wi * 2 + (lane >> 4)] = v;
        const bool stop = wg_bar_or(wg, !ok || *s_abort);
        if (stop) {
          *s_abort = 1;
          atomicExch(a.abort, 1u);
          dead = true;
          break;
        }
        if (sg == 0) {
          const float* pr = pb + rg * WPG * 2;
          if (op.epi == kEpiSwiglu) {
            if (nr >= 2 && lane == 0) {
              float gt = pr[0], up = pr[1];
              for (int j = 1; j < WPG; ++j) {
                gt += pr[j * 2];
                up += pr[j * 2 + 1];
              }
              __stcg(a.h + ((row0 + rbase) >> 1), __fmul_rn(__fdiv_rn(gt, __fadd_rn(1.0f, expf(-gt))), up));
            }
          } else if (lane < 2 && lane < nr) {
            float t = pr[lane];
            for (int j = 1; j < WPG; ++j) t += pr[j * 2 + lane];
            const int row = row0 + rbase + lane;
            if (op.epi == kEpiResidual) {
              const float nv = __fadd_rn(__ldcg(op.y + row), t);  // y is x: every replica
              for (int r = 0; r < a.xr; ++r) op.y[(size_t)r * a.x_stride + row] = nv;
            } else {
              op.y[row] = t;
              if (op.epi == kEpiArgmax && t == t) {
                const unsigned long long key = argmax_key(t, row);
                best_local = key > best_local ? key : best_local;
              }
            }
          }
        }
      }
      // Both warpgroups leave the stage loop together on an abort (the flag is
      // shared); a CTA that is dead still arrives so no barrier waits on it
      // for long, then stops.
      if (op.epi == kEpiArgmax) {
        unsigned long long b = best_local;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const unsigned long long t = __shfl_xor_sync(kFull, b, o);
          b = t > b ? t : b;
        }
        consumer_bar_sync(kNCT);
        unsigned long long* wbest = reinterpret_cast<unsigned long long*>(part);
        if (lane == 0) wbest[warp] = b;
        consumer_bar_sync(kNCT);
        if (tid == 0) {
          unsigned long long m = 0;
          for (int i = 0; i < kNCW; ++i) m = wbest[i] > m ? wbest[i] : m;
          if (m) atomicMax(a.best + (st & 1), m);
        }
      }
      if (op.epi == kEpiSwiglu) {
        // This CTA's h values are stored.  One arrival per Q8_0 block it
        // touched: lane i of warp 0 adds this CTA's pair count for block b0 + i
        // with an acq_rel atomic (release of this CTA's h after the barrier,
        // acquire of the other CTAs'), and warp 0 quantizes every block whose
        // arrival completed its 32 values.
        const int p0 = r0 >> 1, p1 = r1 >> 1;
        const int b0 = p0 >> 5, nblk = p1 > p0 ? ((p1 + 31) >> 5) - b0 : 0;
        consumer_bar_sync(kNCT);
        if (warp == 0) {
          for (int c0 = 0; c0 < nblk; c0 += 32) {
            bool last = false;
            if (c0 + lane < nblk) {
              const int blk = b0 + c0 + lane;
              const unsigned n = (unsigned)(min(p1, (blk + 1) * 32) - max(p0, blk * 32));
              last = atom_add_acq_rel_gpu(a.counters + blk, n) + n == 32u;
            }
            unsigned ballot = __ballot_sync(kFull, last);
            __syncwarp();  // the acquiring lane's view reaches the lanes that read h
            while (ballot) {
              const int qb = b0 + c0 + __ffs(ballot) - 1;
              ballot &= ballot - 1;
              const float4 hv4 = __ldcg(reinterpret_cast<const float4*>(a.h + (size_t)qb * QK) + (lane & 7));
              float d;
              int qsum;
              const unsigned q = quantize_quad(hv4, d, qsum);
              for (int r = 0; r < a.xr; ++r) {
                unsigned char* im = a.img_h + (size_t)r * a.img_h_stride;
                if (lane < 8) reinterpret_cast<unsigned*>(im + (size_t)qb * 48)[lane] = q;
                if (lane == 0) reinterpret_cast<float2*>(im + (size_t)(M >> 6) * 48)[qb] = make_float2(d, __int_as_float(qsum));
              }
              if (lane == 0) a.counters[qb] = 0u;
            }
          }
        }
      }
      gsb += S;
      grid_arrive();
      ++opi;
    }
  }

  // The last step's token and the final position (CTA 0, after every CTA's
  // last operation).
  if (!dead && blockIdx.x == 0) {
    if (grid_wait(opi * gridDim.x) && tid == 0) {
      const int last = pos0 + a.n_steps - 1;
      const unsigned long long b = __ldcg(a.best + ((a.n_steps - 1) & 1));
      if (last + 1 >= a.n_prompt) a.tokens[last + 1] = argmax_row(b);
      a.best[(a.n_steps - 1) & 1] = 0ull;
      *a.pos = pos0 + a.n_steps;
    }
  }
}

// ==========================================================================
// Host side
// ==========================================================================
std::mutex g_mu;

template <int FMT>
cudaError_t launch_t(const PersistArgs& a, size_t smem, int sms, int per_sm, cudaStream_t stream) {
  auto kernel = decode_persistent_kernel<FMT>;
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (dev < 64 && !attr_done[dev]) {
      int optin = 0;
      cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
      cudaFuncAttributes fa;
      cudaError_t e = cudaFuncGetAttributes(&fa, kernel);
      if (e != cudaSuccess) return e;
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)fa.sharedSizeBytes);
      if (e != cudaSuccess) return e;
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
      if (e != cudaSuccess) return e;
      attr_done[dev] = true;
    }
  }
  int occ = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, kThreads, smem);
  if (e != cudaSuccess) return e;
  if (occ < 1) return cudaErrorNotSupported;
  const int grid = sms * (per_sm < occ ? per_sm : occ);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, a);
}

}  // namespace

size_t persist_attn_scratch_bytes(int ctx) {
  return attn_smem_bytes_fixed<256>() + 16 + (size_t)ctx * sizeof(float);
}

// Plans the shared memory: scratch (largest activation image or the attention
// scratch), then NS ring slots of the largest stage.  Two CTAs per SM when it
// fits in about 100 KB, else one CTA with the opt-in maximum.
bool persist_plan(PersistArgs& a, const std::vector<PersistOp>& ops, int fmt, int smem_optin, int* per_sm,
                  size_t* smem) {
  const int ub = fmt == kFmtQ4_0 ? 16 : 32;
  size_t scratch = persist_attn_scratch_bytes(a.ctx), slot = 0;
  for (const PersistOp& op : ops) {
    if (op.kind != kOpMatvec) continue;
    scratch = std::max(scratch, act_image_bytes(op.nb));
    slot = std::max(slot, (size_t)op.R * (size_t)op.nb * (ub + 2));
  }
  scratch = (scratch + 127) & ~(size_t)127;
  slot = (slot + 127) & ~(size_t)127;
  const size_t fixed = kBarBytesP + kPartBytesP + scratch;
  for (int cand = 2; cand >= 1; --cand) {
    const size_t budget = cand == 2 ? 100 * 1024 : (size_t)smem_optin - 1024;
    if (budget <= fixed) continue;
    size_t ns = (budget - fixed) / slot;
    if (ns > 8) ns = 8;
    ns -= ns % kNWG;
    if (ns < 2 * kNWG) continue;
    a.NS = (int)ns;
    a.slot_bytes = (int)slot;
    a.scratch_bytes = (int)scratch;
    *per_sm = cand;
    *smem = fixed + ns * slot;
    return true;
  }
  return false;
}

cudaError_t launch_decode_persistent(const PersistArgs& a, int fmt, size_t smem, int sms, int per_sm,
                                     cudaStream_t stream) {
  return fmt == kFmtQ4_0 ? launch_t<kFmtQ4_0>(a, smem, sms, per_sm, stream)
                         : launch_t<kFmtQ8_0>(a, smem, sms, per_sm, stream);
}

}  // namespace asmllm


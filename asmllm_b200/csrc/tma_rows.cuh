// asmllm_b200/csrc/tma_rows.cuh -- the row-stage variant of the bulk-copy
// matvec: one producer warp fills a CTA-wide ring with stages of R whole rows
// and every consumer warp works on every stage.  Included by tma_matvec.cu
// only (it shares that unit's error word, exchange and argmax helpers).
//
// Same semantics as tma_matvec_kernel: the activation image is the Q8_0
// quantization of x (bit-exact), each (row, block) int32 dot is exact, and
// y[r] = sum_b fma(float(isum), wd * xd) in a fixed order.
//
// Why two kernels: the warp-ring kernel gives each warp its own ring of small
// stages, which keeps rows of up to 128 blocks (K <= 4096) streaming at full
// rate and lets consecutive launches overlap.  For longer rows its stages are
// either whole rows (one or two per warp in flight) or chunks (many small
// copies), and in a chain of dependent launches (a decode step, where every
// matvec reads the previous one's output) it measured 20-40 % slower than
// this design, whose stages are ~16 KB of whole rows shared by 16 warps:
//   * The matrix is cut into stages of R whole rows (R in {8,4,2,1}, the
//     largest with at most 16 KB of quants); a stage is two cp.async.bulk
//     copies, the R rows' quants and their scales.  CTA c takes stages
//     c, c + grid, ... or one contiguous row range (SwiGLU pairs, the
//     tensor-parallel exchange).
//   * 1 producer warp: lane 0 issues stages into the rings of 2 warpgroups
//     (full / empty mbarriers, expect_tx), before griddepcontrol.wait when the
//     weights are static.
//   * Each warpgroup of 8 consumer warps owns alternate stages.  8/RG warps
//     share a group of RW = 2 rows: each takes a strided subset of the blocks,
//     reduces across lanes, and the slices' partials are summed in slice order
//     through shared memory (deterministic).
//   * Every mbarrier wait is bounded; on timeout the kernel sets bit 0 of
//     g_device_error, stops, lets the copies it issued land, and returns.

namespace {
constexpr int kRowsBarBytes = 256;               // 2 x 14 mbarriers + abort flag
constexpr int kRowsPartBytes = 2 * 2 * 8 * 2 * 4;  // row partials [2 parities][2 warpgroups][8 warps][2 rows]
constexpr int kRowsNwg = 2;                       // consumer warpgroups
constexpr int kRowsStageKb = 16;                  // quant bytes per stage (target)
constexpr int kRowsSmemKb = 100;                  // shared memory per CTA (two CTAs per SM)
constexpr int kRowsMaxSlots = 8;                  // ring slots per CTA (cap)
}  // namespace

template <int FMT, bool F16S, bool DBG, int PRO, int EPI, int NWG, int R, int RW>
__global__ void __launch_bounds__((NWG * 8 + 1) * 32, 2)
tma_rows_kernel(const uint8_t* __restrict__ w, const void* __restrict__ scales, const void* __restrict__ act,
                float* __restrict__ y, int M, int nb, int32_t* __restrict__ isums, int NS, int pre,
                const MvFuse fz) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int UB = FMT == kFmtQ4_0 ? 16 : 32;  // weight bytes per block
  constexpr int SS = F16S ? 2 : 4;               // scale bytes per block
  constexpr int UPB = FMT == kFmtQ4_0 ? 1 : 2;   // 16-byte units per block
  constexpr int NCW = NWG * 8;                   // consumer warps
  constexpr int NCT = NCW * 32;                  // consumer threads

  // Shared layout: [barriers + abort flag | row partials | activation image | ring]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);  // full[0..NS), empty[NS..2NS)
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + kRowsBarBytes - 4);
  float* part = reinterpret_cast<float*>(smem + kRowsBarBytes);  // [2][NWG][8][2] partial row sums
  unsigned char* img = smem + kRowsBarBytes + kRowsPartBytes;
  const size_t img_bytes = (act_image_bytes(nb) + 127) & ~(size_t)127;
  unsigned char* stages = img + img_bytes;
  const size_t row_w = (size_t)nb * UB, row_s = (size_t)nb * SS;
  const size_t stage_bytes = (size_t)R * (row_w + row_s);  // R whole rows, then their scales
  constexpr int NRG = R / RW;                              // row groups per stage (RW rows each)
  constexpr int WPG = 8 / NRG;                             // warps sharing a row group (block slices)
  const int NU = nb * UPB;                                 // 16-byte units per row
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
  // contiguous span.  SwiGLU and the tensor-parallel exchange need a
  // contiguous row range per CTA.
  const bool stride = EPI == kEpiStore || EPI == kEpiArgmax || (EPI == kEpiResidual && fz.tp <= 1);
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
      int s = 0;
      for (; s < S && !*s_abort; ++s) {
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
  const int rg = wi / WPG, sg = wi - rg * WPG;  // this warp's row group in a stage and its block slice
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
              const float sc = smem_scale<F16S>(s0 + r * row_s + b * SS);
              const int isum = q4_block_dot(q, xa, xb, qsum8);
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
                sc = smem_scale<F16S>(s0 + r * row_s + b * SS);
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
    const bool stop = WPG < 8 ? group_bar_or(4 + wg * NRG + rg, 32 * WPG, !ok || *s_abort)
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

// ---------------------------------------------------------------- host side
namespace {

struct RowsPlan {
  int R = 0, NS = 0;
  size_t smem = 0;
};

// Stage = R whole consecutive rows (R in {8, 4, 2, 1}, the largest whose
// quants fit in 16 KB); the ring takes what is left of ~100 KB after the
// activation image (two CTAs per SM), else the whole opt-in shared memory.
bool rows_plan(int fmt, bool f16s, int64_t nb, int smem_optin, RowsPlan* p) {
  const int ub = fmt == kFmtQ4_0 ? 16 : 32, ss = f16s ? 2 : 4;
  if (nb <= 0 || nb % (f16s ? 8 : 4) != 0) return false;  // 16-byte aligned scale rows
  const size_t row_w = (size_t)nb * ub, row_s = (size_t)nb * ss;
  if (row_w > 24 * 1024) return false;
  int R = 8;
  while (R > 1 && (size_t)R * row_w > (size_t)kRowsStageKb * 1024) R /= 2;
  const size_t stage = (size_t)R * (row_w + row_s);
  const size_t img = (act_image_bytes(nb) + 127) & ~(size_t)127;
  size_t budget = (size_t)kRowsSmemKb * 1024;
  if (budget > (size_t)smem_optin) budget = smem_optin;
  const size_t fixed = kRowsBarBytes + kRowsPartBytes + img;
  auto slots = [&](size_t b) -> size_t {
    if (b < fixed) return 0;
    size_t n = (b - fixed) / stage;
    if (n > (size_t)kRowsMaxSlots) n = kRowsMaxSlots;
    return n - n % kRowsNwg;  // equal rings per warpgroup
  };
  size_t ns = slots(budget);
  if (ns < 2 * kRowsNwg) ns = slots((size_t)smem_optin - 1024);  // room for the static shared memory
  if (ns < 2 * kRowsNwg) return false;
  p->R = R;
  p->NS = (int)ns;
  p->smem = fixed + ns * stage;
  return true;
}

template <int FMT, bool F16S, bool DBG, int PRO, int EPI, int R>
cudaError_t launch_rows_t(const MatvecArgs& a, const RowsPlan& p, int sms, cudaStream_t stream, bool pdl) {
  constexpr int RW = R >= 2 ? 2 : 1;
  auto kernel = tma_rows_kernel<FMT, F16S, DBG, PRO, EPI, kRowsNwg, R, RW>;
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
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)fa.sharedSizeBytes);
      if (e != cudaSuccess) return e;
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
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
  MvFuse fz = a.fuse ? *a.fuse : MvFuse{};
  void* args[] = {(void*)&w, (void*)&s, (void*)&act, (void*)&y, (void*)&M, (void*)&nb,
                  (void*)&isums, (void*)&NS, (void*)&pre, (void*)&fz};
  // Persistent grid: two CTAs per SM when they fit beside each other.
  const int smem_sm = smem_info(0).sm;
  int per_sm = smem_sm > 0 ? (int)((size_t)smem_sm / (p.smem + 1024)) : 1;
  per_sm = per_sm < 1 ? 1 : per_sm > 2 ? 2 : per_sm;
  long long grid = (long long)sms * per_sm;
  const long long groups = (M + R - 1) / R;
  if (grid > groups) grid = groups;
  if (grid < 1) grid = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3((kRowsNwg * 8 + 1) * 32);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelExC(&cfg, (const void*)kernel, args);
}

template <int FMT, int R>
cudaError_t launch_rows_r(const MatvecArgs& a, const RowsPlan& p, int sms, cudaStream_t stream, bool pdl) {
  const int pro = prologue_of(a);
  if (is_fused(a)) {
    switch (a.epi) {
      case kEpiStore:
        if (pro == kProNorm) return launch_rows_t<FMT, true, false, kProNorm, kEpiStore, R>(a, p, sms, stream, pdl);
        break;
      case kEpiResidual:
        if (pro == kProImage) return launch_rows_t<FMT, true, false, kProImage, kEpiResidual, R>(a, p, sms, stream, pdl);
        if (pro == kProQuant) return launch_rows_t<FMT, true, false, kProQuant, kEpiResidual, R>(a, p, sms, stream, pdl);
        break;
      case kEpiSwiglu:
        if constexpr (R >= 2) {
          if (pro == kProNorm) return launch_rows_t<FMT, true, false, kProNorm, kEpiSwiglu, R>(a, p, sms, stream, pdl);
        }
        break;
      case kEpiArgmax:
        if (pro == kProNorm) return launch_rows_t<FMT, true, false, kProNorm, kEpiArgmax, R>(a, p, sms, stream, pdl);
        break;
      default:
        break;
    }
    return cudaErrorNotSupported;
  }
  const bool fused = a.image == nullptr;
  if (a.isums) {
    return fused ? launch_rows_t<FMT, false, true, kProQuant, kEpiStore, R>(a, p, sms, stream, pdl)
                 : launch_rows_t<FMT, false, true, kProImage, kEpiStore, R>(a, p, sms, stream, pdl);
  }
  if (a.scales_f16) {
    return fused ? launch_rows_t<FMT, true, false, kProQuant, kEpiStore, R>(a, p, sms, stream, pdl)
                 : launch_rows_t<FMT, true, false, kProImage, kEpiStore, R>(a, p, sms, stream, pdl);
  }
  return fused ? launch_rows_t<FMT, false, false, kProQuant, kEpiStore, R>(a, p, sms, stream, pdl)
               : launch_rows_t<FMT, false, false, kProImage, kEpiStore, R>(a, p, sms, stream, pdl);
}

template <int FMT>
cudaError_t launch_rows_fmt(const MatvecArgs& a, const RowsPlan& p, int sms, cudaStream_t stream, bool pdl) {
  switch (p.R) {
    case 8: return launch_rows_r<FMT, 8>(a, p, sms, stream, pdl);
    case 4: return launch_rows_r<FMT, 4>(a, p, sms, stream, pdl);
    case 2: return launch_rows_r<FMT, 2>(a, p, sms, stream, pdl);
    default: return launch_rows_r<FMT, 1>(a, p, sms, stream, pdl);
  }
}

}  // namespace

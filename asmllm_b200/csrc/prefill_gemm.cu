// asmllm_b200/csrc/prefill_gemm.cu -- batched (prefill) Q4_0/Q8_0 x Q8_0
// matrix product on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// Y[n][m] = sum_b (wd[m][b] * xd[n][b]) * isum_b[m][n],
// isum_b[m][n] = sum_{i<32} w[m][32b+i] * xq[n][32b+i]   (an exact integer)
// for N activation rows already quantized to Q8_0 (the activation image of
// asm_act_image_q8_0_async, one row per token).  Per row and token this is
// the reference's NEON combine (THRISHAL12345/asmllm
// src/kernels/arm64/matmul_q4_neon.S:239-255): s = wd * xd (fp32 multiply),
// acc = fma(float(isum), s, acc), blocks in order.  Without a split of K the
// output equals the single-token Q4_0 x Q8_0 result bit for bit; with a split
// (small N, see below) the split partials are added in a fixed order.
//
// Exact integer sums on the fp16 tensor path.  The per-32-block scales differ
// for every (row, token, block), so each block is its own MMA into a fresh
// accumulator and the scales are applied afterwards by CUDA-core threads.
// The operands are the small integers themselves, held exactly in fp16
// (nibble - 8 in [-8, 7], int8 in [-128, 127]); every product is exact, and
// every partial sum of a block is an integer below 2^24 in magnitude, so the
// fp32 accumulator of kind::f16 holds the exact isum -- already a float, so
// the epilogue needs no int -> float conversion (one packed multiply and one
// packed fma per two outputs).  Within a block the 32 positions may be
// visited in any order as long as A and B agree; both use the order
//   k = 8c + j  ->  element 4c + {0, 2, 1, 3, 16, 18, 17, 19}[j],
// which is what the nibble layout (byte i = elements i and i + 16) expands to
// with one mask-or per two weights.
//
// CTA: 128 rows x BN tokens (BN in 16, 32, 64, 128), a contiguous range of
// K blocks.  Warp roles (15 warps):
//   0      producer: one TMA (cp.async.bulk.tensor.2d, 128-byte swizzle) per
//          stage of 128 rows x 128 bytes of raw weights (8 Q4_0 or 4 Q8_0
//          blocks) plus the stage's fp16 scales, into a 4-stage ring.
//   14     tile loader: per block the activation tile (fp16, already in
//          operand layout, tiles.cuh) and its xd, by 16-byte LSU async copies
//          (cp.async + cp.async.mbarrier.arrive).  (Through the TMA unit these
//          small L2-resident copies queued behind the weight stages' HBM
//          latency: ~1.5k cycles each.)
//   1      MMA issuer: two tcgen05.mma kind::f16 (K = 16 each) per block into
//          the block's tensor-memory accumulator; one tcgen05.commit per group.
//   2..    expanders (4 warps, or for narrow tiles 8 in two teams that take alternate groups):
//          raw weights -> fp16 A tiles and each block's wd.
//   ..13   epilogue (8 warps, or 4): warp w reads tensor-memory lanes
//          32*(w%4).. (its rows) and its share of the BN columns, then
//          acc += d * (wd * xd) block by block.
// The roles hand over groups of G blocks (one mbarrier handoff and one commit
// per group): measured with a %clock64 trace of one CTA, a handoff costs a
// few hundred cycles, which per single block made the kernel latency-bound.
// Split K (when the tiles alone do not cover the SMs): the splits of one tile
// form a thread-block cluster along z; each CTA leaves its partial tile in its
// own shared memory and, after a cluster barrier, each CTA adds a slice of
// the tile over all splits in rank order (distributed shared memory) and
// writes y.  No workspace, no atomics, deterministic.
//
// Shared-memory operand layout (no swizzle, K-major core matrices of 8 rows
// x 16 bytes): element (row, k) of a block tile at
//   (row / 8) * 512 + (k / 8) * 128 + (row % 8) * 16 + (k % 8) * 2
// so for the MMA over k in [16h, 16h + 16) the descriptor starts at h * 256,
// its leading byte offset (K direction) is 128 and its stride byte offset
// (8-row groups) is 512.
//
// Every mbarrier wait is bounded; a role that gives up sets bit 0 of the
// device error word and stops, the roles waiting on it give up in turn, the
// producer and the MMA issuer wait (bounded) for what they issued, and the
// CTA releases its tensor memory.  No cluster multicast anywhere.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

#include "common.cuh"
#include "matvec.cuh"
#include "pipeline.cuh"
#include "tiles.cuh"

namespace asmllm {

std::atomic<int> g_opt_gemm_splits{0};

namespace {

constexpr int kGM = 128;                         // rows per CTA (MMA M)
constexpr int kStages = 4;                       // raw weight ring
constexpr int kRawBytes = kGM * 128;             // one raw stage: 128 rows x 128 bytes
constexpr int kScaleBytes = kGM * 16;            // the stage's fp16 scales: 128 rows x 8 blocks
constexpr int kStageBytes = kRawBytes + kScaleBytes;  // a multiple of 1024 (the swizzle period)
constexpr int kATile = kGM * 64;                 // one block of A: 128 rows x 32 fp16
constexpr int kASlot = kATile + kGM * 4;         // A tile | wd[128]
constexpr uint32_t kMagic = 0x64006400u;  // fp16 1024.0 in both halves
constexpr uint32_t kSub8 = 0x64086408u;   // 1032.0: (1024 + nibble) - 1032 = nibble - 8
static_assert(kStageBytes % 1024 == 0, "raw stages keep the 1024-byte swizzle alignment");

// Rings.  Every handoff between roles costs a few hundred cycles (mbarrier
// waits and arrivals, proxy fences, tcgen05 commits from one thread), so the
// roles hand over groups of G blocks: R groups in flight, each with G A slots
// (expanded weights + wd), G B entries (activation tile + xd) and G
// tensor-memory accumulators of BN columns.
template <int BN>
struct Cfg {
  static constexpr int kBTile = BN * 64;
  static constexpr int kBEntry = kBTile + BN * 4;  // B tile | xd[BN]
  // A tiles in tensor memory (written by the expanders with tcgen05.st, read
  // by the MMA from there) where the accumulators leave room: half the
  // shared-memory traffic per block of the shared-memory A path.
  static constexpr bool kTA = BN <= 64;
  // 128-token tiles: 2 groups of 2 blocks rather than 4 of 1 (half the
  // epilogue's handoffs per block; N = 512 products 10-11 % faster).
  static constexpr int kG = BN >= 64 ? 2 : 4;                                 // blocks per group
  static constexpr int kR = BN >= 128 ? 2 : BN >= 64 ? 3 : BN >= 32 ? 2 : 4;  // groups in flight
  // warps 2 .. 13: expanders then epilogue.  Narrow tiles (decode batches) are
  // bound by the weight expansion, wide ones by the epilogue.
  static constexpr int kXW = BN >= 64 ? 4 : 8;  // expander warps
  // With 8 expander warps: two teams of 4 (one thread per row each) that take
  // alternate groups, so two groups are expanded at once (the expansion of one
  // group is latency-bound: shared load -> convert -> tensor-memory store).
  static constexpr int kTeams = kXW == 8 ? 2 : 1;
  static constexpr int kEW = BN >= 64 ? 8 : 4;  // epilogue warps (8: two column halves)
  static constexpr int kLoader = 2 + kXW + kEW;  // the tile loader's warp (the last)
  static constexpr int kThreads = (kLoader + 1) * 32;
  static constexpr int kCols = BN * 4 / kEW;     // accumulator columns per epilogue thread
  static constexpr int kAccCols = kR * kG * BN;
  static constexpr int kACols = kTA ? kR * kG * 16 : 0;  // 32 fp16 per row and block = 16 columns
  static constexpr int kCols32 = kAccCols + kACols;
  static constexpr int kTmemCols = kCols32 <= 32 ? 32 : kCols32 <= 64 ? 64 : kCols32 <= 128 ? 128
                                   : kCols32 <= 256 ? 256 : 512;
  static constexpr int kSlotBytes = kTA ? kGM * 4 : kASlot;  // per block: [A tile] | wd[128]
  static constexpr int kWdOff = kTA ? 0 : kATile;
  static constexpr int kAOff = kStages * kStageBytes;
  // The activation tiles have their own, deeper ring (kRB groups): the tile
  // loader runs that far ahead of the tensor core, off the critical path.
  static constexpr int kRB = kTA ? 6 : kR;
  static constexpr int kBOff = kAOff + kR * kG * kSlotBytes;
  static constexpr int kBarOff = kBOff + kRB * kG * kBEntry;
  static constexpr int kNBars = 2 * kStages + 3 * kR + 2 * kRB;
  static constexpr int kSmem = kBarOff + kNBars * 8 + 16 + 1024;  // barriers, tmem word, abort; 1024-byte alignment
  static_assert(kGM * BN * 4 <= kStages * kStageBytes, "split-K partial tile must fit the raw ring");
  static_assert(kCols32 <= 512, "tensor memory");
  static_assert(4 % kG == 0, "a group never straddles a raw stage (4 or 8 blocks)");
  static_assert(kSmem <= 227 * 1024, "shared memory");
};

// kind::f16: D f32 (bit 4), A and B f16, both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
template <int BN>
struct IdescF16 {
  static constexpr uint32_t value = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kGM >> 4) << 24);
};

__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
  // start >> 4 | LBO 128 B >> 4 | SBO 512 B >> 4 | version 1 (sm_100) | no swizzle
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(512 >> 4) << 32) |
         ((uint64_t)1 << 46);
}

template <int BN>
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(IdescF16<BN>::value), "r"(accumulate)
      : "memory");
}

// A from tensor memory (lanes = rows, two fp16 per 32-bit column along K).
template <int BN>
__device__ __forceinline__ void umma_f16_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(IdescF16<BN>::value), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, uint4 a, uint4 b) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(a.x),
               "r"(a.y), "r"(a.z), "r"(a.w), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w)
               : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, uint4 a, uint4 b, uint4 c, uint4 d) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w), "r"(c.x), "r"(c.y), "r"(c.z),
      "r"(c.w), "r"(d.x), "r"(d.y), "r"(d.z), "r"(d.w)
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void umma_commit(uint32_t mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t mbar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(mbar)
      : "memory");
}

// N consecutive 32-bit columns of this thread's tensor-memory lane.
template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&r)[N]);

#define ASM_TMEM_LD_8(i) "=r"(r[i]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), \
                         "=r"(r[i + 4]), "=r"(r[i + 5]), "=r"(r[i + 6]), "=r"(r[i + 7])
template <>
__device__ __forceinline__ void tmem_ld<8>(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : ASM_TMEM_LD_8(0)
               : "r"(taddr)
               : "memory");
}
template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : ASM_TMEM_LD_8(0), ASM_TMEM_LD_8(8)
      : "r"(taddr)
      : "memory");
}
template <>
__device__ __forceinline__ void tmem_ld<32>(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : ASM_TMEM_LD_8(0), ASM_TMEM_LD_8(8), ASM_TMEM_LD_8(16), ASM_TMEM_LD_8(24)
      : "r"(taddr)
      : "memory");
}
#undef ASM_TMEM_LD_8

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Chunk c (k = 8c .. 8c+7) of a Q4_0 block from word c of its 16 bytes
// (bytes 4c..4c+3: low nibbles = elements 4c..4c+3, high = 4c+16..4c+19).
__device__ __forceinline__ uint4 q4_chunk(uint32_t w) {
  uint4 r;
  r.x = tiles_hsub2((w & 0x000F000Fu) | kMagic, kSub8);          // elements 4c, 4c+2
  r.y = tiles_hsub2(((w >> 8) & 0x000F000Fu) | kMagic, kSub8);   // 4c+1, 4c+3
  r.z = tiles_hsub2(((w >> 4) & 0x000F000Fu) | kMagic, kSub8);   // 4c+16, 4c+18
  r.w = tiles_hsub2(((w >> 12) & 0x000F000Fu) | kMagic, kSub8);  // 4c+17, 4c+19
  return r;
}

__device__ __forceinline__ uint4 lds128(const unsigned char* p) { return *reinterpret_cast<const uint4*>(p); }

__device__ __forceinline__ unsigned long long pack2(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}

__device__ __forceinline__ void unpack2(unsigned long long v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}

// acc += d * (wd * xd) for two tokens, each element rounded as the scalar fmul / fma.
__device__ __forceinline__ unsigned long long scale_acc2(unsigned long long acc, uint32_t d0, uint32_t d1,
                                                         unsigned long long wd2, unsigned long long xd2) {
  unsigned long long s, r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(s) : "l"(wd2), "l"(xd2));
  asm("fma.rn.f32x2 %0, %1, %2, %3;"
      : "=l"(r)
      : "l"(pack2(__uint_as_float(d0), __uint_as_float(d1))), "l"(s), "l"(acc));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

__device__ __forceinline__ float ld_cluster_f32(uint32_t local_saddr, uint32_t rank) {
  uint32_t remote;
  float v;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_saddr), "r"(rank));
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

// Epilogue of one block for one thread: CH columns from tensor memory.
template <int BN, int CH>
__device__ __forceinline__ void epi_chunk(uint32_t taddr, unsigned long long* acc2, unsigned long long wd2,
                                          const float* xd) {
  uint32_t d[CH];
  tmem_ld<CH>(taddr, d);
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < CH / 4; ++i) {
    const float4 x4 = *reinterpret_cast<const float4*>(xd + 4 * i);
    acc2[2 * i] = scale_acc2(acc2[2 * i], d[4 * i], d[4 * i + 1], wd2, pack2(x4.x, x4.y));
    acc2[2 * i + 1] = scale_acc2(acc2[2 * i + 1], d[4 * i + 2], d[4 * i + 3], wd2, pack2(x4.z, x4.w));
  }
}

// Epilogue of one group of G blocks for one thread: CH columns of each
// block's accumulator, scaled in block order (the NEON combine order).  The
// tensor-memory loads of several blocks go out together (one wait::ld), at
// most 64 staging registers at a time (32 for wide rows).
template <int BN, int G, int CH, int SLOT, int WDOFF>
__device__ __forceinline__ void epi_group(uint32_t taddr, int nblk, unsigned long long* acc2,
                                          const unsigned char* aslots, const unsigned char* bentries, int lrow,
                                          int col0) {
  constexpr int kBEntry = BN * 64 + BN * 4;
  constexpr int LC = CH < 32 ? CH : 32;         // columns per load
  constexpr int NC = CH / LC;                   // loads per block
  constexpr int NL = G * NC;                    // loads per group
  constexpr int BATCH = (CH >= 64 ? 32 : 64) / LC;
#pragma unroll
  for (int l0 = 0; l0 < NL; l0 += BATCH) {
    uint32_t d[BATCH][LC];
#pragma unroll
    for (int i = 0; i < BATCH; ++i) {
      const int l = l0 + i, b = l / NC, c = l % NC;
      if (l < NL && b < nblk) tmem_ld<LC>(taddr + (uint32_t)(b * BN + c * LC), d[i]);
    }
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < BATCH; ++i) {
      const int l = l0 + i, b = l / NC, c = l % NC;
      if (l >= NL || b >= nblk) break;
      const float wd = reinterpret_cast<const float*>(aslots + b * SLOT + WDOFF)[lrow];
      const unsigned long long wd2 = pack2(wd, wd);
      const float* xd = reinterpret_cast<const float*>(bentries + b * kBEntry + BN * 64) + col0 + c * LC;
      unsigned long long* a2 = acc2 + c * (LC / 2);
#pragma unroll
      for (int k = 0; k < LC / 4; ++k) {
        const float4 x4 = *reinterpret_cast<const float4*>(xd + 4 * k);
        a2[2 * k] = scale_acc2(a2[2 * k], d[i][4 * k], d[i][4 * k + 1], wd2, pack2(x4.x, x4.y));
        a2[2 * k + 1] = scale_acc2(a2[2 * k + 1], d[i][4 * k + 2], d[i][4 * k + 3], wd2, pack2(x4.z, x4.w));
      }
    }
  }
}

template <int FMT, int BN, bool STMA>
__global__ void __launch_bounds__(Cfg<BN>::kThreads, 1)
q8act_gemm_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap smap,
                  const __half* __restrict__ scales, const unsigned char* __restrict__ tiles, int np,
                  float* __restrict__ y, int M, int N, int nb, int splits, int pre, unsigned* __restrict__ err) {
  using C = Cfg<BN>;
  constexpr int KB = FMT == kFmtQ4_0 ? 8 : 4;  // blocks per raw stage
  constexpr int G = C::kG, R = C::kR;
  static_assert(C::kTeams == 1 || (KB / G <= C::kTeams && R % C::kTeams == 0),
                "a team reads each raw stage at most once and owns every kTeams-th accumulator slot");
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // the 128-byte swizzle of the raw ring repeats every 1024 bytes of shared address
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  unsigned char* raw = smem;
  unsigned char* aring = smem + C::kAOff;
  unsigned char* bring = smem + C::kBOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* raw_full = bars;
  uint64_t* raw_empty = raw_full + kStages;
  uint64_t* in_full = raw_empty + kStages;  // a group's A tiles and wd (expanders)
  uint64_t* mma_done = in_full + R;         // the group's MMAs completed (tcgen05.commit)
  uint64_t* grp_done = mma_done + R;        // the epilogue finished the group: A slots and accumulators free
  uint64_t* b_full = grp_done + R;          // a group's B entries landed (tile loader), ring of RB
  uint64_t* b_done = b_full + C::kRB;       // the epilogue finished with a group's B entries (xd)
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(b_done + C::kRB);
  volatile uint32_t* s_abort = s_tmem + 1;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m0 = blockIdx.x * kGM, n0 = blockIdx.y * BN;
  const int z = blockIdx.z;
  const int nst = (nb + KB - 1) / KB;
  const int st0 = (int)((long long)z * nst / splits), st1 = (int)((long long)(z + 1) * nst / splits);
  const int b0 = st0 * KB;
  const int jb = min(st1 * KB, nb) - b0;  // blocks of this CTA
  const int ns = st1 - st0;
  const int ng = (jb + G - 1) / G;        // groups of this CTA

  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(s_tmem)),
                 "r"((uint32_t)C::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(smem_u32(&raw_full[i]), 1);
      // expander warps: each team that reads the stage (KB / G groups of it, one per team)
      mbar_init(smem_u32(&raw_empty[i]), (C::kXW / C::kTeams) * (KB / G < C::kTeams ? KB / G : C::kTeams));
    }
    for (int i = 0; i < R; ++i) {
      mbar_init(smem_u32(&in_full[i]), C::kXW / C::kTeams);  // the expander warps of the group's team
      mbar_init(smem_u32(&mma_done[i]), 1);
      mbar_init(smem_u32(&grp_done[i]), C::kEW);
    }
    for (int i = 0; i < C::kRB; ++i) {
      mbar_init(smem_u32(&b_full[i]), 32);  // the tile loader's lanes (cp.async arrivals)
      mbar_init(smem_u32(&b_done[i]), 1 + C::kEW);  // MMA commit + epilogue warps
    }
    *s_abort = 0u;
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  pdl_trigger();

  auto fail = [&]() {
    *s_abort = 1u;
    atomicOr(err, kErrRingTimeout);
  };

  if (warp == 0) {
    // ---------------- producer: raw weight stages (TMA) ----------------
    if (lane == 0) {
      int s_issued = 0;
      auto issue_stage = [&](int s) -> bool {
        const int rs = s % kStages;
        if (s >= kStages && !mbar_wait_bounded(smem_u32(&raw_empty[rs]), ((s / kStages) - 1) & 1)) return false;
        const uint32_t full = smem_u32(&raw_full[rs]);
        mbar_arrive_expect_tx(full, kRawBytes + (STMA ? kScaleBytes : 0));
        tma_load_2d(smem_u32(raw + rs * kStageBytes), &wmap, (st0 + s) * 128, m0, full);
        if (STMA) tma_load_2d(smem_u32(raw + rs * kStageBytes + kRawBytes), &smap, ((st0 + s) * KB) & ~7, m0, full);
        return true;
      };
      // weights declared static do not depend on the previous kernel: their first stages go out now
      if (pre)
        for (; s_issued < ns && s_issued < kStages; ++s_issued) issue_stage(s_issued);  // no wait below kStages
      pdl_wait();
      bool ok = true;
      while (ok && s_issued < ns && !*s_abort) {
        ok = issue_stage(s_issued);
        if (ok) ++s_issued;
      }
      if (!ok) fail();
      // every issued copy lands before the CTA moves on (bounded)
      for (int s = s_issued - kStages < 0 ? 0 : s_issued - kStages; s < s_issued; ++s)
        if (!mbar_wait_bounded(smem_u32(&raw_full[s % kStages]), (s / kStages) & 1)) fail();
    } else {
      pdl_wait();
    }
  } else if (warp == C::kLoader) {
    // ---------------- tile loader: activation tiles by LSU async copies (not the TMA
    // queue, where they would wait behind the weight stages' HBM latency) ----------------
    pdl_wait();  // the activation tiles come from the previous kernel
    constexpr int RB = C::kRB;
    for (int g = 0; g < ng; ++g) {
      const int rb = g % RB;
      bool ok = true;
      if (g >= RB) ok = mbar_wait_bounded(smem_u32(&b_done[rb]), ((g / RB) - 1) & 1);
      if (__any_sync(0xFFFFFFFFu, !ok || *s_abort)) {  // one decision per warp
        if (!ok) fail();
        break;
      }
      for (int b = 0; b < G && g * G + b < jb; ++b) {
        unsigned char* be = bring + (rb * G + b) * C::kBEntry;
        const size_t tb = (size_t)(b0 + g * G + b) * np + n0;  // the block's first token
        const unsigned char* st = tiles + tb * 64;
        const unsigned char* sx = tiles + (size_t)nb * np * 64 + tb * 4;
        for (int c = lane; c < C::kBTile / 16; c += 32) cp_async16(be + 16 * c, st + 16 * c);
        for (int c = lane; c < BN * 4 / 16; c += 32) cp_async16(be + C::kBTile + 16 * c, sx + 16 * c);
      }
      // this lane's arrival on b_full happens when its copies have landed
      asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(&b_full[rb])) : "memory");
    }
    cp_async_wait_all();  // nothing in flight when the CTA moves on
  } else if (warp == 1) {
    pdl_wait();
    // ---------------- MMA issuer: one handoff per group of G blocks ----------------
    if (lane == 0) {
      int issued = 0;
      for (int g = 0; g < ng; ++g) {
        const int r = g % R;
        const int rb = g % C::kRB;
        bool ok = mbar_wait_bounded(smem_u32(&in_full[r]), (g / R) & 1);
        if (ok) ok = mbar_wait_bounded(smem_u32(&b_full[rb]), (g / C::kRB) & 1);
        if (ok && g >= R) ok = mbar_wait_bounded(smem_u32(&grp_done[r]), ((g / R) - 1) & 1);  // accumulators free
        if (!ok) {
          fail();
          break;
        }
        if (*s_abort) break;
        fence_proxy_async();  // the B entries were written by generic-proxy async copies
        tc_fence_after();
        for (int b = 0; b < G && g * G + b < jb; ++b) {
          const uint64_t bd = umma_desc(smem_u32(bring + (rb * G + b) * C::kBEntry));
          const uint32_t td = tmem + (uint32_t)((r * G + b) * BN);
          if constexpr (C::kTA) {
            const uint32_t ta = tmem + (uint32_t)(C::kAccCols + (r * G + b) * 16);
            umma_f16_ta<BN>(td, ta, bd, 0u);
            umma_f16_ta<BN>(td, ta + 8, bd + (256 >> 4), 1u);
          } else {
            const uint64_t ad = umma_desc(smem_u32(aring + (r * G + b) * C::kSlotBytes));
            umma_f16<BN>(td, ad, bd, 0u);
            umma_f16<BN>(td, ad + (256 >> 4), bd + (256 >> 4), 1u);
          }
        }
        umma_commit(smem_u32(&mma_done[r]));
        umma_commit(smem_u32(&b_done[rb]));
        issued = g + 1;
      }
      // the tensor core has finished everything issued before tensor memory is released
      if (issued > 0) {
        const int g = issued - 1;
        if (!mbar_wait_bounded(smem_u32(&mma_done[g % R]), (g / R) & 1)) fail();
      }
    }
  } else if (warp < 2 + C::kXW) {
    pdl_wait();
    // ---------------- expanders: one weight row per thread (two per row with 8 warps in one team) ----------------
    constexpr int kTeams = C::kTeams;
    constexpr int kParts = C::kXW / 4 / kTeams;  // threads per row
    constexpr int kCh = 4 / kParts;              // 16-byte chunks of the A row each writes
    // rows of this warp = its tensor-memory lane quarter (the A tiles may live there)
    const int t = 32 * (warp & 3) + lane, xw = (warp - 2) >> 2;
    const int team = kTeams > 1 ? xw : 0, part = kTeams > 1 ? 0 : xw;
    const int row = m0 + t;
    const bool row_ok = row < M;
    const __half* srow = scales + (size_t)(row_ok ? row : 0) * nb;
    for (int g = team; g < ng; g += kTeams) {
      const int r = g % R;
      bool ok = true;
      if (g >= R) ok = mbar_wait_bounded(smem_u32(&grp_done[r]), ((g / R) - 1) & 1);
      if (__any_sync(0xFFFFFFFFu, !ok || *s_abort)) {  // one decision per warp
        if (!ok) fail();
        break;
      }
      if (C::kTA) tc_fence_after();  // after the MMAs that read this group's A columns last time
      // a group never straddles a raw stage (G divides KB): one wait, then the
      // group's blocks unrolled so their loads and arithmetic interleave
      const int j0 = g * G, nblk = min(G, jb - j0);
      const int s = j0 / KB, bi0 = j0 % KB, rs = s % kStages;
      if (bi0 == 0 || kTeams > 1) {  // (a team's group may start inside a stage)
        const bool okr = mbar_wait_bounded(smem_u32(&raw_full[rs]), (s / kStages) & 1);
        if (__any_sync(0xFFFFFFFFu, !okr || *s_abort)) {
          if (!okr) fail();
          break;
        }
      }
      const unsigned char* stage = raw + rs * kStageBytes;
      const unsigned char* rrow = stage + t * 128;
#pragma unroll
      for (int b = 0; b < G; ++b) {
        if (b >= nblk) break;
        const int j = j0 + b, bi = bi0 + b;
        unsigned char* slot = aring + (r * G + b) * C::kSlotBytes;
        unsigned char* adst = slot + (t >> 3) * 512 + (t & 7) * 16 + part * kCh * 128;
        const uint32_t ta = tmem + ((uint32_t)(32 * (warp & 3)) << 16) +
                            (uint32_t)(C::kAccCols + (r * G + b) * 16 + part * kCh * 4);
        if (C::kTA) {  // this thread's chunks as 32-bit tensor-memory columns of its row
          if (kParts == 1) {
            if (FMT == kFmtQ4_0) {
              const uint4 q = lds128(rrow + ((bi ^ (t & 7)) << 4));
              tmem_st16(ta, q4_chunk(q.x), q4_chunk(q.y), q4_chunk(q.z), q4_chunk(q.w));
            } else {
              const uint4 lo = lds128(rrow + (((2 * bi) ^ (t & 7)) << 4));
              const uint4 hi = lds128(rrow + (((2 * bi + 1) ^ (t & 7)) << 4));
              tmem_st16(ta, tiles_i8_chunk(lo.x, hi.x), tiles_i8_chunk(lo.y, hi.y), tiles_i8_chunk(lo.z, hi.z),
                        tiles_i8_chunk(lo.w, hi.w));
            }
          } else {
            if (FMT == kFmtQ4_0) {
              const uint2 q = *reinterpret_cast<const uint2*>(rrow + ((bi ^ (t & 7)) << 4) + part * 8);
              tmem_st8(ta, q4_chunk(q.x), q4_chunk(q.y));
            } else {
              const uint2 lo = *reinterpret_cast<const uint2*>(rrow + (((2 * bi) ^ (t & 7)) << 4) + part * 8);
              const uint2 hi = *reinterpret_cast<const uint2*>(rrow + (((2 * bi + 1) ^ (t & 7)) << 4) + part * 8);
              tmem_st8(ta, tiles_i8_chunk(lo.x, hi.x), tiles_i8_chunk(lo.y, hi.y));
            }
          }
        } else if (kParts == 1) {
          if (FMT == kFmtQ4_0) {
            const uint4 q = lds128(rrow + ((bi ^ (t & 7)) << 4));
            *reinterpret_cast<uint4*>(adst) = q4_chunk(q.x);
            *reinterpret_cast<uint4*>(adst + 128) = q4_chunk(q.y);
            *reinterpret_cast<uint4*>(adst + 256) = q4_chunk(q.z);
            *reinterpret_cast<uint4*>(adst + 384) = q4_chunk(q.w);
          } else {
            const uint4 lo = lds128(rrow + (((2 * bi) ^ (t & 7)) << 4));
            const uint4 hi = lds128(rrow + (((2 * bi + 1) ^ (t & 7)) << 4));
            *reinterpret_cast<uint4*>(adst) = tiles_i8_chunk(lo.x, hi.x);
            *reinterpret_cast<uint4*>(adst + 128) = tiles_i8_chunk(lo.y, hi.y);
            *reinterpret_cast<uint4*>(adst + 256) = tiles_i8_chunk(lo.z, hi.z);
            *reinterpret_cast<uint4*>(adst + 384) = tiles_i8_chunk(lo.w, hi.w);
          }
        } else {  // half a row: words 2*part, 2*part + 1 -> chunks 2*part, 2*part + 1
          if (FMT == kFmtQ4_0) {
            const uint2 q = *reinterpret_cast<const uint2*>(rrow + ((bi ^ (t & 7)) << 4) + part * 8);
            *reinterpret_cast<uint4*>(adst) = q4_chunk(q.x);
            *reinterpret_cast<uint4*>(adst + 128) = q4_chunk(q.y);
          } else {
            const uint2 lo = *reinterpret_cast<const uint2*>(rrow + (((2 * bi) ^ (t & 7)) << 4) + part * 8);
            const uint2 hi = *reinterpret_cast<const uint2*>(rrow + (((2 * bi + 1) ^ (t & 7)) << 4) + part * 8);
            *reinterpret_cast<uint4*>(adst) = tiles_i8_chunk(lo.x, hi.x);
            *reinterpret_cast<uint4*>(adst + 128) = tiles_i8_chunk(lo.y, hi.y);
          }
        }
        float wd;
        if (STMA) {  // the stage's scale box: 8 blocks from ((st0 + s) * KB) & ~7
          const int off = ((st0 + s) * KB) & 7;
          wd = __half2float(reinterpret_cast<const __half*>(stage + kRawBytes + t * 16)[off + bi]);
        } else {
          wd = row_ok ? __half2float(srow[b0 + j]) : 0.0f;
        }
        if (part == 0) reinterpret_cast<float*>(slot + C::kWdOff)[t] = wd;
      }
      if (kTeams > 1 || bi0 + nblk == KB || j0 + nblk == jb) {  // this warp is done with the raw stage
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&raw_empty[rs]));
      }
      if (C::kTA) {
        tmem_wait_st();  // this thread's tensor-memory stores are done
        tc_fence_before();
      } else {
        fence_proxy_async();  // generic-proxy writes become visible to the tensor core
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&in_full[r]));
    }
  } else {
    pdl_wait();  // y may still be read by the previous kernel
    // ---------------- epilogue: scales applied from tensor memory ----------------
    const int ew = warp - 2 - C::kXW, q = warp & 3, ch = ew >> 2;
    const int lrow = 32 * q + lane, row = m0 + lrow;
    const int col0 = ch * C::kCols;
    unsigned long long acc2[C::kCols / 2];
#pragma unroll
    for (int i = 0; i < C::kCols / 2; ++i) acc2[i] = 0ull;  // (+0.0f, +0.0f)
    for (int g = 0; g < ng; ++g) {
      const int r = g % R;
      bool ok = mbar_wait_bounded(smem_u32(&mma_done[r]), (g / R) & 1);
      // (the MMA saw these complete; the waits give this warp the expanders' and copies' writes)
      const int rb = g % C::kRB;
      if (ok) ok = mbar_wait_bounded(smem_u32(&in_full[r]), (g / R) & 1);
      if (ok) ok = mbar_wait_bounded(smem_u32(&b_full[rb]), (g / C::kRB) & 1);
      if (__any_sync(0xFFFFFFFFu, !ok || *s_abort)) {  // one decision per warp
        if (!ok) fail();
        break;
      }
      tc_fence_after();
      const int nblk = min(G, jb - g * G);
      epi_group<BN, G, C::kCols, C::kSlotBytes, C::kWdOff>(
          tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(r * G * BN + col0), nblk, acc2, aring + r * G * C::kSlotBytes,
          bring + rb * G * C::kBEntry, lrow, col0);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(smem_u32(&grp_done[r]));
        mbar_arrive(smem_u32(&b_done[rb]));
      }
    }
    if (splits == 1) {
      if (row < M) {
#pragma unroll
        for (int i = 0; i < C::kCols / 2; ++i) {
          float v0, v1;
          unpack2(acc2[i], v0, v1);
          const int n = n0 + col0 + 2 * i;
          if (n < N) y[(size_t)n * M + row] = v0;
          if (n + 1 < N) y[(size_t)(n + 1) * M + row] = v1;
        }
      }
    } else if (!*s_abort) {
      // Partial tile [BN][128] into the raw ring: once this warp has scaled the
      // last group, every stage was consumed (the expanders read their raw
      // data before publishing the group the last MMAs used).
      float* part = reinterpret_cast<float*>(raw);
#pragma unroll
      for (int i = 0; i < C::kCols / 2; ++i) {
        float v0, v1;
        unpack2(acc2[i], v0, v1);
        part[(col0 + 2 * i) * kGM + lrow] = v0;
        part[(col0 + 2 * i + 1) * kGM + lrow] = v1;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (splits > 1) {
    cluster_sync_all();  // every split's partial tile is in its shared memory
    if (!*s_abort) {
      const int E = kGM * BN;
      const int e0 = (int)((long long)z * E / splits), e1 = (int)((long long)(z + 1) * E / splits);
      const uint32_t pbase = smem_u32(raw);
      for (int e = e0 + tid; e < e1; e += C::kThreads) {
        const int n = e / kGM, rr = e % kGM;
        float s = 0.0f;
        for (int src = 0; src < splits; ++src) s += ld_cluster_f32(pbase + 4u * (uint32_t)e, (uint32_t)src);
        if (m0 + rr < M && n0 + n < N) y[(size_t)(n0 + n) * M + m0 + rr] = s;
      }
    }
    cluster_sync_all();  // no CTA leaves while another reads its partial tile
  }
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)C::kTmemCols)
                 : "memory");
}

// Activation images (asm_act_image_q8_0_async rows) -> activation tiles.
__global__ void __launch_bounds__(256) act_tiles_from_image_kernel(const unsigned char* __restrict__ images,
                                                                   size_t img_stride, int N, int nb, int np,
                                                                   unsigned char* __restrict__ tiles) {
  pdl_trigger();
  pdl_wait();  // the images may come from the previous kernel
  const long long total = (long long)nb * np;
  for (long long i = blockIdx.x * 256LL + threadIdx.x; i < total; i += (long long)gridDim.x * 256) {
    const int b = (int)(i / np), n = (int)(i % np);
    uint4 lo = make_uint4(0u, 0u, 0u, 0u), hi = lo;
    float d = 0.0f;
    if (n < N) {
      const unsigned char* im = images + (size_t)n * img_stride;
      lo = __ldcg(reinterpret_cast<const uint4*>(im + (size_t)b * 48));
      hi = __ldcg(reinterpret_cast<const uint4*>(im + (size_t)b * 48 + 16));
      d = __ldcg(reinterpret_cast<const float*>(im + (size_t)nb * 48) + 2 * b);
    }
    *reinterpret_cast<uint4*>(tiles + tiles_chunk_offset(np, n, b, 0)) = tiles_i8_chunk(lo.x, hi.x);
    *reinterpret_cast<uint4*>(tiles + tiles_chunk_offset(np, n, b, 1)) = tiles_i8_chunk(lo.y, hi.y);
    *reinterpret_cast<uint4*>(tiles + tiles_chunk_offset(np, n, b, 2)) = tiles_i8_chunk(lo.z, hi.z);
    *reinterpret_cast<uint4*>(tiles + tiles_chunk_offset(np, n, b, 3)) = tiles_i8_chunk(lo.w, hi.w);
    reinterpret_cast<float*>(tiles + (size_t)nb * np * 64)[i] = d;
  }
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool encode_2d(CUtensorMap* map, CUtensorMapDataType type, const void* base, uint64_t inner, uint64_t rows,
               uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swz) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (!encode) return false;
  const cuuint64_t gdim[2] = {inner, rows};
  const cuuint64_t gstride[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t estride[2] = {1u, 1u};
  return encode(map, type, 2, const_cast<void*>(base), gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int FMT, int BN, bool STMA>
cudaError_t launch_bn(const CUtensorMap& wmap, const CUtensorMap& smap, const __half* sp, const unsigned char* tiles,
                      int np, float* y, int M, int N, int nb, int pre, cudaStream_t stream, unsigned* err) {
  using C = Cfg<BN>;
  auto kernel = q8act_gemm_kernel<FMT, BN, STMA>;
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
  if (e != cudaSuccess) return e;
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  constexpr int KB = FMT == kFmtQ4_0 ? 8 : 4;
  const int nst = (nb + KB - 1) / KB;
  const long long tiles_n = (long long)((M + kGM - 1) / kGM) * ((N + BN - 1) / BN);
  // One CTA per SM.  The K split S (1..8, at most the stage count) minimises
  // waves(S) * (stages per CTA + fill): waves(S) = ceil(tiles * S / sms), and
  // the fill is a CTA's start-up and drain, ~4 stages (fitted to measured
  // times; ties keep the smaller S).  So 80 tiles of 256 K blocks take
  // S = 3 (240 CTAs in two waves, a third of K each) rather than one wave on
  // 80 SMs, and 448 tiles S = 2 (7 waves of half-K CTAs rather than 4 waves
  // of full-K CTAs, the last of which runs 4).
  long long S = 1;
  {
    double best = 1e300;
    for (int s = 1; s <= 8 && s <= nst; ++s) {
      const long long waves = (tiles_n * s + sms - 1) / sms;
      const double t = (double)waves * ((double)((nst + s - 1) / s) + 4.0);
      if (t < best) {
        best = t;
        S = s;
      }
    }
  }
  if (g_opt_gemm_splits.load() > 0) S = g_opt_gemm_splits.load();
  if (S > 8) S = 8;
  if (S > nst) S = nst;
  if (S < 1) S = 1;
  const int splits = (int)S;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((M + kGM - 1) / kGM), (unsigned)((N + BN - 1) / BN), (unsigned)splits);
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (g_opt_pdl.load()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (splits > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = (unsigned)splits;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kernel, wmap, smap, sp, tiles, np, y, M, N, nb, splits, pre, err);
}

template <int FMT, int BN>
cudaError_t launch_scales(bool stma, const CUtensorMap& wmap, const CUtensorMap& smap, const __half* sp,
                          const unsigned char* tiles, int np, float* y, int M, int N, int nb, int pre,
                          cudaStream_t stream, unsigned* err) {
  if (stma) return launch_bn<FMT, BN, true>(wmap, smap, sp, tiles, np, y, M, N, nb, pre, stream, err);
  return launch_bn<FMT, BN, false>(wmap, smap, sp, tiles, np, y, M, N, nb, pre, stream, err);
}

template <int FMT>
cudaError_t launch_fmt(bool stma, const CUtensorMap& wmap, const CUtensorMap& smap, const __half* sp,
                       const unsigned char* tiles, int np, float* y, int M, int N, int nb, int pre,
                       cudaStream_t stream, unsigned* err) {
  if (N <= 16) return launch_scales<FMT, 16>(stma, wmap, smap, sp, tiles, np, y, M, N, nb, pre, stream, err);
  if (N <= 32) return launch_scales<FMT, 32>(stma, wmap, smap, sp, tiles, np, y, M, N, nb, pre, stream, err);
  if (N <= 64) return launch_scales<FMT, 64>(stma, wmap, smap, sp, tiles, np, y, M, N, nb, pre, stream, err);
  return launch_scales<FMT, 128>(stma, wmap, smap, sp, tiles, np, y, M, N, nb, pre, stream, err);
}

}  // namespace

cudaError_t launch_q8act_gemm_tiles(int fmt, const void* w, const void* scales_f16, const void* tiles, float* y,
                                    int64_t M, int64_t N, int64_t K, bool weights_static, cudaStream_t stream) {
  const int nb = (int)(K / QK);
  const int ub = fmt == kFmtQ4_0 ? 16 : 32;
  // raw weights as a 2-D byte array [M rows][nb * ub bytes]; box 128 x 128 bytes, 128-byte swizzle
  CUtensorMap wmap, smap;
  if (!encode_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, (uint64_t)nb * ub, (uint64_t)M, (uint64_t)nb * ub, 128u,
                 (uint32_t)kGM, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  // fp16 scales [M][nb] by TMA when their rows are 16-byte multiples: box 8 blocks x 128 rows
  bool stma = nb % 8 == 0 && (uintptr_t)scales_f16 % 16 == 0;
  if (stma && !encode_2d(&smap, CU_TENSOR_MAP_DATA_TYPE_UINT16, scales_f16, (uint64_t)nb, (uint64_t)M,
                         (uint64_t)nb * 2, 8u, (uint32_t)kGM, CU_TENSOR_MAP_SWIZZLE_NONE))
    stma = false;
  if (!stma) smap = wmap;  // unused
  unsigned* err = device_error_word();
  if (!err) return cudaErrorUnknown;
  const __half* sp = static_cast<const __half*>(scales_f16);
  const unsigned char* tp = static_cast<const unsigned char*>(tiles);
  const int np = act_tiles_tokens(N), pre = weights_static ? 1 : 0;
  if (fmt == kFmtQ4_0)
    return launch_fmt<kFmtQ4_0>(stma, wmap, smap, sp, tp, np, y, (int)M, (int)N, nb, pre, stream, err);
  return launch_fmt<kFmtQ8_0>(stma, wmap, smap, sp, tp, np, y, (int)M, (int)N, nb, pre, stream, err);
}

cudaError_t launch_act_tiles_from_image(const void* images, size_t img_stride, int64_t N, int64_t K, void* tiles,
                                        cudaStream_t stream) {
  const int nb = (int)(K / QK), np = act_tiles_tokens(N);
  const long long total = (long long)nb * np;
  long long grid = (total + 255) / 256;
  if (grid > 4096) grid = 4096;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_opt_pdl.load() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, act_tiles_from_image_kernel, static_cast<const unsigned char*>(images), img_stride,
                            (int)N, nb, np, static_cast<unsigned char*>(tiles));
}

// Images -> tiles (stream-ordered scratch) -> product.
cudaError_t launch_q8act_gemm(int fmt, const void* w, const void* scales_f16, const void* images, size_t img_stride,
                              float* y, int64_t M, int64_t N, int64_t K, bool weights_static, cudaStream_t stream) {
  void* tiles = nullptr;
  cudaError_t e = scratch_alloc_async(&tiles, act_tiles_bytes(N, K), stream);
  if (e != cudaSuccess) return e;
  e = launch_act_tiles_from_image(images, img_stride, N, K, tiles, stream);
  if (e == cudaSuccess) e = launch_q8act_gemm_tiles(fmt, w, scales_f16, tiles, y, M, N, K, weights_static, stream);
  const cudaError_t f = scratch_free_async(tiles, stream);
  return e != cudaSuccess ? e : f;
}

}  // namespace asmllm

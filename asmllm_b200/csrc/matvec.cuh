// asmllm_b200/csrc/matvec.cuh -- host-side interface of the matvec kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

namespace asmllm {

// GGUF tensor type ids of the two weight formats.
constexpr int kFmtQ4_0 = 2;
constexpr int kFmtQ8_0 = 8;

// Decode-step fusions of the bulk-copy matvec (tma_matvec.cu).
//
// Prologue (how the CTA builds its Q8_0 activation image):
constexpr int kProImage = 0;  // copy a prepared image (MatvecArgs::image)
constexpr int kProQuant = 1;  // quantize fp32 x
constexpr int kProNorm = 2;   // RMSNorm x with norm_w, then quantize
// Epilogue (what happens to a finished row value v):
constexpr int kEpiStore = 0;     // y[r] = v
constexpr int kEpiResidual = 1;  // y[r] += v (y is the residual stream)
constexpr int kEpiSwiglu = 2;    // rows (2i, 2i+1) = (gate_i, up_i): h_i = silu(gate_i) * up_i,
                                 // quantized to Q8_0 into image_out block by block
constexpr int kEpiArgmax = 3;    // y[r] = v, then the next token = argmax over all rows
constexpr int kEpiGather = 4;    // row-split: y[tp_rank * M + r] = v here, and (seq, v) to every
                                 // other rank's gather buffer (completed by launch_rowsplit_wait)

struct MvFuse {
  const float* norm_w = nullptr;  // kProNorm: weight [K]
  float eps = 0.0f;
  // Source row of the prologue: embed + tokens[*pos] * K when embed is set
  // (the first layer of a decode step), else MatvecArgs::x.  CTA 0 copies the
  // source row to x_copy (the residual stream) when x_copy is set.
  const float* embed = nullptr;
  int32_t vocab = 0;
  int32_t* tokens = nullptr;  // [max_tokens]: prompt ids, then generated ids
  int32_t* pos = nullptr;     // current position (device); advanced by kEpiArgmax
  int32_t max_tokens = 0;
  int32_t n_prompt = 0;
  float* x_copy = nullptr;
  // kEpiSwiglu
  float* h = nullptr;                 // [M/2] fp32
  unsigned char* image_out = nullptr; // Q8_0 image of h (nb = M/64 blocks)
  unsigned* counters = nullptr;       // [M/64] zero on entry; left zero
  // kEpiArgmax
  unsigned long long* best = nullptr;  // packed (value, row); zero on entry, left zero
  unsigned* done = nullptr;            // CTAs finished; zero on entry, left zero
  // Tensor parallelism (tp > 1), kEpiResidual and kEpiArgmax only.
  //   kEpiResidual: y here is this rank's partial sum of a row-parallel
  //   projection; every rank writes its partial rows into every rank's
  //   exchange buffer, then each CTA sums the tp partials of its rows in rank
  //   order and adds them to the residual stream (identical on all ranks).
  //   kEpiArgmax: rows are this rank's vocabulary slice (global row = row +
  //   vocab_offset); the ranks' maxima are exchanged the same way.
  // Exchange words are 64-bit (value bits, sequence number): a reader spins
  // (bounded) until the word carries the current sequence, so no fence is
  // needed.  Buffers: [2 parities][tp source ranks][xchg_rows] words, parity
  // = sequence & 1; the sequence is *ar_seq + 1, stored back by the last CTA.
  int tp = 1, tp_rank = 0;
  int xchg_rows = 0;
  int vocab_offset = 0;
  unsigned long long* xchg[8] = {};  // exchange buffer of each rank (peer pointers)
  unsigned* ar_seq = nullptr;        // call counter of this rank (same on all ranks)
  unsigned* ar_done = nullptr;       // CTAs finished; zero on entry, left zero
};
constexpr int kMaxTp = 8;

struct MatvecArgs {
  int fmt = kFmtQ4_0;       // kFmtQ4_0 or kFmtQ8_0
  bool fp32_act = false;    // false: Q8_0 activations (NEON semantics); true: fp32 x (x86)
  bool scales_f16 = false;  // scale plane dtype
  const void* w = nullptr;  // device: Q4_0 [M][K/32][16] or Q8_0 [M][K/32][32]
  const void* scales = nullptr;
  const float* x = nullptr;     // fp32 activation (used when image is null)
  const void* image = nullptr;  // Q8_0 activation image from launch_act_image (Q8_0 families)
  float* y = nullptr;
  int32_t* isums = nullptr;  // optional: per-(row, block) int32 sums (Q8_0 activations only)
  // The weights are not written by the kernel that precedes this launch in the
  // stream, so the kernel may start reading them before that kernel completes.
  bool weights_static = false;
  // Use the register-streaming (LDG) kernel even where the bulk-copy one applies.
  bool isums_force_ldg = false;
  // x is not written, and y neither read nor written, by the kernel that
  // precedes this launch in the stream: the bulk-copy kernel then starts on
  // x without waiting for that kernel (it still waits before it completes).
  bool act_independent = false;
  // w holds packed rows [M][K/32 * (16 or 32) quant bytes, then K/32 fp16
  // scales] (pack_rows); `scales` is unused.  Bulk-copy kernel only.
  bool packed = false;
  int64_t M = 0, K = 0;
  // Decode fusions (bulk-copy kernel, fp16 scales only): the prologue is
  // kProImage when image is set, else kProNorm when fuse->norm_w is set, else
  // kProQuant.
  int epi = kEpiStore;
  const MvFuse* fuse = nullptr;
};

// Device error word bits (read_device_error).
constexpr unsigned kErrRingTimeout = 1u;  // a shared-memory ring barrier wait gave up
constexpr unsigned kErrDecodeRange = 2u;  // decode position or token id out of range: step skipped
constexpr unsigned kErrXchgTimeout = 4u;  // a tensor-parallel exchange wait gave up (a peer never wrote)

// Limit of every exchange / gather wait on the current device, in SM clock
// cycles (0 = the default, about a second).
cudaError_t set_xchg_wait_cycles(long long cycles);

// Completion of a step of row-split matvecs (kEpiGather): waits until every
// peer's rows of each of the n matvecs carry this step's sequence number in
// this rank's gather buffers, copies them into the full outputs, and advances
// the step counter.  own[j] = this rank's gather buffer of matvec j ([2][tp][M[j]]
// words), y_full[j] = its [tp * M[j]] output.
struct RowsplitWait {
  int n = 0, tp = 1, rank = 0;
  const unsigned long long* own[8] = {};
  float* y_full[8] = {};
  long long M[8] = {};
  unsigned* seq = nullptr;   // step counter (same on every rank)
  unsigned* done = nullptr;  // CTAs finished; zero on entry, left zero
};
cudaError_t launch_rowsplit_wait(const RowsplitWait& w, int sms, cudaStream_t stream);

// Bytes of one row of the Q8_0 activation image for nb = K/32 blocks:
// nb 48-byte slots (32 int8 + 16 pad) then nb (d, qsum) float pairs, rounded to 16.
__host__ __device__ inline size_t act_image_bytes(int64_t nb) {
  return ((size_t)nb * 56 + 15) & ~(size_t)15;
}

cudaError_t launch_matvec(const MatvecArgs& a, cudaStream_t stream);
// pf_w / pf_s: optional weight and scale planes of the matvec that will read
// this image; their first bytes are prefetched into L2 while the kernel waits
// for its predecessor (pass nullptr / 0 for none).
cudaError_t launch_act_image(const float* x, void* image, long long nrows, int64_t K,
                             cudaStream_t stream, const void* pf_w = nullptr, size_t pf_w_bytes = 0,
                             const void* pf_s = nullptr, size_t pf_s_bytes = 0);
cudaError_t launch_quantize(const float* x, int8_t* xq, float* xd, long long nblocks,
                            cudaStream_t stream);
cudaError_t launch_gguf_split(int fmt, const uint8_t* raw, uint8_t* qs, void* scales, int f16,
                              long long nblocks, cudaStream_t stream);
// n empty kernels chained as the matvecs chain (PDL attribute, trigger at
// entry, griddepcontrol.wait when `wait`): the launch-dependency floor.
cudaError_t launch_floor_chain(int n, bool pdl, bool wait, cudaStream_t stream);
// qs plane + fp16 scale plane -> packed rows (MatvecArgs::packed); K/32 a multiple of 8.
cudaError_t launch_pack_rows(int fmt, const void* qs, const void* scales_f16, void* out, int64_t M, int64_t K,
                             cudaStream_t stream);
int64_t max_k(int fmt, bool fp32_act, int dev);

// Bulk-copy (TMA) pipeline kernel for the Q8_0-activation families
// (tma_matvec.cu); launch_matvec uses it when the shape allows.
bool tma_matvec_supported(const MatvecArgs& a, int smem_optin);
// True when a asks for a decode fusion (which only the bulk-copy kernel has).
bool matvec_is_fused(const MatvecArgs& a);
cudaError_t launch_tma_matvec(const MatvecArgs& a, int sms, int smem_optin, cudaStream_t stream, bool pdl);
// Y [N][M] for N <= kNarrowMaxN activation images, every weight byte read once
// for all N rows (narrow_gemm.cuh); row n equals the warp-ring matvec of row n.
constexpr int kNarrowMaxN = 8;
cudaError_t launch_gemm_narrow(int fmt, const void* w, const void* scales_f16, const void* images,
                               long long image_stride, float* y, long long M, long long N, long long K, int sms,
                               int smem_optin, cudaStream_t stream);
// Reads (and optionally clears) the device error word the kernels set when a
// bounded wait gives up (bit 0: a shared-memory ring barrier timed out).
cudaError_t read_device_error(unsigned* out, bool clear);
// Points the kernels' error reports on the current device at a mapped pinned
// host word as well (nullptr: none), so a synchronous caller sees them
// without a copy.
cudaError_t set_device_error_mirror(unsigned* host_mapped);
// Stream-ordered scratch for one call (a per-device pool that keeps its
// memory; a graph allocation under stream capture), and trimming the pools.
cudaError_t scratch_alloc_async(void** p, size_t bytes, cudaStream_t stream);
cudaError_t scratch_free_async(void* p, cudaStream_t stream);
void scratch_trim();
// Device address of the error word on the current device (for kernels in
// other translation units); nullptr if it cannot be looked up.
unsigned* device_error_word();

// Attention for one decode position (decode.cu): RoPE, fp16 KV append,
// softmax(q.K^T / sqrt_hd).V per query head, Q8_0 image of the output.
cudaError_t launch_attention_decode(const float* qkv, void* k_cache, void* v_cache, const float* rope_cs,
                                    const int32_t* pos, void* image, int n_heads, int n_kv, int head_dim, int ctx,
                                    float sqrt_hd, cudaStream_t stream, bool pdl);

// Q5_0 x fp32 matvec (q5_matvec.cu): ql [M][K/32][16], qh [M][K/32][4], fp32 scales.
size_t q5_smem_bytes(int64_t K);
cudaError_t launch_q5_matvec(const uint8_t* ql, const uint8_t* qh, const float* scales, const float* x, float* y,
                             int64_t M, int64_t K, cudaStream_t stream);

// Batched Q4_0 / Q8_0 x Q8_0 product on the tensor cores (prefill_gemm.cu):
// y [N][M] from the N-token activation tiles (tiles.cuh), fp16 scales;
// weights_static: the weights do not depend on the previous kernel.
cudaError_t launch_q8act_gemm_tiles(int fmt, const void* w, const void* scales_f16, const void* tiles, float* y,
                                    int64_t M, int64_t N, int64_t K, bool weights_static, cudaStream_t stream);
// N activation-image rows (row stride img_stride bytes) -> activation tiles.
cudaError_t launch_act_tiles_from_image(const void* images, size_t img_stride, int64_t N, int64_t K, void* tiles,
                                        cudaStream_t stream);
// The two above with stream-ordered scratch tiles.
cudaError_t launch_q8act_gemm(int fmt, const void* w, const void* scales_f16, const void* images, size_t img_stride,
                              float* y, int64_t M, int64_t N, int64_t K, bool weights_static, cudaStream_t stream);

// Batched decode glue (batch_decode.cu): one CTA per row (token) of B rows.
struct RowsArgs {
  int rows = 0, dim = 0;
  float* x = nullptr;              // [rows][dim] residual stream
  const float* delta = nullptr;    // [rows][dim]: x += delta first (or null)
  const float* embed = nullptr;    // [vocab][dim]: x = embed[tokens[row][pos]] first (or null)
  const int32_t* tokens = nullptr; // [rows][max_tokens]
  const int32_t* pos = nullptr;
  int max_tokens = 0, vocab = 0;
  const float* norm_w = nullptr;   // [dim]: RMSNorm (or null: quantize x as it is)
  float eps = 1e-5f;
  void* tiles = nullptr;           // activation tiles of the rows (tiles.cuh), np tokens
  int np = 0;
};
cudaError_t launch_rows_norm_tiles(const RowsArgs& a, cudaStream_t stream);
cudaError_t launch_rows_swiglu_tiles(const float* gu, int rows, int ffn, void* tiles, int np, cudaStream_t stream);
cudaError_t launch_attention_batch(const float* qkv, size_t qkv_stride, void* k_cache, void* v_cache,
                                   size_t cache_stride, const float* rope_cs, const int32_t* pos, void* tiles, int np,
                                   int rows, int n_heads, int n_kv, int head_dim, int ctx, float sqrt_hd,
                                   cudaStream_t stream);
cudaError_t launch_rows_argmax(const float* logits, int rows, int n, size_t stride, int offset, long long* keys,
                               cudaStream_t stream);
cudaError_t launch_rows_advance(const long long* keys, int rows, int32_t* tokens, int max_tokens, int32_t* pos,
                                int n_prompt, cudaStream_t stream);

// The reference's decode-glue kernels (glue.cu): RMSNorm, softmax, RoPE on
// one head's q and k in place, SiLU(gate) * up into gate, and single-head
// attention over seq query rows.  Lengths up to glue_max_len().
int64_t glue_max_len();
cudaError_t launch_rmsnorm(const float* x, const float* w, float* y, int64_t n, float eps, cudaStream_t stream);
cudaError_t launch_softmax(const float* x, float* y, int64_t n, cudaStream_t stream);
cudaError_t launch_rope(float* q, float* k, int64_t hd, int64_t pos, float theta, cudaStream_t stream);
cudaError_t launch_silu_hadamard(float* gate, const float* up, int64_t n, cudaStream_t stream);
size_t attention_smem(int64_t seq);
cudaError_t launch_attention(const float* q, const float* k, const float* v, float* y, int64_t seq, int64_t hd,
                             float scale, cudaStream_t stream);

extern std::atomic<int> g_opt_tma;  // 1: bulk-copy kernel where it applies
extern std::atomic<int> g_opt_pdl;  // 1: programmatic dependent launch
extern std::atomic<int> g_opt_image_min_k;  // fp32-x matvecs with K >= this quantize x in a pre-pass (0: never)
extern std::atomic<int> g_opt_gemm_splits;  // batched product: 0 = automatic K split, else exactly this many
// Bulk-copy matvec plan (tma_matvec.cu): rows per stage (0 = automatic), ring
// slots per warp cap (0 = automatic), shared-memory budget per CTA in KB,
// CTAs per SM.
extern std::atomic<int> g_opt_mv_rows;
extern std::atomic<int> g_opt_mv_slots;
extern std::atomic<int> g_opt_mv_smem_kb;
extern std::atomic<int> g_opt_mv_kernel;
extern std::atomic<int> g_opt_image_prefetch_mb;
extern std::atomic<int> g_opt_mv_ctas;

}  // namespace asmllm

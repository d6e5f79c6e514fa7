/*
 * include/asmllm.h -- C ABI of libasmllm.so, the B200 (sm_100a) implementation
 * of asmllm's quantized matvec hot path.
 *
 * The first group keeps the exact names and signatures of the reference
 * library's exports (THRISHAL12345/asmllm, exports list build_kernel.py:85-104,
 * threadpool.h:37-102) so its ctypes callers load this library unchanged.
 * The second group adds what the B200 path needs: stream-ordered entries on
 * device pointers, Q8_0 x Q8_0, the standalone activation quantize, a
 * block-sum probe, GGUF block splitting and an error channel.
 *
 * Conventions for every entry point:
 *   - Q4_0 weights: uint8 [M][K/32][16]; byte j of a block holds element j in
 *     its low nibble and element 16+j in its high nibble; value = nibble - 8
 *     (reference tests/reference/ops.py:16-30).
 *   - Q8_0 weights: int8 [M][K/32][32]; value = q.
 *   - scales: one per (row, block), fp32 [M][K/32] (reference generate.py:91-119);
 *     the *_f16s entries take fp16 scales instead (lossless for GGUF data).
 *   - x: fp32 [K]; y: fp32 [M]; K must be a multiple of 32 (K = 0 gives y = 0).
 *   - "Q4_0 x Q8_0" semantics = reference src/kernels/arm64/matmul_q4_neon.S:
 *     x is quantized per 32-block with d = amax/127, q = sat8(RNE(x*127/amax)),
 *     then y[r] = sum_b float(isum[r][b]) * (wd[r][b]*xd[b]).
 *   - "fp32-x" semantics = reference src/kernels/x86_64/matmul_q{4,8}_avx2.asm:
 *     y[r] = sum_b wd[r][b] * sum_i w[r][b][i]*x[b*32+i].
 *
 * Synchronous entries (the reference names) accept host or device pointers
 * in any mix and return with y written, like the reference.  Host buffers are
 * staged through device memory; weights registered with asm_weights_register
 * stay resident in HBM and are not copied again.  They return void, like the
 * reference; failures are reported on stderr and by asm_get_last_error().
 *
 * *_async entries take device pointers only, enqueue on `stream`
 * (a cudaStream_t; NULL = legacy default stream) and return 0 or an ASM_E_*
 * code.
 */
#ifndef ASMLLM_B200_H
#define ASMLLM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ASMLLM_API __attribute__((visibility("default")))

/* Status codes of the int-returning entries. */
#define ASM_OK 0
#define ASM_E_INVALID 1     /* bad argument (negative size, K % 32 != 0, NULL) */
#define ASM_E_UNSUPPORTED 2 /* size beyond what the kernel supports */
#define ASM_E_CUDA 3        /* CUDA runtime error; text via asm_get_last_error */
#define ASM_E_NOT_DEVICE 4  /* an *_async entry got a non-device pointer */

/* ===================================================================== */
/* 1. Reference ABI (drop-in)                                             */
/* ===================================================================== */

/* Q4_0 x Q8_0 matvec (quantizes x inside, NEON semantics).
 * Replaces asm_matmul_q4: src/kernels/arm64/matmul_q4_neon.S:9-16,25-327
 * (same symbol and signature as src/kernels/x86_64/matmul_q4_avx2.asm:12-19). */
ASMLLM_API void asm_matmul_q4(const uint8_t* qweights, const float* scales,
                              const float* x, float* y, int64_t M, int64_t K);

/* Q4_0 x fp32 matvec (x86 semantics, no activation quantize).
 * Replaces asm_matmul_q4_avx512: src/kernels/x86_64/matmul_q4_avx512.asm:57-279. */
ASMLLM_API void asm_matmul_q4_avx512(const uint8_t* qweights, const float* scales,
                                     const float* x, float* y, int64_t M, int64_t K);

/* Q8_0 x fp32 matvec.
 * Replaces asm_matmul_q8: src/kernels/x86_64/matmul_q8_avx2.asm:12-19,51-194
 * and src/kernels/arm64/matmul_q8_neon.S:8-15,23-78. */
ASMLLM_API void asm_matmul_q8(const int8_t* qweights, const float* scales,
                              const float* x, float* y, int64_t M, int64_t K);

/* Multi-thread entries: num_threads is accepted and ignored (one launch
 * covers all rows).  Replace asm_matmul_q4_mt (src/runtime/threadpool.c:390-486,
 * threadpool.h:49-57) and asm_matmul_q8_mt (threadpool.c:750-767,
 * matmul_q8_avx2.asm:203-300, threadpool.h:59-67). */
ASMLLM_API void asm_matmul_q4_mt(const uint8_t* qweights, const float* scales,
                                 const float* x, float* y, int64_t M, int64_t K,
                                 int num_threads);
ASMLLM_API void asm_matmul_q8_mt(const int8_t* qweights, const float* scales,
                                 const float* x, float* y, int64_t M, int64_t K,
                                 int num_threads);
/* Replaces asm_matmul_q4_avx512_mt (threadpool.c:489-586, built with AVX512_ENABLED):
 * fp32-x semantics like asm_matmul_q4_avx512; num_threads ignored. */
ASMLLM_API void asm_matmul_q4_avx512_mt(const uint8_t* qweights, const float* scales,
                                        const float* x, float* y, int64_t M, int64_t K,
                                        int num_threads);

/* Q5_0 x fp32 matvec: ql uint8 [M][K/32][16] (weight j's low 4 bits in the
 * low nibble of byte j, j < 16, else the high nibble of byte j - 16), qh
 * uint8 [M][K/32][4] (weight j's fifth bit = bit j % 8 of byte j / 8), value
 * (nibble | bit << 4) - 16 times the block scale; x stays fp32.
 * Replaces asm_matmul_q5 (src/kernels/x86_64/matmul_q5_avx2.asm:7-23,91-210;
 * src/kernels/arm64/matmul_q5_neon.S) and asm_matmul_q5_mt
 * (matmul_q5_avx2.asm:241-250; num_threads ignored); layout
 * tests/reference/ops.py:67-92. */
ASMLLM_API void asm_matmul_q5(const uint8_t* ql, const uint8_t* qh, const float* scales,
                              const float* x, float* y, int64_t M, int64_t K);
ASMLLM_API void asm_matmul_q5_mt(const uint8_t* ql, const uint8_t* qh, const float* scales,
                                 const float* x, float* y, int64_t M, int64_t K, int num_threads);

/* Pool management.  init records the thread count (returned by
 * get_num_threads) and creates this device's stream and staging state;
 * shutdown releases them and all registered weights.
 * Replace threadpool.h:37,42,102 (threadpool.c:340-388). */
ASMLLM_API void asm_threadpool_init(int num_threads);
ASMLLM_API void asm_threadpool_shutdown(void);
ASMLLM_API int asm_threadpool_get_num_threads(void);

/* Q8_0 x fp32 dispatch with the current pool; same as asm_matmul_q8.
 * Replaces asm_threadpool_dispatch_q8: threadpool.h:80-87, threadpool.c:588-665. */
ASMLLM_API void asm_threadpool_dispatch_q8(const int8_t* qweights, const float* scales,
                                           const float* x, float* y, int64_t M, int64_t K);

/* Q5_0 x fp32 dispatch with the current pool; same as asm_matmul_q5.
 * Replaces asm_threadpool_dispatch_q5: threadpool.h:89-97, threadpool.c:667-747
 * (exported at build_kernel.py:100). */
ASMLLM_API void asm_threadpool_dispatch_q5(const uint8_t* ql, const uint8_t* qh, const float* scales,
                                           const float* x, float* y, int64_t M, int64_t K);

/* ---- Decode-step glue of the reference's generation driver -----------
 * The kernels AsmEngineForward binds next to asm_matmul_q4
 * (src/runtime/generate.py:221-250) and the correctness harness checks
 * (tests/correctness/test_runner.py:376-467), run on the GPU.  Same names,
 * signatures and in-place conventions; host or device pointers in any mix,
 * synchronous like the matvec entries; errors through asm_get_last_error.
 * Arithmetic is fp32 operation by operation as the reference's numpy
 * definitions (tests/reference/ops.py:103-170); vector sums use numpy's
 * pairwise order, so asm_rmsnorm is bit-exact against numpy; exp, sin, cos
 * and pow are evaluated in double precision and rounded once to fp32, as the
 * reference's x86 kernels do on the x87 unit (numpy's own fp32 versions
 * differ from that by about one ulp).  Lengths up to 2^20. */

/* y = (x / sqrt(mean(x^2) + eps)) * weight.  Replaces asm_rmsnorm
 * (src/kernels/x86_64/rmsnorm_avx2.asm, arm64/rmsnorm_neon.S; build_kernel.py:89). */
ASMLLM_API void asm_rmsnorm(const float* x, const float* weight, float* y, int64_t dim, float eps);
/* RoPE of one head's q and k in place, interleaved pairs (x[2i], x[2i+1]):
 * angle = pos / theta^(2i / head_dim).  Replaces asm_rope
 * (x86_64/rope_avx2.asm, arm64/rope_neon.S; build_kernel.py:90). */
ASMLLM_API void asm_rope(float* q, float* k, int64_t head_dim, int64_t pos, float theta);
/* y = exp(x - max x) / sum(exp(x - max x)).  Replaces asm_softmax
 * (x86_64/softmax_avx2.asm, arm64/softmax_neon.S; build_kernel.py:91). */
ASMLLM_API void asm_softmax(const float* x, float* y, int64_t n);
/* Single-head attention over seq_len query rows: y[i] = softmax_j(q[i].k[j] *
 * scale) . v, every key (no mask); q, k, v, y [seq_len][head_dim].  Replaces
 * asm_attention (x86_64/attention_avx2.asm:7-27, arm64/attention_neon.S;
 * build_kernel.py:92). */
ASMLLM_API void asm_attention(const float* q, const float* k, const float* v, float* y, int64_t seq_len,
                              int64_t head_dim, float scale);
/* gate[i] = (gate[i] / (1 + exp(-gate[i]))) * up[i], in place.  Replaces
 * asm_silu_hadamard (x86_64/swiglu_avx2.asm:7-17, arm64/swiglu_neon.S;
 * build_kernel.py:93). */
ASMLLM_API void asm_silu_hadamard(float* gate, const float* up, int64_t n);

/* ===================================================================== */
/* 2. Additions for the B200 path                                         */
/* ===================================================================== */

/* Q8_0 x Q8_0 matvec (x quantized as in asm_matmul_q4, signed int8 block dot).
 * No reference kernel: specified by composing matmul_q4_neon.S:57-143 with an
 * int8 block dot and the combine of matmul_q4_neon.S:239-255. */
ASMLLM_API void asm_matmul_q8q8(const int8_t* qweights, const float* scales,
                                const float* x, float* y, int64_t M, int64_t K);

/* fp32 -> Q8_0 activation quantize alone: xq int8[K], xd fp32[K/32].
 * Exposes the quantize of matmul_q4_neon.S:57-143 (stack scratch :41-50)
 * for bit-exact testing and for callers that quantize once for several matvecs. */
ASMLLM_API void asm_quantize_q8_0(const float* x, int8_t* xq, float* xd, int64_t K);

/* Q4_0 x fp32 matvec under an explicit name (same as asm_matmul_q4_avx512;
 * the x86 AVX2 asm_matmul_q4 semantics, matmul_q4_avx2.asm:57-287). */
ASMLLM_API void asm_matmul_q4_f32(const uint8_t* qweights, const float* scales,
                                  const float* x, float* y, int64_t M, int64_t K);

/* Keeps a copy of host weights resident in HBM.  Later synchronous calls that
 * pass the same host `qweights` pointer (with the same scales pointer, M and
 * K) use the resident copy instead of copying the weights again.  fmt: 2 =
 * Q4_0, 8 = Q8_0 (GGUF type ids).  Scales are stored as fp16 when every
 * scale converts to fp16 exactly, else as fp32.  The host buffers must not
 * change while registered; register again after changing them.  The
 * registration is keyed by the host address: unregister BEFORE freeing the
 * host buffer.  A buffer freed while registered, and an unrelated array that
 * later gets the same address (with the same scales pointer, M and K), is
 * undefined: such calls compute with the resident copy of the old weights
 * (device memory the library still owns, so nothing faults, but y is wrong).
 * This is the one-time "upload to HBM" of the reference's loader path
 * (src/runtime/generate.py:169-180).  Returns ASM_OK or an ASM_E_* code. */
ASMLLM_API int asm_weights_register(const void* qweights, const float* scales,
                                    int64_t M, int64_t K, int fmt);
ASMLLM_API int asm_weights_unregister(const void* qweights);
/* Number of registered weight tensors and their resident bytes. */
ASMLLM_API int64_t asm_weights_resident_bytes(int* count);

/* Last error text of the calling thread (empty when none); returns its code
 * and clears it.  The reference ABI returns void, so this is its error channel. */
ASMLLM_API int asm_get_last_error(char* buf, size_t n);

/* How the synchronous entries see pointer p right now: 0 = pageable host
 * memory (staged by copies), 1 = pinned host memory (used in place through its
 * mapped device address), 2 = device memory; *device (may be NULL) gets the
 * owning device or -1.  Asked of the CUDA driver on every call and never
 * cached, so a buffer unregistered or freed since an earlier call is seen as
 * it is now.  Host-side query only: launches nothing.  No counterpart in the
 * reference (its entries take host pointers only). */
ASMLLM_API int asm_pointer_kind(const void* p, int* device);

/* ---- Stream-ordered entries on device pointers ---------------------- */

/* Q4_0 x Q8_0 (asm_matmul_q4 semantics).  scales fp32. */
ASMLLM_API int asm_matmul_q4_async(const uint8_t* qweights, const float* scales,
                                   const float* x, float* y, int64_t M, int64_t K,
                                   void* stream);
/* Same with fp16 scales (the resident/repacked layout: 18 bytes per block). */
ASMLLM_API int asm_matmul_q4_f16s_async(const uint8_t* qweights, const uint16_t* scales_f16,
                                        const float* x, float* y, int64_t M, int64_t K,
                                        void* stream);
ASMLLM_API int asm_matmul_q8q8_async(const int8_t* qweights, const float* scales,
                                     const float* x, float* y, int64_t M, int64_t K,
                                     void* stream);
ASMLLM_API int asm_matmul_q8q8_f16s_async(const int8_t* qweights, const uint16_t* scales_f16,
                                          const float* x, float* y, int64_t M, int64_t K,
                                          void* stream);
/* fp32-x semantics. */
ASMLLM_API int asm_matmul_q4_f32_async(const uint8_t* qweights, const float* scales,
                                       const float* x, float* y, int64_t M, int64_t K,
                                       void* stream);
ASMLLM_API int asm_matmul_q8_async(const int8_t* qweights, const float* scales,
                                   const float* x, float* y, int64_t M, int64_t K,
                                   void* stream);
/* Q4_0 (fmt 2) or Q8_0 (fmt 8) x Q8_0 matvec with launch flags; scales fp32
 * or fp16 (scales_are_f16).  Same result as asm_matmul_q4_async /
 * asm_matmul_q8q8_async.  ASM_MV_INDEPENDENT: the caller guarantees that the
 * kernel enqueued just before this one on `stream` neither writes x nor reads
 * or writes y -- for instance consecutive matvecs of different inputs and
 * outputs.  The matvec then quantizes x and computes without waiting for
 * that kernel to finish (it still waits before it completes, so whatever
 * follows in the stream sees both finished), and consecutive independent
 * matvecs overlap.  No counterpart in the reference (its calls are
 * synchronous). */
#define ASM_MV_INDEPENDENT 1u
ASMLLM_API int asm_matvec_ex_async(int fmt, const void* qweights, const void* scales, int scales_are_f16,
                                   const float* x, float* y, int64_t M, int64_t K, unsigned flags,
                                   void* stream);
/* ---- Packed rows: the resident layout the bulk-copy matvec streams best ----
 * Row r of a packed matrix is its K/32 quant blocks (16 bytes per Q4_0
 * block, 32 per Q8_0) followed by its K/32 fp16 scales: the same 18 (34)
 * bytes per block as GGUF, but R consecutive rows form one contiguous range,
 * fetched by a single bulk copy.  K must be a multiple of 256.
 * asm_packed_row_bytes: bytes of one packed row (-1 if fmt or K is invalid).
 * asm_pack_rows_async: device qweights + fp16 scales -> device packed rows
 * (all 16-byte aligned).  asm_matvec_packed_async: Q4_0 / Q8_0 x Q8_0 on
 * packed rows, same result as asm_matmul_q4_f16s_async /
 * asm_matmul_q8q8_f16s_async on the planes; flags as asm_matvec_ex_async.
 * Host weights registered with asm_weights_register are kept packed when
 * their scales are fp16-exact and K is a multiple of 256; the fp32-activation
 * entries (asm_matmul_q4_avx512, asm_matmul_q4_f32, asm_matmul_q8) then stage
 * those host weights per call instead of using the resident copy.  No
 * counterpart in the reference (its kernels read the two planes). */
ASMLLM_API int64_t asm_packed_row_bytes(int fmt, int64_t K);
/* Measurement aid: enqueues n empty kernels (one CTA per SM) chained the way
 * the matvecs chain -- programmatic dependent launch when pdl != 0, each
 * kernel triggering its dependents at entry and, when wait != 0, waiting for
 * the previous kernel (griddepcontrol.wait).  Timing such a chain gives the
 * per-launch dependency floor a chain of dependent matvecs cannot go below.
 * No counterpart in the reference. */
ASMLLM_API int asm_launch_floor_async(int32_t n, int32_t pdl, int32_t wait, void* stream);
ASMLLM_API int asm_pack_rows_async(int fmt, const void* qweights, const uint16_t* scales_f16, void* packed,
                                   int64_t M, int64_t K, void* stream);
ASMLLM_API int asm_matvec_packed_async(int fmt, const void* packed, const float* x, float* y, int64_t M,
                                       int64_t K, unsigned flags, void* stream);
/* Batched quantize: N rows of x fp32[N][K] -> xq int8[N][K], xd fp32[N][K/32]. */
ASMLLM_API int asm_quantize_q8_0_async(const float* x, int8_t* xq, float* xd,
                                       int64_t N, int64_t K, void* stream);
/* Per-block int32 sums of the Q4_0 x Q8_0 (fmt 2) or Q8_0 x Q8_0 (fmt 8)
 * dot for every (row, block), written to isums int32[M][K/32], computed by
 * the matvec kernel itself (its debug instantiation) so tests can check them
 * bit for bit; y is written too. */
ASMLLM_API int asm_block_sums_async(int fmt, const void* qweights, const float* scales,
                                    const float* x, float* y, int32_t* isums,
                                    int64_t M, int64_t K, void* stream);

/* ---- Q8_0 activation image: quantize once, share across matvecs ------- */

/* Bytes of one row of the activation image for K (a multiple of 32): K/32
 * slots of 48 bytes (32 int8 + 16 pad) followed by K/32 (d fp32, qsum int32)
 * pairs, rounded up to 16.  -1 if K is invalid. */
ASMLLM_API int64_t asm_act_image_bytes(int64_t K);
/* x fp32 [N][K] -> image [N][asm_act_image_bytes(K)]: the activation quantize of
 * matmul_q4_neon.S:57-143 (same int8 and d as asm_quantize_q8_0), laid out for
 * the matvec kernels.  x and image 16-byte aligned device buffers. */
ASMLLM_API int asm_act_image_q8_0_async(const float* x, void* image, int64_t N, int64_t K,
                                        void* stream);
/* The same, and in addition, before it waits for the previous kernel in the
 * stream, prefetches into L2 the first bytes (up to 32 MB) of next_w / next_s --
 * meant to be the weight and scale planes of the matvec that will read this
 * image -- so HBM streaming overlaps the quantize step.  A hint only: results
 * do not depend on it.  next_w / next_s may be NULL. */
ASMLLM_API int asm_act_image_q8_0_prefetch_async(const float* x, void* image, int64_t N, int64_t K,
                                                 const void* next_w, int64_t next_w_bytes,
                                                 const void* next_s, int64_t next_s_bytes,
                                                 void* stream);
/* Matvec on a prepared activation image (fmt 2: Q4_0 x Q8_0, fmt 8: Q8_0 x Q8_0);
 * scales fp32 or fp16 (scales_are_f16).  Same result as the x entries. */
ASMLLM_API int asm_matmul_image_async(int fmt, const void* qweights, const void* scales,
                                      int scales_are_f16, const void* image, float* y, int64_t M,
                                      int64_t K, void* stream);

/* GGUF block split (reference generate.py:91-119): raw GGUF Q4_0 blocks
 * (18 bytes: fp16 d + 16 nibble bytes) or Q8_0 blocks (34 bytes: fp16 d +
 * 32 int8) for `nblocks` blocks -> qs plane (16 or 32 bytes per block) and a
 * scale plane, fp32 (scales_are_f16 = 0) or fp16 (= 1). */
ASMLLM_API int asm_gguf_split_async(int fmt, const uint8_t* raw, uint8_t* qs, void* scales,
                                    int scales_are_f16, int64_t nblocks, void* stream);

/* Declares the device range [ptr, ptr+bytes) static: the caller guarantees
 * that no kernel immediately preceding a matvec in its stream writes it (model
 * weights uploaded once).  Matvecs whose weights and scales lie in static
 * ranges start streaming them before the previous kernel in the stream has
 * finished (programmatic dependent launch); others wait first.  Unmark before
 * rewriting the buffer from a kernel.  Host-registered weights
 * (asm_weights_register) are static automatically. */
ASMLLM_API int asm_weights_mark_static(const void* ptr, int64_t bytes);
ASMLLM_API int asm_weights_unmark_static(const void* ptr);

/* Reads and clears the device error word: bit 0 = a kernel's bounded wait on
 * its shared-memory pipeline timed out (the call's output is not valid).
 * Synchronous entries check it themselves; callers of *_async entries can
 * call this after synchronizing. */
ASMLLM_API int asm_device_error(unsigned* flags);

/* Q4_0 x Q8_0 matvec that allocates no device memory, for callers that
 * cannot allocate during the call (a server that reserves all device memory
 * at start-up, a serving loop with a fixed budget, a plugin whose host owns
 * all allocations).  No counterpart in the reference.  Device pointers, stream
 * ordered; scales fp32 or fp16 (scales_are_f16); same result as
 * asm_matmul_q4_async.  The activation-quantize scratch is a fixed device
 * array inside the library, so K is limited to 32768 (ASM_E_UNSUPPORTED
 * beyond).  The first call on a device sets the array's address up: make it
 * before any stream capture.  Calls share the array: calls that overlap on
 * the GPU (on different streams, for instance) race. */
ASMLLM_API int asm_matmul_q4_noalloc_async(const uint8_t* qweights, const void* scales,
                                           int scales_are_f16, const float* x, float* y, int64_t M,
                                           int64_t K, void* stream);

/* ------------------------------------------------------------------------
 * Batch-1 decode step on the GPU.  The reference runs one token through a
 * Llama layer in AsmEngineForward.forward_token (src/runtime/generate.py:
 * 255-326): asm_rmsnorm, three asm_matmul_q4, asm_rope per head, a numpy KV
 * append and attention, asm_matmul_q4 (o), a residual add, asm_rmsnorm, two
 * asm_matmul_q4 (gate, up), asm_silu_hadamard, asm_matmul_q4 (down), a
 * residual add; then the final asm_rmsnorm and the lm_head product with a
 * numpy argmax (generate.py:318-326, 410-411).  Here the same step is five
 * launches per layer: every norm, residual, SwiGLU and argmax is fused into
 * a matvec's prologue or epilogue, and RoPE + KV append + attention +
 * quantization of its output is one kernel.  Device pointers, stream ordered,
 * capturable in a CUDA graph after one call per shape; the position and the
 * token ids live in device memory, so one captured step replays for every
 * token.  No single counterpart in the reference (it composes the calls
 * above from Python).
 * ------------------------------------------------------------------------ */
#define ASM_EPI_STORE 0    /* y[r] = v */
#define ASM_EPI_RESIDUAL 1 /* y[r] += v (y = residual stream) */
#define ASM_EPI_SWIGLU 2   /* rows (2i, 2i+1) = (gate_i, up_i) -> h_i = silu(gate_i)*up_i -> Q8_0 image */
#define ASM_EPI_ARGMAX 3   /* y[r] = v; then tokens[*pos+1] = argmax_r y[r] and *pos += 1 */

/* Device error word bits (asm_device_error). */
#define ASM_DEVERR_RING_TIMEOUT 1u /* a shared-memory ring wait gave up */
#define ASM_DEVERR_DECODE_RANGE 2u /* position >= ctx / max_tokens or token id >= vocab: step skipped */
#define ASM_DEVERR_XCHG_TIMEOUT 4u /* an exchange / gather wait gave up (a peer never wrote) */
#define ASM_EPI_GATHER 4   /* row-split gather (asm_matvec_rowsplit_async only; not a fused epilogue) */

typedef struct asm_fused_matvec {
  int32_t fmt;      /* 2 = Q4_0, 8 = Q8_0 */
  int32_t epilogue; /* ASM_EPI_* */
  const void* qweights;
  const void* scales;   /* fp16 [M][K/32] */
  /* Prologue: `image` (a Q8_0 activation image, asm_act_image_q8_0_async
   * layout) is copied when set; else the fp32 source row -- embed[tokens[*pos]]
   * when `embed` is set, else `x` -- is quantized, after RMSNorm
   * ((x / sqrt(mean(x^2) + eps)) * norm_w, tests/reference/ops.py:103-116)
   * when `norm_w` is set.  `x_copy`, when set, receives the source row (the
   * residual stream of the first layer). */
  const float* x;
  const void* image;
  const float* norm_w;
  const float* embed; /* fp32 [vocab][K] */
  float* x_copy;
  float* y; /* [M]: output (STORE, ARGMAX: logits) or residual stream (RESIDUAL) */
  float* h; /* SWIGLU: fp32 [M/2] */
  void* image_out;    /* SWIGLU: Q8_0 image of h (K' = M/2) */
  uint32_t* counters; /* SWIGLU: [M/64], zero before the first call, left zero */
  uint64_t* best;     /* ARGMAX: zero before the first call, left zero */
  uint32_t* done;     /* ARGMAX: zero before the first call, left zero */
  int32_t* tokens;    /* [max_tokens]: prompt ids then generated ids */
  int32_t* pos;       /* current position */
  float eps;
  int32_t vocab;
  int32_t max_tokens;
  int32_t n_prompt; /* ARGMAX writes tokens[p+1] only when p+1 >= n_prompt */
  int64_t M, K;
  /* Tensor parallelism (tp > 1; RESIDUAL and ARGMAX only).  RESIDUAL: this
   * rank's partial rows of a row-parallel projection go to every rank's
   * exchange buffer, each rank sums the tp partials in rank order and adds
   * them to y (the residual stream, identical on all ranks).  ARGMAX: rows are
   * this rank's vocabulary slice starting at vocab_offset; the ranks' maxima
   * are exchanged and every rank picks the same token.  xchg[r] = rank r's
   * exchange buffer (asm_ipc_alloc / asm_ipc_open), 2 * tp * xchg_rows 64-bit
   * words, zero before first use; ar_seq = this rank's call counter (zero at
   * start, advanced by each exchanging call); ar_done zero. */
  int32_t tp, tp_rank, xchg_rows, vocab_offset;
  void* xchg[8];
  uint32_t* ar_seq;
  uint32_t* ar_done;
} asm_fused_matvec_t;

/* One fused matvec of a decode step (see above).  Q4_0 / Q8_0 weights with
 * fp16 scales; SWIGLU needs M % 64 == 0. */
ASMLLM_API int asm_fused_matvec_async(const asm_fused_matvec_t* p, void* stream);

/* Device buffers shared between the processes of a tensor-parallel group
 * (CUDA IPC over NVLink).  asm_ipc_alloc: zeroed device buffer of `bytes` on
 * the current device plus its 64-byte handle; asm_ipc_open: maps a peer's
 * buffer from its handle (peer access must be possible); asm_ipc_close
 * unmaps it; asm_ipc_free frees an own buffer. */
ASMLLM_API int asm_ipc_alloc(int64_t bytes, void** ptr, void* handle64);
ASMLLM_API int asm_ipc_open(const void* handle64, void** ptr);
ASMLLM_API int asm_ipc_close(void* ptr);
ASMLLM_API int asm_ipc_free(void* ptr);

/* ---- Row-split matvec over a tensor-parallel group (one process per GPU) ----
 * The reference splits M among its threads (src/runtime/threadpool.c:408-486,
 * asm_threadpool_dispatch_q4): worker t computes a contiguous range of output
 * rows and every row lands in the one shared y.  Across GPUs the same split
 * is: rank r holds rows [r*M, (r+1)*M) of a (tp*M) x K matrix, computes them,
 * and the full y is all-gathered.  Here the gather rides on the matvec: each
 * finished row is stored into y_full[rank*M + row] and, as a (sequence,
 * value) 64-bit word, into every other rank's gather buffer over NVLink
 * (peer stores, no multicast); asm_rowsplit_wait_async then waits (bounded)
 * for the peers' words of a step and completes y_full.
 *   xchg[r]: rank r's gather buffer, at least 2 * tp * M 64-bit words, zero
 *            before first use (asm_ipc_alloc / asm_ipc_open; own entry unused
 *            by the matvec).  One buffer per matvec of a step.
 *   seq:     the group's step counter (device, zero at start, same on every
 *            rank), read by the matvecs and advanced by asm_rowsplit_wait_async.
 * ASM_MV_PACKED: qweights are packed rows (asm_pack_rows_async) and
 * scales_f16 is unused; else planes with fp16 scales.  ASM_MV_INDEPENDENT as
 * for asm_matvec_ex_async.  A step is: its matvecs, then one
 * asm_rowsplit_wait_async naming all of them, on one stream.  The next
 * step's matvecs may compute while the wait runs; each matvec stores its rows
 * to the peers only after the kernel before it in the stream has completed,
 * so no rank overwrites a parity a slower rank still reads.  tp = 1 is a
 * plain matvec into y_full. */
#define ASM_MV_PACKED 2u
ASMLLM_API int asm_matvec_rowsplit_async(int fmt, const void* qweights, const uint16_t* scales_f16,
                                         const float* x, float* y_full, int64_t M, int64_t K, int32_t tp,
                                         int32_t rank, void* const* xchg, uint32_t* seq, unsigned flags,
                                         void* stream);
typedef struct asm_rowsplit_wait {
  int32_t n;            /* matvecs of the step (<= 8) */
  int32_t tp, rank;
  const void* own[8];   /* this rank's gather buffer of matvec j */
  float* y_full[8];     /* its full output [tp * M[j]] */
  int64_t M[8];         /* its rows per rank */
  uint32_t* seq;        /* the step counter */
  uint32_t* done;       /* device word, zero before the first call, left zero */
} asm_rowsplit_wait_t;
/* Waits (each word at most the "xchg_wait_us" limit; a peer that never
 * writes sets ASM_DEVERR_XCHG_TIMEOUT) until every peer row of the step's
 * matvecs has arrived, copies them into y_full, advances *seq. */
ASMLLM_API int asm_rowsplit_wait_async(const asm_rowsplit_wait_t* w, void* stream);

/* RoPE + KV append + attention for position *pos of one layer, one CTA per
 * query head (reference generate.py:281-296 with ops.py:119-141 RoPE):
 *   qkv     fp32 [(n_heads + 2 n_kv_heads) * head_dim] (q, k, v heads)
 *   k_cache, v_cache  fp16 [ctx][n_kv_heads][head_dim] (this layer)
 *   rope_cs fp32 [ctx][head_dim/2][2] = (cos, sin) of pos * theta^(-2i/head_dim)
 *   image_out  Q8_0 activation image of the attention output (K = n_heads*head_dim)
 * scores = q.k / sqrt_head_dim (the reference divides by float32 sqrt(hd)).
 * head_dim must be 128; n_heads a multiple of n_kv_heads (grouped KV). */
ASMLLM_API int asm_attention_decode_async(const float* qkv, void* k_cache, void* v_cache,
                                          const float* rope_cs, const int32_t* pos, void* image_out,
                                          int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                                          int32_t ctx, float sqrt_head_dim, void* stream);

/* The whole decode loop as one persistent kernel.  asm_decode_create builds
 * the per-step program of a resident model (the operations above, in
 * order); asm_decode_run_async then runs n_steps decode steps in ONE
 * cooperative launch: CTAs stay resident for all steps, each streams its
 * share of every weight matrix through a shared-memory ring without stopping
 * between operations, and operations are separated by a grid barrier (a
 * bounded device-side counter wait).  Same arithmetic, bit for bit, as the
 * per-operation entries.  Step s runs position *pos + s; its token is
 * tokens[pos] while pos < n_prompt (and for the first step), else the argmax
 * of the step before; generated ids are stored in tokens[] and *pos is
 * advanced by n_steps.  The run is refused on the device (error bit
 * ASM_DEVERR_DECODE_RANGE, nothing done) if it would pass ctx or max_tokens.
 * Weights: fp16 scales; gate/up rows interleaved (gate_0, up_0, gate_1, ...);
 * q/k/v rows stacked [wq; wk; wv].  No counterpart in the reference. */
typedef struct asm_decode_layer {
  const void* wqkv;
  const void* sqkv; /* [(n_heads + 2 n_kv_heads) * head_dim][dim/32] */
  const void* wo;
  const void* so; /* [dim][n_heads * head_dim / 32] */
  const void* wgu;
  const void* sgu; /* [2 ffn][dim/32] */
  const void* wdown;
  const void* sdown; /* [dim][ffn/32] */
  const float* attn_norm;
  const float* ffn_norm; /* [dim] */
  void* k_cache;
  void* v_cache; /* fp16 [ctx][n_kv_heads][head_dim] */
} asm_decode_layer_t;

typedef struct asm_decode_model {
  int32_t fmt; /* 2 = Q4_0, 8 = Q8_0 */
  int32_t n_layers, dim, n_heads, n_kv_heads, head_dim, ffn, vocab, ctx, max_tokens;
  float eps, sqrt_head_dim;
  const asm_decode_layer_t* layers; /* host array [n_layers], copied by create */
  const void* lm_head;
  const void* lm_scales; /* [vocab][dim/32] */
  const float* final_norm;
  const float* embed;   /* fp32 [vocab][dim] */
  const float* rope_cs; /* fp32 [ctx][head_dim/2][2] */
  /* work buffers (device): */
  float* x;          /* [dim] residual stream */
  float* qkv;        /* [(n_heads + 2 n_kv_heads) * head_dim] */
  void* img_attn;    /* asm_act_image_bytes(n_heads * head_dim) */
  float* h;          /* [ffn] */
  void* img_h;       /* asm_act_image_bytes(ffn) */
  uint32_t* counters; /* [ffn/32], zero */
  float* logits;     /* [vocab] */
  uint64_t* best;    /* [2], zero */
  int32_t* tokens;   /* [max_tokens] */
  int32_t* pos;      /* [1] */
} asm_decode_model_t;

ASMLLM_API int asm_decode_create(const asm_decode_model_t* model, void** handle);
ASMLLM_API int asm_decode_run_async(void* handle, int32_t n_steps, int32_t n_prompt, void* stream);
ASMLLM_API int asm_decode_destroy(void* handle);

/* Batched (prefill) Q4_0 / Q8_0 x Q8_0 product on the tensor cores:
 * y [N][M] fp32, row n = the matvec of activation row n, from N rows of
 * Q8_0 activation images (asm_act_image_q8_0_async with N rows; row stride
 * image_stride bytes, a multiple of 16).  Each output is the reference's
 * NEON combine for that row and token (s = wd * xd, acc = fma(float(isum),
 * s, acc) over the blocks in order), so it equals the Q4_0 x Q8_0 matvec of
 * the reference semantics bit for bit -- when K is not split.  When the
 * 128-row x token tiles alone would leave SMs idle (small N), K is split into
 * S <= 8 contiguous ranges of blocks, each an fma chain from zero, and the S
 * partials are added in range order ((0 + p0) + p1) + ...: deterministic,
 * within fp32 rounding of the unsplit result ("gemm_splits" option below).
 * fp16 scales; qweights 16-byte aligned.  No single counterpart in the
 * reference (its batched work is one asm_matmul_q4 call per token). */
ASMLLM_API int asm_gemm_image_async(int fmt, const void* qweights, const void* scales_f16, const void* images,
                                    int64_t image_stride, float* y, int64_t M, int64_t N, int64_t K,
                                    void* stream);

/* The same product for a few tokens (1 <= N <= 8) on the CUDA cores: at
 * such N the work is bound by the weight stream, so every weight byte is read
 * from HBM once and applied to all N activation rows (held in shared memory,
 * N * (K/32 * 40 bytes) must fit it).  Row n of y equals the Q4_0 / Q8_0 x
 * Q8_0 matvec of activation row n computed by the matvec entries' warp-ring
 * kernel (asm_matvec_ex_async with ASM_MV_INDEPENDENT, asm_matvec_packed_async)
 * bit for bit.  Arguments as asm_gemm_image_async; N > 8 is ASM_E_UNSUPPORTED.
 * No single counterpart in the reference. */
ASMLLM_API int asm_gemm_narrow_async(int fmt, const void* qweights, const void* scales_f16, const void* images,
                                     int64_t image_stride, float* y, int64_t M, int64_t N, int64_t K,
                                     void* stream);

/* Activation tiles: N Q8_0-quantized rows of K values laid out as the fp16
 * operand of the tensor-core product (the int8 quants are exact in fp16).
 * np = N rounded up to 16, 32, 64 or a multiple of 128; plane B (K/32 * np *
 * 64 bytes): block b, token n, position k at b*np*64 + (n/8)*512 + (k/8)*128
 * + (n%8)*16 + (k%8)*2 holds the quant of element 32b + perm(k), perm(8c+j)
 * = 4c + {0,2,1,3,16,18,17,19}[j]; plane D (K/32 * np floats) after it: the
 * block scale of (b, n) at b*np + n.  Rows n >= N are zero.
 * asm_act_tiles_bytes returns the size (0 for invalid N, K).
 * asm_gemm_image_async is asm_act_tiles_from_image_async into stream-ordered
 * scratch followed by asm_gemm_tiles_async; callers that produce tiles
 * directly (the batched decode glue below) skip the conversion. */
ASMLLM_API int64_t asm_act_tiles_bytes(int64_t N, int64_t K);
ASMLLM_API int asm_act_tiles_from_image_async(const void* images, int64_t image_stride, int64_t N, int64_t K,
                                              void* tiles, void* stream);
ASMLLM_API int asm_gemm_tiles_async(int fmt, const void* qweights, const void* scales_f16, const void* tiles,
                                    float* y, int64_t M, int64_t N, int64_t K, void* stream);

/* Batched decode glue: B sequences in lockstep at one position (the
 * reference's AsmEngineForward.forward_token, src/runtime/generate.py:255-326,
 * run for B token rows at once; its matvecs become asm_gemm_tiles_async).
 * One row per sequence; every kernel is stream-ordered and reads what the
 * previous one wrote.
 *   asm_rows_norm_tiles_async: per row, x <- embed[tokens[row][*pos]] (when
 *     embed is set) or x + delta (when delta is set), written back to x; then
 *     RMSNorm (x / sqrt(mean(x^2) + eps)) * norm_w (tests/reference/ops.py:
 *     103-116; plain x when norm_w is NULL), quantized to Q8_0 into row `row`
 *     of the rows' activation tiles.  Out-of-range token ids read row 0 and
 *     set ASM_DEVERR_RANGE.
 *   asm_rows_swiglu_tiles_async: gu [rows][2*ffn] with (gate_i, up_i) pairs
 *     (the gate/up product of interleaved weight rows) -> h = (g / (1 +
 *     exp(-g))) * u (generate.py:370) -> tiles of [rows][ffn].
 *   asm_attention_batch_async: asm_attention_decode_async per row: q/k/v of
 *     row r at qkv + r*qkv_stride (floats), its KV cache at k_cache/v_cache +
 *     r*cache_stride (halves); output quantized into the tiles of [rows]
 *     [n_heads*128].
 *   asm_rows_argmax_async: keys[r] = the first maximum of logits row r
 *     (n values at r*stride; NaN ignored) as a signed-orderable 64-bit key of
 *     (value, offset + index): the max over int64 of the keys of several
 *     vocabulary slices is the key of their combined argmax.
 *   asm_rows_advance_async: tokens[r][*pos + 1] = the index of keys[r] when
 *     *pos + 1 >= n_prompt (and < max_tokens); then *pos += 1. */
typedef struct asm_rows {
  int32_t rows;          /* B */
  int32_t dim;           /* values per row, a multiple of 32 */
  float* x;              /* [rows][dim] residual stream */
  const float* delta;    /* [rows][dim] or NULL */
  const float* embed;    /* [vocab][dim] or NULL */
  const int32_t* tokens; /* [rows][max_tokens] (embed) */
  const int32_t* pos;    /* [1] (embed) */
  int32_t max_tokens;
  int32_t vocab;
  const float* norm_w;   /* [dim] or NULL */
  float eps;
  int32_t reserved;
  void* tiles;           /* asm_act_tiles_bytes(rows, dim) */
} asm_rows_t;

ASMLLM_API int asm_rows_norm_tiles_async(const asm_rows_t* d, void* stream);
ASMLLM_API int asm_rows_swiglu_tiles_async(const float* gu, int32_t rows, int32_t ffn, void* tiles, void* stream);
ASMLLM_API int asm_attention_batch_async(const float* qkv, int64_t qkv_stride, void* k_cache, void* v_cache,
                                         int64_t cache_stride, const float* rope_cs, const int32_t* pos, void* tiles,
                                         int32_t rows, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                                         int32_t ctx, float sqrt_head_dim, void* stream);
ASMLLM_API int asm_rows_argmax_async(const float* logits, int32_t rows, int32_t n, int64_t stride, int32_t offset,
                                     int64_t* keys, void* stream);
ASMLLM_API int asm_rows_advance_async(const int64_t* keys, int32_t rows, int32_t* tokens, int32_t max_tokens,
                                      int32_t* pos, int32_t n_prompt, void* stream);

/* Q5_0 x fp32 on device pointers (see asm_matmul_q5), stream ordered. */
ASMLLM_API int asm_matmul_q5_async(const uint8_t* ql, const uint8_t* qh, const float* scales,
                                   const float* x, float* y, int64_t M, int64_t K, void* stream);

/* Kernel-path switches for testing and tuning; returns the previous value
 * (-1 for an unknown name).  "tma": 1 = Q8_0-activation matvecs use the
 * bulk-copy pipeline kernel where the shape allows (default), 0 = the
 * register-streaming kernels.  "pdl": programmatic dependent launch on/off.
 * "image_min_k": Q8_0-activation matvecs given fp32 x with K >= this value
 * quantize x in a separate pre-pass kernel into stream-ordered scratch
 * instead of in every CTA (default 0 = always in the CTAs: with the per-warp
 * ring kernel the pre-pass measured slower at K = 11008 and 28672).
 * "gemm_splits": 0 = the batched product picks its K split (default),
 * S >= 1 = exactly S ranges (clamped to [1, 8] and to the number of 128-byte
 * weight stages).  Results are identical either way up to fp32 summation
 * order.  "sync_map": how the synchronous entries treat pinned host x and y
 * of the current device: bit 0 = the activation pre-pass reads x in place
 * through its mapped address, bit 1 = the matvec writes y in place (default
 * 3); a cleared bit stages that buffer with a copy.
 * Plan of the bulk-copy matvec (results do not depend on them): "mv_rows"
 * rows per stage, 1, 2 or 4 (0 = automatic, default); "mv_slots" cap on the
 * ring slots of each warp (0 = automatic up to 6, default); "mv_smem_kb"
 * shared-memory budget of a CTA in KB (default 110, which leaves room on
 * every SM for a CTA of the next launch; a plan that does not fit takes the
 * whole opt-in shared memory); "mv_ctas" CTAs per SM (default 1).
 * "mv_kernel": which bulk-copy kernel streams a matvec: 0 (default) = the
 * fused decode-step matvecs (asm_fused_matvec_async) and plain matvecs with
 * rows of more than 128 blocks in launches that wait for the previous kernel
 * go to the row-stage kernel (one producer warp, ~16 KB stages of whole rows
 * shared by 16 warps), everything else to the warp-ring kernel; 1 = warp rings always;
 * 2 = row stages wherever they apply (not packed rows, not independent
 * launches).  The two kernels add a row's products in different fixed orders,
 * so y may differ in the last bits between settings (each is deterministic).
 * "sync_fused": 1 = the synchronous Q8_0-activation entries quantize x
 * inside the matvec kernel instead of in a pre-pass into a per-device image
 * (default 0).  "image_prefetch_mb": the activation pre-pass also pulls up to
 * this many MB of the following matvec's weights into L2 (default 0 = off).
 * "xchg_wait_us": limit of every tensor-parallel exchange and row-split
 * gather wait on the current device, in microseconds at about 2 GHz (0 =
 * the default, about a second); a wait that runs out sets
 * ASM_DEVERR_XCHG_TIMEOUT and the kernel returns. */
ASMLLM_API int asm_set_option(const char* name, int value);

/* Largest K each matvec family supports (shared-memory staging of x). */
ASMLLM_API int64_t asm_max_k(int fmt, int fp32_activations);

/* Library version string. */
ASMLLM_API const char* asm_version(void);

#ifdef __cplusplus
}
#endif

#endif /* ASMLLM_B200_H */

// asmllm_b200/csrc/narrow_gemm.cuh -- the batched Q4_0/Q8_0 x Q8_0 product
// for a few tokens (N <= 8), on the CUDA cores: each weight byte is read from
// HBM once for all N activation rows.  Included by tma_matvec.cu only (it
// shares that unit's block-dot and reduction helpers).
//
// At N <= 8 the product is bound by the weight stream (N multiply-adds per
// weight byte), where the tensor-core kernel's role handoffs dominate.  Here a
// warp takes two rows at a time: each lane loads its blocks b = lane + 32 j
// of both rows into registers (chunks of 2 blocks, the next chunk's loads
// issued before the current one is used; Q4_0 nibble masks applied once per
// block), then for every token reads
// that block's activation from shared memory once and applies it to both
// rows.  The N activation images sit in shared memory in the swizzled layout
// of the matvec kernel.  Per row and token the products are added in the
// matvec kernel's order (lane l: its blocks in ascending order, fma into one
// accumulator; then the same butterfly across the warp), so row n of Y equals
// the warp-ring matvec of activation row n bit for bit.

template <int FMT, int NA>
__global__ void __launch_bounds__(256, 2)
narrow_gemm_kernel(const uint8_t* __restrict__ w, const __half* __restrict__ scales,
                   const unsigned char* __restrict__ images, long long img_stride, float* __restrict__ y, int M,
                   int nb) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int UB = FMT == kFmtQ4_0 ? 16 : 32;  // weight bytes per block
  constexpr int QW = UB / 16;                    // uint4 per block
  constexpr int CJ = 2;                          // blocks per lane per chunk
  const size_t img_b = smem_image_bytes(nb);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

  // N activation images: the 48-byte slots' two 16-byte halves into the
  // swizzled quant area, then the (d, q-sum) pairs.
  for (int n = 0; n < NA; ++n) {
    const unsigned char* src = images + (size_t)n * (size_t)img_stride;
    unsigned char* dst = smem + (size_t)n * img_b;
    for (int i = threadIdx.x; i < 2 * nb; i += blockDim.x)
      *reinterpret_cast<uint4*>(dst + xhalf(i >> 1, i & 1)) =
          __ldg(reinterpret_cast<const uint4*>(src + (size_t)(i >> 1) * 48 + (i & 1) * 16));
    for (int b = threadIdx.x; b < nb; b += blockDim.x)
      reinterpret_cast<float2*>(dst + (size_t)nb * 32)[b] = __ldg(reinterpret_cast<const float2*>(src + (size_t)nb * 48) + b);
  }
  __syncthreads();

  const size_t row_w = (size_t)nb * UB;
  const int n_pairs = (M + 1) / 2;
  const int nj = (nb + 31) / 32;  // block slots per lane
  for (int pr = blockIdx.x * (blockDim.x / 32) + warp; pr < n_pairs; pr += gridDim.x * (blockDim.x / 32)) {
    const int row0 = 2 * pr;
    const bool has1 = row0 + 1 < M;
    float acc[NA][2];
#pragma unroll
    for (int n = 0; n < NA; ++n) acc[n][0] = acc[n][1] = 0.0f;
    uint4 q[2][CJ][QW], qn[2][CJ][QW];
    float sc[2][CJ], scn[2][CJ];
    auto load_chunk = [&](int j0, uint4 (&qq)[2][CJ][QW], float (&ss)[2][CJ]) {
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int jj = 0; jj < CJ; ++jj) {
          const int b = lane + 32 * (j0 + jj);
          const bool in = b < nb && (r == 0 || has1);
          const uint4* src = reinterpret_cast<const uint4*>(w + (size_t)(row0 + r) * row_w + (size_t)b * UB);
#pragma unroll
          for (int h = 0; h < QW; ++h) qq[r][jj][h] = in ? __ldg(src + h) : make_uint4(0u, 0u, 0u, 0u);
          ss[r][jj] = in ? __half2float(scales[(size_t)(row0 + r) * nb + b]) : 0.0f;
        }
    };
    load_chunk(0, q, sc);
    for (int j0 = 0; j0 < nj; j0 += CJ) {
      if (j0 + CJ < nj) load_chunk(j0 + CJ, qn, scn);  // the next chunk in flight during this one
#pragma unroll
      for (int jj = 0; jj < CJ; ++jj) {
        const int b = lane + 32 * (j0 + jj);
        const bool in = b < nb;
        const int bb = in ? b : 0;
        // Q4_0: the nibble masks once per block, not once per token
        uint4 lo[2], hi[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const uint4 qq = q[r][jj][0];
          lo[r] = make_uint4(qq.x & 0x0F0F0F0Fu, qq.y & 0x0F0F0F0Fu, qq.z & 0x0F0F0F0Fu, qq.w & 0x0F0F0F0Fu);
          hi[r] = make_uint4(qq.x & 0xF0F0F0F0u, qq.y & 0xF0F0F0F0u, qq.z & 0xF0F0F0F0u, qq.w & 0xF0F0F0F0u);
        }
#pragma unroll
        for (int n = 0; n < NA; ++n) {
          const uint32_t xs = smem_u32(smem + (size_t)n * img_b);
          uint4 xa = lds_v4(xs + (uint32_t)xhalf(bb, 0)), xb = lds_v4(xs + (uint32_t)xhalf(bb, 1));
          const float2 dq = reinterpret_cast<const float2*>(smem + (size_t)n * img_b + (size_t)nb * 32)[bb];
          const float xd = in ? dq.x : 0.0f;
          const int qs8 = in ? __float_as_int(dq.y) * 8 : 0;
          if (!in) xa = xb = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            int isum;
            if (FMT == kFmtQ4_0) {  // as q4_block_dot, on the pre-masked nibbles
              int l = 0, h = 0;
              l = dp4a_us(lo[r].x, (int)xa.x, l);
              h = dp4a_us(hi[r].x, (int)xb.x, h);
              l = dp4a_us(lo[r].y, (int)xa.y, l);
              h = dp4a_us(hi[r].y, (int)xb.y, h);
              l = dp4a_us(lo[r].z, (int)xa.z, l);
              h = dp4a_us(hi[r].z, (int)xb.z, h);
              l = dp4a_us(lo[r].w, (int)xa.w, l);
              h = dp4a_us(hi[r].w, (int)xb.w, h);
              isum = l + (h >> 4) - qs8;
            } else {
              isum = q8_block_dot(q[r][jj][0], q[r][jj][QW - 1], xa, xb);
            }
            acc[n][r] = __fmaf_rn(__int2float_rn(isum), __fmul_rn(sc[r][jj], xd), acc[n][r]);
          }
        }
      }
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int jj = 0; jj < CJ; ++jj) {
          sc[r][jj] = scn[r][jj];
#pragma unroll
          for (int h = 0; h < QW; ++h) q[r][jj][h] = qn[r][jj][h];
        }
    }
#pragma unroll
    for (int n = 0; n < NA; ++n) {
      const float v = rows_reduce<2>(acc[n], lane);
      const int r = lane >> 4;  // lane 0: row0, lane 16: row0 + 1
      if ((lane & 15) == 0 && (r == 0 || has1)) y[(size_t)n * M + row0 + r] = v;
    }
  }
}

namespace {

template <int FMT, int NA>
cudaError_t launch_narrow_t(const uint8_t* w, const __half* s, const unsigned char* images, long long stride,
                            float* y, int M, int nb, int sms, int smem_optin, cudaStream_t stream) {
  auto kernel = narrow_gemm_kernel<FMT, NA>;
  const size_t smem = (size_t)NA * smem_image_bytes(nb);
  if (smem > (size_t)smem_optin) return cudaErrorInvalidValue;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(g_tma_mu);
    auto key = std::make_tuple((const void*)kernel, dev);
    if (!g_tma_attr[key]) {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_optin);
      if (e != cudaSuccess) return e;
      g_tma_attr[key] = true;
    }
  }
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, 256, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) per_sm = 1;
  long long grid = (long long)sms * per_sm;
  const long long warps_needed = ((M + 1) / 2 + 7) / 8;
  if (grid > warps_needed) grid = warps_needed;
  if (grid < 1) grid = 1;
  kernel<<<(unsigned)grid, 256, smem, stream>>>(w, s, images, stride, y, M, nb);
  return cudaGetLastError();
}

template <int FMT>
cudaError_t launch_narrow_fmt(const uint8_t* w, const __half* s, const unsigned char* images, long long stride,
                              float* y, int M, int N, int nb, int sms, int smem_optin, cudaStream_t stream) {
  switch (N) {
    case 1: return launch_narrow_t<FMT, 1>(w, s, images, stride, y, M, nb, sms, smem_optin, stream);
    case 2: return launch_narrow_t<FMT, 2>(w, s, images, stride, y, M, nb, sms, smem_optin, stream);
    case 3: return launch_narrow_t<FMT, 3>(w, s, images, stride, y, M, nb, sms, smem_optin, stream);
    case 4: return launch_narrow_t<FMT, 4>(w, s, images, stride, y, M, nb, sms, smem_optin, stream);
    case 5: return launch_narrow_t<FMT, 5>(w, s, images, stride, y, M, nb, sms, smem_optin, stream);
    case 6: return launch_narrow_t<FMT, 6>(w, s, images, stride, y, M, nb, sms, smem_optin, stream);
    case 7: return launch_narrow_t<FMT, 7>(w, s, images, stride, y, M, nb, sms, smem_optin, stream);
    case 8: return launch_narrow_t<FMT, 8>(w, s, images, stride, y, M, nb, sms, smem_optin, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_gemm_narrow(int fmt, const void* w, const void* scales_f16, const void* images,
                               long long image_stride, float* y, long long M, long long N, long long K, int sms,
                               int smem_optin, cudaStream_t stream) {
  if (N < 1 || N > kNarrowMaxN || K <= 0 || K % 32 != 0 || M <= 0 || M > 0x7fffffffLL) return cudaErrorInvalidValue;
  const int nb = (int)(K / 32);
  const auto* wp = static_cast<const uint8_t*>(w);
  const auto* sp = static_cast<const __half*>(scales_f16);
  const auto* ip = static_cast<const unsigned char*>(images);
  if (fmt == kFmtQ4_0) return launch_narrow_fmt<kFmtQ4_0>(wp, sp, ip, image_stride, y, (int)M, (int)N, nb, sms, smem_optin, stream);
  return launch_narrow_fmt<kFmtQ8_0>(wp, sp, ip, image_stride, y, (int)M, (int)N, nb, sms, smem_optin, stream);
}

// quant.cu -- int4 weight format kernels (quantise, dequantise, prepack for the grouped
// GEMM) and the row gather used by the reference-compatible permute op.
//
// Canonical format (defined by this library; the reference only carries the unused flag
// EngineConfig.use_int4_quantization, python/light_moe/engine/executor.py:44-48):
//   qweight uint8 [rows, K/2]  byte b = (q[2b] + 8) | (q[2b+1] + 8) << 4
//   scales  fp16  [rows, K/g]  s = fp16_rn(max|w| / 7)
//   q = clamp(rint(w / float(s)), -8, 7)     (q = 0 when s == 0)
//   dequantised value = bf16_rn(float(q) * float(s))
// The arithmetic is the same IEEE sequence as oracle/lmoe_oracle.c, so results are bit-exact.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "host_util.h"
#include "w4_layout.cuh"

namespace lmoe {
namespace {

// one warp per (row, group); lane handles pairs p = lane, lane + 32, ...
template <typename Tin>
__global__ void quantize_w4_kernel(const Tin* __restrict__ w, int64_t rows, int K, int g,
                                   uint8_t* __restrict__ q, uint16_t* __restrict__ scales) {
  const int G = K / g;
  const int64_t warp_id = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp_id >= rows * G) return;
  const int64_t r = warp_id / G;
  const int gi = (int)(warp_id % G);
  const Tin* wr = w + r * K + (int64_t)gi * g;
  float m = 0.0f;
  for (int p = lane; p < g / 2; p += 32) {
    float a, b;
    if constexpr (sizeof(Tin) == 4) {
      a = wr[2 * p];
      b = wr[2 * p + 1];
    } else {
      a = __bfloat162float(wr[2 * p]);
      b = __bfloat162float(wr[2 * p + 1]);
    }
    m = fmaxf(m, fmaxf(fabsf(a), fabsf(b)));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const __half s16 = __float2half_rn(__fdiv_rn(m, 7.0f));
  const float sf = __half2float(s16);
  if (lane == 0) scales[r * G + gi] = __half_as_ushort(s16);
  const bool usable = sf != 0.0f && isfinite(sf);
  for (int p = lane; p < g / 2; p += 32) {
    float a, b;
    if constexpr (sizeof(Tin) == 4) {
      a = wr[2 * p];
      b = wr[2 * p + 1];
    } else {
      a = __bfloat162float(wr[2 * p]);
      b = __bfloat162float(wr[2 * p + 1]);
    }
    int qa = 0, qb = 0;
    if (usable) {
      const float xa = rintf(__fdiv_rn(a, sf));
      const float xb = rintf(__fdiv_rn(b, sf));
      qa = xa > 7.0f ? 7 : (xa < -8.0f ? -8 : (int)xa);
      qb = xb > 7.0f ? 7 : (xb < -8.0f ? -8 : (int)xb);
    }
    q[r * (K / 2) + ((int64_t)gi * g) / 2 + p] = (uint8_t)(((qa + 8) & 15) | (((qb + 8) & 15) << 4));
  }
}

// one thread per packed byte -> two bf16 outputs
__global__ void dequantize_w4_kernel(const uint8_t* __restrict__ q, const uint16_t* __restrict__ scales,
                                     int64_t rows, int K, int g, __nv_bfloat162* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nbytes = rows * (K / 2);
  if (i >= nbytes) return;
  const int64_t r = i / (K / 2);
  const int kk = (int)(i % (K / 2)) * 2;
  const uint8_t b = q[i];
  const float sf = __half2float(__ushort_as_half(scales[r * (K / g) + kk / g]));
  const float lo = __fmul_rn((float)((int)(b & 15) - 8), sf);
  const float hi = __fmul_rn((float)((int)(b >> 4) - 8), sf);
  out[i] = __nv_bfloat162(__float2bfloat16_rn(lo), __float2bfloat16_rn(hi));
}

// permuted[r] = hidden[sorted_idx[r] / top_k]; one CTA per row, 16-byte vectors
__global__ void permute_rows_kernel(const uint4* __restrict__ hidden, const int32_t* __restrict__ sorted_idx,
                                    int64_t rows, int vec_per_row, int top_k, uint4* __restrict__ out) {
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const int64_t src = sorted_idx[r] / top_k;
    const uint4* s = hidden + src * vec_per_row;
    uint4* d = out + r * vec_per_row;
    for (int i = threadIdx.x; i < vec_per_row; i += blockDim.x) d[i] = __ldg(s + i);
  }
}

}  // namespace
}  // namespace lmoe

using namespace lmoe;

extern "C" int lmoe_quantize_w4(const void* w, int w_is_fp32, int64_t rows, int K, int group_size, uint8_t* qweight,
                                uint16_t* scales, lmoe_stream_t stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  LMOE_ARG_CHECK(rows >= 0 && K > 0 && group_size > 0 && (group_size % 2) == 0 && (K % group_size) == 0);
  if (rows == 0) return LMOE_OK;
  LMOE_ARG_CHECK(w && qweight && scales);
  const int64_t warps = rows * (K / group_size);
  const int threads = 256;
  const int64_t blocks = (warps * 32 + threads - 1) / threads;
  LMOE_ARG_CHECK(blocks < (int64_t)INT32_MAX);
  if (w_is_fp32)
    quantize_w4_kernel<float><<<(unsigned)blocks, threads, 0, stream>>>(static_cast<const float*>(w), rows, K,
                                                                       group_size, qweight, scales);
  else
    quantize_w4_kernel<__nv_bfloat16><<<(unsigned)blocks, threads, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(w), rows, K, group_size, qweight, scales);
  return cuda_status(cudaGetLastError());
}

extern "C" int lmoe_dequantize_w4(const uint8_t* qweight, const uint16_t* scales, int64_t rows, int K, int group_size,
                                  void* out, lmoe_stream_t stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  LMOE_ARG_CHECK(rows >= 0 && K > 0 && group_size > 0 && (group_size % 2) == 0 && (K % group_size) == 0);
  if (rows == 0) return LMOE_OK;
  LMOE_ARG_CHECK(qweight && scales && out && (reinterpret_cast<uintptr_t>(out) & 3u) == 0);
  const int64_t n = rows * (K / 2);
  const int threads = 256;
  const int64_t blocks = (n + threads - 1) / threads;
  LMOE_ARG_CHECK(blocks < (int64_t)INT32_MAX);
  dequantize_w4_kernel<<<(unsigned)blocks, threads, 0, stream>>>(qweight, scales, rows, K, group_size,
                                                                 static_cast<__nv_bfloat162*>(out));
  return cuda_status(cudaGetLastError());
}

extern "C" int lmoe_permute_rows(const void* hidden, int elem_bytes, const int32_t* sorted_idx, int64_t rows,
                                 int hidden_size, int top_k, void* permuted, lmoe_stream_t stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  LMOE_ARG_CHECK(elem_bytes == 2 || elem_bytes == 4);
  LMOE_ARG_CHECK(rows >= 0 && hidden_size > 0 && ((int64_t)hidden_size * elem_bytes) % 16 == 0 && top_k >= 1);
  if (rows == 0) return LMOE_OK;
  LMOE_ARG_CHECK(hidden && sorted_idx && permuted && aligned16(hidden) && aligned16(permuted));
  const int vec = (int)(((int64_t)hidden_size * elem_bytes) / 16);   // 16-byte pieces per row
  const int threads = vec >= 256 ? 256 : ((vec + 31) / 32) * 32;
  const int64_t grid = rows < 65535 * 4 ? rows : 65535 * 4;
  permute_rows_kernel<<<(unsigned)grid, threads, 0, stream>>>(static_cast<const uint4*>(hidden), sorted_idx, rows,
                                                              vec, top_k, static_cast<uint4*>(permuted));
  return cuda_status(cudaGetLastError());
}

// simt_gemm.cu -- dense fp32 grouped GEMM on CUDA cores, for fp32 callers of the reference's
// grouped_gemm op.
//
// The reference multiplies each expert's rows in the input dtype with cuBLAS
// (csrc/grouped_gemm.cu:30-40, torch::mm_out); for fp32 inputs that is an fp32 GEMM, which the
// tcgen05 tensor cores (16-bit, 8-bit and tf32 operands) cannot reproduce.  This kernel keeps
// fp32 operands and accumulates each output with fp32 FFMA in K order.
//
// Tiles of 64 rows (of one segment) x 64 output columns, 16 K values per step staged in
// shared memory, each of the 256 threads owning 4 x 4 outputs.  The offsets are read on the
// device; every CTA derives the tile list from them (segment-major), so there is no host copy.
#include <cuda_runtime.h>

#include "grouped_gemm.h"
#include "host_util.h"
#include "ptx.cuh"

namespace lmoe {
namespace {

constexpr int kTM = 64, kTN = 64, kTK = 16, kNT = 256;
constexpr uint32_t kSite = 0x400u;

__global__ void __launch_bounds__(kNT) grouped_gemm_f32_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                                const void* offsets, int offsets_i64, int E, int N,
                                                                int K, int64_t R, float* __restrict__ out,
                                                                uint32_t* err) {
  __shared__ int row_off[kMaxGemmExperts + 1];
  __shared__ int tile_start[kMaxGemmExperts + 1];
  __shared__ __align__(16) float xs[kTK][kTM + 4];
  __shared__ __align__(16) float ws[kTK][kTN + 4];
  const int tid = threadIdx.x;
  for (int e = tid; e <= E; e += kNT) {
    const int64_t o = offsets_i64 ? static_cast<const int64_t*>(offsets)[e]
                                  : (int64_t) static_cast<const int32_t*>(offsets)[e];
    row_off[e] = (int)(o < 0 ? -1 : (o > R ? R + 1 : o));
  }
  __syncthreads();
  const int nb = (N + kTN - 1) / kTN;
  if (tid == 0) {
    int acc = 0;
    tile_start[0] = 0;
    for (int e = 0; e < E; ++e) {
      int n_e = row_off[e + 1] - row_off[e];
      if (n_e < 0 || row_off[e] < 0 || row_off[e + 1] > R) {   // rows outside the input: skipped
        if (n_e != 0) report_error(err, kErrBadArg, kSite + 1);
        n_e = 0;
      }
      acc += ((n_e + kTM - 1) / kTM) * nb;
      tile_start[e + 1] = acc;
    }
  }
  __syncthreads();
  const int total = tile_start[E];
  const int tx = tid % (kTN / 4), ty = tid / (kTN / 4);
  int e = 0;
  for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
    while (tile >= tile_start[e + 1]) ++e;
    const int n_e = row_off[e + 1] - row_off[e];
    const int ntb = (n_e + kTM - 1) / kTM;
    const int local = tile - tile_start[e];
    const int fb = local / ntb, tb = local - fb * ntb;
    const int64_t r0 = row_off[e] + (int64_t)tb * kTM;
    const int rows = min(kTM, n_e - tb * kTM);
    const int n0 = fb * kTN;
    const float* wb = w + ((int64_t)e * N) * K;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
    for (int k0 = 0; k0 < K; k0 += kTK) {
      {   // one float4 of x and one of w per thread: 64 rows x 16 K each
        const int r = tid / (kTK / 4), kq = tid % (kTK / 4);
        const int k = k0 + kq * 4;
        float4 xv = make_float4(0.f, 0.f, 0.f, 0.f), wv = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r < rows && k < K) xv = *reinterpret_cast<const float4*>(x + (r0 + r) * K + k);
        if (n0 + r < N && k < K) wv = *reinterpret_cast<const float4*>(wb + (int64_t)(n0 + r) * K + k);
        xs[kq * 4 + 0][r] = xv.x; xs[kq * 4 + 1][r] = xv.y; xs[kq * 4 + 2][r] = xv.z; xs[kq * 4 + 3][r] = xv.w;
        ws[kq * 4 + 0][r] = wv.x; ws[kq * 4 + 1][r] = wv.y; ws[kq * 4 + 2][r] = wv.z; ws[kq * 4 + 3][r] = wv.w;
      }
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < kTK; ++kk) {
        const float4 a4 = *reinterpret_cast<const float4*>(&xs[kk][ty * 4]);
        const float4 b4 = *reinterpret_cast<const float4*>(&ws[kk][tx * 4]);
        const float av[4] = {a4.x, a4.y, a4.z, a4.w}, bv[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = __fmaf_rn(av[i], bv[j], acc[i][j]);
      }
      __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = ty * 4 + i;
      if (r >= rows) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = n0 + tx * 4 + j;
        if (n < N) out[(r0 + r) * N + n] = acc[i][j];
      }
    }
  }
}

}  // namespace

int run_grouped_gemm_f32(const float* x, int64_t total_rows, int K, const float* w, int N, const void* offsets,
                         int offsets_i64, int num_experts, float* out, uint32_t* err, cudaStream_t stream) {
  if (num_experts < 1 || num_experts > kMaxGemmExperts) return LMOE_ERR_UNSUPPORTED;
  if (K <= 0 || K % 4 || N <= 0 || total_rows < 0 || total_rows > INT32_MAX) return LMOE_ERR_INVALID_ARG;
  if (!x || !w || !offsets || !out || !aligned16(x) || !aligned16(w)) return LMOE_ERR_INVALID_ARG;
  if (total_rows == 0) return LMOE_OK;
  DeviceInfo dev;
  const int st = get_device_info(&dev);
  if (st != LMOE_OK) return st;
  // persistent: a few CTAs per SM walk the tile list
  grouped_gemm_f32_kernel<<<dev.num_sms * 4, kNT, 0, stream>>>(x, w, offsets, offsets_i64, num_experts, N, K,
                                                                total_rows, out, err);
  return cuda_status(cudaGetLastError());
}

}  // namespace lmoe

// layer.cu -- C-ABI entry points for the grouped GEMMs and the W4A16 MoE layer, plus the
// small glue kernels between them (routing-table expansion, row gather, int4 prepacking,
// weighted combine).
//
// Layer data flow (all on one stream, no host synchronisation):
//   router     x, Wg          -> ids, weights, counts, offsets, sorted_idx      (router.cu)
//   table      sorted_idx     -> per dispatched row: source token, output slot, weight;
//                                expert offsets extended with the always-on shared experts
//   gather     x              -> xp [R, d]   rows in expert order (permute)
//   gate/up    xp, W13 (int4) -> h  [R, ffn] = silu(x W1^T) * (x W3^T)   (SwiGLU epilogue)
//   down       h,  W2  (int4) -> o  [T*(k+S), d] = weight * (h W2^T), scattered to its slot
//   combine    o              -> y  [T, d]   = sum over the token's slots (fixed order)
// Reference: SparseMoEBlock.forward (python/light_moe/model/moe_block.py:119-169) and
// SparseMoEBlockFast.forward (moe_block.py:216-274).
#include <cuda_bf16.h>

#include "decode_gemm.h"
#include "grouped_gemm.h"
#include "host_util.h"
#include "ptx.cuh"
#include "w4_layout.cuh"

namespace lmoe {
namespace {

// ------------------------------------------------------------------------------------ prepack
// Output super-block (e, fb, sb) of w4_layout.cuh.  Source rows: plain blocks of 128 rows,
// or (paired) 64 rows of A followed by the same 64 rows of B.
__device__ __forceinline__ int64_t prepack_src_row(int e, int rows_in, int fb, int r, int paired) {
  return paired ? (int64_t)e * rows_in + fb * 64 + (r & 63) : (int64_t)e * rows_in + fb * kW4BlockRows + r;
}

// int4 part: one thread per output 16-byte chunk (e, fb, sb, j, h, row).
__global__ void prepack_w4_kernel(const uint8_t* __restrict__ qa, const uint8_t* __restrict__ qb, int E, int rows_in,
                                  int K, int sb_bytes, uint8_t* __restrict__ out, int paired) {
  const int NB = paired ? rows_in / 64 : rows_in / kW4BlockRows;
  const int KSB = K / kW4SuperK;
  const int64_t total = (int64_t)E * NB * KSB * 4 * kW4BlockRows;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int r = (int)(i % kW4BlockRows);
  int64_t rest = i / kW4BlockRows;
  const int jh = (int)(rest % 4);   // k-block j = jh / 2, half h = jh % 2
  rest /= 4;
  const int sb = (int)(rest % KSB);
  rest /= KSB;
  const int fb = (int)(rest % NB);
  const int e = (int)(rest / NB);
  const uint8_t* src = (paired && r >= 64) ? qb : qa;
  const int64_t srow = prepack_src_row(e, rows_in, fb, r, paired);
  const int k0 = sb * kW4SuperK + (jh >> 1) * 64 + (jh & 1) * 32;
  const uint4 c = *reinterpret_cast<const uint4*>(src + srow * (K / 2) + k0 / 2);
  const uint4 o = w4_device_half(c);
  uint8_t* dst = out + ((int64_t)(e * NB + fb) * KSB + sb) * sb_bytes + jh * 2048 + r * 16;
  *reinterpret_cast<uint4*>(dst) = o;
}

// scale part: one thread per (e, fb, sb, group-in-super-block, row).
__global__ void prepack_scales_kernel(const uint16_t* __restrict__ sa, const uint16_t* __restrict__ sb_in, int E,
                                      int rows_in, int K, int g, int sb_bytes, uint8_t* __restrict__ out,
                                      int paired) {
  const int NB = paired ? rows_in / 64 : rows_in / kW4BlockRows;
  const int KSB = K / kW4SuperK;
  const int SG = w4_scale_groups(g);
  const int G = K / g;
  const int64_t total = (int64_t)E * NB * KSB * SG * kW4BlockRows;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int r = (int)(i % kW4BlockRows);
  int64_t rest = i / kW4BlockRows;
  const int gi = (int)(rest % SG);
  rest /= SG;
  const int sb = (int)(rest % KSB);
  rest /= KSB;
  const int fb = (int)(rest % NB);
  const int e = (int)(rest / NB);
  const uint16_t* src = (paired && r >= 64) ? sb_in : sa;
  const int64_t srow = prepack_src_row(e, rows_in, fb, r, paired);
  const int group = (sb * kW4SuperK + gi * (g < kW4SuperK ? g : 0)) / g;
  uint16_t* dst = reinterpret_cast<uint16_t*>(out + ((int64_t)(e * NB + fb) * KSB + sb) * sb_bytes +
                                              kW4SuperInt4Bytes + gi * 256) + r;
  *dst = src[srow * G + group];
}

// ------------------------------------------------------------------------------------ routing table
// rows r < T*k come from the router's sorted order; rows T*k + s*T + t are token t for
// shared expert s.  Slots are [T, k + S]: routed slot j, then shared slot k + s.
__global__ void routing_table_kernel(const int32_t* __restrict__ sorted_idx, const float* __restrict__ weights,
                                     const int32_t* __restrict__ offsets, int T, int k, int E, int S,
                                     int32_t* __restrict__ src_tok, int32_t* __restrict__ dest,
                                     float* __restrict__ scale, int32_t* __restrict__ offsets_ext) {
  const int64_t Rr = (int64_t)T * k;
  const int64_t R = Rr + (int64_t)S * T;
  const int slots = k + S;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < R) {
    if (i < Rr) {
      const int f = sorted_idx[i];
      const int t = f / k;
      const int j = f - t * k;
      src_tok[i] = t;
      dest[i] = t * slots + j;
      scale[i] = weights[f];
    } else {
      const int64_t u = i - Rr;
      const int s = (int)(u / T);
      const int t = (int)(u - (int64_t)s * T);
      src_tok[i] = t;
      dest[i] = t * slots + k + s;
      scale[i] = 1.0f;
    }
  }
  if (i <= E + S) {
    offsets_ext[i] = (i <= E) ? offsets[i] : (int32_t)(Rr + (int64_t)(i - E) * T);
  }
}

__global__ void gather_rows_kernel(const uint4* __restrict__ x, const int32_t* __restrict__ src_tok, int64_t rows,
                                   int vec_per_row, uint4* __restrict__ out) {
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const uint4* s = x + (int64_t)src_tok[r] * vec_per_row;
    uint4* d = out + r * vec_per_row;
    for (int i = threadIdx.x; i < vec_per_row; i += blockDim.x) d[i] = __ldg(s + i);
  }
}

// y[t, :] = sum_{j < slots} o[t*slots + j, :]  (fp32 accumulation in slot order, bf16 out);
// 8 columns (one 16-byte load per slot row) per thread
__global__ void combine_slots16_kernel(const uint4* __restrict__ o, int64_t T, int slots, int d8,
                                       uint4* __restrict__ y) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * d8) return;
  const int64_t t = i / d8;
  const int c = (int)(i - t * d8);
  float acc[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) acc[q] = 0.0f;
  const uint4* p = o + t * slots * d8 + c;
  for (int j = 0; j < slots; ++j) {
    const uint4 v = __ldcs(p + (int64_t)j * d8);   // read once: do not keep in L2
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[q]));
      acc[2 * q] = __fadd_rn(acc[2 * q], f.x);
      acc[2 * q + 1] = __fadd_rn(acc[2 * q + 1], f.y);
    }
  }
  uint32_t r[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(acc[2 * q], acc[2 * q + 1]);
    r[q] = *reinterpret_cast<const uint32_t*>(&h);
  }
  y[i] = make_uint4(r[0], r[1], r[2], r[3]);
}

// the same with 2 columns per thread (outputs that are not 16-byte aligned)
__global__ void combine_slots_kernel(const __nv_bfloat162* __restrict__ o, int64_t T, int slots, int d2,
                                     __nv_bfloat162* __restrict__ y) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * d2) return;
  const int64_t t = i / d2;
  const int c = (int)(i - t * d2);
  float ax = 0.0f, ay = 0.0f;
  const __nv_bfloat162* p = o + t * slots * d2 + c;
  for (int j = 0; j < slots; ++j) {
    const float2 v = __bfloat1622float2(p[(int64_t)j * d2]);
    ax = __fadd_rn(ax, v.x);
    ay = __fadd_rn(ay, v.y);
  }
  y[i] = __floats2bfloat162_rn(ax, ay);
}

// y[t, :] = sum_j w[t*k+j] * rows[pos[t*k+j], :] + sum_s extra[s*T + t, :]  (fp32, fixed order)
__global__ void combine_rows_kernel(const __nv_bfloat162* __restrict__ rows, const int32_t* __restrict__ pos,
                                    const float* __restrict__ w, int64_t T, int k, int d2,
                                    const __nv_bfloat162* __restrict__ extra, int S,
                                    __nv_bfloat162* __restrict__ y) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * d2) return;
  const int64_t t = i / d2;
  const int c = (int)(i - t * d2);
  float ax = 0.0f, ay = 0.0f;
  for (int j = 0; j < k; ++j) {
    const float wj = w[t * k + j];
    const float2 v = __bfloat1622float2(rows[(int64_t)pos[t * k + j] * d2 + c]);
    ax = __fadd_rn(ax, __fmul_rn(wj, v.x));
    ay = __fadd_rn(ay, __fmul_rn(wj, v.y));
  }
  for (int s = 0; s < S; ++s) {
    const float2 v = __bfloat1622float2(extra[((int64_t)s * T + t) * d2 + c]);
    ax = __fadd_rn(ax, v.x);
    ay = __fadd_rn(ay, v.y);
  }
  y[i] = __floats2bfloat162_rn(ax, ay);
}

// Decode path: y[t, :] = sum_j w[t*k+j] * P(pos[t*k+j]) + sum_s P(Rr + s*T + t), where
// P(r) = sum over the K chunks c of part[c][r, :] (fp32, chunk order fixed).  Four columns per
// thread (16-byte loads; d % 4 == 0).
__global__ void combine_partials_kernel(const float4* __restrict__ part, int ksplit, int64_t R,
                                        const int32_t* __restrict__ pos, const float* __restrict__ w, int64_t T,
                                        int k, int S, int d4, uint2* __restrict__ y) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * d4) return;
  const int64_t t = i / d4;
  const int c = (int)(i - t * d4);
  const int64_t Rr = T * k;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int j = 0; j < k + S; ++j) {
    const int64_t r = j < k ? (int64_t)pos[t * k + j] : Rr + (int64_t)(j - k) * T + t;
    const float wj = j < k ? w[t * k + j] : 1.0f;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q = 0; q < ksplit; ++q) {
      const float4 p = __ldcs(part + ((int64_t)q * R + r) * d4 + c);
      v.x = __fadd_rn(v.x, p.x);
      v.y = __fadd_rn(v.y, p.y);
      v.z = __fadd_rn(v.z, p.z);
      v.w = __fadd_rn(v.w, p.w);
    }
    if (j < k) {
      acc.x = __fadd_rn(acc.x, __fmul_rn(wj, v.x));
      acc.y = __fadd_rn(acc.y, __fmul_rn(wj, v.y));
      acc.z = __fadd_rn(acc.z, __fmul_rn(wj, v.z));
      acc.w = __fadd_rn(acc.w, __fmul_rn(wj, v.w));
    } else {
      acc.x = __fadd_rn(acc.x, v.x);
      acc.y = __fadd_rn(acc.y, v.y);
      acc.z = __fadd_rn(acc.z, v.z);
      acc.w = __fadd_rn(acc.w, v.w);
    }
  }
  const __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
  y[i] = make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
}

// K chunks for the decode down projection: the divisor d of the stage count KS (d <= 16)
// that minimises the modelled time in stage units per SM: the static schedule's makespan,
// ceil(tiles * d / SMs) tiles of KS / d stages, plus the fp32 partial sums written and read
// back by the combine (d * rows * N * 8 bytes spread over the SMs, at one stage per
// stage_bytes).
inline int pick_ksplit(int KS, int64_t tiles_per_chunk, int num_sms, int64_t rows, int64_t N, int64_t stage_bytes) {
  int best = 1;
  double best_cost = 1e300;
  for (int d = 1; d <= KS && d <= 16; ++d) {
    if (KS % d) continue;
    const double waves = (double)((tiles_per_chunk * d + num_sms - 1) / num_sms);
    const double cost = waves * (KS / d) + (double)d * rows * N * 8.0 / num_sms / (double)stage_bytes;
    if (cost < best_cost) {
      best_cost = cost;
      best = d;
    }
  }
  return best;
}

constexpr int kDecodeMaxSplit = 16;

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Workspace carve-up of the layer (all 256-byte aligned).
struct LayerWs {
  size_t router, ids, wts, counts, offs, sidx, pos, src, dest, scale, offx, xp, h, o, part, total;
};

LayerWs layer_ws(int64_t T, int d, int ffn, int E, int k, int S) {
  LayerWs w{};
  const int64_t R = T * k + (int64_t)S * T;
  size_t p = 0;
  // the router workspace comes first: its leading error word is shared by every kernel of
  // the layer, so reading word 0 of the layer workspace reports any of them
  w.router = p;
  p = align256(p + lmoe_router_workspace_bytes(T, E));
  w.ids = p; p = align256(p + sizeof(int32_t) * T * k);
  w.wts = p; p = align256(p + sizeof(float) * T * k);
  w.counts = p; p = align256(p + sizeof(int32_t) * E);
  w.offs = p; p = align256(p + sizeof(int32_t) * (E + 1));
  w.sidx = p; p = align256(p + sizeof(int32_t) * T * k);
  w.pos = p; p = align256(p + sizeof(int32_t) * T * k);
  w.src = p; p = align256(p + sizeof(int32_t) * R);
  w.dest = p; p = align256(p + sizeof(int32_t) * R);
  w.scale = p; p = align256(p + sizeof(float) * R);
  w.offx = p; p = align256(p + sizeof(int32_t) * (E + S + 1));
  w.xp = p; p = align256(p + sizeof(uint16_t) * R * d);
  w.h = p; p = align256(p + sizeof(uint16_t) * R * ffn);
  w.o = p; p = align256(p + sizeof(uint16_t) * T * (k + S) * d);
  // decode path (T <= 64): fp32 partial sums of the split-K down projection
  w.part = p;
  if (T <= kDecodeMaxRows) p = align256(p + sizeof(float) * (size_t)kDecodeMaxSplit * R * d);
  w.total = p;
  return w;
}

}  // namespace
}  // namespace lmoe

using namespace lmoe;

// ---------------------------------------------------------------------------------- C ABI

extern "C" int lmoe_w4_prepacked_bytes(int num_experts, int rows, int K, int group_size, int paired,
                                       size_t* packed_bytes) {
  LMOE_ARG_CHECK(num_experts >= 1 && rows > 0 && K > 0 && group_size > 0 && packed_bytes);
  LMOE_ARG_CHECK(K % kW4SuperK == 0 && K % group_size == 0 && group_size % 64 == 0);
  LMOE_ARG_CHECK(group_size >= kW4SuperK || kW4SuperK % group_size == 0);
  LMOE_ARG_CHECK(paired ? rows % 64 == 0 : rows % kW4BlockRows == 0);
  const int64_t out_rows = (int64_t)(paired ? 2 * rows : rows);
  *packed_bytes = (size_t)num_experts * (out_rows / kW4BlockRows) * (K / kW4SuperK) * w4_super_bytes(group_size);
  return LMOE_OK;
}

extern "C" int lmoe_prepack_w4(const uint8_t* qweight_a, const uint16_t* scales_a, const uint8_t* qweight_b,
                               const uint16_t* scales_b, int num_experts, int rows, int K, int group_size,
                               uint8_t* packed, lmoe_stream_t stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  const int paired = qweight_b != nullptr;
  size_t pb = 0;
  int st = lmoe_w4_prepacked_bytes(num_experts, rows, K, group_size, paired, &pb);
  if (st != LMOE_OK) return st;
  LMOE_ARG_CHECK(qweight_a && scales_a && packed);
  LMOE_ARG_CHECK(!paired || scales_b);
  LMOE_ARG_CHECK(aligned16(qweight_a) && (!paired || aligned16(qweight_b)) && aligned16(packed));
  const int threads = 256;
  const int NB = paired ? rows / 64 : rows / kW4BlockRows;
  const int64_t chunks = (int64_t)num_experts * NB * (K / kW4SuperK) * 4 * kW4BlockRows;
  const int sbb = w4_super_bytes(group_size);
  prepack_w4_kernel<<<(unsigned)((chunks + threads - 1) / threads), threads, 0, stream>>>(
      qweight_a, qweight_b, num_experts, rows, K, sbb, packed, paired);
  LMOE_CUDA_TRY(cudaGetLastError());
  const int64_t ns = (int64_t)num_experts * NB * (K / kW4SuperK) * w4_scale_groups(group_size) * kW4BlockRows;
  prepack_scales_kernel<<<(unsigned)((ns + threads - 1) / threads), threads, 0, stream>>>(
      scales_a, scales_b, num_experts, rows, K, group_size, sbb, packed, paired);
  return cuda_status(cudaGetLastError());
}

extern "C" size_t lmoe_gemm_workspace_bytes(void) { return 256; }

extern "C" int lmoe_grouped_gemm(const void* input, int dtype, int64_t total_rows, int K, const void* weights, int N,
                                 const void* expert_offsets, int offsets_are_int64, int num_experts, int zero_fill,
                                 void* output, void* workspace, size_t workspace_bytes, lmoe_stream_t stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  LMOE_ARG_CHECK(dtype == LMOE_DTYPE_BF16 || dtype == LMOE_DTYPE_F16 || dtype == LMOE_DTYPE_F32);
  LMOE_ARG_CHECK(total_rows >= 0 && K > 0 && N > 0 && num_experts >= 1);
  LMOE_ARG_CHECK(input && weights && expert_offsets && output);
  LMOE_ARG_CHECK(aligned16(input) && aligned16(weights));
  LMOE_ARG_CHECK(dtype == LMOE_DTYPE_F32 ? (K % 4 == 0) : (K % 64 == 0));
  if (!workspace || workspace_bytes < 256) return LMOE_ERR_WORKSPACE;
  const size_t esize = dtype == LMOE_DTYPE_F32 ? 4 : 2;
  if (zero_fill && total_rows > 0)
    LMOE_CUDA_TRY(cudaMemsetAsync(output, 0, (size_t)total_rows * N * esize, stream));
  LMOE_CUDA_TRY(cudaMemsetAsync(workspace, 0, 256, stream));
  if (dtype == LMOE_DTYPE_F32)
    return run_grouped_gemm_f32(static_cast<const float*>(input), total_rows, K, static_cast<const float*>(weights),
                                N, expert_offsets, offsets_are_int64, num_experts, static_cast<float*>(output),
                                static_cast<uint32_t*>(workspace), stream);
  GemmProblem p;
  p.x = input;
  p.ldx = K;
  p.total_rows = total_rows;
  p.K = K;
  p.offsets = expert_offsets;
  p.offsets_i64 = offsets_are_int64;
  p.num_experts = num_experts;
  p.num_w = num_experts;
  p.w = weights;
  p.ab_f16 = dtype == LMOE_DTYPE_F16 ? 1 : 0;
  p.N = N;
  p.mode = kModePlain;
  p.out = output;
  p.ldo = N;
  p.err = static_cast<uint32_t*>(workspace);
  return run_grouped_gemm(p, stream);
}

extern "C" int lmoe_grouped_gemm_bf16(const void* input, int64_t total_rows, int K, const void* weights, int N,
                                      const void* expert_offsets, int offsets_are_int64, int num_experts,
                                      int zero_fill, void* output, void* workspace, size_t workspace_bytes,
                                      lmoe_stream_t stream) {
  return lmoe_grouped_gemm(input, LMOE_DTYPE_BF16, total_rows, K, weights, N, expert_offsets, offsets_are_int64,
                           num_experts, zero_fill, output, workspace, workspace_bytes, stream);
}

extern "C" int lmoe_w4a16_grouped_gemm(const void* input, int64_t total_rows, int K, const uint8_t* packed, int N,
                                       int group_size,
                                       const void* expert_offsets, int offsets_are_int64, int num_experts,
                                       const int32_t* segment_expert, int num_weight_matrices, int epilogue,
                                       const int32_t* dest_rows,
                                       const float* row_scale,
                                       int64_t max_rows_per_expert, void* output, int64_t ldo, void* workspace,
                                       size_t workspace_bytes, lmoe_stream_t stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  LMOE_ARG_CHECK(total_rows >= 0 && K > 0 && N > 0 && num_experts >= 1 && num_weight_matrices >= 1);
  LMOE_ARG_CHECK(segment_expert || num_experts <= num_weight_matrices);
  LMOE_ARG_CHECK(input && packed && expert_offsets && output);
  LMOE_ARG_CHECK(aligned16(input) && aligned16(packed));
  LMOE_ARG_CHECK(epilogue >= kModePlain && epilogue <= kModeScatter);
  LMOE_ARG_CHECK(ldo >= (epilogue == kModeSwiGLU ? N / 2 : N));
  if (!workspace || workspace_bytes < 256) return LMOE_ERR_WORKSPACE;
  LMOE_CUDA_TRY(cudaMemsetAsync(workspace, 0, 256, stream));
  GemmProblem p;
  p.x = input;
  p.ldx = K;
  p.total_rows = total_rows;
  p.K = K;
  p.offsets = expert_offsets;
  p.offsets_i64 = offsets_are_int64;
  p.num_experts = num_experts;
  p.seg_expert = segment_expert;
  p.num_w = num_weight_matrices;
  p.wq = packed;
  p.group_size = group_size;
  p.N = N;
  p.mode = epilogue;
  p.out = output;
  p.ldo = ldo;
  p.dest = dest_rows;
  p.row_scale = row_scale;
  p.err = static_cast<uint32_t*>(workspace);
  p.max_rows_per_expert_hint = max_rows_per_expert;
  if (max_rows_per_expert > 0 && max_rows_per_expert <= kDecodeMaxRows && epilogue != kModeScatter) {
    DecodeProblem d;
    d.x = input;
    d.ldx = K;
    d.total_rows = total_rows;
    d.K = K;
    d.offsets = expert_offsets;
    d.offsets_i64 = offsets_are_int64;
    d.num_experts = num_experts;
    d.seg_expert = segment_expert;
    d.num_w = num_weight_matrices;
    d.wq = packed;
    d.group_size = group_size;
    d.N = N;
    d.mode = epilogue == kModeSwiGLU ? kDecodeSwiGLU : kDecodePlain;
    d.out = output;
    d.ldo = ldo;
    d.err = p.err;
    return run_decode_gemm(d, stream);
  }
  return run_grouped_gemm(p, stream);
}

extern "C" int lmoe_combine_rows(const void* rows, const int32_t* positions, const float* weights, int64_t num_tokens,
                                 int top_k, int hidden_size, const void* extra_rows, int num_extra, void* y,
                                 lmoe_stream_t stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  LMOE_ARG_CHECK(num_tokens >= 0 && top_k >= 0 && hidden_size > 0 && (hidden_size % 2) == 0 && num_extra >= 0);
  if (num_tokens == 0) return LMOE_OK;
  LMOE_ARG_CHECK(y && (top_k == 0 || (rows && positions && weights)) && (num_extra == 0 || extra_rows));
  const int threads = 256;
  const int64_t n = num_tokens * (hidden_size / 2);
  combine_rows_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0, stream>>>(
      static_cast<const __nv_bfloat162*>(rows), positions, weights, num_tokens, top_k, hidden_size / 2,
      static_cast<const __nv_bfloat162*>(extra_rows), num_extra, static_cast<__nv_bfloat162*>(y));
  return cuda_status(cudaGetLastError());
}

extern "C" size_t lmoe_moe_layer_workspace_bytes(int64_t num_tokens, int hidden_size, int ffn_size, int num_experts,
                                                 int top_k, int num_shared) {
  if (num_tokens < 0 || hidden_size <= 0 || ffn_size <= 0 || num_experts <= 0 || top_k <= 0 || num_shared < 0)
    return 0;
  return layer_ws(num_tokens, hidden_size, ffn_size, num_experts, top_k, num_shared).total;
}

extern "C" int lmoe_moe_layer_w4a16(const void* x, int64_t num_tokens, int hidden_size, const void* gate_weight,
                                    const float* gate_bias, int num_experts, int top_k, int num_shared,
                                    const uint8_t* w13_packed, const uint8_t* w2_packed, int ffn_size, int group_size,
                                    void* y,
                                    int32_t* ids_out, float* weights_out, void* workspace, size_t workspace_bytes,
                                    lmoe_stream_t stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  const int64_t T = num_tokens;
  const int d = hidden_size, E = num_experts, k = top_k, S = num_shared, F = ffn_size;
  LMOE_ARG_CHECK(T >= 0 && d > 0 && F > 0 && E >= 1 && k >= 1 && S >= 0);
  LMOE_ARG_CHECK(E + S <= kMaxGemmExperts);
  LMOE_ARG_CHECK(d % 128 == 0 && F % 128 == 0 && group_size % 64 == 0 && d % group_size == 0 && F % group_size == 0);
  LMOE_ARG_CHECK(group_size >= kW4SuperK || kW4SuperK % group_size == 0);
  LMOE_ARG_CHECK(x && gate_weight && w13_packed && w2_packed && y);
  LMOE_ARG_CHECK((reinterpret_cast<uintptr_t>(y) & 7) == 0);
  const LayerWs L = layer_ws(T, d, F, E, k, S);
  if (!workspace || workspace_bytes < L.total || !aligned16(workspace)) return LMOE_ERR_WORKSPACE;
  if (T == 0) return LMOE_OK;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  auto at = [&](size_t off) { return static_cast<void*>(ws + off); };
  int32_t* ids = ids_out ? ids_out : static_cast<int32_t*>(at(L.ids));
  float* wts = weights_out ? weights_out : static_cast<float*>(at(L.wts));
  int32_t* counts = static_cast<int32_t*>(at(L.counts));
  int32_t* offs = static_cast<int32_t*>(at(L.offs));
  int32_t* sidx = static_cast<int32_t*>(at(L.sidx));
  int32_t* posn = static_cast<int32_t*>(at(L.pos));
  int32_t* src = static_cast<int32_t*>(at(L.src));
  int32_t* dest = static_cast<int32_t*>(at(L.dest));
  float* scale = static_cast<float*>(at(L.scale));
  int32_t* offx = static_cast<int32_t*>(at(L.offx));
  uint32_t* err = static_cast<uint32_t*>(at(L.router));  // zeroed by the router call
  const int64_t R = T * k + (int64_t)S * T;

  int st = lmoe_fused_gate_topk(x, gate_weight, gate_bias, T, d, E, k, ids, wts, nullptr, counts, offs, sidx,
                                posn, nullptr, at(L.router), lmoe_router_workspace_bytes(T, E), stream_);
  if (st != LMOE_OK) return st;
  {
    const int threads = 256;
    const int64_t n = R > (E + S + 1) ? R : (E + S + 1);
    routing_table_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0, stream>>>(
        sidx, wts, offs, (int)T, k, E, S, src, dest, scale, offx);
    LMOE_CUDA_TRY(cudaGetLastError());
    const int vec = d / 8;
    const int64_t grid = R < 65535 * 4 ? R : 65535 * 4;
    gather_rows_kernel<<<(unsigned)grid, vec >= 256 ? 256 : vec, 0, stream>>>(
        static_cast<const uint4*>(x), src, R, vec, static_cast<uint4*>(at(L.xp)));
    LMOE_CUDA_TRY(cudaGetLastError());
  }
  if (T <= kDecodeMaxRows) {
    // decode: every expert holds at most T <= 64 rows -> warp-level MMA path, split-K down
    DecodeProblem d1;
    d1.x = at(L.xp);
    d1.ldx = d;
    d1.total_rows = R;
    d1.K = d;
    d1.offsets = offx;
    d1.num_experts = E + S;
    d1.num_w = E + S;
    d1.wq = w13_packed;
    d1.group_size = group_size;
    d1.N = 2 * F;
    d1.mode = kDecodeSwiGLU;
    d1.out = at(L.h);
    d1.ldo = F;
    d1.err = err;
    st = run_decode_gemm(d1, stream);
    if (st != LMOE_OK) return st;
    DeviceInfo dev;
    st = get_device_info(&dev);
    if (st != LMOE_OK) return st;
    const int KS2 = F / kW4SuperK;
    // decode tiles: every segment holds at most T <= 64 rows, i.e. at most two 32-row tiles
    const int ksplit = pick_ksplit(KS2, (int64_t)(E + S) * (d / 128), dev.num_sms, R, d, w4_super_bytes(group_size));
    DecodeProblem d2 = d1;
    d2.x = at(L.h);
    d2.ldx = F;
    d2.K = F;
    d2.wq = w2_packed;
    d2.N = d;
    d2.mode = kDecodePartial;
    d2.ksplit = ksplit;
    d2.out = at(L.part);
    d2.ldo = d;
    st = run_decode_gemm(d2, stream);
    if (st != LMOE_OK) return st;
    const int threads = 256;
    const int64_t n = T * (d / 4);
    combine_partials_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0, stream>>>(
        static_cast<const float4*>(at(L.part)), ksplit, R, posn, wts, T, k, S, d / 4, static_cast<uint2*>(y));
    return cuda_status(cudaGetLastError());
  }
  // a routed expert receives at most T rows; shared experts exactly T
  const int64_t hint = T;
  GemmProblem g1;
  g1.x = at(L.xp);
  g1.ldx = d;
  g1.total_rows = R;
  g1.K = d;
  g1.offsets = offx;
  g1.num_experts = E + S;
  g1.num_w = E + S;
  g1.wq = w13_packed;
  g1.group_size = group_size;
  g1.N = 2 * F;
  g1.mode = kModeSwiGLU;
  g1.out = at(L.h);
  g1.ldo = F;
  g1.err = err;
  g1.max_rows_per_expert_hint = hint;
  st = run_grouped_gemm(g1, stream);
  if (st != LMOE_OK) return st;
  GemmProblem g2;
  g2.x = at(L.h);
  g2.ldx = F;
  g2.total_rows = R;
  g2.K = F;
  g2.offsets = offx;
  g2.num_experts = E + S;
  g2.num_w = E + S;
  g2.wq = w2_packed;
  g2.group_size = group_size;
  g2.N = d;
  g2.mode = kModeScatter;
  g2.out = at(L.o);
  g2.ldo = d;
  g2.dest = dest;
  g2.row_scale = scale;
  g2.err = err;
  g2.max_rows_per_expert_hint = hint;
  st = run_grouped_gemm(g2, stream);
  if (st != LMOE_OK) return st;
  {
    const int threads = 256;
    if (d % 8 == 0 && aligned16(y) && aligned16(at(L.o))) {
      const int64_t n = T * (d / 8);
      combine_slots16_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0, stream>>>(
          static_cast<const uint4*>(at(L.o)), T, k + S, d / 8, static_cast<uint4*>(y));
    } else {
      const int64_t n = T * (d / 2);
      combine_slots_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0, stream>>>(
          static_cast<const __nv_bfloat162*>(at(L.o)), T, k + S, d / 2, static_cast<__nv_bfloat162*>(y));
    }
    LMOE_CUDA_TRY(cudaGetLastError());
  }
  return LMOE_OK;
}

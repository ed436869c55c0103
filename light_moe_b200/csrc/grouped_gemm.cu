// grouped_gemm.cu -- persistent grouped GEMMs for MoE experts on B200 (sm_100a).
//
// For every expert e, rows [offsets[e], offsets[e+1]) of an activation matrix X (bf16,
// row-major [R, K]) are multiplied by that expert's weight matrix W_e ([N, K]):
//     Y[r, n] = sum_k X[r, k] * W_e[n, k]
// Reference: csrc/grouped_gemm.cu:11-43 (one cuBLAS mm_out per expert after copying the
// offsets to the host) and python/light_moe/ops/grouped_gemm.py:21-106.  Here one launch
// covers all experts, the offsets are read on the device, and the weights may be int4.
//
// "Swap-AB" formulation: the MMA's M dimension (128) runs over weight rows, N over tokens,
// so decode-sized batches (a handful of tokens per expert) still fill the 128-row MMA, and
// the accumulator tile is [128 weight rows x BN tokens] in tensor memory.
//
// W4A16 weights (the north-star path): packed int4 blocks (w4_layout.cuh) are bulk-copied
// into shared memory, dequantised by dedicated warps into bf16 and written with tcgen05.st
// straight into tensor memory, where tcgen05.mma reads them as the A operand ("TS" form);
// the token tile (B operand) arrives by TMA with the 128-byte swizzle.  Dequantised value =
// bf16_rn(q * s), computed exactly as q*s_hi + q*s_lo with one final rounding (s_hi/s_lo
// split the fp16 scale into two bf16 parts), bit-identical to the CPU oracle.
// bf16 weights (the reference's dense grouped_gemm op): the weight tile arrives by TMA too
// and both operands are read from shared memory ("SS" form).
//
// Warp roles (one CTA per SM, persistent over a static round-robin tile schedule):
//   warp 0            producer: weight blocks (bulk copy or TMA) and token tiles (TMA)
//   warp 1            MMA issuer (one thread)
//   warps 2..2+DQ-1   int4 dequantisers (W4 only): one weight row per thread
//   last 4 warps      epilogue: TMEM -> registers -> (SwiGLU | scale+scatter) -> global
//
// Tile order: expert-major, then feature block, then token block (fastest), so the CTAs
// working at the same time share each weight block through L2.
//
// Epilogue modes:
//   kPlain   out[r, n]                                        = bf16(acc)
//   kSwiGLU  out[r, fb*64 + j]  (tile rows j: gate, j+64: up) = bf16(silu(gate) * up)
//   kScatter out[dest[r], n]                                  = bf16(scale[r] * acc)
#include <cuda_bf16.h>

#include "grouped_gemm.h"
#include "host_util.h"
#include "ptx.cuh"
#include "w4_layout.cuh"

namespace lmoe {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr uint32_t kSite = 0x200u;

struct GemmArgs {
  // weights
  const uint8_t* wq;        // W4: prepacked blocks
  const uint16_t* wscale;   // W4: prepacked scales
  int group_size;           // W4
  int G;                    // W4: K / group_size
  // problem
  const void* offsets;      // [E+1] row ranges of the segments
  int offsets_i64;
  const int32_t* seg_expert; // weight matrix used by each segment (NULL: segment e uses expert e)
  int E, N, K, NB, KB;      // NB = ceil(N / 128) weight-row blocks, KB = K / 64
  int mode;
  __nv_bfloat16* out;
  int64_t ldo;
  const int32_t* dest;
  const float* row_scale;
  uint32_t* err;
  uint32_t tmem_cols;
};

template <int BN, int DQ, int WST, int BST, int AST, int ACC, bool W4>
struct Cfg {
  static constexpr int kDQWarps = W4 ? DQ : 0;
  static constexpr int kEpiWarp0 = 2 + kDQWarps;
  static constexpr int kThreads = (kEpiWarp0 + 4) * 32;
  static constexpr uint32_t kBStageBytes = BN * kBK * 2;
  static constexpr uint32_t kAStageBytes = W4 ? 0u : (uint32_t)(kBM * kBK * 2);   // bf16 weights in smem
  static constexpr uint32_t kWStageBytes = W4 ? (uint32_t)(kW4BlockBytes + kBM * 2) : 0u;
  static constexpr int kWStages = W4 ? WST : BST;   // bf16: weight tile travels with the token tile
  static constexpr uint32_t kXchgBytes = 64 * 17 * 4;
  static constexpr uint32_t kSmemBytes = 1024 + BST * (kBStageBytes + kAStageBytes) + (W4 ? WST * kWStageBytes : 0) +
                                         kXchgBytes + 1024;
  static constexpr uint32_t kTmemColsNeeded = ACC * BN + (W4 ? AST * 32 : 0);
};

struct __align__(8) GemmBars {
  uint64_t w_full[16], w_empty[16];
  uint64_t b_full[8], b_empty[8];
  uint64_t a_full[16], a_empty[16];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
  int total_tiles;
  int tile_start[kMaxGemmExperts + 1];
  int row_off[kMaxGemmExperts + 1];
  int seg_w[kMaxGemmExperts];
};

struct TileInfo {
  int e, w, fb, row0, rows;   // segment, its weight matrix, feature block, first row, rows
};

// Tiles are numbered expert-major, then feature block, then token block (fastest).
template <int BN>
__device__ __forceinline__ TileInfo tile_at(const GemmBars* b, int tile, int& e_hint, int NB) {
  int e = e_hint;
  while (tile >= b->tile_start[e + 1]) ++e;
  e_hint = e;
  const int n_e = b->row_off[e + 1] - b->row_off[e];
  const int ntb = (n_e + BN - 1) / BN;
  const int local = tile - b->tile_start[e];
  TileInfo ti;
  ti.e = e;
  ti.w = b->seg_w[e];
  ti.fb = local / ntb;
  const int tb = local - ti.fb * ntb;
  ti.row0 = b->row_off[e] + tb * BN;
  const int left = n_e - tb * BN;
  ti.rows = left < BN ? left : BN;
  return ti;
}

__device__ __forceinline__ uint32_t bf16x2_bits(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ __nv_bfloat162 bits_bf16x2(uint32_t v) { return *reinterpret_cast<__nv_bfloat162*>(&v); }

// Dequantise one interleaved word (8 K values) into 4 bf16x2 registers.
__device__ __forceinline__ void dequant_word(uint32_t w, __nv_bfloat162 s_hi, __nv_bfloat162 s_lo,
                                             const __nv_bfloat162 off136, uint32_t* out4) {
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint32_t x = ((w >> (4 * p)) & 0x000F000Fu) | 0x43004300u;   // bf16 pair (128 + u)
    const __nv_bfloat162 q = __hsub2(bits_bf16x2(x), off136);           // exact q = u - 8
    const __nv_bfloat162 t = __hmul2(q, s_lo);                           // exact (<= 6 bits)
    out4[p] = bf16x2_bits(__hfma2(q, s_hi, t));                          // one rounding of q*s
  }
}

__device__ __forceinline__ float silu_f(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

template <int BN, int DQ, int WST, int BST, int AST, int ACC, bool W4>
__global__ void __launch_bounds__(Cfg<BN, DQ, WST, BST, AST, ACC, W4>::kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                        const GemmArgs a) {
  using C = Cfg<BN, DQ, WST, BST, AST, ACC, W4>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* b_stages = base;                                           // BST x [BN x 64] bf16 (SW128)
  uint8_t* a_stages = b_stages + BST * C::kBStageBytes;               // bf16 path: BST x [128 x 64]
  uint8_t* w_stages = a_stages + BST * C::kAStageBytes;               // W4 path: WST x (4096 + 256)
  float* xchg = reinterpret_cast<float*>(w_stages + (W4 ? WST * C::kWStageBytes : 0));
  GemmBars* bars = reinterpret_cast<GemmBars*>(reinterpret_cast<uint8_t*>(xchg) + C::kXchgBytes);
  volatile int* abort_flag = &bars->abort;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  if (tid == 0) {
    for (int s = 0; s < C::kWStages; ++s) {
      mbar_init(&bars->w_full[s], 1);
      mbar_init(&bars->w_empty[s], W4 ? 4 : 1);
    }
    for (int s = 0; s < BST; ++s) {
      mbar_init(&bars->b_full[s], 1);
      mbar_init(&bars->b_empty[s], 1);
    }
    for (int s = 0; s < AST; ++s) {
      mbar_init(&bars->a_full[s], W4 ? 4 : 1);
      mbar_init(&bars->a_empty[s], 1);
    }
    for (int s = 0; s < ACC; ++s) {
      mbar_init(&bars->acc_full[s], 1);
      mbar_init(&bars->acc_empty[s], 128);
    }
    mbar_init(&bars->mma_done, 1);
    bars->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_x);
    if (!W4) tma_prefetch_desc(&tm_w);
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, a.tmem_cols);
    tmem_relinquish();
  }
  // expert row offsets and the tile prefix (computed redundantly by every CTA)
  for (int e = tid; e <= a.E; e += C::kThreads) {
    bars->row_off[e] = a.offsets_i64 ? (int)static_cast<const int64_t*>(a.offsets)[e]
                                     : static_cast<const int32_t*>(a.offsets)[e];
    if (e < a.E) bars->seg_w[e] = a.seg_expert ? a.seg_expert[e] : e;
  }
  __syncthreads();
  if (tid == 0) {
    int acc_t = 0;
    bars->tile_start[0] = 0;
    for (int e = 0; e < a.E; ++e) {
      int n_e = bars->row_off[e + 1] - bars->row_off[e];
      if (n_e < 0) {
        report_error(a.err, kErrBadArg, kSite + 9);
        n_e = 0;
      }
      acc_t += ((n_e + BN - 1) / BN) * a.NB;
      bars->tile_start[e + 1] = acc_t;
    }
    bars->total_tiles = acc_t;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const uint32_t tmem_a = tmem + ACC * BN;   // W4: AST stages of 32 columns
  const int total = bars->total_tiles;
  const int KB = a.KB;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t wit = 0, bit = 0;
      int e_hint = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        const TileInfo ti = tile_at<BN>(bars, tile, e_hint, a.NB);
        const uint8_t* wblk = nullptr;
        const uint16_t* sblk = nullptr;
        if (W4) {
          wblk = a.wq + (size_t)(ti.w * a.NB + ti.fb) * KB * kW4BlockBytes;
          sblk = a.wscale + (size_t)(ti.w * a.NB + ti.fb) * a.G * kBM;
        }
        for (int kb = 0; kb < KB; ++kb) {
          if (W4) {
            const int s = wit % WST;
            if (!mbar_wait(&bars->w_empty[s], ((wit / WST) & 1u) ^ 1u, a.err, abort_flag, kSite + 1)) { ok = false; break; }
            uint8_t* wsm = w_stages + s * C::kWStageBytes;
            mbar_arrive_expect_tx(&bars->w_full[s], kW4BlockBytes + kBM * 2);
            bulk_load(wsm, wblk + (size_t)kb * kW4BlockBytes, kW4BlockBytes, &bars->w_full[s]);
            bulk_load(wsm + kW4BlockBytes, sblk + (size_t)((kb * kBK) / a.group_size) * kBM, kBM * 2,
                      &bars->w_full[s]);
            ++wit;
          }
          const int s2 = bit % BST;
          if (!mbar_wait(&bars->b_empty[s2], ((bit / BST) & 1u) ^ 1u, a.err, abort_flag, kSite + 2)) { ok = false; break; }
          uint8_t* bsm = b_stages + s2 * C::kBStageBytes;
          if (W4) {
            mbar_arrive_expect_tx(&bars->b_full[s2], C::kBStageBytes);
          } else {
            mbar_arrive_expect_tx(&bars->b_full[s2], C::kBStageBytes + C::kAStageBytes);
            tma_load_2d(a_stages + s2 * C::kAStageBytes, &tm_w, &bars->b_full[s2], kb * kBK,
                        ti.w * a.N + ti.fb * kBM);
          }
          tma_load_2d(bsm, &tm_x, &bars->b_full[s2], kb * kBK, ti.row0);
          ++bit;
        }
      }
      // drain: no bulk copy may still be landing when the CTA exits
      const uint32_t bfirst = bit > (uint32_t)BST ? bit - BST : 0u;
      for (uint32_t j = bfirst; j < bit; ++j) mbar_wait(&bars->b_full[j % BST], (j / BST) & 1u, a.err, nullptr, kSite + 3);
      if (W4) {
        const uint32_t wfirst = wit > (uint32_t)WST ? wit - WST : 0u;
        for (uint32_t j = wfirst; j < wit; ++j) mbar_wait(&bars->w_full[j % WST], (j / WST) & 1u, a.err, nullptr, kSite + 4);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t ait = 0, bit = 0, lt = 0;
      int e_hint = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, ++lt) {
        const TileInfo ti = tile_at<BN>(bars, tile, e_hint, a.NB);
        const uint32_t n_eff = (uint32_t)((ti.rows + 15) & ~15);
        const uint32_t idesc = idesc_bf16_f32(kBM, n_eff);
        const uint32_t acc = lt % ACC;
        if (!mbar_wait(&bars->acc_empty[acc], ((lt / ACC) & 1u) ^ 1u, a.err, abort_flag, kSite + 5)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + acc * BN;
        for (int kb = 0; kb < KB; ++kb) {
          const int s2 = bit % BST;
          if (W4) {
            const int as = ait % AST;
            if (!mbar_wait(&bars->a_full[as], (ait / AST) & 1u, a.err, abort_flag, kSite + 6)) { ok = false; break; }
          }
          if (!mbar_wait(&bars->b_full[s2], (bit / BST) & 1u, a.err, abort_flag, kSite + 7)) { ok = false; break; }
          tc_fence_after();
          const uint32_t bsm = smem_u32(b_stages + s2 * C::kBStageBytes);
          if (W4) {
            const uint32_t as_col = tmem_a + (ait % AST) * 32;
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
              mma_ts(d_tmem, as_col + kk * 8, sdesc_k_sw128(bsm + kk * 32), idesc, (kb | kk) != 0 ? 1u : 0u);
            mma_commit(&bars->a_empty[ait % AST]);
            ++ait;
          } else {
            const uint32_t asm_ = smem_u32(a_stages + s2 * C::kAStageBytes);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
              mma_ss(d_tmem, sdesc_k_sw128(asm_ + kk * 32), sdesc_k_sw128(bsm + kk * 32), idesc,
                     (kb | kk) != 0 ? 1u : 0u);
          }
          mma_commit(&bars->b_empty[s2]);
          ++bit;
        }
        if (ok) mma_commit(&bars->acc_full[acc]);
      }
      mma_commit(&bars->mma_done);
      mbar_wait(&bars->mma_done, 0, a.err, nullptr, kSite + 8);
    }
  } else if (W4 && warp < C::kEpiWarp0) {
    // ------------------------------------------------------------------ int4 dequantisers
    // DQ / 4 groups of 4 warps (one warp per TMEM lane quarter, one weight row per thread).
    // Group g owns every (DQ/4)-th k-block, so several k-blocks are dequantised at once and
    // the barrier / shared-load / tensor-memory-store latency of one block overlaps the
    // arithmetic of the others.
    constexpr int kGroups = DQ / 4;
    const int grp = (warp - 2) >> 2;
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const __nv_bfloat162 off136 = __floats2bfloat162_rn(136.0f, 136.0f);
    uint32_t it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
      for (int kb = 0; kb < KB; ++kb, ++it) {
        if ((int)(it % kGroups) != grp) continue;
        const int s = it % WST;
        if (!mbar_wait(&bars->w_full[s], (it / WST) & 1u, a.err, abort_flag, kSite + 10)) { ok = false; break; }
        const uint8_t* wsm = w_stages + s * C::kWStageBytes;
        const uint4 v0 = *reinterpret_cast<const uint4*>(wsm + row * 16);
        const uint4 v1 = *reinterpret_cast<const uint4*>(wsm + 2048 + row * 16);
        const uint16_t sbits = reinterpret_cast<const uint16_t*>(wsm + kW4BlockBytes)[row];
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->w_empty[s]);
        // exact split of the fp16 scale into bf16 hi + lo parts
        const float sf = __half2float(__ushort_as_half(sbits));
        const __nv_bfloat16 shi = __float2bfloat16_rz(sf);
        const __nv_bfloat16 slo = __float2bfloat16_rn(__fsub_rn(sf, __bfloat162float(shi)));
        const __nv_bfloat162 s_hi = __nv_bfloat162(shi, shi);
        const __nv_bfloat162 s_lo = __nv_bfloat162(slo, slo);
        uint32_t o0[16], o1[16];
        dequant_word(v0.x, s_hi, s_lo, off136, &o0[0]);
        dequant_word(v0.y, s_hi, s_lo, off136, &o0[4]);
        dequant_word(v0.z, s_hi, s_lo, off136, &o0[8]);
        dequant_word(v0.w, s_hi, s_lo, off136, &o0[12]);
        dequant_word(v1.x, s_hi, s_lo, off136, &o1[0]);
        dequant_word(v1.y, s_hi, s_lo, off136, &o1[4]);
        dequant_word(v1.z, s_hi, s_lo, off136, &o1[8]);
        dequant_word(v1.w, s_hi, s_lo, off136, &o1[12]);
        const int as = it % AST;
        if (!mbar_wait(&bars->a_empty[as], ((it / AST) & 1u) ^ 1u, a.err, abort_flag, kSite + 11)) { ok = false; break; }
        tc_fence_after();
        const uint32_t taddr = tmem_a + ((uint32_t)(q * 32) << 16) + as * 32;
        tmem_st16(taddr, o0);
        tmem_st16(taddr + 16, o1);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->a_full[as]);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int row = q * 32 + lane;
    uint32_t lt = 0;
    int e_hint = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++lt) {
      const TileInfo ti = tile_at<BN>(bars, tile, e_hint, a.NB);
      const int n_eff = (ti.rows + 15) & ~15;
      const uint32_t acc = lt % ACC;
      if (!mbar_wait(&bars->acc_full[acc], (lt / ACC) & 1u, a.err, abort_flag, kSite + 12)) break;
      tc_fence_after();
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + acc * BN;
      const int feat = ti.fb * kBM + row;
      for (int c0 = 0; c0 < n_eff; c0 += 16) {
        uint32_t v[16];
        tmem_ld16(taddr + c0, v);
        if (a.mode == kModeSwiGLU) {
          if (q >= 2) {
#pragma unroll
            for (int i = 0; i < 16; ++i) xchg[(row - 64) * 17 + i] = __uint_as_float(v[i]);
          }
          named_bar_sync(2, 128);
          if (q < 2) {
            const int f = ti.fb * 64 + row;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int c = c0 + i;
              if (c < ti.rows) {
                const float g = __uint_as_float(v[i]);
                const float u = xchg[row * 17 + i];
                a.out[(int64_t)(ti.row0 + c) * a.ldo + f] = __float2bfloat16_rn(silu_f(g) * u);
              }
            }
          }
          named_bar_sync(2, 128);
        } else if (feat < a.N) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int c = c0 + i;
            if (c < ti.rows) {
              const int r = ti.row0 + c;
              float val = __uint_as_float(v[i]);
              int64_t orow = r;
              if (a.mode == kModeScatter) {
                if (a.row_scale) val = __fmul_rn(val, a.row_scale[r]);
                if (a.dest) orow = a.dest[r];
              }
              a.out[orow * a.ldo + feat] = __float2bfloat16_rn(val);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&bars->acc_empty[acc]);
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, a.tmem_cols);
  }
}

template <int BN, int DQ, int WST, int BST, int AST, int ACC, bool W4>
int launch_gemm(const CUtensorMap& tm_x, const CUtensorMap& tm_w, GemmArgs a, int grid, cudaStream_t stream) {
  using C = Cfg<BN, DQ, WST, BST, AST, ACC, W4>;
  static_assert(C::kTmemColsNeeded <= 512, "tensor memory budget");
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "MMA N");
  uint32_t cols = 32;
  while (cols < C::kTmemColsNeeded) cols <<= 1;
  a.tmem_cols = cols;
  const size_t smem = C::kSmemBytes + sizeof(GemmBars);
  auto fn = grouped_gemm_kernel<BN, DQ, WST, BST, AST, ACC, W4>;
  LMOE_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  fn<<<grid, C::kThreads, smem, stream>>>(tm_x, tm_w, a);
  return cuda_status(cudaGetLastError());
}

}  // namespace

// Internal entry used by the C-ABI wrappers below and by the layer driver.
int run_grouped_gemm(const GemmProblem& p, cudaStream_t stream) {
  DeviceInfo dev;
  int st = get_device_info(&dev);
  if (st != LMOE_OK) return st;
  if (dev.cc_major != 10) return LMOE_ERR_DEVICE;
  if (p.num_experts < 1 || p.num_experts > kMaxGemmExperts) return LMOE_ERR_UNSUPPORTED;
  if (p.K < kBK || p.K % kBK) return LMOE_ERR_INVALID_ARG;
  if (p.total_rows < 0 || p.total_rows > INT32_MAX) return LMOE_ERR_INVALID_ARG;
  if (!p.x || !p.offsets || !p.out || !p.err) return LMOE_ERR_INVALID_ARG;
  const bool w4 = p.wq != nullptr;
  if (w4) {
    if (!p.wscale || p.group_size < kBK || p.group_size % kBK || p.K % p.group_size) return LMOE_ERR_UNSUPPORTED;
    if (p.N % kBM) return LMOE_ERR_UNSUPPORTED;
  } else {
    if (!p.w) return LMOE_ERR_INVALID_ARG;
    if (p.mode == kModeSwiGLU) return LMOE_ERR_UNSUPPORTED;
  }
  if (p.mode == kModeSwiGLU && (p.N % kBM)) return LMOE_ERR_INVALID_ARG;
  if (p.total_rows == 0) return LMOE_OK;

  GemmArgs a = {};
  a.wq = p.wq;
  a.wscale = p.wscale;
  a.group_size = p.group_size;
  a.G = w4 ? p.K / p.group_size : 0;
  a.offsets = p.offsets;
  a.offsets_i64 = p.offsets_i64;
  a.seg_expert = p.seg_expert;
  a.E = p.num_experts;
  a.N = p.N;
  a.K = p.K;
  a.NB = (p.N + kBM - 1) / kBM;
  a.KB = p.K / kBK;
  a.mode = p.mode;
  a.out = static_cast<__nv_bfloat16*>(p.out);
  a.ldo = p.ldo;
  a.dest = p.dest;
  a.row_scale = p.row_scale;
  a.err = p.err;

  const bool small = p.max_rows_per_expert_hint > 0 && p.max_rows_per_expert_hint <= 64;
  const int BNsel = small ? 64 : 192;
  CUtensorMap tm_x, tm_w;
  st = encode_tmap_2d(&tm_x, p.x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)p.total_rows, (uint64_t)p.K,
                      (uint64_t)p.ldx * 2, (uint32_t)BNsel, kBK, true);
  if (st != LMOE_OK) return st;
  if (!w4) {
    st = encode_tmap_2d(&tm_w, p.w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)p.num_experts * p.N,
                        (uint64_t)p.K, (uint64_t)p.K * 2, kBM, kBK, true);
    if (st != LMOE_OK) return st;
  } else {
    tm_w = tm_x;
  }
  const int grid = dev.num_sms;
  if (w4) {
    if (small) return launch_gemm<64, 16, 16, 4, 8, 2, true>(tm_x, tm_w, a, grid, stream);
    return launch_gemm<192, 12, 8, 4, 4, 2, true>(tm_x, tm_w, a, grid, stream);
  }
  if (small) return launch_gemm<64, 0, 1, 6, 1, 2, false>(tm_x, tm_w, a, grid, stream);
  return launch_gemm<192, 0, 1, 4, 1, 2, false>(tm_x, tm_w, a, grid, stream);
}

}  // namespace lmoe

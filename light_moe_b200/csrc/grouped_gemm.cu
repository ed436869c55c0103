// grouped_gemm.cu -- persistent grouped GEMMs for MoE experts on B200 (sm_100a).
//
// For every row segment e (one expert's rows), rows [offsets[e], offsets[e+1]) of an
// activation matrix X (bf16, row-major [R, K]) are multiplied by that segment's weight
// matrix W ([N, K]):   Y[r, n] = sum_k X[r, k] * W[n, k]
// Reference: csrc/grouped_gemm.cu:11-43 (one cuBLAS mm_out per expert after copying the
// offsets to the host) and python/light_moe/ops/grouped_gemm.py:21-106.  Here one launch
// covers all experts, the offsets are read on the device, and the weights may be int4.
//
// "Swap-AB": the MMA's M dimension (128) runs over weight rows and N over tokens, so a
// decode-sized batch (a handful of tokens per expert) still fills the 128-row MMA; the
// accumulator tile is [128 weight rows x BN tokens] in tensor memory.
//
// W4A16 weights (the MoE-layer hot path): one prepacked int4 super-block (128 rows x 128 K,
// scales embedded, w4_layout.cuh) per pipeline stage arrives by one bulk copy; dequantiser
// warps turn it into bf16 and write it with tcgen05.st straight into tensor memory, where
// tcgen05.mma reads it as the A operand ("TS" form); the token tile (B operand) arrives by
// TMA with the 128-byte swizzle.  Dequantised value = bf16_rn(q * s), computed exactly as
// q*s_hi + q*s_lo with one final rounding (s_hi / s_lo split the fp16 scale into two bf16
// parts), bit-identical to the CPU oracle.
// bf16 weights (the reference's dense grouped_gemm op): the weight tile arrives by TMA too
// and both operands are read from shared memory ("SS" form).
//
// Warp roles (one CTA per SM, persistent over a static round-robin tile schedule):
//   warp 0            producer: token tiles (TMA) and weights (bulk copy of int4 super-blocks
//                     / TMA of bf16 tiles), the weights up to WST - BST stages ahead
//   warp 1            MMA issuer (one thread) for token columns [0, BN/2) of every tile
//   warp 2            MMA issuer for token columns [BN/2, BN)
//   warps 3..3+DQ-1   int4 dequantisers (W4 only), DQ/4 groups of 4 warps; a group owns
//                     every (DQ/4)-th stage, one weight row per thread
//   next 4 warps      epilogue: TMEM -> registers -> (SwiGLU | scale+scatter) -> global
//   last warp         the MMA issuers' waiter: waits on the stage and accumulator barriers
//                     and publishes a counter the issuers poll
// Every stage covers 128 K values (two 64-wide swizzle atoms), so each mbarrier wait,
// expect-tx and commit is amortised over eight 128 x N x 16 MMAs per issuer.
//
// Epilogue: 32 accumulator columns per tensor-memory load wait; the results of each 32-column
// step are staged token-major in shared memory and written as whole token rows (128 B for
// SwiGLU, 256 B otherwise) with 16-byte stores; for SwiGLU the gate lanes (0-63) and up lanes
// (64-127) exchange half of the step's columns so all four epilogue warps compute.
//
// Tile order: segment-major; inside a segment the larger operand is the slow index (feature
// blocks for the gate/up projection, token blocks for the down projection of a prefill
// batch), so the CTAs working at the same time share its tiles through L2.
//
// Epilogue modes:
//   kPlain   out[r, n]                                        = bf16(acc)
//   kSwiGLU  out[r, fb*64 + j]  (tile rows j: gate, j+64: up) = bf16(silu(gate) * up)
//   kScatter out[dest[r], n]                                  = bf16(scale[r] * acc)
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "grouped_gemm.h"
#include "host_util.h"
#include "ptx.cuh"
#include "w4_dequant.cuh"
#include "w4_layout.cuh"

namespace lmoe {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;     // one 128-byte swizzle atom of bf16
constexpr int kSK = 128;    // K values per pipeline stage
constexpr uint32_t kSite = 0x200u;

struct GemmArgs {
  const uint8_t* wq;          // W4: prepacked super-blocks
  int group_size;             // W4
  uint32_t sb_bytes;          // W4: bytes per super-block
  const void* offsets;        // [E+1] row ranges of the segments
  int offsets_i64;
  const int32_t* seg_expert;  // weight matrix of each segment (NULL: segment e uses matrix e)
  int E, N, K, NB, KS;        // NB = ceil(N / 128) weight-row blocks, KS = K / 128 stages per tile
  int mode;
  __nv_bfloat16* out;
  int64_t ldo;
  const int32_t* dest;
  const float* row_scale;
  uint32_t* err;
  uint32_t tmem_cols;
  int vec_out;                // N % 128 == 0, ldo % 8 == 0, out 16-byte aligned: staged 16-byte stores
  int ab_f16;                 // dense operands fp16 (else bf16); plain outputs written as fp16
  int num_w;                  // weight matrices available
  int64_t R;                  // activation rows
  int raster_rows;            // segments with more rows run token-block-major (tile_at)
  // scatter to several buffers: dest[r] = (buffer << 24) | row of buffer dest_bases[buffer]
  // (peer memory included: the outputs of an expert-parallel step go straight back to the
  // rank that owns the token); NULL: dest[r] is a row of out
  const uint64_t* dest_bases;
  int dest_count;             // entries of dest_bases
};

// Output row base of a scattered row.
__device__ __forceinline__ __nv_bfloat16* scatter_row(const GemmArgs& a, int32_t dest) {
  if (a.dest_bases)
    return reinterpret_cast<__nv_bfloat16*>(a.dest_bases[(uint32_t)dest >> 24]) + (int64_t)(dest & 0xffffff) * a.ldo;
  return a.out + (int64_t)dest * a.ldo;
}

// fp32 -> the 16-bit output type (bf16, or fp16 for fp16 operands), as bf16 storage.
__device__ __forceinline__ __nv_bfloat16 cvt_out(float v, int f16) {
  return f16 ? __ushort_as_bfloat16(__half_as_ushort(__float2half_rn(v))) : __float2bfloat16_rn(v);
}

constexpr int gcd_int(int a, int b) { return b == 0 ? a : gcd_int(b, a % b); }
constexpr int lcm_int(int a, int b) { return a / gcd_int(a, b) * b; }

template <int BN, int DQ, int WST, int BST, int AST, int ACC, bool W4, int BOX>
struct Cfg {
  static constexpr int kDQWarps = W4 ? DQ : 0;
  static constexpr int kGroups = W4 ? DQ / 4 : 1;
  static constexpr int kEpiWarp0 = 3 + kDQWarps;
  static constexpr int kWaitWarp = kEpiWarp0 + 4;
  static constexpr int kIssue2Warp = 2;   // second MMA issuer: token columns [BN/2, BN)
  static constexpr int kThreads = (kWaitWarp + 1) * 32;
  static constexpr uint32_t kBStageBytes = 2u * BN * kBK * 2;                        // [2][BN][64] bf16
  static constexpr uint32_t kWStageBytes = W4 ? (uint32_t)(kW4SuperInt4Bytes + 512)  // int4 + <= 2 scale groups
                                              : (uint32_t)(2 * kBM * kBK * 2);       // bf16 [2][128][64]
  // epilogue scratch: SwiGLU exchange buffers of [64 features][32 columns + 1] fp32 (two for
  // the W4 configurations, so one barrier per 32 columns; one for bf16, whose weight stages
  // leave less room), then the tile's routing weights and destination rows [BN] each
  static constexpr int kXchgBufs = W4 ? 2 : 1;
  static constexpr int kXchgFloats = kXchgBufs * 64 * 33;
  static constexpr uint32_t kXchgBytes = (uint32_t)kXchgFloats * 4 + BN * 8;
  static constexpr uint32_t kSmemBytes = 1024 + BST * kBStageBytes + WST * kWStageBytes + kXchgBytes + 1024;
  static constexpr uint32_t kTmemColsNeeded = ACC * BN + (W4 ? AST * 64 : 0);
  // dequantise a whole stage into registers before waiting for its TMEM stage when the
  // register file allows it (65536 registers / threads >= ~128)
  static constexpr bool kEarlyDequant = kThreads <= 512;
  // "stage done" ring: one barrier per stage modulo kRing, a multiple of the A (W4) or weight
  // (bf16) ring and of the token ring, so one commit per issuer and stage frees both slots
  static constexpr int kAR = W4 ? AST : WST;
  static constexpr int kRing = lcm_int(kAR, BST);
  static_assert(kRing <= 16, "stage-done ring");
  static_assert(BN % BOX == 0 && BOX % 8 == 0 && BN % 16 == 0, "token tile = whole boxes of whole swizzle atoms");
  static_assert(!W4 || DQ % 4 == 0, "dequantiser groups of four warps");
  // A stage ring may only be waited on by one group: an mbarrier parity wait is exact only
  // while the waiter is at most one phase ahead, so every stage must have a single owner.
  static_assert(!W4 || (WST % kGroups == 0 && AST % kGroups == 0), "stages per dequantiser group");
};

struct __align__(8) GemmBars {
  uint64_t w_full[16], w_empty[16];
  uint64_t b_full[16];
  uint64_t a_full[8];
  uint64_t stage_done[16];     // both issuers' MMAs of stage it finished (index it % kRing)
  uint64_t acc_full[2], acc_empty[2];
  uint64_t mma_done[2];
  uint32_t ready;              // stages published to the MMA issuer by the waiter warp
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

// Tiles are numbered segment-major; inside a segment, feature block then token block
// (fastest) when the segment's weight matrix is the larger operand, token block then
// feature block (fastest) when its activation rows are: the CTAs working at the same time
// then share the larger operand through L2 and each tile of it is read from HBM about once.
// (Activations rows x K x 2 bytes against weights N x K x 2 bytes, or N x K / 2 for int4:
// token blocks first when rows > raster_rows = N, or N / 4.)
template <int BN>
__device__ __forceinline__ TileInfo tile_at(const GemmBars* b, int tile, int& e_hint, int NB, int raster_rows) {
  int e = e_hint;
  while (tile >= b->tile_start[e + 1]) ++e;
  e_hint = e;
  const int n_e = b->row_off[e + 1] - b->row_off[e];
  const int ntb = (n_e + BN - 1) / BN;
  const int local = tile - b->tile_start[e];
  TileInfo ti;
  ti.e = e;
  ti.w = b->seg_w[e];
  int tb;
  if (n_e > raster_rows) {
    tb = local / NB;
    ti.fb = local - tb * NB;
  } else {
    ti.fb = local / ntb;
    tb = local - ti.fb * ntb;
  }
  ti.row0 = b->row_off[e] + tb * BN;
  const int left = n_e - tb * BN;
  ti.rows = left < BN ? left : BN;
  return ti;
}

__device__ __forceinline__ float silu_f(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

template <int BN, int DQ, int WST, int BST, int AST, int ACC, bool W4, int BOX>
__global__ void __launch_bounds__(Cfg<BN, DQ, WST, BST, AST, ACC, W4, BOX>::kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                        const GemmArgs a) {
  using C = Cfg<BN, DQ, WST, BST, AST, ACC, W4, BOX>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* b_stages = base;                                    // BST x [2][BN][64] bf16 (SW128)
  uint8_t* w_stages = b_stages + BST * C::kBStageBytes;        // WST x (int4 super-block | bf16 [2][128][64])
  float* xchg = reinterpret_cast<float*>(w_stages + WST * C::kWStageBytes);
  GemmBars* bars = reinterpret_cast<GemmBars*>(reinterpret_cast<uint8_t*>(xchg) + C::kXchgBytes);
  volatile int* abort_flag = &bars->abort;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  if (tid == 0) {
    for (int s = 0; s < WST; ++s) {
      mbar_init(&bars->w_full[s], 1);
      mbar_init(&bars->w_empty[s], 4);   // W4: the 4 warps of the owning dequantiser group
    }
    for (int s = 0; s < BST; ++s) {
      mbar_init(&bars->b_full[s], 1);

    }
    for (int s = 0; s < AST; ++s) {
      mbar_init(&bars->a_full[s], 4);

    }
    for (int s = 0; s < ACC; ++s) {
      mbar_init(&bars->acc_full[s], 2);
      mbar_init(&bars->acc_empty[s], 128);
    }
    for (int s = 0; s < C::kRing; ++s) mbar_init(&bars->stage_done[s], 2);   // one commit per MMA issuer
    mbar_init(&bars->mma_done[0], 1);
    mbar_init(&bars->mma_done[1], 1);
    bars->abort = 0;
    bars->ready = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&tm_x);
  if (!W4 && warp == 0 && lane == 0) tma_prefetch_desc(&tm_w);
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, a.tmem_cols);
    tmem_relinquish();
  }
  // segment row offsets, weight map and the tile prefix (computed redundantly by every CTA)
  for (int e = tid; e <= a.E; e += C::kThreads) {
    const int64_t o = a.offsets_i64 ? static_cast<const int64_t*>(a.offsets)[e]
                                    : (int64_t) static_cast<const int32_t*>(a.offsets)[e];
    bars->row_off[e] = (int)(o < 0 ? -1 : (o > a.R ? a.R + 1 : o));   // out of range -> caught below
    if (e < a.E) bars->seg_w[e] = a.seg_expert ? a.seg_expert[e] : e;
  }
  __syncthreads();
  if (tid == 0) {
    int acc_t = 0;
    bars->tile_start[0] = 0;
    for (int e = 0; e < a.E; ++e) {
      int n_e = bars->row_off[e + 1] - bars->row_off[e];
      // a hole (weight matrix -1, rows in range) is skipped silently; a segment whose rows
      // or weight matrix lie outside the buffers is skipped and reported
      const bool rows_ok = n_e >= 0 && bars->row_off[e] >= 0 && bars->row_off[e + 1] <= a.R;
      if (rows_ok && bars->seg_w[e] == -1) {
        n_e = 0;
      } else if (!rows_ok || bars->seg_w[e] < 0 || bars->seg_w[e] >= a.num_w) {
        if (n_e != 0) report_error(a.err, kErrBadArg, kSite + 9);
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
  const uint32_t tmem_a = tmem + ACC * BN;   // W4: AST stages of 64 columns
  const int total = bars->total_tiles;
  const int KS = a.KS;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    // One thread issues both streams: the weight copies (one bulk copy of an int4
    // super-block, or two TMA boxes of bf16) run up to kWLead stages ahead of the token
    // tiles, which have the shorter ring.
    if (lane == 0) {
      constexpr int kWLead = WST > BST ? WST - BST : 0;
      uint32_t it = 0, it_w = 0;
      int e_hint = 0, w_hint = 0, tile_w = blockIdx.x, ks_w = 0;
      TileInfo ti_w = {};
      if (tile_w < total) ti_w = tile_at<BN>(bars, tile_w, w_hint, a.NB, a.raster_rows);
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        const TileInfo ti = tile_at<BN>(bars, tile, e_hint, a.NB, a.raster_rows);
        const int nbox = (ti.rows + BOX - 1) / BOX;   // only the boxes that cover this tile's rows
        const uint32_t bytes = (uint32_t)(2 * nbox * BOX * kBK * 2);
        for (int ks = 0; ks < KS; ++ks, ++it) {
          // weights of stages up to it + kWLead
          while (tile_w < total && it_w <= it + kWLead) {
            const int s = it_w % WST;
            const bool w_free =
                W4 ? mbar_wait(&bars->w_empty[s], ((it_w / WST) & 1u) ^ 1u, a.err, abort_flag, kSite + 3)
                   : (it_w < (uint32_t)WST ||
                      mbar_wait(&bars->stage_done[(it_w - WST) % C::kRing], ((it_w - WST) / C::kRing) & 1u, a.err,
                                abort_flag, kSite + 3));
            if (!w_free) { ok = false; break; }
            uint8_t* wsm = w_stages + s * C::kWStageBytes;
            if (W4) {
              const uint8_t* wblk = a.wq + (size_t)(ti_w.w * a.NB + ti_w.fb) * KS * a.sb_bytes;
              mbar_arrive_expect_tx(&bars->w_full[s], a.sb_bytes);
              bulk_load(wsm, wblk + (size_t)ks_w * a.sb_bytes, a.sb_bytes, &bars->w_full[s]);
            } else {
              mbar_arrive_expect_tx(&bars->w_full[s], 2 * kBM * kBK * 2);
#pragma unroll
              for (int j = 0; j < 2; ++j)
                tma_load_2d(wsm + j * kBM * kBK * 2, &tm_w, &bars->w_full[s], (2 * ks_w + j) * kBK,
                            ti_w.w * a.N + ti_w.fb * kBM);
            }
            ++it_w;
            if (++ks_w == KS) {
              ks_w = 0;
              tile_w += gridDim.x;
              if (tile_w < total) ti_w = tile_at<BN>(bars, tile_w, w_hint, a.NB, a.raster_rows);
            }
          }
          if (!ok) break;
          const int s = it % BST;
          if (it >= (uint32_t)BST &&
              !mbar_wait(&bars->stage_done[(it - BST) % C::kRing], ((it - BST) / C::kRing) & 1u, a.err, abort_flag,
                         kSite + 1)) { ok = false; break; }
          uint8_t* bsm = b_stages + s * C::kBStageBytes;
          mbar_arrive_expect_tx(&bars->b_full[s], bytes);
#pragma unroll
          for (int j = 0; j < 2; ++j)
            for (int bx = 0; bx < nbox; ++bx)
              tma_load_2d(bsm + (j * BN + bx * BOX) * kBK * 2, &tm_x, &bars->b_full[s], (2 * ks + j) * kBK,
                          ti.row0 + bx * BOX);
        }
      }
      // no copy of this CTA may still be in flight when it exits
      const uint32_t first = it > (uint32_t)BST ? it - BST : 0u;
      for (uint32_t j = first; j < it; ++j) mbar_wait(&bars->b_full[j % BST], (j / BST) & 1u, a.err, nullptr, kSite + 2);
      const uint32_t first_w = it_w > (uint32_t)WST ? it_w - WST : 0u;
      for (uint32_t j = first_w; j < it_w; ++j) mbar_wait(&bars->w_full[j % WST], (j / WST) & 1u, a.err, nullptr, kSite + 4);
    }
  } else if (warp == 1 || warp == C::kIssue2Warp) {
    // ------------------------------------------------------------------ MMA issuers
    // Two issuing threads, each owning half of the token columns of every tile: an issuing
    // thread blocks for the duration of each MMA it issues, so while one commits or polls
    // the other keeps the tensor pipe busy.
    const int half = warp == 1 ? 0 : 1;
    if (lane == 0) {
      uint32_t it = 0, lt = 0;
      int e_hint = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, ++lt) {
        const TileInfo ti = tile_at<BN>(bars, tile, e_hint, a.NB, a.raster_rows);
        const int n_eff = (ti.rows + 15) & ~15;
        int n_mine = n_eff - half * (BN / 2);   // this issuer's columns, a multiple of 16
        n_mine = n_mine < 0 ? 0 : (n_mine > BN / 2 ? BN / 2 : n_mine);
        const uint32_t idesc = idesc_f16kind_f32(kBM, n_mine > 0 ? (uint32_t)n_mine : 16u, a.ab_f16);
        const uint32_t acc = lt % ACC;
        const uint32_t d_tmem = tmem + acc * BN + half * (BN / 2);
        for (int ks = 0; ks < KS; ++ks, ++it) {
          const int sb = it % BST;
          const int sa = it % (W4 ? AST : WST);
          // the waiter warp publishes a stage once its operands have landed and, at a tile
          // start, once the accumulator buffer is free
          if (!counter_wait(&bars->ready, it, a.err, abort_flag, kSite + 6)) { ok = false; break; }
          tc_fence_after();
          const uint32_t bsm = smem_u32(b_stages + sb * C::kBStageBytes) + half * (BN / 2) * kBK * 2;
#pragma unroll
          for (int j = 0; j < 2 && n_mine > 0; ++j) {
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk) {
              const uint64_t bdesc = sdesc_k_sw128(bsm + j * BN * kBK * 2 + kk * 32);
              const uint32_t accum = (ks | j | kk) != 0 ? 1u : 0u;
              if (W4) {
                mma_ts(d_tmem, tmem_a + sa * 64 + j * 32 + kk * 8, bdesc, idesc, accum);
              } else {
                const uint32_t asm_ = smem_u32(w_stages + sa * C::kWStageBytes) + j * kBM * kBK * 2;
                mma_ss(d_tmem, sdesc_k_sw128(asm_ + kk * 32), bdesc, idesc, accum);
              }
            }
          }
          mma_commit(&bars->stage_done[it % C::kRing]);   // frees the A / weight and token slots
        }
        if (ok) mma_commit(&bars->acc_full[acc]);
      }
      mma_commit(&bars->mma_done[half]);
      mbar_wait(&bars->mma_done[half], 0, a.err, nullptr, kSite + 8);
    }
  } else if (W4 && warp < C::kEpiWarp0) {
    // ------------------------------------------------------------------ int4 dequantisers
    // Group g owns every kGroups-th stage, so several stages are dequantised at once and
    // the barrier / shared-load / tensor-memory-store latency of one overlaps the others.
    const int grp = (warp - 3) >> 2;
    const int q = warp & 3;          // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;   // weight row within the tile
    const int sg = w4_scale_groups(a.group_size);
    const __nv_bfloat162 off136 = __floats2bfloat162_rn(136.0f, 136.0f);
    uint32_t it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
      for (int ks = 0; ks < KS; ++ks, ++it) {
        if ((int)(it % C::kGroups) != grp) continue;
        const int s = it % WST;
        if (!mbar_wait(&bars->w_full[s], (it / WST) & 1u, a.err, abort_flag, kSite + 10)) { ok = false; break; }
        const uint8_t* wsm = w_stages + s * C::kWStageBytes;
        uint4 v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = *reinterpret_cast<const uint4*>(wsm + i * 2048 + row * 16);
        const uint16_t* scl = reinterpret_cast<const uint16_t*>(wsm + kW4SuperInt4Bytes);
        const uint16_t sb0 = scl[row];
        const uint16_t sb1 = scl[(sg > 1 ? 128 : 0) + row];   // second k-block: next group when g == 64
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->w_empty[s]);
        const int as = it % AST;
        const uint32_t taddr = tmem_a + ((uint32_t)(q * 32) << 16) + as * 64;
        if constexpr (C::kEarlyDequant) {
          // enough registers: dequantise the whole stage first, then wait for the TMEM stage
          uint32_t o[4][16];
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            __nv_bfloat162 s_hi, s_lo;
            split_scale(j == 0 ? sb0 : sb1, s_hi, s_lo);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              dequant_half(v[2 * j + h], s_hi, s_lo, off136, o[2 * j + h]);
            }
          }
          if (it >= (uint32_t)AST &&
              !mbar_wait(&bars->stage_done[(it - AST) % C::kRing], ((it - AST) / C::kRing) & 1u, a.err, abort_flag,
                         kSite + 11)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < 4; ++c) tmem_st16(taddr + c * 16, o[c]);
        } else {
          // register-limited (many warps): the first k-block is dequantised before the wait
          // for the TMEM stage, the second 16 columns at a time after it
          uint32_t o[2][16];
          {
            __nv_bfloat162 s_hi, s_lo;
            split_scale(sb0, s_hi, s_lo);
            dequant_half(v[0], s_hi, s_lo, off136, o[0]);
            dequant_half(v[1], s_hi, s_lo, off136, o[1]);
          }
          if (it >= (uint32_t)AST &&
              !mbar_wait(&bars->stage_done[(it - AST) % C::kRing], ((it - AST) / C::kRing) & 1u, a.err, abort_flag,
                         kSite + 11)) { ok = false; break; }
          tc_fence_after();
          tmem_st16(taddr, o[0]);
          tmem_st16(taddr + 16, o[1]);
          {
            __nv_bfloat162 s_hi, s_lo;
            split_scale(sb1, s_hi, s_lo);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              uint32_t o1[16];
              dequant_half(v[2 + h], s_hi, s_lo, off136, o1);
              tmem_st16(taddr + (2 + h) * 16, o1);
            }
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->a_full[as]);
      }
    }
  } else if (warp == C::kWaitWarp) {
    // ------------------------------------------------------------------ MMA issuer's waiter
    // An mbarrier wait in the MMA-issuing thread costs ~270 cycles even when the phase has
    // long completed (a shared-memory load ~40), so this warp does the issuer's waits and
    // publishes the count of ready stages.
    if (lane == 0) {
      uint32_t it = 0, lt = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, ++lt) {
        const uint32_t acc = lt % ACC;
        if (!mbar_wait(&bars->acc_empty[acc], ((lt / ACC) & 1u) ^ 1u, a.err, abort_flag, kSite + 5)) break;
        for (int ks = 0; ks < KS; ++ks, ++it) {
          const int sb = it % BST;
          const int sa = it % (W4 ? AST : WST);
          const bool ready = W4 ? mbar_wait(&bars->a_full[sa], (it / AST) & 1u, a.err, abort_flag, kSite + 13)
                                : mbar_wait(&bars->w_full[sa], (it / WST) & 1u, a.err, abort_flag, kSite + 13);
          if (!ready || !mbar_wait(&bars->b_full[sb], (it / BST) & 1u, a.err, abort_flag, kSite + 7)) {
            ok = false;
            break;
          }
          st_release_shared(&bars->ready, it + 1);
        }
      }
    }
  } else if (warp >= C::kEpiWarp0) {
    // ------------------------------------------------------------------ epilogue
    // 32 accumulator columns (tokens) per step under one TMEM load wait.  SwiGLU: the gate
    // rows (TMEM lanes 0-63) hand the gate values of columns 16-31 to the up rows (lanes
    // 64-127), which hand back the up values of columns 0-15, so all four warps compute and
    // store.  Scatter: the tile's routing weights and destination rows are staged in shared
    // memory once per tile.
    const int q = warp & 3;
    const int row = q * 32 + lane;
    float* tscale = xchg + C::kXchgFloats;                        // [BN]
    int32_t* tdest = reinterpret_cast<int32_t*>(tscale + BN);     // [BN]
    uint32_t lt = 0, chunk = 0;
    int e_hint = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++lt) {
      const TileInfo ti = tile_at<BN>(bars, tile, e_hint, a.NB, a.raster_rows);
      const int n_eff = (ti.rows + 15) & ~15;
      const uint32_t acc = lt % ACC;
      if (!mbar_wait(&bars->acc_full[acc], (lt / ACC) & 1u, a.err, abort_flag, kSite + 12)) break;
      tc_fence_after();
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + acc * BN;
      const int feat = ti.fb * kBM + row;
      if (a.mode == kModeScatter) {
        named_bar_sync(2, 128);   // the previous tile's tables are no longer read
        for (int c = row; c < ti.rows; c += 128) {
          const int r = ti.row0 + c;
          tscale[c] = a.row_scale ? a.row_scale[r] : 1.0f;
          int32_t dv = a.dest ? a.dest[r] : r;
          if (a.dest_bases && (int)((uint32_t)dv >> 24) >= a.dest_count) {   // no such buffer: skip the row
            report_error(a.err, kErrBadArg, kSite + 14);
            dv = -1;
          }
          tdest[c] = dv;
        }
        named_bar_sync(2, 128);
      }
      for (int c0 = 0; c0 < n_eff; c0 += 32, ++chunk) {
        uint32_t v0[16], v1[16];
        tmem_ld16x2(taddr + c0, taddr + c0 + 16, v0, v1);   // c0 + 32 <= BN: inside the buffer
        if (a.mode == kModeSwiGLU && C::kXchgBufs == 2 && a.vec_out) {
          // as below with one exchange buffer, the 32 x 64 bf16 results staged in shared memory
          // (token-major) and written as whole 128-byte token rows with 16-byte stores
          float* xb = xchg;                                                     // [64][33]
          __nv_bfloat16* stg = reinterpret_cast<__nv_bfloat16*>(xchg + 64 * 33);   // [32][64], 4 KB
          const int f = q < 2 ? row : row - 64;
          if (q < 2) {
#pragma unroll
            for (int i = 0; i < 16; ++i) xb[f * 33 + 16 + i] = __uint_as_float(v1[i]);
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) xb[f * 33 + i] = __uint_as_float(v0[i]);
          }
          named_bar_sync(2, 128);
          const int cl = q < 2 ? 0 : 16;   // this thread's 16 columns within the 32
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float g = q < 2 ? __uint_as_float(v0[i]) : xb[f * 33 + 16 + i];
            const float u = q < 2 ? xb[f * 33 + i] : __uint_as_float(v1[i]);
            stg[(cl + i) * 64 + f] = __float2bfloat16_rn(silu_f(g) * u);
          }
          named_bar_sync(2, 128);   // exchange reads and stage writes are done
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int idx = row + 128 * j;    // 16-byte piece: token idx / 8, features 8 * (idx % 8) ..
            const int c = idx >> 3;
            if (c0 + c < ti.rows)
              *reinterpret_cast<uint4*>(a.out + (int64_t)(ti.row0 + c0 + c) * a.ldo + ti.fb * 64 + (idx & 7) * 8) =
                  *reinterpret_cast<const uint4*>(stg + c * 64 + (idx & 7) * 8);
          }
        } else if (a.mode == kModeSwiGLU) {
          float* xb = xchg + (C::kXchgBufs == 2 ? (int)(chunk & 1u) * (64 * 33) : 0);
          const int f = q < 2 ? row : row - 64;   // feature within the tile's 64
          if (q < 2) {
#pragma unroll
            for (int i = 0; i < 16; ++i) xb[f * 33 + 16 + i] = __uint_as_float(v1[i]);
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) xb[f * 33 + i] = __uint_as_float(v0[i]);
          }
          named_bar_sync(2, 128);
          const int cb = c0 + (q < 2 ? 0 : 16);
          const int fo = ti.fb * 64 + f;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int c = cb + i;
            if (c < ti.rows) {
              const float g = q < 2 ? __uint_as_float(v0[i]) : xb[f * 33 + 16 + i];
              const float u = q < 2 ? xb[f * 33 + i] : __uint_as_float(v1[i]);
              a.out[(int64_t)(ti.row0 + c) * a.ldo + fo] = __float2bfloat16_rn(silu_f(g) * u);
            }
          }
          if (C::kXchgBufs == 1) named_bar_sync(2, 128);   // single buffer: reads done before reuse
        } else if (a.vec_out) {
          // stage the 32 x 128 output block in shared memory (token-major), then write whole
          // 256-byte token rows with 16-byte stores instead of 64 bytes per store
          __nv_bfloat16* stg = reinterpret_cast<__nv_bfloat16*>(xchg);   // [32][128], 8 KB
#pragma unroll
          for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int c = 16 * h + i;
              float val = __uint_as_float(h ? v1[i] : v0[i]);
              if (a.mode == kModeScatter && a.row_scale && c0 + c < ti.rows) val = __fmul_rn(val, tscale[c0 + c]);
              stg[c * kBM + row] = cvt_out(val, a.ab_f16);
            }
          }
          named_bar_sync(2, 128);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int idx = row + 128 * j;    // 16-byte piece: token idx / 16, features 8 * (idx % 16) ..
            const int c = idx >> 4;
            if (c0 + c < ti.rows && (a.mode != kModeScatter || tdest[c0 + c] >= 0)) {
              __nv_bfloat16* orow = a.mode == kModeScatter ? scatter_row(a, tdest[c0 + c])
                                                           : a.out + (int64_t)(ti.row0 + c0 + c) * a.ldo;
              *reinterpret_cast<uint4*>(orow + ti.fb * kBM + (idx & 15) * 8) =
                  *reinterpret_cast<const uint4*>(stg + c * kBM + (idx & 15) * 8);
            }
          }
          named_bar_sync(2, 128);   // the stage is rewritten by the next 32 columns
        } else if (feat < a.N) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int c = c0 + 16 * h + i;
              if (c < ti.rows && (a.mode != kModeScatter || tdest[c] >= 0)) {
                float val = __uint_as_float(h ? v1[i] : v0[i]);
                __nv_bfloat16* orow = a.out + (int64_t)(ti.row0 + c) * a.ldo;
                if (a.mode == kModeScatter) {
                  if (a.row_scale) val = __fmul_rn(val, tscale[c]);
                  orow = scatter_row(a, tdest[c]);
                }
                orow[feat] = cvt_out(val, a.ab_f16);
              }
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

template <int BN, int DQ, int WST, int BST, int AST, int ACC, bool W4, int BOX>
int launch_gemm(const CUtensorMap& tm_x, const CUtensorMap& tm_w, GemmArgs a, int grid, cudaStream_t stream) {
  using C = Cfg<BN, DQ, WST, BST, AST, ACC, W4, BOX>;
  static_assert(C::kTmemColsNeeded <= 512, "tensor memory budget");
  static_assert(C::kSmemBytes + sizeof(GemmBars) <= 232448, "shared memory budget");
  static_assert(WST <= 16 && BST <= 16 && AST <= 8 && ACC <= 2, "barrier arrays");
  static_assert(!W4 || (AST >= 1 && WST >= DQ / 4), "every dequantiser group needs a weight stage");
  uint32_t cols = 32;
  while (cols < C::kTmemColsNeeded) cols <<= 1;
  a.tmem_cols = cols;
  const size_t smem = C::kSmemBytes + sizeof(GemmBars);
  auto fn = grouped_gemm_kernel<BN, DQ, WST, BST, AST, ACC, W4, BOX>;
  {
    const int st = set_max_dynamic_smem(reinterpret_cast<const void*>(fn), smem);
    if (st != LMOE_OK) return st;
  }
  fn<<<grid, C::kThreads, smem, stream>>>(tm_x, tm_w, a);
  return cuda_status(cudaGetLastError());
}

}  // namespace

// Internal entry used by the C-ABI wrappers and by the layer driver.
int run_grouped_gemm(const GemmProblem& p, cudaStream_t stream) {
  DeviceInfo dev;
  int st = get_device_info(&dev);
  if (st != LMOE_OK) return st;
  if (dev.cc_major != 10) return LMOE_ERR_DEVICE;
  if (p.num_experts < 1 || p.num_experts > kMaxGemmExperts) return LMOE_ERR_UNSUPPORTED;
  if (p.K < kSK || p.K % kSK) return LMOE_ERR_UNSUPPORTED;
  if (p.total_rows < 0 || p.total_rows > INT32_MAX) return LMOE_ERR_INVALID_ARG;
  if (!p.x || !p.offsets || !p.out || !p.err) return LMOE_ERR_INVALID_ARG;
  const bool w4 = p.wq != nullptr;
  if (w4) {
    const int g = p.group_size;
    if (g < kBK || g % kBK || p.K % g || (g < kSK && kSK % g)) return LMOE_ERR_UNSUPPORTED;
    if (p.N % kBM) return LMOE_ERR_UNSUPPORTED;
  } else {
    if (!p.w) return LMOE_ERR_INVALID_ARG;
    if (p.mode == kModeSwiGLU) return LMOE_ERR_UNSUPPORTED;
  }
  if (p.mode == kModeSwiGLU && (p.N % kBM)) return LMOE_ERR_INVALID_ARG;
  if (p.total_rows == 0) return LMOE_OK;

  GemmArgs a = {};
  a.wq = p.wq;
  a.group_size = p.group_size;
  a.sb_bytes = w4 ? (uint32_t)w4_super_bytes(p.group_size) : 0u;
  a.offsets = p.offsets;
  a.offsets_i64 = p.offsets_i64;
  a.seg_expert = p.seg_expert;
  a.E = p.num_experts;
  a.N = p.N;
  a.K = p.K;
  a.NB = (p.N + kBM - 1) / kBM;
  a.KS = p.K / kSK;
  a.mode = p.mode;
  a.out = static_cast<__nv_bfloat16*>(p.out);
  a.ldo = p.ldo;
  a.dest = p.dest;
  a.row_scale = p.row_scale;
  a.err = p.err;
  a.vec_out = (p.N % kBM == 0 && p.ldo % 8 == 0 && (reinterpret_cast<uintptr_t>(p.out) & 15) == 0) ? 1 : 0;
  a.ab_f16 = (!w4 && p.ab_f16) ? 1 : 0;
  a.num_w = p.num_w > 0 ? p.num_w : p.num_experts;
  a.R = p.total_rows;
  a.raster_rows = w4 ? p.N / 4 : p.N;
  a.dest_bases = p.mode == kModeScatter ? p.dest_bases : nullptr;
  a.dest_count = p.dest_count;

  const bool small = p.max_rows_per_expert_hint > 0 && p.max_rows_per_expert_hint <= 64;
  // token-tile TMA box: 16 rows for decode-sized tiles (load only what the tile holds),
  // the whole 192-row tile otherwise
  const int box = small ? 16 : 192;
  const CUtensorMapDataType tdt = a.ab_f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap tm_x, tm_w;
  st = encode_tmap_2d(&tm_x, p.x, tdt, 2, (uint64_t)p.total_rows, (uint64_t)p.K, (uint64_t)p.ldx * 2, (uint32_t)box,
                      kBK, true);
  if (st != LMOE_OK) return st;
  if (!w4) {
    st = encode_tmap_2d(&tm_w, p.w, tdt, 2, (uint64_t)a.num_w * p.N, (uint64_t)p.K, (uint64_t)p.K * 2, kBM, kBK,
                        true);
    if (st != LMOE_OK) return st;
  } else {
    tm_w = tm_x;
  }
  const int grid = gemm_grid(dev);
  if (w4) {
    //                          BN  DQ WST BST AST ACC  W4   BOX
    if (small) return launch_gemm<64, 16, 12, 6, 4, 2, true, 16>(tm_x, tm_w, a, grid, stream);
    return launch_gemm<192, 8, 6, 3, 2, 2, true, 192>(tm_x, tm_w, a, grid, stream);
  }
  if (small) return launch_gemm<64, 0, 4, 4, 1, 2, false, 16>(tm_x, tm_w, a, grid, stream);
  return launch_gemm<192, 0, 2, 3, 1, 2, false, 192>(tm_x, tm_w, a, grid, stream);
}

}  // namespace lmoe

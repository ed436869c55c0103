// decode_gemm.cu -- W4A16 grouped GEMM for decode-sized segments (at most 64 rows each).
//
// Same inputs as grouped_gemm.cu: segments of rows of X (bf16 [R, K]), the prepacked int4
// super-blocks (w4_layout.cuh, scales embedded) -- one weight copy serves both kernels.
// Reference semantics: csrc/grouped_gemm.cu:11-43 (one GEMM per expert segment) applied to
// the dequantised int4 weights (w = q * s per group of K values; the int4 format itself is
// defined by this library, the reference only has the unused flag
// python/light_moe/engine/executor.py:44-48).
//
// Why a second kernel.  With a handful of tokens per expert the GEMM is a weight stream:
// 8.5 KB of int4 per 128 x 128 super-block, ~23 bytes per SM per cycle at HBM speed, i.e.
// ~380 cycles per super-block.  Measured on B200:
//   * a tcgen05.mma (M=128, K=16, N <= 128) costs ~44 cycles of issue per issuing thread,
//     whatever N is; two threads issuing to separate accumulators overlap (~24 cycles per
//     MMA per SM).  The eight MMAs of a super-block therefore fit the budget only with two
//     issuers, so warp 2 issues k-block 0 and warp 3 k-block 1 of every stage.
//   * dequantising with the scale folded in (bf16_rn(q * s), three fp16 ops per pair) does
//     not fit next to the rest; here the dequantisers only turn nibbles into integer-valued
//     bf16 q (one shift, one LOP3, one exact bf16 subtraction per pair), the MMAs write the
//     per-k-block partial sums P = sum_k q * x into a tensor-memory ring, and the epilogue
//     warps apply the fp16 scale in fp32: acc += s * P.  The result equals
//     sum_k (q * s) * x up to fp32 rounding (it never rounds the weights to bf16).
//
//   * a tcgen05.commit costs about as much issue time as an MMA, and an mbarrier wait in
//     the issuing thread ~270 cycles even when the phase has long completed, so an issuer
//     polls a shared-memory counter (published by warp 16 after its barrier wait), issues
//     its four MMAs and commits once per stage.  The q stage, the token stage and the
//     partial-sum slot share one ring index; "stage ready" (a_full) collects the
//     dequantisers' arrivals, the token TMA bytes and the epilogue's release of the slot's
//     previous round, and "stage done" (mma_done) collects both issuers' commits and the
//     dequantisers' "scales written" arrivals, so the epilogue also waits once per stage.
//
// CTA = one 128-row weight block x up to 32 tokens of one segment (x one K chunk when
// split-K is used), streamed in 128-K stages.  Warp roles (544 threads, one CTA per SM):
//   warp 0        token producer: two TMA boxes (16 or 32 rows x 64 K) per stage
//   warp 1        weight producer: one bulk copy of the int4 super-block per stage
//   warps 2, 3    MMA issuers for k-block 0 / 1 of every stage (tcgen05 "TS": A = q from
//                 tensor memory, B = tokens from shared memory)
//   warps 4..11   dequantisers, two groups of four (group g owns ring slots s with
//                 s % 2 == g), one weight row per thread; they also pass each row's fp16
//                 scales of the stage to the epilogue through a shared-memory ring of
//                 2 x kRing slots (a slot is rewritten only after the epilogue has released
//                 the partial sums of the round before)
//   warps 12..15  epilogue: partial sums -> registers (scaled), output at the tile end
//   warp 16       waits on the stage-ready barrier for the issuers and publishes a counter
//                 they poll (an mbarrier wait in an MMA-issuing thread costs ~270 cycles,
//                 a shared-memory load ~40)
// Epilogues: SwiGLU (gate rows 0..63 / up rows 64..127 of the paired layout), plain bf16,
// or fp32 partial sums per K chunk for split-K (reduced in a fixed order by the combine
// kernel, so results are deterministic).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "decode_gemm.h"
#include "host_util.h"
#include "ptx.cuh"
#include "w4_layout.cuh"

namespace lmoe {
namespace {

constexpr int kBM = 128;             // weight rows per tile
constexpr int kBN = 32;              // tokens per tile (segments with more rows use several)
constexpr int kDQ = 8;               // dequantiser warps
constexpr int kGroups = kDQ / 4;
constexpr int kWST = 16;             // int4 super-block stages (shared memory)
constexpr int kRing = 4;             // q (tensor memory, 64 columns), token (shared memory) and
                                     // partial-sum (tensor memory, 2 x kBN columns) stages
constexpr int kWarpX = 0, kWarpW = 1, kWarpM0 = 2, kWarpDQ = 4, kWarpEpi = kWarpDQ + kDQ;
constexpr int kWarpSync = kWarpEpi + 4;   // waits on a_full for the issuers
constexpr int kThreads = (kWarpSync + 1) * 32;
constexpr uint32_t kBStageBytes = 2u * kBN * 64 * 2;          // [2 k-blocks][32 tokens][64] bf16, SW128
constexpr uint32_t kWStageBytes = kW4SuperInt4Bytes + 512;    // int4 + up to two scale groups
constexpr uint32_t kXchgBytes = 64 * (kBN + 1) * 4;           // SwiGLU exchange [64 rows][33]
constexpr uint32_t kScaleBytes = 2 * kRing * 2 * kBM * 4;     // fp32 scales [2 x ring][k-block][row]
constexpr uint32_t kTmemP = kRing * 64;                       // partial sums after the q stages
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSite = 0x300u;
static_assert(kTmemP + kRing * 2 * kBN <= kTmemCols, "tensor memory budget");
static_assert(kWST % kGroups == 0 && kRing % kGroups == 0, "every stage has one owning dequantiser group");
// Parity waits are exact only while a waiter is at most one phase behind its barrier:
//   a_full[s]   (warp 16, for the issuers) -- the next round needs the epilogue's release of
//               this round, which needs this round's MMAs, issued after warp 16 published
//   mma_done[s] (epilogue) -- the next round's MMAs need the epilogue's release;
//               (dequantisers, token producer, waiting for the previous round) -- this
//               round needs their own arrivals
// The scale ring has 2 x kRing slots: the slot of iteration i is rewritten at i + 2 kRing,
// after mma_done of i + kRing, whose MMAs waited for the epilogue's release of i.

struct DecodeArgs {
  const uint8_t* wq;
  int group_size;
  uint32_t sb_bytes;
  const void* offsets;
  int offsets_i64;
  const int32_t* seg_expert;
  int E, N, K, NB, KS, ksplit;
  int mode;
  void* out;          // bf16 (plain / SwiGLU) or fp32 [ksplit][R][N] (partials)
  int64_t ldo;
  int64_t R;
  int num_w;          // weight matrices available
  uint32_t* err;
};

struct __align__(8) DecodeBars {
  uint64_t w_full[kWST], w_empty[kWST];
  uint64_t a_full[kRing];      // q written (4 dequantiser warps), tokens landed (producer +
                               // bytes), previous round's partial sums read (4 epilogue warps)
  uint64_t mma_done[kRing];    // both issuers' MMAs finished (2 commits), scales written (4)
  uint64_t done[2];
  uint32_t ready;              // stages whose a_full phase has completed (published by kWarpSync)
  uint32_t tmem_base;
  int abort;
  int total_tiles;
  int tile_start[kMaxGemmExperts + 1];
  int row_off[kMaxGemmExperts + 1];
  int seg_w[kMaxGemmExperts];
};

constexpr uint32_t kSmemBytes =
    1024 + kRing * kBStageBytes + kWST * kWStageBytes + kXchgBytes + kScaleBytes + sizeof(DecodeBars);
static_assert(kSmemBytes <= 232448, "shared memory budget");

struct DTile {
  int e, w, fb, kc, row0, rows;
};

// Tiles: segment-major, then weight block, then K chunk, then token tile (fastest, so the
// token tiles of one weight block run side by side and share it through L2).
__device__ __forceinline__ DTile dtile_at(const DecodeBars* b, int tile, int& e_hint, int ksplit) {
  int e = e_hint;
  while (tile >= b->tile_start[e + 1]) ++e;
  e_hint = e;
  const int n_e = b->row_off[e + 1] - b->row_off[e];
  const int ntb = (n_e + kBN - 1) / kBN;
  int local = tile - b->tile_start[e];
  DTile t;
  t.e = e;
  t.w = b->seg_w[e];
  const int tb = local % ntb;
  local /= ntb;
  t.kc = local % ksplit;
  t.fb = local / ksplit;
  t.row0 = b->row_off[e] + tb * kBN;
  const int left = n_e - tb * kBN;
  t.rows = left < kBN ? left : kBN;
  return t;
}

__device__ __forceinline__ uint32_t bf16x2_bits(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ __nv_bfloat162 bits_bf16x2(uint32_t v) { return *reinterpret_cast<__nv_bfloat162*>(&v); }

// One 16-byte half-row (32 K values, w4_layout.cuh) -> the 16 bf16x2 registers of its K pairs
// as integers q = u - 8: pair m = 4i + c lives in word c, slot i.
__device__ __forceinline__ void dequant_q_half(const uint4 v, const __nv_bfloat162 off136, uint32_t (&o)[16]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int c = 0; c < 4; ++c) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t x = ((w[c] >> (4 * i)) & 0x000F000Fu) | 0x43004300u;   // bf16 pair (128 + u)
      o[4 * i + c] = bf16x2_bits(__hsub2(bits_bf16x2(x), off136));         // exact q = u - 8
    }
  }
}

__device__ __forceinline__ float silu_f(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

__global__ void __launch_bounds__(kThreads, 1)
    w4_decode_kernel(const __grid_constant__ CUtensorMap tm_x16, const __grid_constant__ CUtensorMap tm_x32,
                     const DecodeArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* b_stages = base;                                  // kRing x [2][32][64] bf16 (SW128)
  uint8_t* w_stages = b_stages + kRing * kBStageBytes;       // kWST x int4 super-block
  float* xchg = reinterpret_cast<float*>(w_stages + kWST * kWStageBytes);
  float* scl = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(xchg) + kXchgBytes);   // [2 kRing][2][128]
  DecodeBars* bars = reinterpret_cast<DecodeBars*>(reinterpret_cast<uint8_t*>(scl) + kScaleBytes);
  volatile int* abort_flag = &bars->abort;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  if (tid == 0) {
    for (int s = 0; s < kWST; ++s) {
      mbar_init(&bars->w_full[s], 1);
      mbar_init(&bars->w_empty[s], 4);    // the four warps of the owning dequantiser group
    }
    for (int s = 0; s < kRing; ++s) {
      mbar_init(&bars->a_full[s], 4 + 1 + 4);
      mbar_init(&bars->mma_done[s], 2 + 4);
    }
    mbar_init(&bars->done[0], 1);
    mbar_init(&bars->done[1], 1);
    bars->abort = 0;
    bars->ready = 0;
    fence_mbar_init();
    // the epilogue's share of every slot's first round: there is no earlier round to release
    for (int s = 0; s < kRing; ++s)
      for (int i = 0; i < 4; ++i) mbar_arrive(&bars->a_full[s]);
  }
  if (warp == kWarpX && lane == 0) {
    tma_prefetch_desc(&tm_x16);
    tma_prefetch_desc(&tm_x32);
  }
  if (warp == kWarpM0) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  for (int e = tid; e <= a.E; e += kThreads) {
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
      // a segment whose rows or weight matrix lie outside the buffers is skipped
      if (n_e < 0 || bars->row_off[e] < 0 || bars->row_off[e + 1] > a.R || bars->seg_w[e] < 0 ||
          bars->seg_w[e] >= a.num_w) {
        if (n_e != 0) report_error(a.err, kErrBadArg, kSite + 9);
        n_e = 0;
      }
      acc_t += ((n_e + kBN - 1) / kBN) * a.NB * a.ksplit;
      bars->tile_start[e + 1] = acc_t;
    }
    bars->total_tiles = acc_t;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const int total = bars->total_tiles;
  const int ks_per = a.KS / a.ksplit;

  if (warp == kWarpX) {
    // ------------------------------------------------------------------ token producer
    if (lane == 0) {
      uint32_t it = 0;
      int e_hint = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        const DTile t = dtile_at(bars, tile, e_hint, a.ksplit);
        const int box = t.rows <= 16 ? 16 : 32;
        const CUtensorMap* tm = box == 16 ? &tm_x16 : &tm_x32;
        const uint32_t bytes = (uint32_t)(2 * box * 128);
        for (int ks = 0; ks < ks_per; ++ks, ++it) {
          const int s = it % kRing;
          if (!mbar_wait(&bars->mma_done[s], ((it / kRing) & 1u) ^ 1u, a.err, abort_flag, kSite + 1)) {
            ok = false;
            break;
          }
          uint8_t* bsm = b_stages + s * kBStageBytes;
          const int kglob = (t.kc * ks_per + ks) * kW4SuperK;
          mbar_arrive_expect_tx(&bars->a_full[s], bytes);
          tma_load_2d(bsm, tm, &bars->a_full[s], kglob, t.row0);
          tma_load_2d(bsm + kBN * 128, tm, &bars->a_full[s], kglob + 64, t.row0);
        }
      }
      // no copy of this CTA may still be in flight when it exits (the phase also needs the
      // other arrivals, which a run without errors always makes)
      const uint32_t first = it > (uint32_t)kRing ? it - kRing : 0u;
      for (uint32_t j = first; j < it; ++j) mbar_wait(&bars->a_full[j % kRing], (j / kRing) & 1u, a.err, nullptr, kSite + 2);
    }
  } else if (warp == kWarpW) {
    // ------------------------------------------------------------------ weight producer
    if (lane == 0) {
      uint32_t it = 0;
      int e_hint = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        const DTile t = dtile_at(bars, tile, e_hint, a.ksplit);
        const uint8_t* wblk = a.wq + ((size_t)(t.w * a.NB + t.fb) * a.KS + (size_t)t.kc * ks_per) * a.sb_bytes;
        for (int ks = 0; ks < ks_per; ++ks, ++it) {
          const int s = it % kWST;
          if (!mbar_wait(&bars->w_empty[s], ((it / kWST) & 1u) ^ 1u, a.err, abort_flag, kSite + 3)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&bars->w_full[s], a.sb_bytes);
          bulk_load(w_stages + s * kWStageBytes, wblk + (size_t)ks * a.sb_bytes, a.sb_bytes, &bars->w_full[s]);
        }
      }
      const uint32_t first = it > (uint32_t)kWST ? it - kWST : 0u;
      for (uint32_t j = first; j < it; ++j) mbar_wait(&bars->w_full[j % kWST], (j / kWST) & 1u, a.err, nullptr, kSite + 4);
    }
  } else if (warp < kWarpDQ) {
    // ------------------------------------------------------------------ MMA issuers
    const int kb = warp - kWarpM0;   // the k-block of every stage this warp issues
    if (lane == 0) {
      uint32_t it = 0;
      int e_hint = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        const DTile t = dtile_at(bars, tile, e_hint, a.ksplit);
        const uint32_t idesc = idesc_bf16_f32(kBM, (uint32_t)((t.rows + 15) & ~15));
        for (int ks = 0; ks < ks_per; ++ks, ++it) {
          const int s = it % kRing;
          if (!counter_wait(&bars->ready, it, a.err, abort_flag, kSite + 5)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem + kTmemP + (uint32_t)(2 * s + kb) * kBN;
          const uint32_t a_tmem = tmem + (uint32_t)s * 64 + (uint32_t)kb * 32;
          const uint64_t bdesc = sdesc_k_sw128(smem_u32(b_stages + s * kBStageBytes) + kb * kBN * 128);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)   // +32 bytes along K = +2 in the descriptor's address field
            mma_ts(d_tmem, a_tmem + kk * 8, bdesc + (uint64_t)(2 * kk), idesc, kk > 0 ? 1u : 0u);
          mma_commit(&bars->mma_done[s]);   // frees the q and token stages, publishes the partial sums
        }
      }
      mma_commit(&bars->done[kb]);
      mbar_wait(&bars->done[kb], 0, a.err, nullptr, kSite + 8);
    }
  } else if (warp == kWarpSync) {
    // ------------------------------------------------------------------ issuers' waiter
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        for (int ks = 0; ks < ks_per; ++ks, ++it) {
          if (!mbar_wait(&bars->a_full[it % kRing], (it / kRing) & 1u, a.err, abort_flag, kSite + 14)) {
            ok = false;
            break;
          }
          st_release_shared(&bars->ready, it + 1);
        }
      }
    }
  } else if (warp < kWarpEpi) {
    // ------------------------------------------------------------------ dequantisers
    const int grp = (warp - kWarpDQ) >> 2;
    const int q = warp & 3;          // tensor-memory lane quarter this warp may access
    const int row = q * 32 + lane;   // weight row within the tile
    const __nv_bfloat162 off136 = __floats2bfloat162_rn(136.0f, 136.0f);
    const int s1_idx = w4_scale_groups(a.group_size) > 1 ? kBM : 0;   // k-block 1: next group when g == 64
    uint32_t it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
      for (int ks = 0; ks < ks_per; ++ks, ++it) {
        const int s = it % kRing;
        if (s % kGroups != grp) continue;
        const uint32_t ph = (it / kRing) & 1u;
        const int sw = it % kWST;
        if (!mbar_wait(&bars->w_full[sw], (it / kWST) & 1u, a.err, abort_flag, kSite + 10)) {
          ok = false;
          break;
        }
        const uint8_t* wsm = w_stages + sw * kWStageBytes;
        uint4 v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = *reinterpret_cast<const uint4*>(wsm + i * 2048 + row * 16);
        const uint16_t* ssm = reinterpret_cast<const uint16_t*>(wsm + kW4SuperInt4Bytes);
        const float s0 = __half2float(__ushort_as_half(ssm[row]));
        const float s1 = __half2float(__ushort_as_half(ssm[s1_idx + row]));
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->w_empty[sw]);
        // the q stage is free once the MMAs of the previous round of this slot are done
        if (!mbar_wait(&bars->mma_done[s], ph ^ 1u, a.err, abort_flag, kSite + 11)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)s * 64;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint32_t o[16];
          dequant_q_half(v[i], off136, o);
          tmem_st16(taddr + i * 16, o);
        }
        tmem_wait_st();
        const int ss = it % (2 * kRing);
        scl[(2 * ss) * kBM + row] = s0;
        scl[(2 * ss + 1) * kBM + row] = s1;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&bars->mma_done[s]);   // scales of this round written
          mbar_arrive(&bars->a_full[s]);     // q of this round written
        }
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16) + kTmemP;
    uint32_t it = 0;
    int e_hint = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
      const DTile t = dtile_at(bars, tile, e_hint, a.ksplit);
      const int n_eff = (t.rows + 15) & ~15;
      bool ok = true;
      float acc[kBN];
#pragma unroll
      for (int j = 0; j < kBN; ++j) acc[j] = 0.f;
      for (int ks = 0; ks < ks_per; ++ks, ++it) {
        const int s = it % kRing, sp = 2 * s, ss = it % (2 * kRing);
        if (!mbar_wait(&bars->mma_done[s], (it / kRing) & 1u, a.err, abort_flag, kSite + 12)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float s0 = scl[(2 * ss) * kBM + row];
        const float s1 = scl[(2 * ss + 1) * kBM + row];
        // both k-blocks' partial sums, 16 columns at a time; the slot is released as soon as
        // the last columns are in registers
#pragma unroll
        for (int c0 = 0; c0 < kBN; c0 += 16) {
          if (c0 < n_eff) {
            uint32_t p0[16], p1[16];
            tmem_ld16x2(lane_base + (uint32_t)sp * kBN + c0, lane_base + (uint32_t)(sp + 1) * kBN + c0, p0, p1);
            if (c0 + 16 >= n_eff) {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&bars->a_full[s]);   // counts toward the slot's next round
            }
#pragma unroll
            for (int j = 0; j < 16; ++j)
              acc[c0 + j] = __fmaf_rn(s1, __uint_as_float(p1[j]), __fmaf_rn(s0, __uint_as_float(p0[j]), acc[c0 + j]));
          }
        }
      }
      // ---------------------------------------------------------------- output
      // thread = weight row, acc[j] = token row0 + j; every epilogue warp takes every barrier
      if (a.mode == kDecodeSwiGLU) {
        if (ok && q >= 2) {
#pragma unroll
          for (int j = 0; j < kBN; ++j) xchg[(row - 64) * (kBN + 1) + j] = acc[j];
        }
        named_bar_sync(1, 128);
        if (ok && q < 2) {
          __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out);
#pragma unroll
          for (int j = 0; j < kBN; ++j)
            if (j < t.rows)
              out[(int64_t)(t.row0 + j) * a.ldo + t.fb * 64 + row] =
                  __float2bfloat16_rn(silu_f(acc[j]) * xchg[row * (kBN + 1) + j]);
        }
      } else if (ok && a.mode == kDecodePlain) {
        __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out);
#pragma unroll
        for (int j = 0; j < kBN; ++j)
          if (j < t.rows) out[(int64_t)(t.row0 + j) * a.ldo + t.fb * kBM + row] = __float2bfloat16_rn(acc[j]);
      } else if (ok) {   // fp32 partial sums of K chunk kc
        float* out = static_cast<float*>(a.out) + (int64_t)t.kc * a.R * a.ldo;
#pragma unroll
        for (int j = 0; j < kBN; ++j)
          if (j < t.rows) out[(int64_t)(t.row0 + j) * a.ldo + t.fb * kBM + row] = acc[j];
      }
      // xchg is free for the next tile; the four warps leave together after a failure
      if (named_bar_any(1, 128, !ok)) break;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kWarpM0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

int run_decode_gemm(const DecodeProblem& p, cudaStream_t stream) {
  DeviceInfo dev;
  int st = get_device_info(&dev);
  if (st != LMOE_OK) return st;
  if (dev.cc_major != 10) return LMOE_ERR_DEVICE;
  if (p.num_experts < 1 || p.num_experts > kMaxGemmExperts) return LMOE_ERR_UNSUPPORTED;
  if (p.K < kW4SuperK || p.K % kW4SuperK || p.N % kBM) return LMOE_ERR_UNSUPPORTED;
  const int g = p.group_size;
  if (g < 64 || g % 64 || p.K % g || (g < kW4SuperK && kW4SuperK % g)) return LMOE_ERR_UNSUPPORTED;
  if (!p.x || !p.wq || !p.offsets || !p.out || !p.err) return LMOE_ERR_INVALID_ARG;
  if (p.total_rows < 0 || p.total_rows > INT32_MAX) return LMOE_ERR_INVALID_ARG;
  const int KS = p.K / kW4SuperK;
  if (p.ksplit < 1 || KS % p.ksplit) return LMOE_ERR_INVALID_ARG;
  if (p.mode == kDecodeSwiGLU && p.ksplit != 1) return LMOE_ERR_INVALID_ARG;
  if (p.total_rows == 0) return LMOE_OK;

  DecodeArgs a = {};
  a.wq = p.wq;
  a.group_size = g;
  a.sb_bytes = (uint32_t)w4_super_bytes(g);
  a.offsets = p.offsets;
  a.offsets_i64 = p.offsets_i64;
  a.seg_expert = p.seg_expert;
  a.E = p.num_experts;
  a.N = p.N;
  a.K = p.K;
  a.NB = p.N / kBM;
  a.KS = KS;
  a.ksplit = p.ksplit;
  a.mode = p.mode;
  a.out = p.out;
  a.ldo = p.ldo;
  a.R = p.total_rows;
  a.num_w = p.num_w > 0 ? p.num_w : p.num_experts;
  a.err = p.err;
  CUtensorMap tm_x16, tm_x32;
  st = encode_tmap_2d(&tm_x16, p.x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)p.total_rows, (uint64_t)p.K,
                      (uint64_t)p.ldx * 2, 16, 64, true);
  if (st != LMOE_OK) return st;
  st = encode_tmap_2d(&tm_x32, p.x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)p.total_rows, (uint64_t)p.K,
                      (uint64_t)p.ldx * 2, 32, 64, true);
  if (st != LMOE_OK) return st;
  {
    const int st = set_max_dynamic_smem(reinterpret_cast<const void*>(w4_decode_kernel), kSmemBytes);
    if (st != LMOE_OK) return st;
  }
  w4_decode_kernel<<<dev.num_sms, kThreads, kSmemBytes, stream>>>(tm_x16, tm_x32, a);
  return cuda_status(cudaGetLastError());
}

}  // namespace lmoe

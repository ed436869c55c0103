// decode_gemm.cu -- W4A16 grouped GEMM for decode-sized segments (at most 64 rows each).
//
// Same inputs as grouped_gemm.cu: segments of rows of X (bf16 [R, K]), the prepacked int4
// super-blocks (w4_layout.cuh, scales embedded) -- one weight copy serves both kernels.
// Reference semantics: csrc/grouped_gemm.cu:11-43 (one GEMM per expert segment) applied to
// the dequantised int4 weights (w = q * s per group of K values; the int4 format itself is
// defined by this library, the reference only has the unused flag
// python/light_moe/engine/executor.py:44-48).
//
// With a handful of tokens per expert the GEMM is a weight stream: 8.5 KB of int4 per
// 128 x 128 super-block, ~22 bytes per SM per cycle at HBM speed, i.e. ~380 cycles per
// super-block.  Costs measured on B200 that shape the pipeline:
//   * a tcgen05.mma (M=128, K=16, N <= 128) blocks its issuing thread ~44 cycles whatever N
//     is; two threads issuing to separate accumulators overlap (~24 cycles per MMA per SM);
//   * a tcgen05.commit costs about as much issue time as an MMA; an mbarrier wait in an
//     MMA-issuing thread ~270 cycles even on a completed phase, a shared-memory load ~40.
// So:
//   * the dequantisers only turn nibbles into integer-valued bf16 q (one shift, one LOP3 and
//     one exact bf16 subtraction per pair) in tensor memory; the MMAs write the partial sum
//     P = sum_k q * x of each 128-K stage (one scale group) into a tensor-memory slot and the
//     epilogue warps apply the fp16 scale in fp32: acc += s * P (with 64-wide groups, two
//     partial sums per stage, one per k-block).  This equals sum_k (q * s) * x up to fp32
//     rounding;
//   * stages alternate between two MMA issuers and two dequantiser groups by parity: issuer
//     i issues all eight MMAs of its stages (one accumulator per scale group, one commit),
//     fed by dequantiser group i.  The issuers never wait on an mbarrier: they poll two
//     counters in shared memory, "q of stage it written and its tokens landed" (published by
//     their dequantiser group after a named barrier) and "partial-sum slot released"
//     (published by the epilogue after a named barrier);
//   * the q / token ring (kQS stages) and the partial-sum ring (kPS slots) are separate, so
//     the round trips dequantise -> MMA -> q slot free and MMA -> epilogue read -> partial
//     slot free each span several stages.
//
// CTA = one 128-row weight block x up to 32 tokens of one segment (x one K chunk when
// split-K is used), streamed in 128-K stages.  Warp roles (512 threads, one CTA per SM):
//   warp 0        token producer: two TMA boxes (16 or 32 rows x 64 K) per stage
//   warp 1        weight producer: one bulk copy of the int4 super-block per stage
//   warps 2, 3    MMA issuers of the even / odd stages (tcgen05 "TS": A = q from tensor
//                 memory, B = tokens from shared memory)
//   warps 4..11   dequantisers, group g = warps 4+4g..7+4g owns the stages of parity g, one
//                 weight row per thread; it also hands each row's fp16 scales of the stage
//                 to the epilogue through a shared-memory ring
//   warps 12..15  epilogue: partial sums -> registers (scaled), output at the tile end
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
constexpr int kWST = 16;             // int4 super-block stages (shared memory)
constexpr int kWarpX = 0, kWarpW = 1, kWarpM0 = 2, kWarpDQ = 4, kWarpEpi = 12;
constexpr int kThreads = (kWarpEpi + 4) * 32;
constexpr uint32_t kBStageBytes = 2u * kBN * 64 * 2;          // [2 k-blocks][32 tokens][64] bf16, SW128
constexpr uint32_t kWStageBytes = kW4SuperInt4Bytes + 512;    // int4 + up to two scale groups
constexpr uint32_t kXchgBytes = 64 * (kBN + 1) * 4;           // SwiGLU exchange [64 rows][33]
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSite = 0x300u;
constexpr uint32_t kBarEpi = 1, kBarDQ0 = 2;                  // named barriers (kBarDQ0 + group)

__host__ __device__ constexpr int cgcd(int a, int b) { return b == 0 ? a : cgcd(b, a % b); }

// Ring geometry per scale groups per stage (SG = 1: groups of >= 128 K values; SG = 2: 64).
template <int SG>
struct Geo {
  static constexpr int kQS = SG == 1 ? 6 : 4;                 // q (tensor memory) + token stages
  static constexpr int kPS = 4;                               // partial-sum slots
  static constexpr int kPCols = SG * kBN;                     // tensor-memory columns per slot
  static constexpr int kRing = kQS / cgcd(kQS, kPS) * kPS;    // stage_done barriers: lcm(kQS, kPS)
  static constexpr int kSR = kQS + kPS;                       // scale-ring slots
  static constexpr uint32_t kTmemP = kQS * 64;                // partial sums after the q stages
  static constexpr uint32_t kScaleBytes = kSR * SG * kBM * 4;
  static_assert(kTmemP + kPS * kPCols <= kTmemCols, "tensor memory budget");
  static_assert(kQS % 2 == 0 && kPS % 2 == 0 && kWST % 2 == 0 && kRing % 2 == 0,
                "every ring slot belongs to the stages of one parity (one issuer, one dequantiser group)");
  static_assert(kRing <= 16 && kQS <= 8, "barrier arrays");
};

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

// Parity waits are exact only while a waiter is at most one phase behind its barrier:
//   stage_done[b] (stages b, b + kRing, ...; the issuer's commit + the 4 dequantiser warps'
//     "scales written"): the epilogue waits for stage it -- stage it + kRing needs the
//     partial-sum slot the epilogue releases after reading stage it + kRing - kPS >= it;
//     the dequantisers and the token producer wait for stage it - kQS before reusing its
//     q / token slot -- stage it - kQS + kRing needs this stage's q and tokens first;
//   tok_full[s] (dequantisers of stage it): the tokens of it + kQS are only loaded after
//     stage it is done, which needs the dequantisers' q of stage it first;
//   w_full / w_empty: a producer / consumer ring with one consumer group per slot.
// A dequantiser arrival for stage it lands in the phase of stage it: the phase of stage
// it - kRing (same parity, so the same issuer, committed before stage it - kQS) completed
// before the dequantisers' wait for stage it - kQS returned.
struct __align__(8) DecodeBars {
  uint64_t w_full[kWST], w_empty[kWST];
  uint64_t tok_full[8];
  uint64_t stage_done[16];
  uint64_t done[2];
  uint32_t q_ready[2];         // per parity: it + 1 of the last stage whose q and tokens are ready
  uint32_t p_rel;              // stages whose partial sums the epilogue has read
  uint32_t tmem_base;
  int abort;
  int total_tiles;
  int tile_start[kMaxGemmExperts + 1];
  int row_off[kMaxGemmExperts + 1];
  int seg_w[kMaxGemmExperts];
};

template <int SG>
constexpr uint32_t decode_smem_bytes() {
  return 1024 + Geo<SG>::kQS * kBStageBytes + kWST * kWStageBytes + kXchgBytes + Geo<SG>::kScaleBytes +
         (uint32_t)sizeof(DecodeBars);
}
static_assert(decode_smem_bytes<1>() <= 232448 && decode_smem_bytes<2>() <= 232448, "shared memory budget");

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

template <int SG>
__global__ void __launch_bounds__(kThreads, 1)
    w4_decode_kernel(const __grid_constant__ CUtensorMap tm_x16, const __grid_constant__ CUtensorMap tm_x32,
                     const DecodeArgs a) {
  using G = Geo<SG>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* b_stages = base;                                  // kQS x [2][32][64] bf16 (SW128)
  uint8_t* w_stages = b_stages + G::kQS * kBStageBytes;      // kWST x int4 super-block
  float* xchg = reinterpret_cast<float*>(w_stages + kWST * kWStageBytes);
  float* scl = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(xchg) + kXchgBytes);   // [kSR][SG][128]
  DecodeBars* bars = reinterpret_cast<DecodeBars*>(reinterpret_cast<uint8_t*>(scl) + G::kScaleBytes);
  volatile int* abort_flag = &bars->abort;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  if (tid == 0) {
    for (int s = 0; s < kWST; ++s) {
      mbar_init(&bars->w_full[s], 1);
      mbar_init(&bars->w_empty[s], 4);    // the four warps of the owning dequantiser group
    }
    for (int s = 0; s < G::kQS; ++s) mbar_init(&bars->tok_full[s], 1);
    for (int s = 0; s < G::kRing; ++s) mbar_init(&bars->stage_done[s], 1 + 4);   // commit + scales written
    mbar_init(&bars->done[0], 1);
    mbar_init(&bars->done[1], 1);
    bars->abort = 0;
    bars->q_ready[0] = 0;
    bars->q_ready[1] = 0;
    bars->p_rel = 0;
    fence_mbar_init();
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
          const int s = it % G::kQS;
          // the slot's previous tokens (stage it - kQS) have been read by their MMAs
          if (it >= (uint32_t)G::kQS) {
            const uint32_t j = it - G::kQS;
            if (!mbar_wait(&bars->stage_done[j % G::kRing], (j / G::kRing) & 1u, a.err, abort_flag, kSite + 1)) {
              ok = false;
              break;
            }
          }
          uint8_t* bsm = b_stages + s * kBStageBytes;
          const int kglob = (t.kc * ks_per + ks) * kW4SuperK;
          mbar_arrive_expect_tx(&bars->tok_full[s], bytes);
          tma_load_2d(bsm, tm, &bars->tok_full[s], kglob, t.row0);
          tma_load_2d(bsm + kBN * 128, tm, &bars->tok_full[s], kglob + 64, t.row0);
        }
      }
      // no copy of this CTA may still be in flight when it exits
      const uint32_t first = it > (uint32_t)G::kQS ? it - G::kQS : 0u;
      for (uint32_t j = first; j < it; ++j)
        mbar_wait(&bars->tok_full[j % G::kQS], (j / G::kQS) & 1u, a.err, nullptr, kSite + 2);
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
      for (uint32_t j = first; j < it; ++j)
        mbar_wait(&bars->w_full[j % kWST], (j / kWST) & 1u, a.err, nullptr, kSite + 4);
    }
  } else if (warp < kWarpDQ) {
    // ------------------------------------------------------------------ MMA issuers
    const uint32_t par = (uint32_t)(warp - kWarpM0);   // this issuer's stage parity
    if (lane == 0) {
      uint32_t it = 0;
      int e_hint = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        const DTile t = dtile_at(bars, tile, e_hint, a.ksplit);
        const uint32_t idesc = idesc_bf16_f32(kBM, (uint32_t)((t.rows + 15) & ~15));
        for (int ks = 0; ks < ks_per; ++ks, ++it) {
          if ((it & 1u) != par) continue;
          const int sq = it % G::kQS, sp = it % G::kPS;
          // q and tokens of this stage are ready, and the partial sums of stage it - kPS
          // (the slot's previous use) have been read
          bool ready = counter_wait(&bars->q_ready[par], it, a.err, abort_flag, kSite + 5);
          if (ready && it >= (uint32_t)G::kPS)
            ready = counter_wait(&bars->p_rel, it - G::kPS, a.err, abort_flag, kSite + 6);
          if (!ready) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem + G::kTmemP + (uint32_t)sp * G::kPCols;
          const uint32_t a_tmem = tmem + (uint32_t)sq * 64;
          const uint32_t bsm = smem_u32(b_stages + sq * kBStageBytes);
#pragma unroll
          for (int kb = 0; kb < 2; ++kb) {
            const uint64_t bdesc = sdesc_k_sw128(bsm + kb * kBN * 128);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {   // +32 bytes along K = +2 in the descriptor's address field
              const uint32_t accum = SG == 2 ? (kk > 0 ? 1u : 0u) : ((kb | kk) != 0 ? 1u : 0u);
              mma_ts(d_tmem + (SG == 2 ? (uint32_t)kb * kBN : 0u), a_tmem + kb * 32 + kk * 8,
                     bdesc + (uint64_t)(2 * kk), idesc, accum);
            }
          }
          mma_commit(&bars->stage_done[it % G::kRing]);   // frees q / tokens, publishes the partial sums
        }
      }
      mma_commit(&bars->done[par]);
      mbar_wait(&bars->done[par], 0, a.err, nullptr, kSite + 8);
    }
  } else if (warp < kWarpEpi) {
    // ------------------------------------------------------------------ dequantisers
    const int grp = (warp - kWarpDQ) >> 2;
    const int q = warp & 3;          // tensor-memory lane quarter this warp may access
    const int row = q * 32 + lane;   // weight row within the tile
    const __nv_bfloat162 off136 = __floats2bfloat162_rn(136.0f, 136.0f);
    uint32_t it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
      for (int ks = 0; ks < ks_per; ++ks, ++it) {
        if ((int)(it & 1u) != grp) continue;
        const int sq = it % G::kQS;
        const int sw = it % kWST;
        bool fail = !mbar_wait(&bars->w_full[sw], (it / kWST) & 1u, a.err, abort_flag, kSite + 10);
        uint4 v[4];
        float s0 = 0.f, s1 = 0.f;
        if (!fail) {
          const uint8_t* wsm = w_stages + sw * kWStageBytes;
#pragma unroll
          for (int i = 0; i < 4; ++i) v[i] = *reinterpret_cast<const uint4*>(wsm + i * 2048 + row * 16);
          const uint16_t* ssm = reinterpret_cast<const uint16_t*>(wsm + kW4SuperInt4Bytes);
          s0 = __half2float(__ushort_as_half(ssm[row]));
          if (SG == 2) s1 = __half2float(__ushort_as_half(ssm[kBM + row]));
        }
        __syncwarp();
        if (!fail && lane == 0) mbar_arrive(&bars->w_empty[sw]);
        // the q slot is free once the MMAs of stage it - kQS are done
        if (!fail && it >= (uint32_t)G::kQS) {
          const uint32_t j = it - G::kQS;
          fail = !mbar_wait(&bars->stage_done[j % G::kRing], (j / G::kRing) & 1u, a.err, abort_flag, kSite + 11);
        }
        if (!fail) {
          tc_fence_after();
          const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)sq * 64;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint32_t o[16];
            dequant_q_half(v[i], off136, o);
            tmem_st16(taddr + i * 16, o);
          }
          tmem_wait_st();
          float* sc = scl + (it % G::kSR) * SG * kBM;
          sc[row] = s0;
          if (SG == 2) sc[kBM + row] = s1;
          fail = !mbar_wait(&bars->tok_full[sq], (it / G::kQS) & 1u, a.err, abort_flag, kSite + 12);
        }
        tc_fence_before();
        __syncwarp();
        if (!fail && lane == 0) mbar_arrive(&bars->stage_done[it % G::kRing]);   // scales of this stage written
        // the group's four warps agree; then one thread publishes the stage to its issuer
        if (named_bar_any(kBarDQ0 + grp, 128, fail)) {
          ok = false;
          break;
        }
        if (q == 0 && lane == 0) st_release_shared(&bars->q_ready[grp], it + 1);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16) + G::kTmemP;
    uint32_t it = 0;
    int e_hint = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
      const DTile t = dtile_at(bars, tile, e_hint, a.ksplit);
      const int n_eff = (t.rows + 15) & ~15;
      float acc[kBN];
#pragma unroll
      for (int j = 0; j < kBN; ++j) acc[j] = 0.f;
      for (int ks = 0; ks < ks_per; ++ks, ++it) {
        const int sp = it % G::kPS;
        const bool fail =
            !mbar_wait(&bars->stage_done[it % G::kRing], (it / G::kRing) & 1u, a.err, abort_flag, kSite + 13);
        // group 0 (or the only group): columns 0-15 / 16-31; group 1 (64-wide groups) likewise
        uint32_t a0[16], a1[16], b0[16], b1[16];
        float s0 = 0.f, s1 = 0.f;
        if (!fail) {
          tc_fence_after();
          const float* sc = scl + (it % G::kSR) * SG * kBM;
          s0 = sc[row];
          if (SG == 2) s1 = sc[kBM + row];
          const uint32_t pa = lane_base + (uint32_t)sp * G::kPCols;
          if (n_eff > 16) {
            tmem_ld16x2(pa, pa + 16, a0, a1);
            if (SG == 2) tmem_ld16x2(pa + kBN, pa + kBN + 16, b0, b1);
          } else if (SG == 2) {
            tmem_ld16x2(pa, pa + kBN, a0, b0);
          } else {
            tmem_ld16(pa, a0);
          }
          tc_fence_before();
        }
        // the four warps have read the slot: release it to the issuers
        if (named_bar_any(kBarEpi, 128, fail)) {
          ok = false;
          break;
        }
        if (q == 0 && lane == 0) st_release_shared(&bars->p_rel, it + 1);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          acc[j] = __fmaf_rn(s0, __uint_as_float(a0[j]), acc[j]);
          if (SG == 2) acc[j] = __fmaf_rn(s1, __uint_as_float(b0[j]), acc[j]);
        }
        if (n_eff > 16) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            acc[16 + j] = __fmaf_rn(s0, __uint_as_float(a1[j]), acc[16 + j]);
            if (SG == 2) acc[16 + j] = __fmaf_rn(s1, __uint_as_float(b1[j]), acc[16 + j]);
          }
        }
      }
      if (!ok) break;
      // ---------------------------------------------------------------- output
      // thread = weight row, acc[j] = token row0 + j; every epilogue warp takes every barrier
      if (a.mode == kDecodeSwiGLU) {
        if (q >= 2) {
#pragma unroll
          for (int j = 0; j < kBN; ++j) xchg[(row - 64) * (kBN + 1) + j] = acc[j];
        }
        named_bar_sync(kBarEpi, 128);
        if (q < 2) {
          __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out);
#pragma unroll
          for (int j = 0; j < kBN; ++j)
            if (j < t.rows)
              out[(int64_t)(t.row0 + j) * a.ldo + t.fb * 64 + row] =
                  __float2bfloat16_rn(silu_f(acc[j]) * xchg[row * (kBN + 1) + j]);
        }
        named_bar_sync(kBarEpi, 128);   // xchg is free for the next tile
      } else if (a.mode == kDecodePlain) {
        __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out);
#pragma unroll
        for (int j = 0; j < kBN; ++j)
          if (j < t.rows) out[(int64_t)(t.row0 + j) * a.ldo + t.fb * kBM + row] = __float2bfloat16_rn(acc[j]);
      } else {   // fp32 partial sums of K chunk kc
        float* out = static_cast<float*>(a.out) + (int64_t)t.kc * a.R * a.ldo;
#pragma unroll
        for (int j = 0; j < kBN; ++j)
          if (j < t.rows) out[(int64_t)(t.row0 + j) * a.ldo + t.fb * kBM + row] = acc[j];
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kWarpM0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <int SG>
int launch_decode(const CUtensorMap& tm16, const CUtensorMap& tm32, const DecodeArgs& a, int grid,
                  cudaStream_t stream) {
  constexpr uint32_t smem = decode_smem_bytes<SG>();
  auto fn = w4_decode_kernel<SG>;
  const int st = set_max_dynamic_smem(reinterpret_cast<const void*>(fn), smem);
  if (st != LMOE_OK) return st;
  fn<<<grid, kThreads, smem, stream>>>(tm16, tm32, a);
  return cuda_status(cudaGetLastError());
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
  if (w4_scale_groups(g) == 2) return launch_decode<2>(tm_x16, tm_x32, a, dev.num_sms, stream);
  return launch_decode<1>(tm_x16, tm_x32, a, dev.num_sms, stream);
}

}  // namespace lmoe

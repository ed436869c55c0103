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
// 128 x 128 super-block, ~25 bytes per SM per cycle at HBM speed, i.e. ~350 cycles per
// super-block.  Costs measured on B200 that shape the pipeline:
//   * a tcgen05.mma in the "TS" form (A from tensor memory, M = 128, K = 16, N <= 32) holds
//     its issuing thread ~60 cycles whatever N is; up to four threads issuing to separate
//     accumulators overlap almost linearly;
//   * a single thread runs a dependent chain of integer work and branches at ~10 cycles per
//     instruction, and a bulk or tensor TMA issue blocks it ~50-120 cycles: one thread that
//     issued the weight copy and two token boxes of every stage managed one stage per
//     ~1100 cycles, a third of the HBM rate;
//   * turning nibbles into bf16 integers is integer-pipe work (an AND, or a shift and an
//     AND, per four K pairs and one byte permute per pair): a large share of the HBM
//     budget of a stage, so it has to overlap everything else;
//   * a register that fed a tcgen05.st cannot be rewritten before the store has drained, so
//     a stage is dequantised whole into 64 registers first and then stored;
//   * the register file holds 20 warps at 96 registers per thread.
// So:
//   * the dequantisers write q = u - 8 (exact bf16 integers) into tensor memory; the MMAs
//     write the partial sum P = sum_k q * x of each 128-K stage into a tensor-memory slot
//     and the epilogue applies the fp16 group scale in fp32: acc += s * P (two partial sums
//     per stage for 64-wide groups).  This equals sum_k (q * s) * x up to fp32 rounding;
//   * three dequantiser groups and three MMA issuers own the stages it = 0, 1, 2 (mod 3);
//     every hand-off an issuer depends on is a counter in shared memory, one per writing
//     warp (release store / relaxed poll + acquire fence), so the issuers never wait on an
//     mbarrier and no named barrier couples the warps of a group;
//   * the copies are spread over four threads: one producer thread issues only the weight
//     stream (one bulk copy per stage), and each MMA issuer loads the tokens of its own
//     stages (one 3-D TMA box per stage, six stages ahead), so no thread issues more than
//     ~200 cycles of copies per stage;
//   * the dequantisers hand the row's fp16 group scales to the epilogue through a 12-stage
//     ring in shared memory (a load from L2 in the epilogue's loop cost a round trip per
//     stage).
//
// CTA = one 128-row weight block x up to 32 tokens of one segment (x one K chunk when
// split-K is used), streamed in 128-K stages.  Warp roles (640 threads, one CTA per SM):
//   warp 0        weight producer: one bulk copy of the int4 super-block per stage
//   warps 1..3    MMA issuers of the stages it = 0, 1, 2 (mod 3) (tcgen05 "TS": A = q from
//                 tensor memory, B = tokens from shared memory); each also loads the tokens
//                 of its stages ([2 k-blocks][16 or 32 rows][64 K], one 3-D TMA box)
//   warps 4..15   dequantisers, group g = warps 4+4g..7+4g owns the stages it = g (mod 3),
//                 one weight row per thread
//   warps 16..19  epilogue: partial sums -> registers (scaled), output at the tile end
// Epilogues: SwiGLU (gate rows 0..63 / up rows 64..127 of the paired layout), plain bf16,
// or fp32 partial sums per K chunk for split-K (reduced in a fixed order by the combine
// kernel, so results are deterministic).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "decode_gemm.h"
#include "host_util.h"
#include "ptx.cuh"
#include "w4_dequant.cuh"
#include "w4_layout.cuh"

namespace lmoe {
namespace {

constexpr int kBM = 128;             // weight rows per tile
constexpr int kBN = 32;              // tokens per tile (segments with more rows use several)
constexpr int kGroups = 3;           // dequantiser groups = MMA issuers
constexpr int kWST = 4 * kGroups;    // int4 super-block stages (shared memory)
constexpr int kTS = 4 * kGroups;     // token stages (shared memory)
constexpr int kRing = 12;            // stage_done barriers
constexpr int kTokLead = 6;          // an issuer loads the tokens of stage it + kTokLead before stage it's MMAs
constexpr int kWarpP = 0, kWarpM0 = 1, kWarpDQ = kWarpM0 + kGroups, kWarpEpi = kWarpDQ + 4 * kGroups;
constexpr int kThreads = (kWarpEpi + 4) * 32;
constexpr uint32_t kBStageBytes = 2u * kBN * 64 * 2;          // [2 k-blocks][32 tokens][64] bf16, SW128
constexpr uint32_t kWStageBytes = kW4SuperInt4Bytes + 512;    // int4 + up to two scale groups
constexpr uint32_t kXchgBytes = 64 * (kBN + 1) * 4;           // SwiGLU exchange [64 rows][33]
constexpr int kSR = 12;                                        // scale-ring slots (stages)
constexpr uint32_t kScaleBytes = kSR * 2 * 128 * 4;            // [kSR][<= 2 groups][128 rows] fp32
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSite = 0x300u;
constexpr uint32_t kBarEpi = 1;                               // named barrier of the epilogue warps

static_assert(kThreads == 640, "20 warps: 96 registers per thread");
static_assert(kWarpDQ % 4 == 0 && kWarpEpi % 4 == 0, "a warp's tensor-memory lane quarter is its index mod 4");

// Ring geometry per scale groups per stage (SG = 1: groups of >= 128 K values; SG = 2: 64).
template <int SG>
struct Geo {
  static constexpr int kQS = SG == 1 ? 6 : 3;                 // q stages (tensor memory, 64 columns each)
  static constexpr int kPS = 4;                               // partial-sum slots
  static constexpr int kPCols = SG * kBN;                     // tensor-memory columns per slot
  static constexpr uint32_t kTmemP = kQS * 64;                // partial sums after the q stages
  static_assert(kTmemP + kPS * kPCols <= kTmemCols, "tensor memory budget");
  static_assert(kQS % kGroups == 0 && kWST % kGroups == 0, "a q / weight slot serves one dequantiser group");
  static_assert(kRing % kQS == 0 && kRing % kPS == 0 && kRing % kTS == 0, "stage_done covers every ring");
  static_assert(kSR >= kQS + kPS, "a scale-ring slot is rewritten only after the epilogue read it");
  static_assert(kTS % kGroups == 0 && kTokLead % kGroups == 0 && kTokLead + kGroups <= kTS,
                "a token slot is reloaded by the issuer that used it, after its MMAs");
  static_assert(kTS - kTokLead >= kPS && kTokLead + kPS <= kTS,
                "the partial-sum check of a stage covers the MMAs of the token slot it reloads");
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
//   stage_done[b] (stages b, b + kRing, ...; the MMA commit and the four dequantiser warps'
//     "scales written" each; a dequantiser warp arrives for stage it after its wait for
//     stage it - kQS, which follows the commit of stage it - kRing from the same issuer, and
//     after its own arrival for stage it - kRing, so every arrival lands in its stage's
//     phase): the epilogue waits for
//     stage it -- stage it + kRing needs the partial-sum slot the epilogue frees after
//     reading stage it + kRing - kPS > it; the dequantisers wait for stage it - kQS before
//     reusing its q slot -- stage it - kQS + kRing needs this stage's q first;
//   tok_full[s] (dequantiser warp 0 of the stage's group): the tokens of stage it + kTS
//     are loaded by the stage's issuer before its MMAs of stage it + kTS - kTokLead, which
//     come after the MMAs of stage it, which need this wait first;
//   w_full / w_empty: a producer / consumer ring, one consumer group per slot.
struct __align__(16) DecodeBars {
  uint32_t q_ready[kGroups][4];   // per dequantiser warp: it + 1 of its last stage whose q is
                                  // in tensor memory (warp 0 of a group: and whose tokens landed)
  uint32_t p_rel[4];              // per epilogue warp: stages whose partial sums it has read
  uint64_t w_full[kWST], w_empty[kWST];
  uint64_t tok_full[kTS];
  uint64_t stage_done[kRing];
  uint64_t done[kGroups];
  uint32_t tmem_base;
  int abort;
  int total_tiles;
  int tile_start[kMaxGemmExperts + 1];
  int row_off[kMaxGemmExperts + 1];
  int seg_w[kMaxGemmExperts];
};

constexpr uint32_t decode_smem_bytes() {
  return 1024 + kTS * kBStageBytes + kWST * kWStageBytes + kXchgBytes + kScaleBytes + (uint32_t)sizeof(DecodeBars);
}
static_assert(decode_smem_bytes() <= 232448, "shared memory budget");

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

// A role's position in the CTA's stage sequence (tiles blockIdx.x, + gridDim.x, ...; K
// stages within a tile).
struct Cursor {
  int tile, ks, e_hint;
  uint32_t it;
  DTile t;
};

__device__ __forceinline__ bool cursor_start(Cursor& c, const DecodeBars* b, int total, int ksplit) {
  c.tile = blockIdx.x;
  c.ks = 0;
  c.e_hint = 0;
  c.it = 0;
  if (c.tile >= total) return false;
  c.t = dtile_at(b, c.tile, c.e_hint, ksplit);
  return true;
}

__device__ __forceinline__ bool cursor_next(Cursor& c, const DecodeBars* b, int total, int ksplit, int ks_per) {
  ++c.it;
  if (++c.ks < ks_per) return true;
  c.ks = 0;
  c.tile += gridDim.x;
  if (c.tile >= total) return false;
  c.t = dtile_at(b, c.tile, c.e_hint, ksplit);
  return true;
}

// One 16-byte half-row (32 K values, w4_layout.cuh) -> the 16 bf16x2 registers of its K pairs
// in K order as integers q = u - 8.
__device__ __forceinline__ void dequant_q_half(const uint4 v, const __nv_bfloat162 off136, uint32_t (&o)[16]) {
  w4_unpack_half(v, o);
#pragma unroll
  for (int m = 0; m < 16; ++m) o[m] = bf16x2_bits(__hsub2(bits_bf16x2(o[m]), off136));   // exact
}

__device__ __forceinline__ float silu_f(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

template <int SG>
__global__ void __launch_bounds__(kThreads, 1)
    w4_decode_kernel(const __grid_constant__ CUtensorMap tm_x16, const __grid_constant__ CUtensorMap tm_x32,
                     const DecodeArgs a) {
  using G = Geo<SG>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* b_stages = base;                                  // kTS x [2][32][64] bf16 (SW128)
  uint8_t* w_stages = b_stages + kTS * kBStageBytes;         // kWST x int4 super-block
  float* xchg = reinterpret_cast<float*>(w_stages + kWST * kWStageBytes);
  float* scl = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(xchg) + kXchgBytes);   // [kSR][SG][128]
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
    for (int s = 0; s < kTS; ++s) mbar_init(&bars->tok_full[s], 1);
    for (int s = 0; s < kRing; ++s) mbar_init(&bars->stage_done[s], 1 + 4);   // MMA commit + scales written
    for (int g = 0; g < kGroups; ++g) mbar_init(&bars->done[g], 1);
    bars->abort = 0;
    fence_mbar_init();
  }
  if (tid < kGroups * 4) (&bars->q_ready[0][0])[tid] = 0;
  if (tid < 4) bars->p_rel[tid] = 0;
  if (warp == kWarpM0 + 1 && lane == 0) {
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
      // a hole (weight matrix -1, rows in range) is skipped silently; a segment whose rows
      // or weight matrix lie outside the buffers is skipped and reported
      const bool rows_ok = n_e >= 0 && bars->row_off[e] >= 0 && bars->row_off[e + 1] <= a.R;
      if (rows_ok && bars->seg_w[e] == -1) {
        n_e = 0;
      } else if (!rows_ok || bars->seg_w[e] < 0 || bars->seg_w[e] >= a.num_w) {
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

  if (warp == kWarpP) {
    // ------------------------------------------------------------------ weight producer
    if (lane == 0) {
      uint32_t it = 0;
      int e_hint = 0;
      int s = 0;
      uint32_t ph = 0;   // phase parity of slot s's current use
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        const DTile t = dtile_at(bars, tile, e_hint, a.ksplit);
        const uint8_t* src = a.wq + ((size_t)(t.w * a.NB + t.fb) * a.KS + (size_t)t.kc * ks_per) * a.sb_bytes;
        for (int ks = 0; ks < ks_per; ++ks, ++it, src += a.sb_bytes) {
          // the slot's previous stage it - kWST has been read by its dequantiser group
          if (it >= (uint32_t)kWST && !mbar_wait(&bars->w_empty[s], ph ^ 1u, a.err, abort_flag, kSite + 3)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&bars->w_full[s], a.sb_bytes);
          bulk_load(w_stages + s * kWStageBytes, src, a.sb_bytes, &bars->w_full[s]);
          if (++s == kWST) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      // no copy of this CTA may still be in flight when it exits
      for (uint32_t j = it > (uint32_t)kWST ? it - kWST : 0u; j < it; ++j)
        mbar_wait(&bars->w_full[j % kWST], (j / kWST) & 1u, a.err, nullptr, kSite + 4);
    }
  } else if (warp < kWarpDQ) {
    // ------------------------------------------------------------------ MMA issuers
    // Issuer `me` owns the stages it = me (mod kGroups): it loads their tokens (one 3-D TMA
    // box per stage, kTokLead stages ahead) and issues their MMAs.
    const uint32_t me = (uint32_t)(warp - kWarpM0);
    if (lane == 0) {
      Cursor tc;   // next stage of this issuer whose tokens are to be loaded
      bool t_on = cursor_start(tc, bars, total, a.ksplit);
      for (uint32_t k = 0; k < me && t_on; ++k) t_on = cursor_next(tc, bars, total, a.ksplit, ks_per);
      // tokens of stage tc.it; its slot's previous stage tc.it - kTS must be done (the caller
      // has made sure); then advance tc by kGroups stages
      auto load_tokens = [&]() {
        const uint32_t j = tc.it;
        const int s = j % kTS;
        const int box = tc.t.rows <= 16 ? 16 : 32;
        mbar_arrive_expect_tx(&bars->tok_full[s], (uint32_t)(2 * box * 128));
        tma_load_3d(b_stages + s * kBStageBytes, box == 16 ? &tm_x16 : &tm_x32, &bars->tok_full[s], 0, tc.t.row0,
                    (tc.t.kc * ks_per + tc.ks) * 2);
        for (int k = 0; k < kGroups && t_on; ++k) t_on = cursor_next(tc, bars, total, a.ksplit, ks_per);
      };
      while (t_on && tc.it < (uint32_t)kTokLead) load_tokens();
      // walk only this issuer's stages (a single thread here runs its bookkeeping slowly:
      // no iterations over the other issuers' stages)
      Cursor c;
      bool on = cursor_start(c, bars, total, a.ksplit);
      for (uint32_t k = 0; k < me && on; ++k) on = cursor_next(c, bars, total, a.ksplit, ks_per);
      uint32_t p_seen = 0;
      while (on) {
        const uint32_t it = c.it;
        const uint32_t n_eff = (uint32_t)((c.t.rows + 15) & ~15);
        const uint32_t idesc = idesc_bf16_f32(kBM, n_eff);
        const uint32_t kb_bytes = (c.t.rows <= 16 ? 16u : 32u) * 128u;   // k-block stride of the token box
        // q of stage it in tensor memory (all four warps of the group) and its tokens
        // landed; the partial-sum slot's previous stage it - kPS read by the epilogue
        bool ready = counter4_wait(bars->q_ready[me], it, nullptr, a.err, abort_flag, kSite + 5);
        if (ready && it >= (uint32_t)G::kPS && p_seen <= it - G::kPS)
          ready = counter4_wait(bars->p_rel, it - G::kPS, &p_seen, a.err, abort_flag, kSite + 6);
        if (!ready) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + G::kTmemP + (it % G::kPS) * G::kPCols;
        const uint32_t a_tmem = tmem + (it % G::kQS) * 64;
        const uint32_t bsm = smem_u32(b_stages + (it % kTS) * kBStageBytes);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
          const uint64_t bdesc = sdesc_k_sw128(bsm + kb * kb_bytes);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {   // +32 bytes along K = +2 in the descriptor's address field
            const uint32_t accum = SG == 2 ? (kk > 0 ? 1u : 0u) : ((kb | kk) != 0 ? 1u : 0u);
            mma_ts(d_tmem + (SG == 2 ? (uint32_t)kb * kBN : 0u), a_tmem + kb * 32 + kk * 8,
                   bdesc + (uint64_t)(2 * kk), idesc, accum);
          }
        }
        mma_commit(&bars->stage_done[it % kRing]);   // frees q / tokens, publishes the partial sums
        // tokens of stage it + kTokLead: its slot held stage it + kTokLead - kTS, whose partial
        // sums the epilogue has read (p_seen > it - kPS >= it + kTokLead - kTS), so its MMAs
        // are done; before kPS stages the slot has not been used yet
        if (t_on && tc.it == it + kTokLead) load_tokens();
        for (int k = 0; k < kGroups && on; ++k) on = cursor_next(c, bars, total, a.ksplit, ks_per);
      }
      mma_commit(&bars->done[me]);
      mbar_wait(&bars->done[me], 0, a.err, nullptr, kSite + 8);
      // no token copy of this issuer may still be in flight when the CTA exits
      const uint32_t first = tc.it > (uint32_t)kTS ? tc.it - kTS : 0u;
      for (uint32_t j = first; j < tc.it; ++j)
        if (j % kGroups == me) mbar_wait(&bars->tok_full[j % kTS], (j / kTS) & 1u, a.err, nullptr, kSite + 2);
    }
  } else if (warp < kWarpEpi) {
    // ------------------------------------------------------------------ dequantisers
    const int grp = (warp - kWarpDQ) >> 2;
    const int q = warp & 3;          // tensor-memory lane quarter this warp may access
    const int row = q * 32 + lane;   // weight row within the tile
    const __nv_bfloat162 off136 = __floats2bfloat162_rn(136.0f, 136.0f);
    const int my_tiles = total > (int)blockIdx.x ? (total - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
    const uint32_t n_st = (uint32_t)my_tiles * (uint32_t)ks_per;
    for (uint32_t it = (uint32_t)grp; it < n_st; it += kGroups) {
      const int sw = it % kWST;
      bool fail = !mbar_wait(&bars->w_full[sw], (it / kWST) & 1u, a.err, abort_flag, kSite + 10);
      fail = __any_sync(0xffffffffu, fail);
      if (fail) break;
      uint32_t o[4][16];
      float s0, s1 = 0.f;
      {
        const uint8_t* wsm = w_stages + sw * kWStageBytes;
        uint4 v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = *reinterpret_cast<const uint4*>(wsm + i * 2048 + row * 16);
        const uint16_t* ssm = reinterpret_cast<const uint16_t*>(wsm + kW4SuperInt4Bytes);
        s0 = __half2float(__ushort_as_half(ssm[row]));
        if (SG == 2) s1 = __half2float(__ushort_as_half(ssm[kBM + row]));
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->w_empty[sw]);
#pragma unroll
        for (int i = 0; i < 4; ++i) dequant_q_half(v[i], off136, o[i]);
      }
      // the q slot is free once the MMAs of stage it - kQS are done
      if (it >= (uint32_t)G::kQS) {
        const uint32_t j = it - G::kQS;
        fail = !mbar_wait(&bars->stage_done[j % kRing], (j / kRing) & 1u, a.err, abort_flag, kSite + 11);
        fail = __any_sync(0xffffffffu, fail);
        if (fail) break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (it % G::kQS) * 64;
#pragma unroll
      for (int i = 0; i < 4; ++i) tmem_st16(taddr + i * 16, o[i]);
      // the scale-ring slot's previous stage it - kSR was read by the epilogue before it
      // released stage it - kSR's partial sums, which stage it - kQS's MMAs waited for
      float* sc = scl + (it % kSR) * (2 * kBM);
      sc[row] = s0;
      if (SG == 2) sc[kBM + row] = s1;
      tmem_wait_st();
      if (q == 0) {
        fail = !mbar_wait(&bars->tok_full[it % kTS], (it / kTS) & 1u, a.err, abort_flag, kSite + 12);
        fail = __any_sync(0xffffffffu, fail);
        if (fail) break;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        st_release_shared(&bars->q_ready[grp][q], it + 1);
        mbar_arrive(&bars->stage_done[it % kRing]);   // this warp's scales of stage it are written
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16) + G::kTmemP;
    uint32_t it = 0;
    int e_hint = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
      const DTile t = dtile_at(bars, tile, e_hint, a.ksplit);
      const int n_eff = (t.rows + 15) & ~15;
      float acc[kBN];
#pragma unroll
      for (int j = 0; j < kBN; ++j) acc[j] = 0.f;
      bool ok = true;
      for (int ks = 0; ks < ks_per; ++ks, ++it) {
        bool fail = !mbar_wait(&bars->stage_done[it % kRing], (it / kRing) & 1u, a.err, abort_flag, kSite + 13);
        if (__any_sync(0xffffffffu, fail)) {
          ok = false;
          break;
        }
        const float* sc = scl + (it % kSR) * (2 * kBM);
        const float s0 = sc[row];
        const float s1 = SG == 2 ? sc[kBM + row] : 0.f;
        tc_fence_after();
        const uint32_t pa = lane_base + (it % G::kPS) * G::kPCols;
        if (SG == 1) {
          // columns 0-15 / 16-31 of the slot
          uint32_t a0[16], a1[16];
          if (n_eff > 16) tmem_ld16x2(pa, pa + 16, a0, a1);
          else tmem_ld16(pa, a0);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) st_release_shared(&bars->p_rel[q], it + 1);   // this warp's lanes of the slot are read
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[j] = __fmaf_rn(s0, __uint_as_float(a0[j]), acc[j]);
          if (n_eff > 16) {
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[16 + j] = __fmaf_rn(s0, __uint_as_float(a1[j]), acc[16 + j]);
          }
        } else {
          // scale group 0 in columns 0-31, group 1 in columns 32-63; tokens 0-15 then 16-31
          uint32_t a0[16], b0[16];
          tmem_ld16x2(pa, pa + kBN, a0, b0);
#pragma unroll
          for (int j = 0; j < 16; ++j)
            acc[j] = __fmaf_rn(s1, __uint_as_float(b0[j]), __fmaf_rn(s0, __uint_as_float(a0[j]), acc[j]));
          if (n_eff > 16) {
            tmem_ld16x2(pa + 16, pa + kBN + 16, a0, b0);
#pragma unroll
            for (int j = 0; j < 16; ++j)
              acc[16 + j] =
                  __fmaf_rn(s1, __uint_as_float(b0[j]), __fmaf_rn(s0, __uint_as_float(a0[j]), acc[16 + j]));
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) st_release_shared(&bars->p_rel[q], it + 1);
        }
      }
      // the four epilogue warps agree before the output (the SwiGLU exchange has barriers)
      if (named_bar_any(kBarEpi, 128, !ok)) break;
      // ---------------------------------------------------------------- output
      // thread = weight row, acc[j] = token row0 + j; every epilogue warp takes every barrier
      // (token halves 16-31 only when the tile has more than 16 rows)
      const int halves = n_eff > 16 ? 2 : 1;
      if (a.mode == kDecodeSwiGLU) {
        if (q >= 2) {
#pragma unroll
          for (int h = 0; h < 2; ++h)
            if (h < halves) {
#pragma unroll
              for (int j = 16 * h; j < 16 * h + 16; ++j) xchg[(row - 64) * (kBN + 1) + j] = acc[j];
            }
        }
        named_bar_sync(kBarEpi, 128);
        if (q < 2) {
          __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out) + (int64_t)t.row0 * a.ldo + t.fb * 64 + row;
#pragma unroll
          for (int h = 0; h < 2; ++h)
            if (h < halves) {
#pragma unroll
              for (int j = 16 * h; j < 16 * h + 16; ++j)
                if (j < t.rows) out[(int64_t)j * a.ldo] = __float2bfloat16_rn(silu_f(acc[j]) * xchg[row * (kBN + 1) + j]);
            }
        }
        named_bar_sync(kBarEpi, 128);   // xchg is free for the next tile
      } else if (a.mode == kDecodePlain) {
        __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out) + (int64_t)t.row0 * a.ldo + t.fb * kBM + row;
#pragma unroll
        for (int h = 0; h < 2; ++h)
          if (h < halves) {
#pragma unroll
            for (int j = 16 * h; j < 16 * h + 16; ++j)
              if (j < t.rows) out[(int64_t)j * a.ldo] = __float2bfloat16_rn(acc[j]);
          }
      } else {   // fp32 partial sums of K chunk kc
        float* out = static_cast<float*>(a.out) + (int64_t)t.kc * a.R * a.ldo + (int64_t)t.row0 * a.ldo +
                     t.fb * kBM + row;
#pragma unroll
        for (int h = 0; h < 2; ++h)
          if (h < halves) {
#pragma unroll
            for (int j = 16 * h; j < 16 * h + 16; ++j)
              if (j < t.rows) out[(int64_t)j * a.ldo] = acc[j];
          }
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
  constexpr uint32_t smem = decode_smem_bytes();
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
  // tokens: [2 k-blocks][16 or 32 rows][64] per stage, one 3-D box
  CUtensorMap tm_x16, tm_x32;
  st = encode_tmap_kblocks(&tm_x16, p.x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)p.total_rows, (uint64_t)p.K,
                           (uint64_t)p.ldx * 2, 16, 2);
  if (st != LMOE_OK) return st;
  st = encode_tmap_kblocks(&tm_x32, p.x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)p.total_rows, (uint64_t)p.K,
                           (uint64_t)p.ldx * 2, 32, 2);
  if (st != LMOE_OK) return st;
  const int grid = gemm_grid(dev);
  if (w4_scale_groups(g) == 2) return launch_decode<2>(tm_x16, tm_x32, a, grid, stream);
  return launch_decode<1>(tm_x16, tm_x32, a, grid, stream);
}

}  // namespace lmoe

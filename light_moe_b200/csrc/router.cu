// router.cu -- the fused MoE router for B200 (sm_100a).
//
// One kernel computes, for every token:
//   logits = x . W^T (+ b)          tcgen05 MMA, bf16 x bf16 -> fp32 in tensor memory
//   p      = softmax(logits)        fp32, exp of (logit - max), sequential sum, reciprocal
//   top-k  by p                     ties keep the lower expert id
//   w      = p_topk / sum(p_topk)   reciprocal-multiply renormalisation
// and, over all tokens, the per-expert histogram, its exclusive scan (offsets) and the
// stable permutation sorted_idx (expert, token, slot) of the flattened assignment list.
//
// Reference semantics: csrc/fused_moe_ops.cu:145-231 (fused_gate_topk_cuda,
// fused_softmax_topk_kernel, fused_gate_topk_permute_cuda) and
// python/light_moe/ops/moe_gate.py:39-77, :202-214.  The reference runs a cuBLAS fp32 GEMM
// after two dtype-conversion copies, a CUDA-core softmax/top-k kernel for E in {8,16} and
// top-2 only, and ~2E+6 ATen launches for counts/offsets/argsort; here it is one kernel.
//
// Structure (persistent, one CTA per SM, up to 128 tokens per tile, 10 warps):
//   warp 0     TMA producer: two x tiles [128 x 64] and two W tiles [Epad x 64] per stage
//              (128B swizzle; 256 contiguous bytes of every token row per stage)
//   warp 1     MMA issuer: 8 x tcgen05.mma (M=128, N=Epad, K=16) per stage into one of two
//              TMEM accumulators
//   warps 2-5  epilogue: one token row per thread (TMEM lane), softmax / top-k / renormalise,
//              per-tile expert bitmap for the permutation
//   warps 6-9  epilogue helpers (more than 16 experts): the upper half of each row's expert
//              columns (exponentials, partial top-k), exchanged through shared memory
// When the permutation is requested the kernel is launched cooperatively and, after a grid
// barrier, every CTA scans the per-tile counts and scatters its tokens into sorted_idx.
#include <cuda_bf16.h>

#include <mutex>

#include "host_util.h"
#include "lmoe_math.cuh"
#include "ptx.cuh"

namespace lmoe {
namespace {

constexpr int kBM = 128;          // MMA rows per tile; a tile holds bm <= kBM tokens (see router_tile_rows)
constexpr int kBK = 64;           // hidden elements per TMA box (one 128-byte swizzle row)
constexpr int kBoxes = 2;         // boxes per pipeline stage: 128 hidden elements per stage
constexpr int kEpiWarps = 4;      // epilogue warps that own the token rows (one per TMEM lane quarter)
constexpr int kThreads = 64 + 2 * 32 * kEpiWarps;   // producer, MMA issuer, owners, helpers: 10 warps
constexpr uint32_t kEpiAllBar = 6;   // named barrier of all epilogue threads (ids 1-5: owners, pairs)
constexpr int kMaxStages = 8;
constexpr int kMaxExperts = 256;
constexpr uint32_t kSite = 0x100u;

struct RouterArgs {
  const float* bias;
  int32_t* ids;
  float* weights;
  __nv_bfloat16* weights_bf16;
  float* logits;
  float* probs;           // optional full softmax probabilities [T, E]
  int32_t* counts;
  int32_t* offsets;
  int32_t* sorted_idx;
  int32_t* positions;     // optional inverse of sorted_idx: positions[t*k+j] = its sorted row
  int32_t* tile_counts;   // [num_tiles, E]
  uint32_t* tile_bits;    // [num_tiles, E, 4] : bit r of word r/32 set if token row r picked e
  uint32_t* grid_sync;    // arrival counter for the grid barrier (zeroed by the host)
  uint32_t* err;          // device error word (zeroed by the host)
  int T, d, E, Epad, k, num_tiles, stages;
  int bm;                 // tokens per tile (multiple of 8, <= kBM); MMA rows >= bm are ignored
  uint32_t stage_bytes;   // kBoxes x tiles + kBoxes W tiles, multiple of 1024
  uint32_t w_box_bytes;   // one W tile [Epad x kBK]
  uint32_t tmem_cols;
  int do_perm;
  int ab_f16;             // x and W are fp16 (else bf16) on the tensor-core path
};

struct __align__(8) RouterHdr {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
  float bias[kMaxExperts];
  uint32_t bits[kMaxExperts * 4];
  int32_t total[kMaxExperts];
  int32_t offs[kMaxExperts + 1];
};

__device__ __forceinline__ int32_t warp_inclusive_scan(int32_t v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  return v;
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_gpu_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Permutation phase when every CTA routed exactly one tile (tile = blockIdx.x): the tile's
// expert ids and per-expert row bitmaps are still in shared memory, so only the
// [num_tiles, E] count table is read back.  Per expert, a warp sums the counts of the tiles
// before this one and of all tiles (lanes over tiles, then a shuffle reduction: integer
// sums, order-exact); then the exclusive scan of the totals and the scatter of the tile's
// tokens, as in perm_phase.  `area` holds the count table and the prefixes (16-byte aligned)
// below the tile's ids.
template <int KMAX, int NT>
__device__ __forceinline__ void perm_phase_one_tile(const RouterArgs& a, int32_t* area, const int32_t* tile_ids,
                                                    const uint32_t* bits, int32_t* total, int32_t* offs) {
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int tile = (int)blockIdx.x;
  const int n = a.num_tiles * a.E;
  // all of a thread's 16-byte loads in flight at once (one L2 round trip for the table)
  constexpr int kBatch = 8;
  for (int i0 = tid * 4; i0 < n; i0 += NT * 4 * kBatch) {
    int4 v[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int i = i0 + u * NT * 4;
      if (i + 3 < n) v[u] = __ldcg(reinterpret_cast<const int4*>(a.tile_counts + i));
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int i = i0 + u * NT * 4;
      if (i + 3 < n) {
        *reinterpret_cast<int4*>(area + i) = v[u];
      } else {
        for (int r = i; r < n; ++r) area[r] = __ldcg(a.tile_counts + r);   // ragged tail
      }
    }
  }
  __syncthreads();
  int32_t* pref = area + ((n + 3) & ~3);   // [E] counts of this expert in the tiles before this one
  for (int e = warp; e < a.E; e += NT / 32) {
    int32_t before = 0, all = 0;
    for (int tt = lane; tt < a.num_tiles; tt += 32) {
      const int32_t c = area[tt * a.E + e];
      all += c;
      if (tt < tile) before += c;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      before += __shfl_xor_sync(0xffffffffu, before, o);
      all += __shfl_xor_sync(0xffffffffu, all, o);
    }
    if (lane == 0) {
      pref[e] = before;
      total[e] = all;
    }
  }
  __syncthreads();
  if (warp == 0) {
    int32_t run = 0;
    for (int e0 = 0; e0 < a.E; e0 += 32) {
      const int e = e0 + lane;
      const int32_t c = e < a.E ? total[e] : 0;
      const int32_t v = warp_inclusive_scan(c, lane);
      if (e < a.E) offs[e] = run + v - c;
      run += __shfl_sync(0xffffffffu, v, 31);
    }
    if (lane == 0) offs[a.E] = run;
  }
  __syncthreads();
  if (blockIdx.x == 0) {
    for (int e = tid; e < a.E; e += NT) {
      a.counts[e] = total[e];
      a.offsets[e] = offs[e];
    }
    if (tid == 0) a.offsets[a.E] = offs[a.E];
  }
  for (int row = tid; row < a.bm; row += NT) {
    const int64_t t = (int64_t)tile * a.bm + row;
    if (t >= a.T) continue;
    const int w = row >> 5;
    const uint32_t below = (1u << (row & 31)) - 1u;
#pragma unroll
    for (int j = 0; j < KMAX; ++j) {
      if (j < a.k) {
        const int e = tile_ids[row * KMAX + j];
        int rank = __popc(bits[e * 4 + w] & below);
#pragma unroll
        for (int i = 0; i < 3; ++i)
          if (i < w) rank += __popc(bits[e * 4 + i]);
        const int32_t pos = offs[e] + pref[e] + rank;
        a.sorted_idx[pos] = (int32_t)(t * a.k + j);
        if (a.positions) a.positions[t * a.k + j] = pos;
      }
    }
  }
}

// Permutation phase, run once every tile's counts and bitmaps are in global memory: the
// per-expert totals and, for each tile this CTA owns (blockIdx.x + i * gridDim.x), the
// count of earlier tiles, from the [num_tiles, E] count table staged through shared memory
// in chunks of tiles (16-byte loads, all of a thread's loads in flight at once); thread e
// walks column e of a chunk in tile order.  Integer sums: the result is order-exact.  Then
// the exclusive scan of the totals and the scatter of this CTA's tokens into sorted_idx
// (rank of a token within its tile and expert = popcount of the lower bits of the bitmap).
// `area` holds area_ints ints of shared memory (16-byte aligned); NT threads take part.
template <int KMAX, int NT>
__device__ __forceinline__ void perm_phase(const RouterArgs& a, int32_t* area, int area_ints, int32_t* total,
                                           int32_t* offs) {
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int own_max = (a.num_tiles + (int)gridDim.x - 1) / (int)gridDim.x;
  int32_t* pref = area;                              // [own tiles, E]
  const int pref_ints = (own_max * a.E + 3) & ~3;
  int32_t* chunk = pref + pref_ints;                 // [chunk tiles, E], 16-byte aligned
  const int chunk_ints = area_ints - pref_ints;
  const int chunk_tiles = min(((chunk_ints / a.E) & ~3), (a.num_tiles + 3) & ~3);   // >= 4 (host)
  constexpr int kEPer = (kMaxExperts + NT - 1) / NT;
  int32_t run[kEPer];
#pragma unroll
  for (int j = 0; j < kEPer; ++j) run[j] = 0;
  for (int c0 = 0; c0 < a.num_tiles; c0 += chunk_tiles) {
    const int nt = min(chunk_tiles, a.num_tiles - c0);
    const int n = nt * a.E;
    const int32_t* src = a.tile_counts + (int64_t)c0 * a.E;   // c0 * E * 4 is 16-byte aligned
    constexpr int kBatch = 8;
    for (int i0 = tid * 4; i0 < n; i0 += NT * 4 * kBatch) {
      int4 v[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int i = i0 + u * NT * 4;
        if (i + 3 < n) v[u] = __ldcg(reinterpret_cast<const int4*>(src + i));
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int i = i0 + u * NT * 4;
        if (i + 3 < n) {
          *reinterpret_cast<int4*>(chunk + i) = v[u];
        } else {
          for (int r = i; r < n; ++r) chunk[r] = __ldcg(src + r);   // ragged tail (E % 4 != 0)
        }
      }
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kEPer; ++j) {
      const int e = tid + j * NT;
      if (e < a.E) {
        int32_t r = run[j];
        int own = (c0 + (int)gridDim.x - 1 - (int)blockIdx.x) / (int)gridDim.x;   // owned tiles before c0
        int next = (int)blockIdx.x + own * (int)gridDim.x;                      // next owned tile
        for (int tt = 0; tt < nt; ++tt) {
          const int tile = c0 + tt;
          if (tile == next) {
            pref[own * a.E + e] = r;
            ++own;
            next += (int)gridDim.x;
          }
          r += chunk[tt * a.E + e];
        }
        run[j] = r;
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int j = 0; j < kEPer; ++j) {
    const int e = tid + j * NT;
    if (e < a.E) total[e] = run[j];
  }
  __syncthreads();
  // exclusive scan of the per-expert totals: warp 0, 32 experts per round
  if (warp == 0) {
    int32_t run = 0;
    for (int e0 = 0; e0 < a.E; e0 += 32) {
      const int e = e0 + lane;
      const int32_t c = e < a.E ? total[e] : 0;
      const int32_t v = warp_inclusive_scan(c, lane);
      if (e < a.E) offs[e] = run + v - c;
      run += __shfl_sync(0xffffffffu, v, 31);
    }
    if (lane == 0) offs[a.E] = run;
  }
  __syncthreads();
  if (blockIdx.x == 0) {
    for (int e = tid; e < a.E; e += NT) {
      a.counts[e] = total[e];
      a.offsets[e] = offs[e];
    }
    if (tid == 0) a.offsets[a.E] = offs[a.E];
  }
  int own = 0;
  for (int tile = blockIdx.x; tile < a.num_tiles; tile += gridDim.x, ++own) {
    for (int row = tid; row < a.bm; row += NT) {
      const int64_t t = (int64_t)tile * a.bm + row;
      if (t >= a.T) continue;
      const int w = row >> 5;
      const uint32_t below = (1u << (row & 31)) - 1u;
      // the row's k expert ids, then their k tile bitmaps: two rounds of loads in flight
      int ev[KMAX];
      uint4 bv[KMAX];
#pragma unroll
      for (int j = 0; j < KMAX; ++j)
        if (j < a.k) ev[j] = __ldcg(&a.ids[t * a.k + j]);
#pragma unroll
      for (int j = 0; j < KMAX; ++j)
        if (j < a.k) bv[j] = __ldcg(reinterpret_cast<const uint4*>(a.tile_bits) + (int64_t)tile * a.E + ev[j]);
#pragma unroll
      for (int j = 0; j < KMAX; ++j) {
        if (j < a.k) {
          const uint32_t b[4] = {bv[j].x, bv[j].y, bv[j].z, bv[j].w};
          int rank = __popc(b[w] & below);
#pragma unroll
          for (int i = 0; i < 3; ++i)
            if (i < w) rank += __popc(b[i]);
          const int32_t pos = offs[ev[j]] + pref[own * a.E + ev[j]] + rank;
          a.sorted_idx[pos] = (int32_t)(t * a.k + j);
          if (a.positions) a.positions[t * a.k + j] = pos;
        }
      }
    }
  }
}

template <int KMAX>
__global__ void __launch_bounds__(kThreads, 1)
    router_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                  const RouterArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  RouterHdr* h = reinterpret_cast<RouterHdr*>(base + a.stages * a.stage_bytes);
  uint8_t* xchg = reinterpret_cast<uint8_t*>(h + 1);   // owner / helper exchange (split epilogue only)
  volatile int* abort_flag = &h->abort;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int nk = (a.d + kBK * kBoxes - 1) / (kBK * kBoxes);   // stages per tile
  // Every CTA routes at most one tile: after its accumulator is full the stage area is free,
  // so the epilogue keeps the tile's expert ids at its end (and the bitmap in the header) for
  // the permutation phase, which then reads back only the count table.
  const int area_ints = (int)(((size_t)a.stages * a.stage_bytes) / 4);
  const bool one_tile = a.num_tiles <= (int)gridDim.x &&
                        ((a.num_tiles * a.E + 3) & ~3) + a.E + kBM * KMAX <= area_ints;
  int32_t* tile_ids = reinterpret_cast<int32_t*>(base) + area_ints - kBM * KMAX;   // [row][KMAX]
  constexpr uint32_t kXBox = kBM * kBK * 2;

  if (tid == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&h->full[s], 1);
      mbar_init(&h->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&h->acc_full[b], 1);
      mbar_init(&h->acc_empty[b], 128);
    }
    mbar_init(&h->mma_done, 1);
    h->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_w);
  }
  if (warp == 1) {
    tmem_alloc(&h->tmem_base, a.tmem_cols);
    tmem_relinquish();
  }
  for (int e = tid; e < a.E; e += kThreads) h->bias[e] = a.bias ? a.bias[e] : 0.0f;
  for (int i = tid; i < a.E * 4; i += kThreads) h->bits[i] = 0u;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = h->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < a.num_tiles && ok; tile += gridDim.x) {
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const int s = it % a.stages;
          const uint32_t ph = (it / a.stages) & 1u;
          if (!mbar_wait(&h->empty[s], ph ^ 1u, a.err, abort_flag, kSite + 1)) { ok = false; break; }
          uint8_t* xs = base + s * a.stage_bytes;
          uint8_t* ws = xs + kBoxes * kXBox;
          const int nb = min(kBoxes, a.d / kBK - kc * kBoxes);   // the last stage may hold one box
          // an x box is bm rows (bm * 128 bytes, rows past T zero-filled); rows bm..127 of the
          // slot keep stale bytes, which only reach accumulator rows that are never read
          mbar_arrive_expect_tx(&h->full[s], (uint32_t)nb * ((uint32_t)a.bm * kBK * 2 + a.w_box_bytes));
          for (int b = 0; b < nb; ++b) {
            tma_load_2d(xs + b * kXBox, &tm_x, &h->full[s], (kc * kBoxes + b) * kBK, tile * a.bm);
            tma_load_2d(ws + b * a.w_box_bytes, &tm_w, &h->full[s], (kc * kBoxes + b) * kBK, 0);
          }
        }
      }
      // never leave the CTA with bulk copies still landing in shared memory
      const uint32_t issued = it;
      const uint32_t first = issued > (uint32_t)a.stages ? issued - a.stages : 0u;
      for (uint32_t j = first; j < issued; ++j) {
        const int s = j % a.stages;
        mbar_wait(&h->full[s], (j / a.stages) & 1u, a.err, nullptr, kSite + 2);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16kind_f32(kBM, a.Epad, a.ab_f16);
      uint32_t it = 0, lt = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < a.num_tiles && ok; tile += gridDim.x, ++lt) {
        const uint32_t acc = lt & 1u;
        if (!mbar_wait(&h->acc_empty[acc], ((lt >> 1) & 1u) ^ 1u, a.err, abort_flag, kSite + 3)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + acc * a.Epad;
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const int s = it % a.stages;
          if (!mbar_wait(&h->full[s], (it / a.stages) & 1u, a.err, abort_flag, kSite + 4)) { ok = false; break; }
          tc_fence_after();
          const uint32_t xa = smem_u32(base + s * a.stage_bytes);
          const uint32_t wa = xa + kBoxes * kXBox;
          const int nb = min(kBoxes, a.d / kBK - kc * kBoxes);
#pragma unroll
          for (int b = 0; b < kBoxes; ++b) {
            if (b < nb) {
#pragma unroll
              for (int kk = 0; kk < kBK / 16; ++kk) {
                mma_ss(d_tmem, sdesc_k_sw128(xa + b * kXBox + kk * 32),
                       sdesc_k_sw128(wa + b * a.w_box_bytes + kk * 32), idesc, (kc | b | kk) != 0 ? 1u : 0u);
              }
            }
          }
          mma_commit(&h->empty[s]);
        }
        if (ok) mma_commit(&h->acc_full[acc]);
      }
      // all issued MMAs must retire before the tensor memory is released
      mma_commit(&h->mma_done);
      mbar_wait(&h->mma_done, 0, a.err, nullptr, kSite + 5);
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    // Warp w serves TMEM lane quarter w & 3.  Warps 2-5 own the token rows; when the experts
    // span more than one 16-column chunk, warps 6-9 take the upper chunks of the same rows
    // (exponentials and a partial top-k), so each pass has two threads per row.
    const int q = warp & 3;
    const int row = q * 32 + lane;           // token row within the tile
    const bool owner = warp < 2 + kEpiWarps;
    const int nch = a.Epad / 16;
    const bool split = nch >= 2;
    const int ch_a = split ? (nch + 1) / 2 : nch;   // chunks [0, ch_a) to the owner
    const int c_lo = owner ? 0 : ch_a * 16;
    const int c_hi = owner ? ch_a * 16 : a.Epad;
    const uint32_t pair_bar = 2 + q;         // the owner warp and its helper (64 threads)
    const uint32_t epi_threads = split ? 2 * 32 * kEpiWarps : 32 * kEpiWarps;
    float* x_m = reinterpret_cast<float*>(xchg);                  // [2][128]
    float* x_inv = x_m + 2 * kBM;                                 // [128]
    float* x_tv = x_inv + kBM;                                    // [KMAX][128]
    int* x_ti = reinterpret_cast<int*>(x_tv + KMAX * kBM);        // [KMAX][128]
    uint32_t lt = 0;
    for (int tile = blockIdx.x; (owner || split) && tile < a.num_tiles; tile += gridDim.x, ++lt) {
      const uint32_t acc = lt & 1u;
      // every epilogue thread leaves together if any of them gave up waiting
      const bool fail = !mbar_wait(&h->acc_full[acc], (lt >> 1) & 1u, a.err, abort_flag, kSite + 6);
      if (named_bar_any(kEpiAllBar, epi_threads, fail)) break;
      tc_fence_after();
      const int64_t t = (int64_t)tile * a.bm + row;
      const bool valid = row < a.bm && t < a.T;
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + acc * a.Epad;
      uint32_t r[16];
      float tv[KMAX];
      int ti[KMAX];
#pragma unroll
      for (int j = 0; j < KMAX; ++j) { tv[j] = -INFINITY; ti[j] = 0; }
      if (!split) {
        // one 16-column chunk per row: one tensor-memory load, everything else in registers
        // (the same operations in the same order as the chunked passes below)
        tmem_ld16(taddr, r);
        float v[16];
        float m = -INFINITY;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          v[i] = 0.0f;
          if (i < a.E) {
            const float l = __fadd_rn(__uint_as_float(r[i]), h->bias[i]);
            v[i] = l;
            m = fmaxf(m, l);
            if (a.logits && valid) a.logits[t * a.E + i] = l;
          }
        }
        float sum = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          if (i < a.E) {
            v[i] = softmax_exp(__fsub_rn(v[i], m));
            sum = __fadd_rn(sum, v[i]);
          }
        }
        const float inv = __frcp_rn(sum);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          if (i < a.E) {
            const float p = __fmul_rn(v[i], inv);
            if (a.probs && valid) a.probs[t * a.E + i] = p;
            topk_insert<KMAX>(tv, ti, p, i);
          }
        }
      } else {
        // pass 1: logits (+bias), running max over this thread's chunks
        float m = -INFINITY;
        for (int c0 = c_lo; c0 < c_hi; c0 += 16) {
          tmem_ld16(taddr + c0, r);
  #pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int e = c0 + i;
            if (e < a.E) {
              const float l = __fadd_rn(__uint_as_float(r[i]), h->bias[e]);
              m = fmaxf(m, l);
              if (a.logits && valid) a.logits[t * a.E + e] = l;
            }
          }
        }
        if (split) {   // the maximum is exact in any order
          x_m[(owner ? 0 : kBM) + row] = m;
          named_bar_sync(pair_bar, 64);
          m = fmaxf(x_m[row], x_m[kBM + row]);
        }
        // pass 2: exp(l - max) of this thread's chunks, written back over the logits
        for (int c0 = c_lo; c0 < c_hi; c0 += 16) {
          tmem_ld16(taddr + c0, r);
  #pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int e = c0 + i;
            const float l = __fadd_rn(__uint_as_float(r[i]), h->bias[e < a.E ? e : 0]);
            r[i] = e < a.E ? __float_as_uint(softmax_exp(__fsub_rn(l, m))) : 0u;
          }
          tmem_st16(taddr + c0, r);
        }
        tmem_wait_st();
        if (split) {
          tc_fence_before();
          named_bar_sync(pair_bar, 64);
          tc_fence_after();
        }
        // the owner sums all exponentials sequentially over experts 0..E-1
        float inv = 0.0f;
        if (owner) {
          float sum = 0.0f;
          for (int c0 = 0; c0 < a.Epad; c0 += 16) {
            tmem_ld16(taddr + c0, r);
  #pragma unroll
            for (int i = 0; i < 16; ++i)
              if (c0 + i < a.E) sum = __fadd_rn(sum, __uint_as_float(r[i]));
          }
          inv = __frcp_rn(sum);
        }
        if (split) {
          if (owner) x_inv[row] = inv;
          named_bar_sync(pair_bar, 64);
          if (!owner) inv = x_inv[row];
        }
        // pass 3: probabilities and top-k over this thread's chunks
        for (int c0 = c_lo; c0 < c_hi; c0 += 16) {
          tmem_ld16(taddr + c0, r);
  #pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int e = c0 + i;
            if (e < a.E) {
              const float p = __fmul_rn(__uint_as_float(r[i]), inv);
              if (a.probs && valid) a.probs[t * a.E + e] = p;
              topk_insert<KMAX>(tv, ti, p, e);
            }
          }
        }
        if (split) {
          // the helper's list (higher expert ids, descending) is inserted after the owner's:
          // the merged list equals the sequential insertion over all experts
          tc_fence_before();
          if (!owner) {
  #pragma unroll
            for (int j = 0; j < KMAX; ++j) {
              x_tv[j * kBM + row] = tv[j];
              x_ti[j * kBM + row] = ti[j];
            }
          }
          named_bar_sync(pair_bar, 64);
          if (owner) {
  #pragma unroll
            for (int j = 0; j < KMAX; ++j) topk_insert<KMAX>(tv, ti, x_tv[j * kBM + row], x_ti[j * kBM + row]);
          }
        }
      }
      if (!owner) continue;
      // the accumulator can be reused by the MMA warp (the helper finished reading it
      // before the last pair barrier)
      tc_fence_before();
      mbar_arrive(&h->acc_empty[acc]);
      float ssum = 0.0f;
#pragma unroll
      for (int j = 0; j < KMAX; ++j)
        if (j < a.k) ssum = __fadd_rn(ssum, tv[j]);
      const float invs = __frcp_rn(ssum);
      if (valid) {
#pragma unroll
        for (int j = 0; j < KMAX; ++j) {
          if (j < a.k) {
            const float w = __fmul_rn(tv[j], invs);
            a.ids[t * a.k + j] = ti[j];
            if (a.weights) a.weights[t * a.k + j] = w;
            if (a.weights_bf16) a.weights_bf16[t * a.k + j] = __float2bfloat16_rn(w);
            if (a.do_perm) {
              atomicOr(&h->bits[ti[j] * 4 + (row >> 5)], 1u << (row & 31));
              if (one_tile) tile_ids[row * KMAX + j] = ti[j];
            }
          }
        }
      }
      if (a.do_perm) {
        named_bar_sync(1, 32 * kEpiWarps);
        for (int e = row; e < a.E; e += kBM) {
          uint32_t b[4];
          int cnt = 0;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            b[i] = h->bits[e * 4 + i];
            cnt += __popc(b[i]);
            if (!one_tile) h->bits[e * 4 + i] = 0u;   // one tile per CTA: kept for the scatter
          }
          a.tile_counts[(int64_t)tile * a.E + e] = cnt;
          uint4 bv = make_uint4(b[0], b[1], b[2], b[3]);
          reinterpret_cast<uint4*>(a.tile_bits)[(int64_t)tile * a.E + e] = bv;
        }
        named_bar_sync(1, 32 * kEpiWarps);
      }
    }
  }

  __syncthreads();

  // ---------------------------------------------------------------- permutation phase
  if (a.do_perm) {
    if (tid == 0) {
      // release: the CTA's counts and bitmaps (ordered before by the barrier above) become
      // visible with the arrival; acquire on the poll that sees every arrival
      red_release_gpu_add(a.grid_sync, 1u);
      const uint64_t t0 = globaltimer_ns();
      uint32_t spins = 0;
      while (ld_acquire_gpu(a.grid_sync) < gridDim.x) {
        if (((++spins) & 255u) == 0u && globaltimer_ns() - t0 > kWaitBudgetNs) {
          report_error(a.err, kErrTimeout, kSite + 7);
          h->abort = 1;
          break;
        }
      }
    }
    __syncthreads();
    if (!*abort_flag) {
      if (one_tile)
        perm_phase_one_tile<KMAX, kThreads>(a, reinterpret_cast<int32_t*>(base), tile_ids, h->bits, h->total,
                                            h->offs);
      else
        perm_phase<KMAX, kThreads>(a, reinterpret_cast<int32_t*>(base), area_ints, h->total, h->offs);
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, a.tmem_cols);
  }
}

// ---------------------------------------------------------------------------------------
// Logits on CUDA cores.
//  * Small batches (at most kSmallTokens tokens, i.e. one 128-token tile): the tensor-core
//    kernel above would run on a single SM, streaming the whole batch through one CTA.
//    Instead one warp per (token, expert) computes the logit as a dot product (16-byte
//    loads, fp32 accumulation, fixed butterfly reduction: deterministic).
//  * Inputs that are not both bf16 or both fp16 (fp32 hidden states or gate weight, or a mix
//    of types): the reference converts both operands to fp32 and multiplies them in fp32
//    (csrc/fused_moe_ops.cu:158-159), which a kind::f16 tensor-core MMA cannot reproduce
//    (it takes one 16-bit type for both operands).  A tiled fp32 FFMA GEMM computes the
//    logits from the caller's values; each logit is one sequential fp32 sum over the hidden
//    dimension (deterministic).
// The routing itself (softmax / top-k / renormalise, counts, offsets, permutation) then
// runs from the fp32 logits with the same arithmetic as the tensor-core epilogue.
// ---------------------------------------------------------------------------------------
constexpr int kSmallTokens = 128;

// Eight consecutive elements (16-byte aligned) as fp32.
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&f)[8]) {
  const uint4 v = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
    f[2 * j] = t.x;
    f[2 * j + 1] = t.y;
  }
}
__device__ __forceinline__ void load8(const __half* p, float (&f)[8]) {
  const uint4 v = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
    f[2 * j] = t.x;
    f[2 * j + 1] = t.y;
  }
}
__device__ __forceinline__ void load8(const float* p, float (&f)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

template <typename TX, typename TW>
__global__ void __launch_bounds__(256) router_small_logits_kernel(const TX* __restrict__ x, const TW* __restrict__ w,
                                                                   const float* __restrict__ bias, int T, int d,
                                                                   int E, float* __restrict__ logits) {
  const int t = blockIdx.x;
  const int e = blockIdx.y * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T || e >= E) return;
  const TX* xr = x + (int64_t)t * d;
  const TW* wr = w + (int64_t)e * d;
  float acc = 0.0f;
  for (int i = lane; i < d / 8; i += 32) {
    float xf[8], wf[8];
    load8(xr + 8 * i, xf);
    load8(wr + 8 * i, wf);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc = __fmaf_rn(xf[j], wf[j], acc);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
  if (lane == 0) logits[(int64_t)t * E + e] = bias ? __fadd_rn(acc, bias[e]) : acc;
}

// logits[t, e] = sum_i x[t, i] * w[e, i] (+ bias[e]): tiles of TM tokens x EW experts, 32
// hidden values per step staged in shared memory as fp32; each thread owns 4 tokens x 4
// experts and adds the products of one logit in hidden order (fp32 FFMA).
template <typename TX, typename TW, int TM, int EW>
__global__ void __launch_bounds__((TM / 4) * (EW / 4)) router_simt_logits_kernel(
    const TX* __restrict__ x, const TW* __restrict__ w, const float* __restrict__ bias, int T, int d, int E,
    float* __restrict__ logits) {
  constexpr int kNT = (TM / 4) * (EW / 4);
  constexpr int kKS = 32;
  __shared__ __align__(16) float xs[kKS][TM];
  __shared__ __align__(16) float ws[kKS][EW];
  const int tid = threadIdx.x;
  const int tx = tid % (EW / 4);   // expert quad
  const int ty = tid / (EW / 4);   // token quad
  const int64_t t0 = (int64_t)blockIdx.x * TM;
  const int e0 = blockIdx.y * EW;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
  for (int k0 = 0; k0 < d; k0 += kKS) {
    for (int i = tid; i < TM * (kKS / 8); i += kNT) {
      const int r = i / (kKS / 8), seg = i % (kKS / 8);
      float f[8];
      if (t0 + r < T) {
        load8(x + (t0 + r) * d + k0 + seg * 8, f);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) f[j] = 0.0f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) xs[seg * 8 + j][r] = f[j];
    }
    for (int i = tid; i < EW * (kKS / 8); i += kNT) {
      const int r = i / (kKS / 8), seg = i % (kKS / 8);
      float f[8];
      if (e0 + r < E) {
        load8(w + (int64_t)(e0 + r) * d + k0 + seg * 8, f);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) f[j] = 0.0f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ws[seg * 8 + j][r] = f[j];
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < kKS; ++kk) {
      const float4 xv = *reinterpret_cast<const float4*>(&xs[kk][ty * 4]);
      const float4 wv = *reinterpret_cast<const float4*>(&ws[kk][tx * 4]);
      const float xa[4] = {xv.x, xv.y, xv.z, xv.w}, wa[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = __fmaf_rn(xa[i], wa[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t t = t0 + ty * 4 + i;
    if (t >= T) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = e0 + tx * 4 + j;
      if (e < E) logits[t * E + e] = bias ? __fadd_rn(acc[i][j], bias[e]) : acc[i][j];
    }
  }
}

// Softmax / top-k / renormalisation of one token's fp32 logits, the same operation sequence
// as the tensor-core epilogue: max, sum of exp(l - max) in expert order, reciprocal,
// probabilities into the insertion top-k, reciprocal of the sum of the k selected.
template <int KMAX>
__device__ __forceinline__ void route_row(const float* __restrict__ l, int E, int k, float (&tv)[KMAX],
                                          int (&ti)[KMAX], float& invs, float* __restrict__ probs) {
  float m = -INFINITY;
  for (int e = 0; e < E; ++e) m = fmaxf(m, l[e]);
  float sum = 0.0f;
  for (int e = 0; e < E; ++e) sum = __fadd_rn(sum, softmax_exp(__fsub_rn(l[e], m)));
  const float inv = __frcp_rn(sum);
#pragma unroll
  for (int j = 0; j < KMAX; ++j) { tv[j] = -INFINITY; ti[j] = 0; }
  for (int e = 0; e < E; ++e) {
    const float p = __fmul_rn(softmax_exp(__fsub_rn(l[e], m)), inv);
    if (probs) probs[e] = p;
    topk_insert<KMAX>(tv, ti, p, e);
  }
  float ssum = 0.0f;
#pragma unroll
  for (int j = 0; j < KMAX; ++j)
    if (j < k) ssum = __fadd_rn(ssum, tv[j]);
  invs = __frcp_rn(ssum);
}

template <int KMAX>
__global__ void __launch_bounds__(kSmallTokens) router_small_route_kernel(const float* __restrict__ logits, int T,
                                                                           int E, int k, RouterArgs a) {
  __shared__ int32_t sids[kSmallTokens * 16];
  __shared__ int32_t scnt[kMaxExperts];
  __shared__ int32_t snext[kMaxExperts];
  const int t = threadIdx.x;
  for (int e = t; e < E; e += blockDim.x) scnt[e] = 0;
  if (t < T) {
    float tv[KMAX], invs;
    int ti[KMAX];
    route_row<KMAX>(logits + (int64_t)t * E, E, k, tv, ti, invs, a.probs ? a.probs + (int64_t)t * E : nullptr);
#pragma unroll
    for (int j = 0; j < KMAX; ++j) {
      if (j < k) {
        const float wj = __fmul_rn(tv[j], invs);
        a.ids[t * k + j] = ti[j];
        if (a.weights) a.weights[t * k + j] = wj;
        if (a.weights_bf16) a.weights_bf16[t * k + j] = __float2bfloat16_rn(wj);
        sids[t * k + j] = ti[j];
      }
    }
  }
  if (!a.do_perm) return;
  __syncthreads();
  const int n = T * k;
  for (int f = t; f < n; f += blockDim.x) atomicAdd(&scnt[sids[f]], 1);
  __syncthreads();
  if (t == 0) {
    int run = 0;
    for (int e = 0; e < E; ++e) {
      a.counts[e] = scnt[e];
      a.offsets[e] = run;
      snext[e] = run;
      run += scnt[e];
    }
    a.offsets[E] = run;
  }
  __syncthreads();
  // warp 0 walks the flat indices in order, 32 at a time: equal experts in a chunk take
  // consecutive slots in lane order, so the result is ordered by (expert, token, slot)
  if (t < 32) {
    for (int c = 0; c < n; c += 32) {
      const int f = c + t;
      const int e = f < n ? sids[f] : E;
      const uint32_t peers = __match_any_sync(0xffffffffu, e);
      const int rank = __popc(peers & ((1u << t) - 1u));
      const int base = e < E ? snext[e] : 0;
      __syncwarp();
      if (f < n) {
        a.sorted_idx[base + rank] = f;
        if (a.positions) a.positions[f] = base + rank;
        if (rank == 0) snext[e] = base + __popc(peers);
      }
      __syncwarp();
    }
  }
}

// Any batch size from fp32 logits: one 128-token tile per CTA, one token per thread; with
// the permutation requested it writes the tile's per-expert counts and token bitmaps in the
// tensor-core kernel's format, for router_perm_kernel.
template <int KMAX>
__global__ void __launch_bounds__(kBM) router_route_logits_kernel(const float* __restrict__ logits, RouterArgs a) {
  __shared__ uint32_t bits[kMaxExperts * 4];
  const int row = threadIdx.x;
  const int tile = blockIdx.x;
  const int64_t t = (int64_t)tile * kBM + row;
  for (int i = row; i < a.E * 4; i += kBM) bits[i] = 0u;
  __syncthreads();
  if (t < a.T) {
    float tv[KMAX], invs;
    int ti[KMAX];
    route_row<KMAX>(logits + t * a.E, a.E, a.k, tv, ti, invs, a.probs ? a.probs + t * a.E : nullptr);
#pragma unroll
    for (int j = 0; j < KMAX; ++j) {
      if (j < a.k) {
        const float w = __fmul_rn(tv[j], invs);
        a.ids[t * a.k + j] = ti[j];
        if (a.weights) a.weights[t * a.k + j] = w;
        if (a.weights_bf16) a.weights_bf16[t * a.k + j] = __float2bfloat16_rn(w);
        if (a.do_perm) atomicOr(&bits[ti[j] * 4 + (row >> 5)], 1u << (row & 31));
      }
    }
  }
  if (!a.do_perm) return;
  __syncthreads();
  for (int e = row; e < a.E; e += kBM) {
    const uint4 bv = make_uint4(bits[e * 4], bits[e * 4 + 1], bits[e * 4 + 2], bits[e * 4 + 3]);
    a.tile_counts[(int64_t)tile * a.E + e] = __popc(bv.x) + __popc(bv.y) + __popc(bv.z) + __popc(bv.w);
    reinterpret_cast<uint4*>(a.tile_bits)[(int64_t)tile * a.E + e] = bv;
  }
}

// The permutation phase of the tensor-core kernel as a kernel of its own (launched after
// router_route_logits_kernel on the same stream, so no grid barrier is needed).
template <int KMAX>
__global__ void __launch_bounds__(kThreads) router_perm_kernel(RouterArgs a, int area_ints) {
  extern __shared__ int4 perm_area[];
  __shared__ int32_t total[kMaxExperts];
  __shared__ int32_t offs[kMaxExperts + 1];
  perm_phase<KMAX, kThreads>(a, reinterpret_cast<int32_t*>(perm_area), area_ints, total, offs);
}

// Tile height: 128 tokens, or fewer when there are fewer than 128 tokens per SM, so that
// every SM streams a share of x (a multiple of 8 rows: whole 128-byte swizzle atoms).
// The SM count is capped at kMaxGridTiles so the tile count stays bounded without
// querying the device (router_max_tiles, used for the workspace size).
constexpr int kMaxGridTiles = 256;

int router_tile_rows(int64_t T, int num_sms) {
  const int64_t s = num_sms < kMaxGridTiles ? num_sms : kMaxGridTiles;
  int64_t bm = (T + s - 1) / s;
  bm = (bm + 7) & ~int64_t(7);
  return (int)(bm > kBM ? kBM : (bm < 8 ? 8 : bm));
}

// Upper bound on ceil(T / router_tile_rows(T, any SM count)).
constexpr int64_t router_max_tiles(int64_t T) {
  const int64_t full = (T + kBM - 1) / kBM;
  const int64_t small = (T + 7) / 8 < kMaxGridTiles ? (T + 7) / 8 : kMaxGridTiles;
  return full > small ? full : small;
}

template <int KMAX>
int launch_router(const CUtensorMap& tm_x, const CUtensorMap& tm_w, const RouterArgs& a, int grid, size_t smem,
                  cudaStream_t stream) {
  auto fn = router_kernel<KMAX>;
  {
    const int st = set_max_dynamic_smem(reinterpret_cast<const void*>(fn), smem);
    if (st != LMOE_OK) return st;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = a.do_perm ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, fn, tm_x, tm_w, a));
}

// ---------------------------------------------------------------------------------------
// Router scratch in a fixed device array, for lmoe_fused_gate_topk_static: callers that may
// not allocate device memory at all (a custom allocator that owns every byte, a serving
// loop that forbids allocation after start-up) get the router without passing a workspace.
// Limits: at most kStaticMaxTokens tokens per call (num_experts <= 256 always fits).
// ---------------------------------------------------------------------------------------
constexpr int64_t kStaticMaxTokens = 16384;
constexpr size_t kStaticScratchBytes =
    ((256 + (size_t)router_max_tiles(kStaticMaxTokens) * kMaxExperts * sizeof(int32_t) + 255) & ~size_t(255)) +
    (size_t)router_max_tiles(kStaticMaxTokens) * kMaxExperts * 4 * sizeof(uint32_t);   // 1.25 MB + 256 B

static __device__ __align__(256) uint8_t g_router_scratch[kStaticScratchBytes];

constexpr int kMaxScratchDevices = 64;
std::mutex g_scratch_mu;
struct ScratchSlot {
  unsigned long long ctx_id;   // CUDA context the address belongs to (0 = none yet)
  void* ptr;
};
ScratchSlot g_scratch[kMaxScratchDevices] = {};

// Device address of g_router_scratch in the current device's current context.  The lookup
// runs on the first call in a context and again whenever the context changes (for example
// after cudaDeviceReset made a new primary context); other calls only read the cached
// pointer.
int router_scratch(void** out) {
  int dev = 0;
  LMOE_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxScratchDevices) return LMOE_ERR_UNSUPPORTED;
  unsigned long long ctx = 0;
  int st = current_context_id(&ctx);
  if (st != LMOE_OK) return st;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (ctx == 0 || g_scratch[dev].ctx_id != ctx || !g_scratch[dev].ptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_router_scratch);   // binds the primary context
    if (e != cudaSuccess) return cuda_status(e);
    if (!p) return LMOE_ERR_DEVICE;
    st = current_context_id(&ctx);
    if (st != LMOE_OK) return st;
    g_scratch[dev] = {ctx, p};
  }
  *out = g_scratch[dev].ptr;
  return LMOE_OK;
}

}  // namespace
}  // namespace lmoe

using namespace lmoe;

namespace {

bool dtype_ok(int dt) { return dt == LMOE_DTYPE_BF16 || dt == LMOE_DTYPE_F16 || dt == LMOE_DTYPE_F32; }

// Both operands bf16, or both fp16: the tensor-core kernel computes the logits.
bool tensor_core_logits(int x_dtype, int w_dtype) {
  return x_dtype == w_dtype && (x_dtype == LMOE_DTYPE_BF16 || x_dtype == LMOE_DTYPE_F16);
}

// Bytes of the per-tile count table and bitmaps (after the 256-byte header).
size_t router_tile_bytes(int64_t tiles, int E) {
  size_t bytes = 256 + (size_t)tiles * E * sizeof(int32_t);   // error word, grid barrier, counts
  bytes = (bytes + 255) & ~size_t(255);
  return bytes + (size_t)tiles * E * 4 * sizeof(uint32_t);
}

template <typename TX, typename TW>
int launch_logits(const void* hidden, const void* gate_weight, const float* bias, int64_t T, int d, int E,
                  float* logits, cudaStream_t stream) {
  const TX* x = static_cast<const TX*>(hidden);
  const TW* w = static_cast<const TW*>(gate_weight);
  if (T <= kSmallTokens) {
    router_small_logits_kernel<TX, TW><<<dim3((unsigned)T, (E + 7) / 8), 256, 0, stream>>>(x, w, bias, (int)T, d, E,
                                                                                            logits);
  } else if (E <= 16) {
    router_simt_logits_kernel<TX, TW, 128, 16>
        <<<dim3((unsigned)((T + 127) / 128), 1), 128, 0, stream>>>(x, w, bias, (int)T, d, E, logits);
  } else {
    router_simt_logits_kernel<TX, TW, 64, 64>
        <<<dim3((unsigned)((T + 63) / 64), (E + 63) / 64), 256, 0, stream>>>(x, w, bias, (int)T, d, E, logits);
  }
  return cuda_status(cudaGetLastError());
}

template <typename TX>
int launch_logits_w(const void* hidden, const void* gate_weight, int w_dtype, const float* bias, int64_t T, int d,
                    int E, float* logits, cudaStream_t stream) {
  if (w_dtype == LMOE_DTYPE_BF16) return launch_logits<TX, __nv_bfloat16>(hidden, gate_weight, bias, T, d, E, logits, stream);
  if (w_dtype == LMOE_DTYPE_F16) return launch_logits<TX, __half>(hidden, gate_weight, bias, T, d, E, logits, stream);
  return launch_logits<TX, float>(hidden, gate_weight, bias, T, d, E, logits, stream);
}

int launch_logits_any(const void* hidden, int x_dtype, const void* gate_weight, int w_dtype, const float* bias,
                      int64_t T, int d, int E, float* logits, cudaStream_t stream) {
  if (x_dtype == LMOE_DTYPE_BF16)
    return launch_logits_w<__nv_bfloat16>(hidden, gate_weight, w_dtype, bias, T, d, E, logits, stream);
  if (x_dtype == LMOE_DTYPE_F16) return launch_logits_w<__half>(hidden, gate_weight, w_dtype, bias, T, d, E, logits, stream);
  return launch_logits_w<float>(hidden, gate_weight, w_dtype, bias, T, d, E, logits, stream);
}

template <int KMAX>
int launch_route_from_logits(const float* lg, RouterArgs a, int num_sms, cudaStream_t stream) {
  if (a.T <= kSmallTokens) {
    router_small_route_kernel<KMAX><<<1, kSmallTokens, 0, stream>>>(lg, a.T, a.E, a.k, a);
    return cuda_status(cudaGetLastError());
  }
  router_route_logits_kernel<KMAX><<<a.num_tiles, kBM, 0, stream>>>(lg, a);
  LMOE_CUDA_TRY(cudaGetLastError());
  if (!a.do_perm) return LMOE_OK;
  // the permutation kernel's shared area: the owned tiles' prefixes and a chunk of count rows
  const int grid = a.num_tiles < num_sms ? a.num_tiles : num_sms;
  const int own_max = (a.num_tiles + grid - 1) / grid;
  const int pref_ints = (own_max * a.E + 3) & ~3;
  int chunk_tiles = (((64 * 1024) / 4) / a.E) & ~3;
  chunk_tiles = chunk_tiles < 4 ? 4 : chunk_tiles;
  const int area_ints = pref_ints + chunk_tiles * a.E;
  const size_t smem = (size_t)area_ints * sizeof(int32_t);
  auto fn = router_perm_kernel<KMAX>;
  const int st = set_max_dynamic_smem(reinterpret_cast<const void*>(fn), smem);
  if (st != LMOE_OK) return st;
  fn<<<grid, kThreads, smem, stream>>>(a, area_ints);
  return cuda_status(cudaGetLastError());
}

int route_from_logits(const float* lg, const RouterArgs& a, int num_sms, cudaStream_t stream) {
  if (a.k <= 2) return launch_route_from_logits<2>(lg, a, num_sms, stream);
  if (a.k <= 4) return launch_route_from_logits<4>(lg, a, num_sms, stream);
  if (a.k <= 8) return launch_route_from_logits<8>(lg, a, num_sms, stream);
  return launch_route_from_logits<16>(lg, a, num_sms, stream);
}

}  // namespace

extern "C" size_t lmoe_router_workspace_bytes_typed(int64_t num_tokens, int num_experts, int x_dtype, int w_dtype) {
  if (num_tokens < 0 || num_experts <= 0 || !dtype_ok(x_dtype) || !dtype_ok(w_dtype)) return 0;
  const size_t logits = (((size_t)num_tokens * num_experts * sizeof(float)) + 255) & ~size_t(255);
  if (num_tokens <= kSmallTokens) {
    // the fp32 logits after the 256-byte header
    const size_t small = 256 + logits;
    const size_t tiles = router_tile_bytes(router_max_tiles(num_tokens), num_experts);
    return tiles > small ? tiles : small;
  }
  if (tensor_core_logits(x_dtype, w_dtype)) return router_tile_bytes(router_max_tiles(num_tokens), num_experts);
  // CUDA-core logits: 128-token tiles, then the fp32 logits
  const size_t tiles = (router_tile_bytes((num_tokens + kBM - 1) / kBM, num_experts) + 255) & ~size_t(255);
  return tiles + logits;
}

extern "C" size_t lmoe_router_workspace_bytes(int64_t num_tokens, int num_experts) {
  return lmoe_router_workspace_bytes_typed(num_tokens, num_experts, LMOE_DTYPE_BF16, LMOE_DTYPE_BF16);
}

extern "C" int lmoe_fused_gate_topk_typed(const void* hidden, int x_dtype, const void* gate_weight, int w_dtype,
                                          const float* gate_bias, int64_t num_tokens, int hidden_size,
                                          int num_experts, int top_k, int32_t* ids, float* weights,
                                          void* weights_bf16, int32_t* counts, int32_t* offsets, int32_t* sorted_idx,
                                          int32_t* positions, float* logits, float* probs, void* workspace,
                                          size_t workspace_bytes, lmoe_stream_t stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  LMOE_ARG_CHECK(dtype_ok(x_dtype) && dtype_ok(w_dtype));
  LMOE_ARG_CHECK(num_tokens >= 0 && num_tokens <= (int64_t)INT32_MAX / 16);
  LMOE_ARG_CHECK(num_experts >= 1 && num_experts <= kMaxExperts);
  LMOE_ARG_CHECK(top_k >= 1 && top_k <= 16 && top_k <= num_experts);
  LMOE_ARG_CHECK(hidden_size >= kBK && hidden_size % kBK == 0);
  const bool do_perm = counts || offsets || sorted_idx;
  if (num_tokens == 0) {
    // ids / weights / sorted_idx are empty (possibly NULL); only counts and offsets exist
    if (do_perm) LMOE_ARG_CHECK(counts && offsets);
    if (do_perm) {
      LMOE_CUDA_TRY(cudaMemsetAsync(counts, 0, sizeof(int32_t) * num_experts, stream));
      LMOE_CUDA_TRY(cudaMemsetAsync(offsets, 0, sizeof(int32_t) * (num_experts + 1), stream));
    }
    return LMOE_OK;
  }
  LMOE_ARG_CHECK(ids != nullptr);
  if (do_perm) LMOE_ARG_CHECK(counts && offsets && sorted_idx);
  LMOE_ARG_CHECK(hidden && gate_weight && aligned16(hidden) && aligned16(gate_weight));
  const size_t need = lmoe_router_workspace_bytes_typed(num_tokens, num_experts, x_dtype, w_dtype);
  if (!workspace || workspace_bytes < need || !aligned16(workspace)) return LMOE_ERR_WORKSPACE;

  DeviceInfo dev;
  int st = get_device_info(&dev);
  if (st != LMOE_OK) return st;
  if (dev.cc_major != 10) return LMOE_ERR_DEVICE;

  const int E = num_experts;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (num_tokens <= kSmallTokens || !tensor_core_logits(x_dtype, w_dtype)) {
    // CUDA-core logits into the caller's buffer or the workspace, then routing from them
    LMOE_CUDA_TRY(cudaMemsetAsync(ws, 0, 256, stream));
    RouterArgs a = {};
    a.ids = ids;
    a.weights = weights;
    a.weights_bf16 = static_cast<__nv_bfloat16*>(weights_bf16);
    a.counts = counts;
    a.offsets = offsets;
    a.sorted_idx = sorted_idx;
    a.positions = do_perm ? positions : nullptr;
    a.probs = probs;
    a.do_perm = do_perm ? 1 : 0;
    a.err = reinterpret_cast<uint32_t*>(ws);
    a.T = (int)num_tokens;
    a.d = hidden_size;
    a.E = E;
    a.k = top_k;
    a.bm = kBM;
    a.num_tiles = (int)((num_tokens + kBM - 1) / kBM);
    float* lg = logits;
    if (!lg) {
      const size_t off = num_tokens <= kSmallTokens
                             ? 256
                             : (router_tile_bytes(a.num_tiles, E) + 255) & ~size_t(255);
      lg = reinterpret_cast<float*>(ws + off);
    }
    if (num_tokens > kSmallTokens) {
      a.tile_counts = reinterpret_cast<int32_t*>(ws + 256);
      size_t tb_off = 256 + (size_t)a.num_tiles * E * sizeof(int32_t);
      tb_off = (tb_off + 255) & ~size_t(255);
      a.tile_bits = reinterpret_cast<uint32_t*>(ws + tb_off);
    }
    st = launch_logits_any(hidden, x_dtype, gate_weight, w_dtype, gate_bias, num_tokens, hidden_size, E, lg, stream);
    if (st != LMOE_OK) return st;
    return route_from_logits(lg, a, dev.num_sms, stream);
  }
  const int Epad = ((E + 15) / 16) * 16;
  const int bm = router_tile_rows(num_tokens, dev.num_sms);
  const int num_tiles = (int)((num_tokens + bm - 1) / bm);
  const uint32_t w_box_bytes = (uint32_t)Epad * kBK * 2;           // multiple of 2048
  const uint32_t stage_bytes = kBoxes * (kBM * kBK * 2 + w_box_bytes);
  // header, then (more than one 16-column chunk of experts) the owner / helper exchange:
  // max [2][128], 1/sum [128], partial top-k values and ids [KMAX][128] each
  const int kmax = top_k <= 2 ? 2 : top_k <= 4 ? 4 : top_k <= 8 ? 8 : 16;
  const size_t xchg = Epad > 16 ? (size_t)(3 + 2 * kmax) * kBM * 4 : 0;
  const size_t hdr = (sizeof(RouterHdr) + xchg + 1023) & ~size_t(1023);
  int stages = (int)((dev.max_smem_optin - hdr - 1024) / stage_bytes);
  stages = stages > kMaxStages ? kMaxStages : stages;
  if (stages < 2) return LMOE_ERR_UNSUPPORTED;
  const size_t smem = 1024 + (size_t)stages * stage_bytes + sizeof(RouterHdr) + xchg;
  uint32_t tmem_cols = 32;
  while (tmem_cols < (uint32_t)(2 * Epad)) tmem_cols <<= 1;
  const int grid = num_tiles < dev.num_sms ? num_tiles : dev.num_sms;
  if (do_perm) {
    // the stage area holds the owned tiles' prefixes and a chunk of at least 4 count rows
    const size_t own_max = (size_t)((num_tiles + grid - 1) / grid);
    const size_t pref_ints = (own_max * E + 3) & ~size_t(3);
    if ((pref_ints + 4 * (size_t)E) * sizeof(int32_t) > (size_t)stages * stage_bytes) return LMOE_ERR_UNSUPPORTED;
  }

  LMOE_CUDA_TRY(cudaMemsetAsync(ws, 0, 256, stream));
  RouterArgs a = {};
  a.bias = gate_bias;
  a.ids = ids;
  a.weights = weights;
  a.weights_bf16 = static_cast<__nv_bfloat16*>(weights_bf16);
  a.logits = logits;
  a.probs = probs;
  a.counts = counts;
  a.offsets = offsets;
  a.sorted_idx = sorted_idx;
  a.positions = do_perm ? positions : nullptr;
  a.err = reinterpret_cast<uint32_t*>(ws);
  a.grid_sync = reinterpret_cast<uint32_t*>(ws) + 1;
  a.tile_counts = reinterpret_cast<int32_t*>(ws + 256);
  size_t tb_off = 256 + (size_t)num_tiles * E * sizeof(int32_t);
  tb_off = (tb_off + 255) & ~size_t(255);
  a.tile_bits = reinterpret_cast<uint32_t*>(ws + tb_off);
  a.T = (int)num_tokens;
  a.d = hidden_size;
  a.E = E;
  a.Epad = Epad;
  a.k = top_k;
  a.bm = bm;
  a.num_tiles = num_tiles;
  a.stages = stages;
  a.stage_bytes = stage_bytes;
  a.w_box_bytes = w_box_bytes;
  a.tmem_cols = tmem_cols;
  a.do_perm = do_perm ? 1 : 0;

  a.ab_f16 = x_dtype == LMOE_DTYPE_F16 ? 1 : 0;

  const CUtensorMapDataType tdt = a.ab_f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap tm_x, tm_w;
  st = encode_tmap_2d(&tm_x, hidden, tdt, 2, (uint64_t)num_tokens, (uint64_t)hidden_size, (uint64_t)hidden_size * 2,
                      (uint32_t)bm, kBK, true);
  if (st != LMOE_OK) return st;
  st = encode_tmap_2d(&tm_w, gate_weight, tdt, 2, (uint64_t)E, (uint64_t)hidden_size, (uint64_t)hidden_size * 2,
                      (uint32_t)Epad, kBK, true);
  if (st != LMOE_OK) return st;

  if (top_k <= 2) return launch_router<2>(tm_x, tm_w, a, grid, smem, stream);
  if (top_k <= 4) return launch_router<4>(tm_x, tm_w, a, grid, smem, stream);
  if (top_k <= 8) return launch_router<8>(tm_x, tm_w, a, grid, smem, stream);
  return launch_router<16>(tm_x, tm_w, a, grid, smem, stream);
}

extern "C" int lmoe_fused_gate_topk(const void* hidden, const void* gate_weight, const float* gate_bias,
                                    int64_t num_tokens, int hidden_size, int num_experts, int top_k,
                                    int32_t* ids, float* weights, void* weights_bf16, int32_t* counts,
                                    int32_t* offsets, int32_t* sorted_idx, int32_t* positions, float* logits,
                                    void* workspace, size_t workspace_bytes, lmoe_stream_t stream) {
  return lmoe_fused_gate_topk_typed(hidden, LMOE_DTYPE_BF16, gate_weight, LMOE_DTYPE_BF16, gate_bias, num_tokens,
                                    hidden_size, num_experts, top_k, ids, weights, weights_bf16, counts, offsets,
                                    sorted_idx, positions, logits, nullptr, workspace, workspace_bytes, stream);
}

extern "C" int lmoe_fused_gate_topk_static(const void* hidden, const void* gate_weight, const float* gate_bias,
                                           int64_t num_tokens, int hidden_size, int num_experts, int top_k,
                                           int32_t* ids, float* weights, void* weights_bf16, int32_t* counts,
                                           int32_t* offsets, int32_t* sorted_idx, int32_t* positions,
                                           float* logits, lmoe_stream_t stream) {
  if (num_tokens > kStaticMaxTokens) return LMOE_ERR_WORKSPACE;   // beyond the fixed scratch
  static_assert(kStaticScratchBytes % 256 == 0, "scratch size");
  void* scratch = nullptr;
  const int st = router_scratch(&scratch);
  if (st != LMOE_OK) return st;
  // same kernel and checks as the workspace entry point; the scratch header (error word and
  // grid barrier) is cleared there on the stream before every launch
  return lmoe_fused_gate_topk(hidden, gate_weight, gate_bias, num_tokens, hidden_size, num_experts, top_k, ids,
                              weights, weights_bf16, counts, offsets, sorted_idx, positions, logits, scratch,
                              kStaticScratchBytes, stream);
}

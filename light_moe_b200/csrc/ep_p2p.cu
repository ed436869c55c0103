// ep_p2p.cu -- the expert-parallel exchange over peer memory (NVLink / NVSwitch): no NCCL
// and no host synchronisation on the data path.
//
// Every rank owns one "symmetric" buffer (same size and layout on all ranks, allocated here
// with cudaMalloc and mapped into the other ranks' processes through CUDA IPC handles):
//   flags  [3][ep] uint32   epoch flags written by the peers: counts, rows, returned rows
//   cnt    [ep][E] int32    every rank's routed-row counts per global expert
//   rows   [ep*Tc*k + S*Tc][d] bf16   rows for this rank's experts, expert-major (expert l:
//                                     source 0's rows, source 1's, ...), then the shared
//                                     experts' copies of this rank's own tokens at ep*Tc*k
//   meta   [ep*Tc*k + S*Tc] int32  for each routed row: (source rank << 24) | source slot
//                                   (t*k + j); for shared row u: (ep << 24) | u (set once)
//   ret    [Tc*k][d] bf16   this rank's own slots, each written back by the rank that ran it
// (Tc = capacity tokens per rank and step, the same on every rank.)
//
// One step, in stream order on every rank (epoch e = a device counter bumped by step 1):
//   1. exchange_counts  write this rank's counts[E] into every peer's cnt[me], raise their
//                       count flag; wait for every peer's; then every rank holds the same
//                       [ep][E] matrix and derives its segment offsets and, for each of its
//                       own sorted rows, the destination position in the owner's rows
//   2. dispatch         the permutation and the send in one kernel: sorted row i (token t,
//                       choice j, expert e) is copied from x[t] straight into the owning
//                       rank's rows at its final expert-major position (16-byte stores over
//                       NVLink), with its meta; the last CTA raises the peers' row flags
//   3. wait(rows)       then the grouped GEMMs run on the local rows buffer
//   4. send_back        every routed output row goes straight into its source rank's ret
//                       slot; the last CTA raises the sources' return flags
//   5. wait(returns)    then the weighted combine reads ret locally
// Buffers are single.  A peer writes this rank's count matrix, rows and meta for step e+1
// only after finishing its step e, which needed this rank's returned rows of step e, sent
// after this rank's last reads of them (counts exchange, down GEMM, send-back).  It writes
// this rank's ret region for step e+1 only after receiving this rank's step-e+1 rows, which
// this rank dispatches after its step-e combine.  So no data is overwritten while it is
// read.  Flags only grow (epochs), so a wait is "flag >= epoch".
//
// Reference: the exchange of python/light_moe/distributed/expert_parallel.py:186-244 and
// :275-319 (padded NCCL all-to-alls of whole token sets); here only routed rows move, once
// each way, and the permutation / un-permutation ride on the copies.
// Every wait is bounded (kWaitBudgetNs): a missing peer leaves an error code in the state's
// error word and the kernel returns; no fault, trap or endless spin.
#include <cuda_bf16.h>

#include <cstring>

#include "grouped_gemm.h"
#include "host_util.h"
#include "ptx.cuh"

namespace lmoe {
namespace {

constexpr int kP2PMaxRanks = 64;
constexpr int kP2PMaxExperts = 256;
constexpr uint32_t kSite = 0x600u;
enum P2PFlag : int { kFlagCounts = 0, kFlagRows = 1, kFlagReturns = 2 };

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct P2PLayout {
  size_t flags, cnt, rows, meta, ret, total;
  int64_t routed_rows;   // ep * Tc * k: start of the shared experts' rows
};

P2PLayout p2p_layout(int ep, int E, int64_t Tc, int k, int S, int d) {
  P2PLayout L{};
  size_t p = 0;
  L.flags = p; p = align256(p + sizeof(uint32_t) * 3 * ep);
  L.cnt = p; p = align256(p + sizeof(int32_t) * (size_t)ep * E);
  L.routed_rows = (int64_t)ep * Tc * k;
  L.rows = p; p = align256(p + sizeof(uint16_t) * (size_t)(L.routed_rows + (int64_t)S * Tc) * d);
  L.meta = p; p = align256(p + sizeof(int32_t) * (size_t)(L.routed_rows + (int64_t)S * Tc));
  L.ret = p; p = align256(p + sizeof(uint16_t) * (size_t)(Tc * k) * d);
  L.total = p;
  return L;
}

// Arguments shared by the kernels.  peers[r] = rank r's buffer as mapped in this process
// (peers[me] is the local allocation).  state: [0] epoch, [1] error word, [2] / [3] CTA
// completion counters of dispatch / send_back.
struct P2PArgs {
  const uint64_t* peers;
  int me, ep, E, epr, k, S, d;
  int64_t Tc, T;
  size_t off_flags, off_cnt, off_rows, off_meta, off_ret;
  int64_t routed_rows;
  int32_t* state;
};

__device__ __forceinline__ uint8_t* peer_base(const P2PArgs& a, int r) {
  return reinterpret_cast<uint8_t*>(a.peers[r]);
}

__device__ __forceinline__ uint32_t* flag_ptr(const P2PArgs& a, int r, int kind, int src) {
  return reinterpret_cast<uint32_t*>(peer_base(a, r) + a.off_flags) + kind * a.ep + src;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One warp copies one row of `vec` 16-byte words, eight loads per lane in flight before
// their stores (a load-then-store chain per word would pay a memory round trip each).
__device__ __forceinline__ void copy_row(uint4* __restrict__ dst, const uint4* __restrict__ src, int vec,
                                         int lane) {
  constexpr int kU = 8;
  for (int c0 = lane; c0 < vec; c0 += 32 * kU) {
    uint4 v[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u)
      if (c0 + 32 * u < vec) v[u] = __ldg(src + c0 + 32 * u);
#pragma unroll
    for (int u = 0; u < kU; ++u)
      if (c0 + 32 * u < vec) dst[c0 + 32 * u] = v[u];
  }
}

// Threads 0..ep-1 each wait for the flag of one source rank to reach the epoch (bounded);
// every thread of the CTA must call it.  Returns false (error recorded) when a flag never
// arrived.
__device__ bool wait_flags(const P2PArgs& a, int kind, uint32_t epoch, uint32_t site) {
  __shared__ int s_fail;
  if (threadIdx.x == 0) s_fail = 0;
  __syncthreads();
  if ((int)threadIdx.x < a.ep) {
    const uint32_t* f = flag_ptr(a, a.me, kind, threadIdx.x);
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while ((int32_t)(ld_acquire_sys(f) - epoch) < 0) {
      if (((++spins) & 63u) == 0u && globaltimer_ns() - t0 > kWaitBudgetNs) {
        report_error(reinterpret_cast<uint32_t*>(a.state + 1), kErrTimeout, site);
        atomicExch(&s_fail, 1);
        break;
      }
    }
  }
  __syncthreads();
  return s_fail == 0;
}

// Raise flag `kind` of this rank in every peer, after every CTA of the grid finished its
// stores (the last CTA to finish does it); counter is the grid's completion counter.
__device__ void signal_when_grid_done(const P2PArgs& a, int kind, int32_t* counter, uint32_t epoch) {
  __threadfence_system();   // this thread's peer stores before the CTA's arrival
  __syncthreads();
  if (threadIdx.x == 0) {
    const int32_t done = atomicAdd(counter, 1);
    if (done == (int32_t)gridDim.x - 1) {
      __threadfence_system();
      for (int r = 0; r < a.ep; ++r) st_release_sys(flag_ptr(a, r, kind, a.me), epoch);
      *counter = 0;   // the next launch starts from zero (stream order)
    }
  }
}


// Step 1 (one CTA): bump the epoch, publish this rank's counts to every peer, wait for all
// of theirs, then derive this rank's segment offsets [epr + 2 + S] (experts, the hole up to
// the shared rows, shared segments of T rows) and, per global expert e, the position in the
// owner's rows where this rank's rows for e start (-1: skip the step, counts inconsistent).
__global__ void __launch_bounds__(256) exchange_counts_kernel(P2PArgs a, const int32_t* __restrict__ counts,
                                                              int32_t* __restrict__ seg_offsets,
                                                              int32_t* __restrict__ dst_base) {
  __shared__ uint32_t s_epoch;
  __shared__ int s_bad;
  const int tid = threadIdx.x;
  if (tid == 0) {
    s_epoch = (uint32_t)a.state[0] + 1u;
    a.state[0] = (int32_t)s_epoch;
    s_bad = 0;
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  for (int i = tid; i < a.ep * a.E; i += blockDim.x) {
    const int r = i / a.E, e = i - r * a.E;
    reinterpret_cast<int32_t*>(peer_base(a, r) + a.off_cnt)[a.me * a.E + e] = counts[e];
  }
  if (tid < a.ep * a.E) __threadfence_system();   // only the threads that stored to peers
  __syncthreads();
  if (tid == 0)
    for (int r = 0; r < a.ep; ++r) st_release_sys(flag_ptr(a, r, kFlagCounts, a.me), epoch);
  const bool ok = wait_flags(a, kFlagCounts, epoch, kSite + 1);
  const int32_t* cnt = reinterpret_cast<const int32_t*>(peer_base(a, a.me) + a.off_cnt);   // [ep][E]
  // every rank checks the same matrix, so all of them skip a bad step alike
  if (ok) {
    for (int s = tid; s < a.ep; s += blockDim.x) {
      int64_t tot = 0;
      for (int e = 0; e < a.E; ++e) {
        const int32_t c = cnt[s * a.E + e];
        if (c < 0) s_bad = 1;
        tot += c;
      }
      if (tot > a.Tc * a.k) s_bad = 1;   // a source never sends more than Tc * k rows
    }
  }
  __syncthreads();
  const bool good = ok && !s_bad;
  if (ok && !good && tid == 0) report_error(reinterpret_cast<uint32_t*>(a.state + 1), kErrBadArg, kSite + 2);
  if (tid == 0) {
    int64_t acc = 0;
    seg_offsets[0] = 0;
    for (int l = 0; l < a.epr; ++l) {
      const int e = a.me * a.epr + l;
      if (good)
        for (int s = 0; s < a.ep; ++s) acc += cnt[s * a.E + e];
      seg_offsets[l + 1] = (int32_t)acc;
    }
    seg_offsets[a.epr + 1] = (int32_t)a.routed_rows;   // hole: the unused routed rows
    for (int s = 0; s < a.S; ++s) seg_offsets[a.epr + 2 + s] = (int32_t)(a.routed_rows + (int64_t)(s + 1) * a.T);
  }
  for (int e = tid; e < a.E; e += blockDim.x) {
    const int r = e / a.epr;
    int64_t base = 0;
    for (int e2 = r * a.epr; e2 < e; ++e2)
      for (int s = 0; s < a.ep; ++s) base += cnt[s * a.E + e2];
    for (int s = 0; s < a.me; ++s) base += cnt[s * a.E + e];
    dst_base[e] = good ? (int32_t)base : -1;
  }
}

// Step 2: sorted row i < T*k (token t = f / k, choice f % k with f = sorted_idx[i], expert
// e = ids[f]) goes to rank e / epr at dst_base[e] + (i - offsets[e]); rows T*k + s*T + t copy
// token t into this rank's own shared-expert rows.  One warp per row, 16-byte copies.
__global__ void __launch_bounds__(256) dispatch_kernel(P2PArgs a, const uint4* __restrict__ x,
                                                       const int32_t* __restrict__ sorted_idx,
                                                       const int32_t* __restrict__ ids,
                                                       const int32_t* __restrict__ offsets,
                                                       const int32_t* __restrict__ dst_base) {
  const uint32_t epoch = (uint32_t)a.state[0];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int vec = a.d / 8;
  const int64_t routed = a.T * a.k;
  const int64_t total = routed + (int64_t)a.S * a.T;
  for (int64_t i = (int64_t)blockIdx.x * 8 + warp; i < total; i += (int64_t)gridDim.x * 8) {
    const uint4* src;
    uint4* dst;
    if (i < routed) {
      const int32_t f = sorted_idx[i];
      if (f < 0 || f >= routed) { if (lane == 0) report_error(reinterpret_cast<uint32_t*>(a.state + 1), kErrBadArg, kSite + 3); continue; }
      const int e = ids[f];
      if (e < 0 || e >= a.E) { if (lane == 0) report_error(reinterpret_cast<uint32_t*>(a.state + 1), kErrBadArg, kSite + 3); continue; }
      const int32_t base = dst_base[e];
      if (base < 0) continue;   // step skipped (reported by exchange_counts)
      const int64_t pos = base + (i - offsets[e]);
      if (pos < 0 || pos >= a.routed_rows) { if (lane == 0) report_error(reinterpret_cast<uint32_t*>(a.state + 1), kErrBadArg, kSite + 4); continue; }
      uint8_t* pb = peer_base(a, e / a.epr);
      src = x + (int64_t)(f / a.k) * vec;
      dst = reinterpret_cast<uint4*>(pb + a.off_rows) + pos * vec;
      if (lane == 0) reinterpret_cast<int32_t*>(pb + a.off_meta)[pos] = (a.me << 24) | f;
    } else {
      const int64_t u = i - routed;
      const int64_t s = u / a.T, t = u - s * a.T;
      src = x + t * vec;
      dst = reinterpret_cast<uint4*>(peer_base(a, a.me) + a.off_rows) + (a.routed_rows + s * a.T + t) * vec;
    }
    copy_row(dst, src, vec, lane);
  }
  signal_when_grid_done(a, kFlagRows, a.state + 2, epoch);
}

// Step 4: routed output row q (q < seg_offsets[epr]) goes back to its source's ret slot.
__global__ void __launch_bounds__(256) send_back_kernel(P2PArgs a, const uint4* __restrict__ out,
                                                        const int32_t* __restrict__ seg_offsets) {
  const uint32_t epoch = (uint32_t)a.state[0];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int vec = a.d / 8;
  const int64_t R = seg_offsets[a.epr];
  const int32_t* meta = reinterpret_cast<const int32_t*>(peer_base(a, a.me) + a.off_meta);
  for (int64_t q = (int64_t)blockIdx.x * 8 + warp; q < R && q < a.routed_rows; q += (int64_t)gridDim.x * 8) {
    const int32_t m = meta[q];
    const int s = (int)((uint32_t)m >> 24);
    const int32_t slot = m & 0xffffff;
    if (s >= a.ep || slot >= a.Tc * a.k) { if (lane == 0) report_error(reinterpret_cast<uint32_t*>(a.state + 1), kErrBadArg, kSite + 5); continue; }
    uint4* dst = reinterpret_cast<uint4*>(peer_base(a, s) + a.off_ret) + (int64_t)slot * vec;
    const uint4* src = out + q * vec;
    copy_row(dst, src, vec, lane);
  }
  signal_when_grid_done(a, kFlagReturns, a.state + 3, epoch);
}

// Once: the shared rows' destinations, (ep << 24) | u for shared row u (buffer ep of the
// down GEMM's destination table is this rank's shared-expert output).
__global__ void init_meta_kernel(P2PArgs a) {
  int32_t* meta = reinterpret_cast<int32_t*>(peer_base(a, a.me) + a.off_meta) + a.routed_rows;
  const int64_t n = (int64_t)a.S * a.Tc;
  for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < n; u += (int64_t)gridDim.x * blockDim.x)
    meta[u] = (a.ep << 24) | (int32_t)u;
}

// After the down GEMM wrote its routed rows straight into the sources' ret regions: raise
// the sources' return flags (the GEMM's stores are complete at its kernel boundary).
__global__ void signal_returns_kernel(P2PArgs a) {
  if (threadIdx.x == 0) {
    __threadfence_system();
    const uint32_t epoch = (uint32_t)a.state[0];
    for (int r = 0; r < a.ep; ++r) st_release_sys(flag_ptr(a, r, kFlagReturns, a.me), epoch);
  }
}

// Steps 3 and 5: wait until every peer raised flag `kind` for this step.
__global__ void __launch_bounds__(64) wait_kernel(P2PArgs a, int kind) {
  wait_flags(a, kind, (uint32_t)a.state[0], kSite + 8 + kind);
}

}  // namespace
}  // namespace lmoe

using namespace lmoe;

// ---------------------------------------------------------------------------------- C ABI

namespace {

int p2p_args(const uint64_t* peers, int me, int ep, int num_experts, int64_t capacity_tokens, int top_k,
             int num_shared, int hidden, int64_t num_tokens, int32_t* state, P2PArgs* a) {
  LMOE_ARG_CHECK(peers && state);
  LMOE_ARG_CHECK(ep >= 1 && ep <= kP2PMaxRanks && me >= 0 && me < ep);
  LMOE_ARG_CHECK(num_experts >= 1 && num_experts <= kP2PMaxExperts && num_experts % ep == 0);
  LMOE_ARG_CHECK(top_k >= 1 && top_k <= num_experts && num_shared >= 0 && hidden >= 8 && hidden % 8 == 0);
  LMOE_ARG_CHECK(capacity_tokens >= 1 && num_tokens >= 0 && num_tokens <= capacity_tokens);
  // meta packs (source rank << 24) | slot; segment offsets are int32
  LMOE_ARG_CHECK(capacity_tokens * top_k < (1 << 24));
  const P2PLayout L = p2p_layout(ep, num_experts, capacity_tokens, top_k, num_shared, hidden);
  LMOE_ARG_CHECK(L.routed_rows + (int64_t)num_shared * capacity_tokens <= INT32_MAX);
  a->peers = peers;
  a->me = me;
  a->ep = ep;
  a->E = num_experts;
  a->epr = num_experts / ep;
  a->k = top_k;
  a->S = num_shared;
  a->d = hidden;
  a->Tc = capacity_tokens;
  a->T = num_tokens;
  a->off_flags = L.flags;
  a->off_cnt = L.cnt;
  a->off_rows = L.rows;
  a->off_meta = L.meta;
  a->off_ret = L.ret;
  a->routed_rows = L.routed_rows;
  a->state = state;
  return LMOE_OK;
}

int copy_grid(int64_t rows) {
  DeviceInfo dev;
  const int sms = get_device_info(&dev) == LMOE_OK ? dev.num_sms : 148;
  const int64_t want = (rows + 7) / 8;   // eight rows (warps) per CTA
  return (int)(want < 1 ? 1 : (want > 4 * sms ? 4 * sms : want));
}

}  // namespace

extern "C" size_t lmoe_p2p_buffer_bytes(int ep, int num_experts, int64_t capacity_tokens, int top_k, int num_shared,
                                        int hidden) {
  if (ep < 1 || num_experts < 1 || capacity_tokens < 1 || top_k < 1 || num_shared < 0 || hidden < 1) return 0;
  return p2p_layout(ep, num_experts, capacity_tokens, top_k, num_shared, hidden).total;
}

extern "C" int lmoe_p2p_buffer_offsets(int ep, int num_experts, int64_t capacity_tokens, int top_k, int num_shared,
                                       int hidden, size_t* rows_offset, size_t* ret_offset) {
  LMOE_ARG_CHECK(ep >= 1 && num_experts >= 1 && capacity_tokens >= 1 && top_k >= 1 && num_shared >= 0 && hidden >= 1);
  LMOE_ARG_CHECK(rows_offset && ret_offset);
  const P2PLayout L = p2p_layout(ep, num_experts, capacity_tokens, top_k, num_shared, hidden);
  *rows_offset = L.rows;
  *ret_offset = L.ret;
  return LMOE_OK;
}

extern "C" int lmoe_p2p_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  LMOE_ARG_CHECK(bytes > 0 && ptr && ipc_handle);
  void* p = nullptr;
  LMOE_CUDA_TRY(cudaMalloc(&p, bytes));
  cudaError_t e = cudaMemset(p, 0, bytes);   // flags start at epoch 0
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_status(e);
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return LMOE_OK;
}

extern "C" int lmoe_p2p_open(const void* ipc_handle, void** ptr) {
  LMOE_ARG_CHECK(ipc_handle && ptr);
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  LMOE_CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return LMOE_OK;
}

extern "C" int lmoe_p2p_close(void* ptr) {
  LMOE_ARG_CHECK(ptr);
  return cuda_status(cudaIpcCloseMemHandle(ptr));
}

extern "C" int lmoe_p2p_free(void* ptr) {
  LMOE_ARG_CHECK(ptr);
  return cuda_status(cudaFree(ptr));
}

extern "C" int lmoe_p2p_exchange_counts(const uint64_t* peers, int me, int ep, int num_experts,
                                        int64_t capacity_tokens, int top_k, int num_shared, int hidden,
                                        int64_t num_tokens, int32_t* state, const int32_t* counts,
                                        int32_t* seg_offsets, int32_t* dst_base, lmoe_stream_t stream_) {
  P2PArgs a;
  const int st = p2p_args(peers, me, ep, num_experts, capacity_tokens, top_k, num_shared, hidden, num_tokens, state,
                          &a);
  if (st != LMOE_OK) return st;
  LMOE_ARG_CHECK(counts && seg_offsets && dst_base);
  exchange_counts_kernel<<<1, 256, 0, reinterpret_cast<cudaStream_t>(stream_)>>>(a, counts, seg_offsets, dst_base);
  return cuda_status(cudaGetLastError());
}

extern "C" int lmoe_p2p_dispatch(const uint64_t* peers, int me, int ep, int num_experts, int64_t capacity_tokens,
                                 int top_k, int num_shared, int hidden, int64_t num_tokens, int32_t* state,
                                 const void* x, const int32_t* sorted_idx, const int32_t* ids,
                                 const int32_t* offsets, const int32_t* dst_base, lmoe_stream_t stream_) {
  P2PArgs a;
  const int st = p2p_args(peers, me, ep, num_experts, capacity_tokens, top_k, num_shared, hidden, num_tokens, state,
                          &a);
  if (st != LMOE_OK) return st;
  LMOE_ARG_CHECK(dst_base && (num_tokens == 0 || (x && aligned16(x) && sorted_idx && ids && offsets)));
  const int grid = copy_grid(num_tokens * (top_k + num_shared));
  dispatch_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream_)>>>(
      a, static_cast<const uint4*>(x), sorted_idx, ids, offsets, dst_base);
  return cuda_status(cudaGetLastError());
}

extern "C" int lmoe_p2p_wait(const uint64_t* peers, int me, int ep, int num_experts, int64_t capacity_tokens,
                             int top_k, int num_shared, int hidden, int64_t num_tokens, int32_t* state, int which,
                             lmoe_stream_t stream_) {
  P2PArgs a;
  const int st = p2p_args(peers, me, ep, num_experts, capacity_tokens, top_k, num_shared, hidden, num_tokens, state,
                          &a);
  if (st != LMOE_OK) return st;
  LMOE_ARG_CHECK(which == kFlagRows || which == kFlagReturns);
  wait_kernel<<<1, 64, 0, reinterpret_cast<cudaStream_t>(stream_)>>>(a, which);
  return cuda_status(cudaGetLastError());
}

extern "C" int lmoe_p2p_send_back(const uint64_t* peers, int me, int ep, int num_experts, int64_t capacity_tokens,
                                  int top_k, int num_shared, int hidden, int64_t num_tokens, int32_t* state,
                                  const void* out, const int32_t* seg_offsets, lmoe_stream_t stream_) {
  P2PArgs a;
  const int st = p2p_args(peers, me, ep, num_experts, capacity_tokens, top_k, num_shared, hidden, num_tokens, state,
                          &a);
  if (st != LMOE_OK) return st;
  LMOE_ARG_CHECK(out && aligned16(out) && seg_offsets);
  const int grid = copy_grid(a.routed_rows);
  send_back_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream_)>>>(a, static_cast<const uint4*>(out),
                                                                               seg_offsets);
  return cuda_status(cudaGetLastError());
}

extern "C" int lmoe_p2p_init(const uint64_t* peers, int me, int ep, int num_experts, int64_t capacity_tokens,
                             int top_k, int num_shared, int hidden, int32_t* state, lmoe_stream_t stream_) {
  P2PArgs a;
  const int st = p2p_args(peers, me, ep, num_experts, capacity_tokens, top_k, num_shared, hidden, 0, state, &a);
  if (st != LMOE_OK) return st;
  if (num_shared == 0) return LMOE_OK;
  const int64_t n = (int64_t)num_shared * capacity_tokens;
  const int grid = (int)((n + 255) / 256 < 1024 ? (n + 255) / 256 : 1024);
  init_meta_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream_)>>>(a);
  return cuda_status(cudaGetLastError());
}

extern "C" int lmoe_p2p_down_gemm(const uint64_t* peers, int me, int ep, int num_experts, int64_t capacity_tokens,
                                  int top_k, int num_shared, int hidden, int64_t num_tokens, int32_t* state,
                                  void* buffer, const void* h, int ffn_size, const uint8_t* w2_packed, int group_size,
                                  const int32_t* seg_offsets, const int32_t* seg_expert, int num_segments,
                                  int num_weight_matrices, const uint64_t* dest_bases, lmoe_stream_t stream_) {
  P2PArgs a;
  const int st = p2p_args(peers, me, ep, num_experts, capacity_tokens, top_k, num_shared, hidden, num_tokens, state,
                          &a);
  if (st != LMOE_OK) return st;
  LMOE_ARG_CHECK(buffer && h && aligned16(h) && w2_packed && aligned16(w2_packed) && seg_offsets && seg_expert &&
                 dest_bases);
  LMOE_ARG_CHECK(num_segments >= 1 && num_weight_matrices >= 1 && ffn_size > 0);
  const uint64_t own = reinterpret_cast<uint64_t>(buffer);   // this rank's buffer (= peers[me])
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  GemmProblem p;
  p.x = h;
  p.ldx = ffn_size;
  p.total_rows = a.routed_rows + (int64_t)num_shared * capacity_tokens;
  p.K = ffn_size;
  p.offsets = seg_offsets;
  p.num_experts = num_segments;
  p.seg_expert = seg_expert;
  p.num_w = num_weight_matrices;
  p.wq = w2_packed;
  p.group_size = group_size;
  p.N = hidden;
  p.mode = kModeScatter;
  p.out = reinterpret_cast<void*>(own + a.off_ret);   // alignment reference; rows go through dest_bases
  p.ldo = hidden;
  p.dest = reinterpret_cast<const int32_t*>(own + a.off_meta);
  p.dest_bases = dest_bases;
  p.dest_count = ep + 1;
  p.err = reinterpret_cast<uint32_t*>(state + 1);
  p.max_rows_per_expert_hint = 0;
  const int gs = run_grouped_gemm(p, stream);
  if (gs != LMOE_OK) return gs;
  signal_returns_kernel<<<1, 32, 0, stream>>>(a);
  return cuda_status(cudaGetLastError());
}

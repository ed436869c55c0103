// dispatch.cu -- index plans of the fixed-capacity expert-parallel exchange (decode steps).
//
// Every rank sends every rank a block of C rows (its rows routed to that rank, then padding),
// so the all-to-alls have equal, host-known splits and nothing is copied to the host.  Two
// small kernels turn the per-(rank, expert) counts into the indices the row gathers, the
// grouped GEMMs and the weighted combine need, on the device:
//
//   send plan (before the exchange; counts of this rank's rows per destination expert):
//     send_index[r * C + c]   the sorted row (router order: expert, token, slot) of slot c of
//                             the block for rank r, or 0 for padding (a valid row, never read
//                             back);
//     combine_pos[t * k + j]  the slot of the block that carries token t's j-th choice;
//   receive plan (after the counts' all-to-all; rows received per source rank and local
//   expert):
//     regroup[p]   the received row at expert-major position p: local expert 0's rows from
//                  source 0, 1, ..., then expert 1's, ..., then every source's padding;
//     restore[q]   its inverse (received row q -> expert-major position);
//     seg_offsets  [epr + 1 + S + 1]: the experts' segments, the padding hole, then S shared
//                  segments of T rows each (rows appended after the ep * C received ones).
//
// Reference: the reference pads every rank's tokens to equal splits and sends them to every
// rank (python/light_moe/distributed/expert_parallel.py:186-244); here only routed rows carry
// data.  Integer work only; results are exact.
#include "host_util.h"

namespace lmoe {
namespace {

constexpr int kPlanThreads = 512;
constexpr int kMaxPlanEntries = 3072;   // ep x (experts per rank + 1) entries of the receive plan
constexpr int kMaxPlanRanks = 1024;

__global__ void __launch_bounds__(kPlanThreads) send_plan_kernel(const int32_t* __restrict__ counts,
                                                                  const int32_t* __restrict__ sorted_idx,
                                                                  const int32_t* __restrict__ positions, int64_t T,
                                                                  int k, int ep, int epr, int64_t C,
                                                                  int32_t* __restrict__ send_index,
                                                                  int32_t* __restrict__ combine_pos) {
  __shared__ int32_t start[kMaxPlanRanks + 1];   // first sorted row of each destination rank
  __shared__ int32_t fill[kMaxPlanRanks];        // rows of each destination's block (<= C)
  if (threadIdx.x == 0) {
    int64_t acc = 0;
    for (int r = 0; r < ep; ++r) {
      int64_t cnt = 0;
      for (int e = 0; e < epr; ++e) cnt += max(counts[r * epr + e], 0);
      start[r] = (int32_t)acc;
      fill[r] = (int32_t)min(cnt, C);   // a block never takes more than C rows
      acc += cnt;
    }
    start[ep] = (int32_t)acc;
  }
  __syncthreads();
  const int64_t n_send = (int64_t)ep * C;
  for (int64_t i = threadIdx.x; i < n_send; i += blockDim.x) {
    const int r = (int)(i / C);
    const int64_t c = i - (int64_t)r * C;
    send_index[i] = c < fill[r] && start[r] + c < T * k ? sorted_idx[start[r] + c] : 0;
  }
  const int64_t n_rows = T * k;
  for (int64_t j = threadIdx.x; j < n_rows; j += blockDim.x) {
    const int32_t sr = positions[j];   // sorted row of (token, choice) j
    int r = 0;                         // its destination rank: start[r] <= sr < start[r + 1]
    while (r + 1 < ep && start[r + 1] <= sr) ++r;
    const int64_t c = min((int64_t)sr - start[r], C - 1);
    combine_pos[j] = (int32_t)((int64_t)r * C + c);
  }
}

__global__ void __launch_bounds__(kPlanThreads) receive_plan_kernel(const int32_t* __restrict__ recv_counts, int ep,
                                                                     int epr, int64_t C, int num_shared, int64_t T,
                                                                     int32_t* __restrict__ regroup,
                                                                     int32_t* __restrict__ restore,
                                                                     int32_t* __restrict__ seg_offsets) {
  // entries (expert e, source s) in expert-major order, e = epr is the padding of source s;
  // counts are clamped so every source's entries fill exactly its C rows
  __shared__ int32_t cnt[kMaxPlanEntries];         // rows of each entry
  __shared__ int32_t dst_start[kMaxPlanEntries + 1];
  __shared__ int32_t src_start[kMaxPlanEntries];
  const int n_ent = (epr + 1) * ep;
  if (threadIdx.x == 0) {
    for (int s = 0; s < ep; ++s) {
      int64_t used = 0;
      for (int e = 0; e < epr; ++e) {
        const int64_t c = min(max((int64_t)recv_counts[s * epr + e], (int64_t)0), C - used);
        cnt[e * ep + s] = (int32_t)c;
        src_start[e * ep + s] = (int32_t)((int64_t)s * C + used);
        used += c;
      }
      cnt[epr * ep + s] = (int32_t)(C - used);
      src_start[epr * ep + s] = (int32_t)((int64_t)s * C + used);
    }
    int64_t acc = 0;
    seg_offsets[0] = 0;
    for (int e = 0; e <= epr; ++e) {
      for (int s = 0; s < ep; ++s) {
        dst_start[e * ep + s] = (int32_t)acc;
        acc += cnt[e * ep + s];
      }
      seg_offsets[e + 1] = (int32_t)acc;   // experts 0..epr-1, then the hole (e = epr)
    }
    dst_start[n_ent] = (int32_t)acc;
    for (int s = 0; s < num_shared; ++s) seg_offsets[epr + 2 + s] = (int32_t)(acc + (int64_t)(s + 1) * T);
  }
  __syncthreads();
  const int64_t n = (int64_t)ep * C;
  for (int64_t p = threadIdx.x; p < n; p += blockDim.x) {
    int lo = 0, hi = n_ent - 1;   // last entry with dst_start <= p (empty entries share a start)
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (dst_start[mid] <= p) lo = mid;
      else hi = mid - 1;
    }
    const int64_t q = src_start[lo] + (p - dst_start[lo]);
    regroup[p] = (int32_t)q;
    restore[q] = (int32_t)p;
  }
}

}  // namespace
}  // namespace lmoe

extern "C" int lmoe_capacity_send_plan(const int32_t* counts, const int32_t* sorted_idx, const int32_t* positions,
                                       int64_t num_tokens, int top_k, int ep, int experts_per_rank,
                                       int64_t capacity_rows, int32_t* send_index, int32_t* combine_pos,
                                       lmoe_stream_t stream_) {
  using namespace lmoe;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  LMOE_ARG_CHECK(num_tokens >= 0 && top_k >= 1 && ep >= 1 && experts_per_rank >= 1 && capacity_rows >= 1);
  LMOE_ARG_CHECK(ep <= kMaxPlanRanks && num_tokens * top_k <= capacity_rows);
  LMOE_ARG_CHECK((int64_t)ep * capacity_rows <= INT32_MAX);
  LMOE_ARG_CHECK(counts && send_index && (num_tokens == 0 || (sorted_idx && positions && combine_pos)));
  send_plan_kernel<<<1, kPlanThreads, 0, stream>>>(counts, sorted_idx, positions, num_tokens, top_k, ep,
                                                    experts_per_rank, capacity_rows, send_index, combine_pos);
  return cuda_status(cudaGetLastError());
}

extern "C" int lmoe_capacity_receive_plan(const int32_t* recv_counts, int ep, int experts_per_rank,
                                          int64_t capacity_rows, int num_shared, int64_t num_tokens,
                                          int32_t* regroup, int32_t* restore, int32_t* seg_offsets,
                                          lmoe_stream_t stream_) {
  using namespace lmoe;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  LMOE_ARG_CHECK(ep >= 1 && experts_per_rank >= 1 && capacity_rows >= 1 && num_shared >= 0 && num_tokens >= 0);
  LMOE_ARG_CHECK((int64_t)(experts_per_rank + 1) * ep <= kMaxPlanEntries);
  LMOE_ARG_CHECK((int64_t)ep * capacity_rows + (int64_t)num_shared * num_tokens <= INT32_MAX);
  LMOE_ARG_CHECK(recv_counts && regroup && restore && seg_offsets);
  receive_plan_kernel<<<1, kPlanThreads, 0, stream>>>(recv_counts, ep, experts_per_rank, capacity_rows, num_shared,
                                                       num_tokens, regroup, restore, seg_offsets);
  return cuda_status(cudaGetLastError());
}

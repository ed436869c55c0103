// grouped_gemm.h -- internal interface of the persistent grouped GEMM (grouped_gemm.cu).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace lmoe {

constexpr int kMaxGemmExperts = 256;

enum GemmMode : int {
  kModePlain = 0,    // out[r, n] = acc
  kModeSwiGLU = 1,   // tile rows j / j+64 = gate / up of feature fb*64+j: out[r, f] = silu(g) * u
  kModeScatter = 2,  // out[dest[r], n] = row_scale[r] * acc
};

struct GemmProblem {
  // activations: bf16 [total_rows, K], row pitch ldx elements
  const void* x = nullptr;
  int64_t ldx = 0;
  int64_t total_rows = 0;
  int K = 0;
  // expert row ranges [num_experts + 1] (int32, or int64 when offsets_i64)
  const void* offsets = nullptr;
  int offsets_i64 = 0;
  int num_experts = 0;  // number of row segments
  // weight matrix of each segment (NULL: segment e uses matrix e); lets rows that arrive
  // grouped by (source rank, expert) be multiplied without a local re-sort
  const int32_t* seg_expert = nullptr;
  int num_w = 0;        // weight matrices available; segments mapping outside [0, num_w) are skipped
  // weights: either W4 prepacked super-blocks (wq, scales embedded) or bf16 [num_experts, N, K] (w)
  const uint8_t* wq = nullptr;
  int group_size = 0;
  const void* w = nullptr;
  int ab_f16 = 0;       // dense weights and activations are fp16 (else bf16); output of the same type
  int N = 0;  // weight rows per expert (for SwiGLU: 2 * features)
  // epilogue
  int mode = kModePlain;
  void* out = nullptr;
  int64_t ldo = 0;
  const int32_t* dest = nullptr;
  // scatter into several buffers: dest[r] = (buffer << 24) | row of dest_bases[buffer]
  const uint64_t* dest_bases = nullptr;
  int dest_count = 0;
  const float* row_scale = nullptr;
  uint32_t* err = nullptr;
  // a known upper bound of rows per expert (0 = unknown); small values pick the decode tiles
  int64_t max_rows_per_expert_hint = 0;
};

int run_grouped_gemm(const GemmProblem& p, cudaStream_t stream);

// Dense fp32 grouped GEMM on CUDA cores (fp32 FFMA): out[r, n] = sum_k x[r, k] * w[e, n, k]
// for the rows r of segment e; K % 4 == 0, x / w / out 16-byte aligned.
int run_grouped_gemm_f32(const float* x, int64_t total_rows, int K, const float* w, int N, const void* offsets,
                         int offsets_i64, int num_experts, float* out, uint32_t* err, cudaStream_t stream);

}  // namespace lmoe

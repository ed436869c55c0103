// decode_gemm.h -- internal interface of the decode-sized W4A16 grouped GEMM (decode_gemm.cu).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "grouped_gemm.h"

namespace lmoe {

enum DecodeMode : int {
  kDecodePlain = 0,    // out bf16 [R, ldo]
  kDecodeSwiGLU = 1,   // paired gate/up rows -> out bf16 [R, ldo] = silu(gate) * up
  kDecodePartial = 2,  // out fp32 [ksplit][R][ldo]: partial sums of each K chunk
};

struct DecodeProblem {
  const void* x = nullptr;      // bf16 [total_rows, K], row pitch ldx
  int64_t ldx = 0;
  int64_t total_rows = 0;
  int K = 0;
  const void* offsets = nullptr;  // [num_experts + 1]; every segment must hold <= 64 rows
  int offsets_i64 = 0;
  int num_experts = 0;
  const int32_t* seg_expert = nullptr;
  int num_w = 0;                // weight matrices available (segments mapping outside are skipped)
  const uint8_t* wq = nullptr;  // prepacked super-blocks
  int group_size = 0;
  int N = 0;                    // weight rows per matrix (multiple of 128)
  int mode = kDecodePlain;
  int ksplit = 1;               // K chunks (divides K / 128); > 1 only with kDecodePartial
  void* out = nullptr;
  int64_t ldo = 0;
  uint32_t* err = nullptr;
};

constexpr int kDecodeMaxRows = 64;

int run_decode_gemm(const DecodeProblem& p, cudaStream_t stream);

}  // namespace lmoe

// lmoe_math.cuh -- device arithmetic that must match the CPU oracle bit for bit.
//
// Every operation is an explicitly rounded IEEE-754 single-precision operation
// (__fmul_rn / __fadd_rn / __fmaf_rn / __frcp_rn), so the compiler cannot contract or
// reorder it; the oracle (oracle/lmoe_oracle.c, built with -ffp-contract=off) performs the
// same sequence on the CPU.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace lmoe {

// exp(x) for x <= 0 (softmax arguments).  Cody & Waite argument reduction
// x = n*ln2 + r, n = rint(x*log2 e), |r| <= ln2/2, with ln2 split as LN2_HI + LN2_LO
// (LN2_HI has 12 trailing zero bits so n*LN2_HI is exact), followed by the degree-7 Taylor
// polynomial of exp evaluated with fused multiply-adds and a scaling by 2^n.  Within 2 ulp
// of exp(x); results below the subnormal range flush to +0.
__device__ __forceinline__ float softmax_exp(float x) {
  if (!(x > -104.0f)) return 0.0f;
  if (x > 0.0f) x = 0.0f;
  const float t = __fmul_rn(x, __uint_as_float(0x3fb8aa3bu));
  const float n = rintf(t);
  float r = __fmaf_rn(-n, __uint_as_float(0x3f317000u), x);
  r = __fmaf_rn(-n, __uint_as_float(0x3805fdf4u), r);
  float p = __uint_as_float(0x39500d01u);
  p = __fmaf_rn(p, r, __uint_as_float(0x3ab60b61u));
  p = __fmaf_rn(p, r, __uint_as_float(0x3c088889u));
  p = __fmaf_rn(p, r, __uint_as_float(0x3d2aaaabu));
  p = __fmaf_rn(p, r, __uint_as_float(0x3e2aaaabu));
  p = __fmaf_rn(p, r, __uint_as_float(0x3f000000u));
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const int ni = static_cast<int>(n);
  if (ni >= -126) return __fmul_rn(p, __uint_as_float(static_cast<uint32_t>(ni + 127) << 23));
  const float p2 = __fmul_rn(p, __uint_as_float(static_cast<uint32_t>(ni + 64 + 127) << 23));
  return __fmul_rn(p2, __uint_as_float(static_cast<uint32_t>(127 - 64) << 23));
}

// Insert (v, e) into a descending list of KMAX entries; an equal value never displaces an
// earlier entry, so among equal probabilities the lower expert id stays first.
template <int KMAX>
__device__ __forceinline__ void topk_insert(float (&tv)[KMAX], int (&ti)[KMAX], float v, int e) {
#pragma unroll
  for (int j = KMAX - 1; j >= 0; --j) {
    const bool gt_prev = (j > 0) ? (v > tv[j > 0 ? j - 1 : 0]) : false;
    const bool gt_cur = v > tv[j];
    const float nv = gt_prev ? tv[j > 0 ? j - 1 : 0] : (gt_cur ? v : tv[j]);
    const int ni = gt_prev ? ti[j > 0 ? j - 1 : 0] : (gt_cur ? e : ti[j]);
    tv[j] = nv;
    ti[j] = ni;
  }
}

}  // namespace lmoe

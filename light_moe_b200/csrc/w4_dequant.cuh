// w4_dequant.cuh -- int4 -> bf16 dequantisation of the prepacked super-block layout
// (w4_layout.cuh), shared by the grouped GEMM and the decode GEMM.
//
// Dequantised value = bf16_rn(q * s) with q = u - 8 (u the stored nibble) and s the fp16
// group scale, computed exactly: q is an exact bf16 integer (magic-number trick), s is split
// into bf16 hi (top 8 significant bits, round toward zero) + lo (the exact remainder), and
// q*s = fma(q, s_hi, q * s_lo) rounds once because q * s_lo is exact (|q| <= 8, s_lo has at
// most 3 significant bits beyond bf16's 8).  Bit-identical to the CPU oracle's
// bf16_rn(float(q) * float(s)).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

namespace lmoe {

__device__ __forceinline__ uint32_t bf16x2_bits(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ __nv_bfloat162 bits_bf16x2(uint32_t v) { return *reinterpret_cast<__nv_bfloat162*>(&v); }

// One 16-byte half-row (w4_layout.cuh) -> the bf16x2 bits of (128 + u) for its 16 K pairs
// in K order (o[m] = pair m: K 2m in the low half, 2m + 1 in the high half).
__device__ __forceinline__ void w4_unpack_half(const uint4 v, uint32_t (&o)[16]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint32_t lo = w[c] & 0x0F0F0F0Fu;           // pairs 4c, 4c+1
    const uint32_t hi = (w[c] >> 4) & 0x0F0F0F0Fu;    // pairs 4c+2, 4c+3
    o[4 * c + 0] = __byte_perm(lo, 0x43434343u, 0x5140);
    o[4 * c + 1] = __byte_perm(lo, 0x43434343u, 0x7362);
    o[4 * c + 2] = __byte_perm(hi, 0x43434343u, 0x5140);
    o[4 * c + 3] = __byte_perm(hi, 0x43434343u, 0x7362);
  }
}

// Dequantise one 16-byte half-row (32 K values) into the 16 bf16x2 registers of its K pairs
// in K order.
__device__ __forceinline__ void dequant_half(const uint4 v, __nv_bfloat162 s_hi, __nv_bfloat162 s_lo,
                                             const __nv_bfloat162 off136, uint32_t (&o)[16]) {
  w4_unpack_half(v, o);
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    const __nv_bfloat162 q = __hsub2(bits_bf16x2(o[m]), off136);   // exact q = u - 8
    const __nv_bfloat162 t = __hmul2(q, s_lo);                      // exact (<= 6 bits)
    o[m] = bf16x2_bits(__hfma2(q, s_hi, t));                        // one rounding of q*s
  }
}

// Exact split of an fp16 scale into bf16 hi (top 8 significant bits) + lo (the rest).
__device__ __forceinline__ void split_scale(uint16_t sbits, __nv_bfloat162& s_hi, __nv_bfloat162& s_lo) {
  const float sf = __half2float(__ushort_as_half(sbits));
  const __nv_bfloat16 hi = __float2bfloat16_rz(sf);
  const __nv_bfloat16 lo = __float2bfloat16_rn(__fsub_rn(sf, __bfloat162float(hi)));
  s_hi = __nv_bfloat162(hi, hi);
  s_lo = __nv_bfloat162(lo, lo);
}

}  // namespace lmoe

// w4_layout.cuh -- the device ("prepacked") int4 weight layout streamed by the W4A16
// grouped GEMM.
//
// The canonical format (qweight [rows, K/2], scales [rows, K/g], see quant.cu) is
// re-arranged once, offline, so that the GEMM streams one contiguous "super-block" per
// pipeline stage with a single 1-D bulk copy and dequantises with one LOP3 per bf16 pair:
//
//   super-block = 128 weight rows x 128 K values of one expert
//     [ int4:   2 k-blocks x 2 halves x 128 rows x 16 bytes          8192 bytes ]
//     [ scales: SG groups x 128 rows x fp16, SG = max(1, 128 / g)    256*SG bytes ]
//   k-block j (K values 64j..64j+63 of the super-block), half h (32h..32h+31 of the
//   k-block): the 16 bytes of row r sit at j*4096 + h*2048 + r*16, so the thread owning a
//   row reads 16 consecutive bytes and consecutive threads read consecutive 16-byte chunks
//   (no shared-memory bank conflicts);
//   scales: group i of the super-block at 8192 + i*256 + r*2 (for g > 128 every
//   super-block carries the scale of the group that contains it);
//   packed [E][NB = rows/128][K/128][super-block]
//
//   inside each 32-bit word (8 consecutive K values k0..k7) the nibbles are interleaved
//     bits [0,4)=k0 [4,8)=k2 [8,12)=k4 [12,16)=k6 [16,20)=k1 [20,24)=k3 [24,28)=k5 [28,32)=k7
//   so (word >> 4p) & 0x000F000F places k_{2p} and k_{2p+1} in the two bf16 halves.
//
// Gate/up ("paired") prepacking interleaves two matrices A (gate, w1) and B (up, w3) of
// F rows each by 64-row blocks: block fb holds rows fb*64.. of A in rows 0..63 and the same
// rows of B in rows 64..127, so one 128-row GEMM tile produces gate and up for 64 features.
#pragma once
#include <cstdint>

namespace lmoe {

constexpr int kW4BlockRows = 128;
constexpr int kW4SuperK = 128;                                   // K values per super-block
constexpr int kW4KBlockBytes = kW4BlockRows * 64 / 2;            // 4096: one 64-wide k-block
constexpr int kW4SuperInt4Bytes = 2 * kW4KBlockBytes;            // 8192

__host__ __device__ constexpr int w4_scale_groups(int g) { return g >= kW4SuperK ? 1 : kW4SuperK / g; }
__host__ __device__ constexpr int w4_super_bytes(int g) { return kW4SuperInt4Bytes + 256 * w4_scale_groups(g); }

// Canonical 32-bit word (bytes b_i = k_{2i} | k_{2i+1} << 4) -> interleaved word.
__host__ __device__ __forceinline__ uint32_t w4_interleave_word(uint32_t c) {
  uint32_t lo = c & 0x0F0F0F0Fu;          // k0, k2, k4, k6 in the low nibble of each byte
  uint32_t hi = (c >> 4) & 0x0F0F0F0Fu;   // k1, k3, k5, k7
  lo = (lo | (lo >> 4)) & 0x00FF00FFu;    // byte0 = k0|k2<<4, byte2 = k4|k6<<4
  hi = (hi | (hi >> 4)) & 0x00FF00FFu;
  lo = (lo & 0xFFu) | ((lo >> 8) & 0xFF00u);
  hi = (hi & 0xFFu) | ((hi >> 8) & 0xFF00u);
  return lo | (hi << 16);
}

}  // namespace lmoe

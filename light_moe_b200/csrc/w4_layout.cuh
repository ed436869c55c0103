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
//   inside each 16-byte half-row (32 consecutive K values = 16 pairs (2m, 2m+1), m = 0..15;
//   lo(m) / hi(m) the nibbles of K 2m / 2m+1) the nibbles are regrouped so that one AND or
//   one shift+AND exposes four pairs in four bytes: 32-bit word c (c = 0..3) holds pairs
//   4c..4c+3 as
//     byte 0 = lo(4c)   | lo(4c+2) << 4      byte 1 = hi(4c)   | hi(4c+2) << 4
//     byte 2 = lo(4c+1) | lo(4c+3) << 4      byte 3 = hi(4c+1) | hi(4c+3) << 4
//   so w & 0x0F0F0F0F = [lo(4c), hi(4c), lo(4c+1), hi(4c+1)] and (w >> 4) & 0x0F0F0F0F the
//   same for pairs 4c+2, 4c+3, and one byte permute per pair builds the bf16 pair
//   (128 + lo, 128 + hi) with the exponent byte 0x43 (w4_dequant.cuh).  A thread that owns a
//   whole row reads its 16 bytes and gets the 16 pairs in K order.
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

// Canonical 16 bytes of a half-row (byte m = lo(m) | hi(m) << 4, m = 0..15) -> device words.
// Word c is built from canonical word c alone (pairs 4c..4c+3).
__host__ __device__ __forceinline__ uint32_t w4_device_word(uint32_t v) {
  const uint32_t b0 = v & 0xFFu, b1 = (v >> 8) & 0xFFu, b2 = (v >> 16) & 0xFFu, b3 = v >> 24;
  const uint32_t d0 = (b0 & 0x0Fu) | ((b2 & 0x0Fu) << 4);
  const uint32_t d1 = (b0 >> 4) | (b2 & 0xF0u);
  const uint32_t d2 = (b1 & 0x0Fu) | ((b3 & 0x0Fu) << 4);
  const uint32_t d3 = (b1 >> 4) | (b3 & 0xF0u);
  return d0 | (d1 << 8) | (d2 << 16) | (d3 << 24);
}

__host__ __device__ __forceinline__ uint4 w4_device_half(uint4 canon) {
  return make_uint4(w4_device_word(canon.x), w4_device_word(canon.y), w4_device_word(canon.z),
                    w4_device_word(canon.w));
}

}  // namespace lmoe

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
//   inside each 16-byte half-row (32 consecutive K values, octets i = 0..3 of 8 values) the
//   nibbles are transposed and interleaved: 32-bit word c (c = 0..3) holds, in slot i, the
//   pair (k = 8i + 2c, 8i + 2c + 1):  bits [4i, 4i+4) = k 8i+2c,  bits [16+4i, 20+4i) = k 8i+2c+1.
//   So (word >> 4i) & 0x000F000F places one K pair in the two bf16 halves, and
//   * a thread that owns a whole row (tcgen05 path) gets every pair of its 32 K values from
//     its 16 bytes (pair m = 4i + c comes from word c, slot i);
//   * ldmatrix of 8 rows x 16 bytes gives mma.sync thread (g, c) word c of row g: exactly the
//     A-fragment pairs (k 2c, 2c+1) of the half's four octets (two 16-wide k steps).
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

// Bytes b_i = (k_{2i} | k_{2i+1} << 4), i = 0..3 -> low nibbles in bits [4i, 4i+4), high
// nibbles in bits [16+4i, 20+4i).
__host__ __device__ __forceinline__ uint32_t w4_split_nibbles(uint32_t c) {
  uint32_t lo = c & 0x0F0F0F0Fu;
  uint32_t hi = (c >> 4) & 0x0F0F0F0Fu;
  lo = (lo | (lo >> 4)) & 0x00FF00FFu;
  hi = (hi | (hi >> 4)) & 0x00FF00FFu;
  lo = (lo & 0xFFu) | ((lo >> 8) & 0xFF00u);
  hi = (hi & 0xFFu) | ((hi >> 8) & 0xFF00u);
  return lo | (hi << 16);
}

// Canonical 16 bytes of a half-row (byte b = k 2b | k 2b+1 << 4, b = 0..15) -> device words.
// Word c gathers canonical byte 4i + c of every octet i (a 4 x 4 byte transpose) and splits
// the nibbles.
__host__ __device__ __forceinline__ uint4 w4_device_half(uint4 canon) {
  const uint32_t w[4] = {canon.x, canon.y, canon.z, canon.w};
  uint32_t t[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t v = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) v |= ((w[i] >> (8 * c)) & 0xFFu) << (8 * i);
    t[c] = w4_split_nibbles(v);
  }
  return make_uint4(t[0], t[1], t[2], t[3]);
}

}  // namespace lmoe

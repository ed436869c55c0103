// host_util.h -- host-side helpers shared by the C-ABI entry points: status codes, device
// properties, and TMA tensor-map encoding through the driver entry point (so the library
// does not link libcuda directly).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>

#include "lmoe_b200.h"

namespace lmoe {

// Map a CUDA runtime error to the C-ABI status (positive CUDA error code).
inline int cuda_status(cudaError_t e) { return e == cudaSuccess ? LMOE_OK : static_cast<int>(e); }

#define LMOE_CUDA_TRY(expr)                         \
  do {                                              \
    cudaError_t _e = (expr);                        \
    if (_e != cudaSuccess) return static_cast<int>(_e); \
  } while (0)

#define LMOE_ARG_CHECK(cond)                    \
  do {                                          \
    if (!(cond)) return LMOE_ERR_INVALID_ARG;   \
  } while (0)

// Per-device cached properties.
struct DeviceInfo {
  int device = -1;
  int num_sms = 0;
  int cc_major = 0;
  int cc_minor = 0;
  size_t max_smem_optin = 0;
};

int get_device_info(DeviceInfo* out);

// CTAs of a persistent GEMM launch: one per SM, capped by lmoe_set_gemm_sm_limit.
int gemm_grid(const DeviceInfo& dev);

// Process-unique id of the calling thread's current CUDA context (cuCtxGetId); 0 when no
// context is bound to the thread yet.
int current_context_id(unsigned long long* id);

// cudaFuncSetAttribute(fn, MaxDynamicSharedMemorySize, smem) on the current device, skipped
// when this (kernel, device) already allows at least `smem` bytes: the attribute call costs
// microseconds of host time on every launch otherwise.
int set_max_dynamic_smem(const void* fn, size_t smem);

// Encode a 2-D row-major tensor map: `rows` x `cols` elements of `elem_bytes` bytes,
// row pitch `row_stride_bytes`, box `box_cols` x `box_rows`, 128-byte swizzle when
// `swizzle128` (box_cols * elem_bytes must then be 128).  Returns a C-ABI status.
int encode_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint32_t elem_bytes,
                   uint64_t rows, uint64_t cols, uint64_t row_stride_bytes, uint32_t box_rows, uint32_t box_cols,
                   bool swizzle128);

// Encode a row-major `rows` x `cols` matrix (row pitch `row_stride_bytes`) as a 3-D tensor
// of 128-byte column blocks: dims {block elements, rows, cols / block elements}, so one box
// {block elements, box_rows, box_blocks} lands in shared memory as [box_blocks][box_rows]
// [128 bytes] with the 128-byte swizzle -- several K blocks of a row tile in one copy.
int encode_tmap_kblocks(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint32_t elem_bytes,
                        uint64_t rows, uint64_t cols, uint64_t row_stride_bytes, uint32_t box_rows,
                        uint32_t box_blocks);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace lmoe

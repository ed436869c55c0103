// host_util.cu -- device-info cache, TMA descriptor encoding and the small C-ABI utilities.
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>

#include "host_util.h"

namespace lmoe {

namespace {
constexpr int kMaxDevices = 64;
DeviceInfo g_info[kMaxDevices];
std::mutex g_info_mu;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
PFN_cuCtxGetCurrent_v4000 g_ctx_current = nullptr;
PFN_cuCtxGetId_v12000 g_ctx_id = nullptr;
std::once_flag g_ctx_once;
}  // namespace

int current_context_id(unsigned long long* id) {
  std::call_once(g_ctx_once, []() {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &fn, 4000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_ctx_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(fn);
    fn = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &fn, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_ctx_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(fn);
  });
  if (!g_ctx_current || !g_ctx_id) return LMOE_ERR_DEVICE;
  CUcontext ctx = nullptr;
  if (g_ctx_current(&ctx) != CUDA_SUCCESS) return LMOE_ERR_DEVICE;
  if (!ctx) {   // no context bound to this thread yet
    *id = 0;
    return LMOE_OK;
  }
  unsigned long long v = 0;
  if (g_ctx_id(ctx, &v) != CUDA_SUCCESS) return LMOE_ERR_DEVICE;
  *id = v;
  return LMOE_OK;
}

namespace {
std::atomic<int> g_gemm_sm_limit{0};
}  // namespace

int gemm_grid(const DeviceInfo& dev) {
  const int cap = g_gemm_sm_limit.load(std::memory_order_relaxed);
  return cap > 0 && cap < dev.num_sms ? cap : dev.num_sms;
}

int get_device_info(DeviceInfo* out) {
  int dev = 0;
  LMOE_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return LMOE_ERR_DEVICE;
  {
    std::lock_guard<std::mutex> lk(g_info_mu);
    if (g_info[dev].device == dev) {
      *out = g_info[dev];
      return LMOE_OK;
    }
  }
  DeviceInfo d;
  d.device = dev;
  LMOE_CUDA_TRY(cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev));
  LMOE_CUDA_TRY(cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev));
  LMOE_CUDA_TRY(cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev));
  int smem = 0;
  LMOE_CUDA_TRY(cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
  d.max_smem_optin = (size_t)smem;
  std::lock_guard<std::mutex> lk(g_info_mu);
  g_info[dev] = d;
  *out = d;
  return LMOE_OK;
}

namespace {
struct SmemAttr {
  const void* fn;
  int device;
  size_t smem;
};
constexpr int kMaxSmemAttrs = 256;
SmemAttr g_smem_attr[kMaxSmemAttrs];
int g_smem_attr_n = 0;
std::mutex g_smem_attr_mu;
}  // namespace

int set_max_dynamic_smem(const void* fn, size_t smem) {
  int dev = 0;
  LMOE_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_smem_attr_mu);
  int slot = -1;
  for (int i = 0; i < g_smem_attr_n; ++i) {
    if (g_smem_attr[i].fn == fn && g_smem_attr[i].device == dev) {
      if (g_smem_attr[i].smem >= smem) return LMOE_OK;
      slot = i;
      break;
    }
  }
  LMOE_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  if (slot < 0 && g_smem_attr_n < kMaxSmemAttrs) slot = g_smem_attr_n++;
  if (slot >= 0) g_smem_attr[slot] = {fn, dev, smem};   // a full table only loses the shortcut
  return LMOE_OK;
}

namespace {
// Encoded tensor maps by (address, type, shape, strides, box, swizzle): a layer call encodes
// the same few maps every time, and a map depends on nothing else, so an entry never goes
// stale.  Direct-mapped, 256 slots.
struct TmapKey {
  const void* base;
  uint64_t dims[3];
  uint64_t strides[2];
  uint32_t box[3];
  uint32_t dtype, rank, swizzle;
  bool operator==(const TmapKey& o) const {
    return base == o.base && dtype == o.dtype && rank == o.rank && swizzle == o.swizzle &&
           dims[0] == o.dims[0] && dims[1] == o.dims[1] && dims[2] == o.dims[2] && strides[0] == o.strides[0] &&
           strides[1] == o.strides[1] && box[0] == o.box[0] && box[1] == o.box[1] && box[2] == o.box[2];
  }
};
struct TmapSlot {
  bool used = false;
  TmapKey key;
  CUtensorMap map;
};
constexpr int kTmapSlots = 256;
TmapSlot g_tmap[kTmapSlots];
std::mutex g_tmap_mu;

uint32_t tmap_slot(const TmapKey& k) {
  uint64_t h = 1469598103934665603ull;
  auto mix = [&](uint64_t v) { h = (h ^ v) * 1099511628211ull; };
  mix(reinterpret_cast<uintptr_t>(k.base));
  for (int i = 0; i < 3; ++i) mix(k.dims[i]);
  mix(k.strides[0]);
  mix(k.strides[1]);
  for (int i = 0; i < 3; ++i) mix(k.box[i]);
  mix(k.dtype);
  mix(k.rank);
  mix(k.swizzle);
  return (uint32_t)(h ^ (h >> 32)) % kTmapSlots;
}

bool tmap_lookup(const TmapKey& k, CUtensorMap* out) {
  std::lock_guard<std::mutex> lk(g_tmap_mu);
  const TmapSlot& e = g_tmap[tmap_slot(k)];
  if (!e.used || !(e.key == k)) return false;
  *out = e.map;
  return true;
}

void tmap_store(const TmapKey& k, const CUtensorMap& m) {
  std::lock_guard<std::mutex> lk(g_tmap_mu);
  TmapSlot& e = g_tmap[tmap_slot(k)];
  e.used = true;
  e.key = k;
  e.map = m;
}
}  // namespace

int encode_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint32_t elem_bytes,
                   uint64_t rows, uint64_t cols, uint64_t row_stride_bytes, uint32_t box_rows, uint32_t box_cols,
                   bool swizzle128) {
  std::call_once(g_encode_once, []() {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  });
  if (!g_encode) return LMOE_ERR_DEVICE;
  if (!aligned16(base) || (row_stride_bytes % 16) != 0) return LMOE_ERR_INVALID_ARG;
  if (box_rows == 0 || box_rows > 256 || box_cols == 0 || box_cols > 256) return LMOE_ERR_INVALID_ARG;
  if (swizzle128 && box_cols * elem_bytes != 128) return LMOE_ERR_INVALID_ARG;
  const TmapKey key = {base, {cols, rows, 0}, {row_stride_bytes, 0}, {box_cols, box_rows, 0}, (uint32_t)dtype, 2u,
                       swizzle128 ? 1u : 0u};
  if (tmap_lookup(key, map)) return LMOE_OK;
  cuuint64_t gdim[2] = {cols, rows};
  cuuint64_t gstride[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estride[2] = {1, 1};
  CUresult r = g_encode(map, dtype, 2, const_cast<void*>(base), gdim, gstride, box, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return LMOE_ERR_INVALID_ARG;
  tmap_store(key, *map);
  return LMOE_OK;
}

int encode_tmap_kblocks(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint32_t elem_bytes,
                        uint64_t rows, uint64_t cols, uint64_t row_stride_bytes, uint32_t box_rows,
                        uint32_t box_blocks) {
  // the driver entry point is resolved by encode_tmap_2d's first call
  if (!g_encode) {
    CUtensorMap tmp;
    encode_tmap_2d(&tmp, base, dtype, elem_bytes, 1, 128 / elem_bytes, row_stride_bytes, 1, 128 / elem_bytes, true);
  }
  if (!g_encode) return LMOE_ERR_DEVICE;
  const uint64_t blk = 128 / elem_bytes;   // elements per 128-byte block
  if (!aligned16(base) || (row_stride_bytes % 16) != 0 || cols % blk != 0) return LMOE_ERR_INVALID_ARG;
  if (box_rows == 0 || box_rows > 256 || box_blocks == 0 || box_blocks > 256) return LMOE_ERR_INVALID_ARG;
  const TmapKey key = {base, {blk, rows, cols / blk}, {row_stride_bytes, 128}, {(uint32_t)blk, box_rows, box_blocks},
                       (uint32_t)dtype, 3u, 1u};
  if (tmap_lookup(key, map)) return LMOE_OK;
  cuuint64_t gdim[3] = {blk, rows, cols / blk};
  cuuint64_t gstride[2] = {row_stride_bytes, 128};
  cuuint32_t box[3] = {(cuuint32_t)blk, box_rows, box_blocks};
  cuuint32_t estride[3] = {1, 1, 1};
  CUresult r = g_encode(map, dtype, 3, const_cast<void*>(base), gdim, gstride, box, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return LMOE_ERR_INVALID_ARG;
  tmap_store(key, *map);
  return LMOE_OK;
}

}  // namespace lmoe

extern "C" int lmoe_version(void) { return 100; }

extern "C" const char* lmoe_status_string(int status) {
  switch (status) {
    case LMOE_OK: return "ok";
    case LMOE_ERR_INVALID_ARG: return "invalid argument (shape, dtype, alignment or null pointer)";
    case LMOE_ERR_UNSUPPORTED: return "unsupported configuration";
    case LMOE_ERR_WORKSPACE: return "workspace missing or too small";
    case LMOE_ERR_DEVICE: return "device is not sm_100 or a kernel reported an error";
    default: break;
  }
  if (status > 0) return cudaGetErrorString(static_cast<cudaError_t>(status));
  return "unknown status";
}

extern "C" int lmoe_set_gemm_sm_limit(int max_ctas) {
  if (max_ctas < 0) return LMOE_ERR_INVALID_ARG;
  lmoe::g_gemm_sm_limit.store(max_ctas, std::memory_order_relaxed);
  return LMOE_OK;
}

extern "C" int lmoe_get_gemm_sm_limit(void) { return lmoe::g_gemm_sm_limit.load(std::memory_order_relaxed); }

extern "C" int lmoe_read_error(const void* workspace, uint32_t* out, lmoe_stream_t stream) {
  if (!workspace || !out) return LMOE_ERR_INVALID_ARG;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  LMOE_CUDA_TRY(cudaMemcpyAsync(out, workspace, sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
  LMOE_CUDA_TRY(cudaStreamSynchronize(s));
  return LMOE_OK;
}

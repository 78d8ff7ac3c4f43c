// Host helpers and library-info entry points of libce_b200.so.
#include "ce_host.h"

#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/ce_api.h"

namespace ce {
namespace host {

namespace {
thread_local char g_last_error[256] = "";
constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices] = {0};
std::mutex g_mu;

struct SmemEntry {
  const void* func;
  int device;
  int bytes;
};
SmemEntry g_smem[256];
int g_smem_n = 0;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
}  // namespace

const char* last_error() { return g_last_error; }

int fail(int status, const char* msg) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s", msg);
  return status;
}

int fail_cuda(const char* where) {
  cudaError_t e = cudaGetLastError();
  std::snprintf(g_last_error, sizeof(g_last_error), "%s: %s", where, cudaGetErrorString(e));
  return CE_ERR_CUDA;
}

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
  if (g_sm_count[dev] > 0) return g_sm_count[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
  g_sm_count[dev] = n;
  return n;
}

bool set_smem_attr(const void* func, int bytes) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  std::lock_guard<std::mutex> lock(g_mu);
  for (int i = 0; i < g_smem_n; ++i)
    if (g_smem[i].func == func && g_smem[i].device == dev && g_smem[i].bytes >= bytes) return true;
  if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
    return false;
  if (g_smem_n < 256) g_smem[g_smem_n++] = {func, dev, bytes};
  return true;
}

bool set_max_shared_carveout_attr(const void* func) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  std::lock_guard<std::mutex> lock(g_mu);
  // carveout entries share the cache with bytes = -1
  for (int i = 0; i < g_smem_n; ++i)
    if (g_smem[i].func == func && g_smem[i].device == dev && g_smem[i].bytes == -1) return true;
  if (cudaFuncSetAttribute(func, cudaFuncAttributePreferredSharedMemoryCarveout,
                           static_cast<int>(cudaSharedmemCarveoutMaxShared)) != cudaSuccess)
    return false;
  if (g_smem_n < 256) g_smem[g_smem_n++] = {func, dev, -1};
  return true;
}

static bool encoder() {
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return false;
    g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  }
  return true;
}

bool encode_map(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                const uint64_t* dims, const uint64_t* strides, const uint32_t* box, bool swizzle128) {
  if (rank < 1 || rank > 5 || !encoder()) return false;
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) st[i] = strides[i];
  CUresult r = g_encode(map, dtype, rank, const_cast<void*>(base), d, st, b, e,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool encode_rows_map(CUtensorMap* map, const void* base, uint64_t rows, uint32_t cols,
                     uint32_t box_rows) {
  const uint64_t dims[2] = {cols, rows};
  const uint64_t strides[1] = {static_cast<uint64_t>(cols) * 2};
  const uint32_t box[2] = {cols, box_rows};
  return encode_map(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, true);
}

}  // namespace host
}  // namespace ce

extern "C" const char* ce_version(void) { return "cache_eviction_b200 0.1 (sm_100a)"; }

extern "C" const char* ce_status_string(int status) {
  switch (status) {
    case CE_OK: return "ok";
    case CE_ERR_ARG: return "invalid argument";
    case CE_ERR_UNSUPPORTED: return "unsupported shape";
    case CE_ERR_CUDA: return "CUDA error";
    case CE_ERR_WORKSPACE: return "workspace too small";
    default: return "unknown status";
  }
}

extern "C" const char* ce_last_error(void) { return ce::host::last_error(); }

extern "C" int ce_prepare_device(void) {
  int st = ce::host::decode_prepare_device();
  if (st == CE_OK) st = ce::host::select_prepare_device();
  if (st == CE_OK) st = ce::host::fill_prepare_device();
  if (st == CE_OK) st = ce::host::pool_prepare_device();
  return st;
}

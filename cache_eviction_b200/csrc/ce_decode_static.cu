// ce_decode_attn_score_static: the fused decode attention + H2O score for
// callers that cannot allocate device memory.
//
// Some callers cannot call cudaMalloc (or any allocating routine) at the point
// where they run a decode step: a serving process that hands all of HBM to its
// KV-cache pool at start-up and has nothing left to carve a workspace from, a
// plugin whose host forbids device allocations after initialisation so that
// memory use stays fixed, or code that runs inside a CUDA graph capture in
// global mode, where allocation calls are rejected.  ce_decode_attn_score
// still needs such a caller to pass a workspace; this entry point does not.
//
// Its scratch is the file-scope array below, CE_DECODE_STATIC_SCRATCH_BYTES
// long.  The entry point checks that the call fits the array, finds the
// array's device address and hands it to ce_decode_attn_score as the
// workspace; nothing else changes.
//
// When the array takes device memory: with lazy module loading (the CUDA 12
// default, CUDA_MODULE_LOADING=LAZY) the driver places it when this file's
// module is first used, which is the set-up below (the first call on a
// device, or a call with bs == 0); with eager loading, when the context is
// created.  It then stays until the process exits.  The set-up also loads the
// decode kernels themselves.  A caller that gives the rest of HBM to its pool
// therefore makes its set-up call first.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/ce_api.h"
#include "ce_host.h"

namespace {

// The scratch itself.  In host code this name is only a stand-in for the
// device array (its address is not a device address); the real address comes
// from cudaGetSymbolAddress, once per device and context.
static __device__ __align__(256) unsigned char g_decode_scratch[CE_DECODE_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;

// The device address found at set-up, with the context it belongs to: after
// cudaDeviceReset the device gets a new primary context (and a new copy of the
// array), so an address cached for the old one is looked up again.
struct Slot {
  void* ptr = nullptr;
  unsigned long long context = 0;
};
Slot g_slot[kMaxDevices];
std::mutex g_mu;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

// Unique id of the calling thread's current context, or 0 when there is none
// (or the driver cannot say, in which case every call repeats the set-up).
unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static bool looked_up = false;
  if (!looked_up) {
    looked_up = true;
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(fn);
    fn = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(fn);
    cudaGetLastError();  // a failed lookup leaves nothing pending for later launches
  }
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx ||
      get_id(ctx, &id) != CUDA_SUCCESS)
    return 0;
  return id;
}

// Device address of this device's copy of the scratch.  The first call made
// with a device current (and the first after its context was replaced) runs
// the set-up: it looks the address up, which places the array under lazy
// loading, and loads the decode kernels.
int scratch_address(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return ce::host::fail_cuda("ce_decode_attn_score_static: no current device");
  std::lock_guard<std::mutex> lock(g_mu);
  Slot& slot = g_slot[dev];
  const unsigned long long ctx = current_context_id();
  if (!slot.ptr || ctx == 0 || ctx != slot.context) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_decode_scratch) != cudaSuccess || !ptr) {
      slot = Slot{};
      return ce::host::fail_cuda("ce_decode_attn_score_static: cudaGetSymbolAddress of the static scratch");
    }
    const int st = ce::host::decode_prepare_device();
    if (st != CE_OK) {
      slot = Slot{};
      return st;
    }
    slot.ptr = ptr;
    slot.context = current_context_id();  // the lookup made the primary context current
  }
  *out = slot.ptr;
  return CE_OK;
}

}  // namespace

extern "C" int ce_decode_attn_score_static(
    const void* q, int64_t q_sb, int64_t q_sh, const void* k_pool, const void* v_pool,
    int64_t pool_units, const int32_t* kv_indptr, const int32_t* kv_indices,
    const int32_t* kv_tokens, int64_t kv_capacity, const float* sinks,
    const int32_t* mode_of_row, const int64_t* rows, float sm_scale, int32_t bs,
    int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, int32_t page_size,
    float* scores, int64_t score_sg, int32_t zero_new, void* out, int32_t out_f32, int64_t o_sb,
    int64_t o_sh, float* lse_out, int32_t score_flags, int32_t* err, void* stream) {
  if (score_flags & CE_SCORE_DEFER)
    return ce::host::fail(CE_ERR_ARG, "ce_decode_attn_score_static: deferred scores need a caller workspace");
  if (bs < 0) return ce::host::fail(CE_ERR_ARG, "ce_decode_attn_score_static: negative batch");
  void* scratch = nullptr;
  if (bs == 0) return scratch_address(&scratch);  // set-up only: nothing is launched
  const int64_t need = ce_decode_workspace_bytes(bs, kv_capacity, num_q_heads, num_kv_heads,
                                                 page_size, score_flags);
  if (need < 0) return ce::host::fail(CE_ERR_ARG, "ce_decode_attn_score_static: bad sizes");
  if (need > static_cast<int64_t>(CE_DECODE_STATIC_SCRATCH_BYTES))
    return ce::host::fail(CE_ERR_WORKSPACE,
                          "ce_decode_attn_score_static: this batch needs more scratch than the "
                          "static maximum (CE_DECODE_STATIC_SCRATCH_BYTES); use "
                          "ce_decode_attn_score with a caller workspace");
  const int st = scratch_address(&scratch);
  if (st != CE_OK) return st;
  // Nothing in the scratch has to start at zero: every byte the kernels read
  // is written earlier in the same call, so the previous call's contents are
  // harmless.
  return ce_decode_attn_score(q, q_sb, q_sh, k_pool, v_pool, pool_units, kv_indptr, kv_indices,
                              kv_tokens, kv_capacity, sinks, mode_of_row, rows, sm_scale, bs,
                              num_q_heads, num_kv_heads, head_dim, page_size, scores, score_sg,
                              zero_new, out, out_f32, o_sb, o_sh, lse_out, score_flags, scratch,
                              static_cast<int64_t>(CE_DECODE_STATIC_SCRATCH_BYTES), err, stream);
}

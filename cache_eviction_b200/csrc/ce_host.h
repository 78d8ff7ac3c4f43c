// Host-side helpers shared by the C-ABI entry points (no device code).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace ce {
namespace host {

// Records a message for ce_status_string's companion ce_last_error and
// returns `status` unchanged.
int fail(int status, const char* msg);
// Message of the last failing entry point on this host thread.
const char* last_error();
// Records the pending CUDA error text and returns CE_ERR_CUDA.
int fail_cuda(const char* where);

// Multiprocessor count of the current device (cached per device).
int sm_count();

// Raise a kernel's dynamic shared-memory limit once per device.
bool set_smem_attr(const void* func, int bytes);
template <class F>
bool set_smem(F* func, int bytes) {
  return set_smem_attr(reinterpret_cast<const void*>(func), bytes);
}

// Prefer the largest shared-memory carveout for a kernel, once per device: a
// small kernel that runs beside a large-shared-memory one must not leave an
// SM configured for less shared memory than the large one needs.
bool set_max_shared_carveout_attr(const void* func);
template <class F>
bool set_max_shared_carveout(F* func) {
  return set_max_shared_carveout_attr(reinterpret_cast<const void*>(func));
}

// Tiled tensor map of `rank` dims (innermost first): dims, byte strides of
// dims 1..rank-1, box sizes; element strides 1, zero fill out of bounds,
// 128-byte swizzle or none.
bool encode_map(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                const uint64_t* dims, const uint64_t* strides, const uint32_t* box, bool swizzle128);

// 2D bf16 tensor map over `rows` rows of `cols` elements (dense), box
// {cols, box_rows}, 128-byte swizzle, zero fill out of bounds.
bool encode_rows_map(CUtensorMap* map, const void* base, uint64_t rows, uint32_t cols,
                     uint32_t box_rows);

// Loads every kernel that ce_decode_attn_score launches on the current device
// and sets their launch attributes, which that entry point otherwise does on
// its first call (defined in ce_decode.cu).  Returns a CE_* status.
int decode_prepare_device();

// The same for the selection / boundary kernels (ce_select.cu), the CSR
// kernel (ce_fill.cu) and the unit-pool kernels (ce_pool.cu).
int select_prepare_device();
int fill_prepare_device();
int pool_prepare_device();

}  // namespace host
}  // namespace ce

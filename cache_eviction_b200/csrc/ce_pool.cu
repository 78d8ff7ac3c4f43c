// Unit pool of a continuous batch: a device-resident stack of free units.
//
// The reference hands slots to requests through SGLang's token allocator: a
// decode step allocates the new token's slot, an eviction boundary returns its
// leftover slots (allocator.free_full, code/cache_eviction/
// sglang_evict_runtime.py:476-482) and a finished request returns the rest
// (release, runtime:719-742).  Here the same bookkeeping is two small kernels
// over a stack that lives on the GPU, so a decode step (including a step
// replayed from a CUDA graph) allocates without a host round trip:
//
//   ce_pool_alloc  every batch entry whose newest token starts a unit pops
//                  one unit and writes it to req_to_unit[row, pos / page];
//   ce_pool_push   returns lists of units (one list per row) to the stack.
//
// Both serve entries / rows in their batch order (ranks by a block scan), so
// which unit goes where is deterministic.  The stack is `units[0 .. top)`;
// `top` is a device int32.  An empty stack or a full one flags
// CE_EW_CAPACITY and leaves the entry unallocated (unit 0, the padding unit)
// or the unit unreturned.
#include <cuda_runtime.h>

#include "ce_common.cuh"
#include "ce_host.h"

namespace ce {
namespace pool {

constexpr int THREADS = 1024;

// Exclusive block scan of one int per thread; returns the thread's offset and
// the block total in `total`.
__device__ int block_scan(int v, int* sh, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) sh[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int s = lane < THREADS / 32 ? sh[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    if (lane < THREADS / 32) sh[lane] = s;   // inclusive warp totals
  }
  __syncthreads();
  total = sh[THREADS / 32 - 1];
  const int before = warp ? sh[warp - 1] : 0;
  __syncthreads();
  return before + x - v;
}

__global__ void __launch_bounds__(THREADS) alloc_kernel(int32_t* units, int32_t* top, int32_t* r2u,
                                                       int64_t r2u_stride, int64_t r2u_width,
                                                       const int64_t* rows, const int64_t* seq_lens, int bs,
                                                       int page, int32_t* err) {
  __shared__ int sh[THREADS / 32];
  __shared__ int base_sh;
  if (threadIdx.x == 0) base_sh = *top;
  __syncthreads();
  int base = base_sh;
  for (int b0 = 0; b0 < bs; b0 += THREADS) {
    const int b = b0 + threadIdx.x;
    int64_t row = -1, slot = -1;
    if (b < bs) {
      const int64_t pos = seq_lens[b] - 1;   // the newest token
      if (pos >= 0 && pos % page == 0) {
        row = rows[b];
        slot = pos / page;
      }
    }
    int total = 0;
    const int rank = block_scan(slot >= 0 ? 1 : 0, sh, total);
    if (slot >= 0) {
      const int at = base - 1 - rank;       // pops from the top, batch order
      if (at < 0 || slot >= r2u_width) {
        flag_error(err, CE_EW_CAPACITY);
        if (slot < r2u_width) r2u[row * r2u_stride + slot] = 0;
      } else {
        r2u[row * r2u_stride + slot] = units[at];
      }
    }
    base = max(0, base - total);
  }
  if (threadIdx.x == 0) *top = base;
}

__global__ void __launch_bounds__(THREADS) push_kernel(int32_t* units, int32_t* top, int64_t capacity,
                                                      const int32_t* lists, const int32_t* counts,
                                                      int64_t count_stride, int nrows, int64_t stride,
                                                      int32_t* err) {
  __shared__ int base_sh;
  if (threadIdx.x == 0) base_sh = *top;
  __syncthreads();
  int64_t base = base_sh;
  for (int r = 0; r < nrows; ++r) {
    const int n = max(0, counts[r * count_stride]);
    if (n > stride) {
      if (threadIdx.x == 0) flag_error(err, CE_EW_SHAPE);
      continue;
    }
    for (int i = threadIdx.x; i < n; i += THREADS) {
      const int64_t at = base + i;
      if (at < capacity)
        units[at] = lists[r * stride + i];
      else
        flag_error(err, CE_EW_CAPACITY);
    }
    base = base + n < capacity ? base + n : capacity;
  }
  __syncthreads();
  if (threadIdx.x == 0) *top = static_cast<int32_t>(base);
}

}  // namespace pool
}  // namespace ce

using namespace ce;

int ce::host::pool_prepare_device() {
  cudaFuncAttributes a;
  if (cudaFuncGetAttributes(&a, pool::alloc_kernel) != cudaSuccess ||
      cudaFuncGetAttributes(&a, pool::push_kernel) != cudaSuccess)
    return host::fail_cuda("unit pool kernels: set-up");
  return CE_OK;
}

extern "C" int ce_pool_alloc(int32_t* units, int32_t* top, int32_t* req_to_unit, int64_t r2u_stride,
                             int64_t r2u_width, const int64_t* rows, const int64_t* seq_lens, int32_t bs,
                             int32_t page_size, int32_t* err, void* stream) {
  if (bs < 0 || page_size <= 0 || r2u_width < 0) return host::fail(CE_ERR_ARG, "ce_pool_alloc: bad sizes");
  if (bs == 0) return CE_OK;
  if (!units || !top || !req_to_unit || !rows || !seq_lens) return host::fail(CE_ERR_ARG, "ce_pool_alloc: null pointer");
  pool::alloc_kernel<<<1, pool::THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      units, top, req_to_unit, r2u_stride, r2u_width, rows, seq_lens, bs, page_size, err);
  if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("ce_pool_alloc launch");
  return CE_OK;
}

extern "C" int ce_pool_push(int32_t* units, int32_t* top, int64_t capacity, const int32_t* lists,
                            int64_t list_stride, const int32_t* counts, int64_t count_stride, int32_t nrows,
                            int32_t* err, void* stream) {
  if (nrows < 0 || capacity < 0 || list_stride < 0) return host::fail(CE_ERR_ARG, "ce_pool_push: bad sizes");
  if (nrows == 0) return CE_OK;
  if (!units || !top || !lists || !counts) return host::fail(CE_ERR_ARG, "ce_pool_push: null pointer");
  pool::push_kernel<<<1, pool::THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      units, top, capacity, lists, counts, count_stride, nrows, list_stride, err);
  if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("ce_pool_push launch");
  return CE_OK;
}

// K4: ragged CSR page table for full-attention decode.
//
// Same contract as the overlay's fill (code/cache_eviction/sglang_evict_runtime.py:136-152):
// each batch entry reads its compacted residents table[row, :count] and then its
// tail req_to_unit[row, frontier:ceil(len/page)], so every KV head reads one index
// list.  One block per batch entry; the entry's offset is the sum of the lengths
// of the entries before it (a block reduction), so the whole build is one launch
// with no host round trip and can be captured in a CUDA graph.
#include <cuda_runtime.h>

#include "ce_common.cuh"
#include "ce_host.h"

namespace ce {
namespace fill {

constexpr int THREADS = 256;

struct Params {
  const int32_t* table;
  int64_t table_stride;
  const int32_t* r2u;
  int64_t r2u_stride;
  const int32_t* frontier;
  const int32_t* count;
  const int64_t* rows;
  const int64_t* seq_lens;
  int bs, page;
  int32_t* indptr;
  void* indices;
  int idx64;
  int64_t capacity;
  int32_t* tokens;
  int32_t* err;
};

__device__ __forceinline__ int64_t entry_len(const Params& p, int b) {
  const int64_t row = p.rows[b];
  const int64_t len = p.seq_lens[b];
  const int64_t units = (len + p.page - 1) / p.page;
  const int64_t tail = units - p.frontier[row];
  return static_cast<int64_t>(p.count[row]) + (tail > 0 ? tail : 0);
}

__global__ void __launch_bounds__(THREADS) fill_kernel(const Params p) {
  __shared__ int64_t red[THREADS / 32];
  const int b = blockIdx.x;
  int64_t part = 0;
  for (int i = threadIdx.x; i < b; i += THREADS) part += entry_len(p, i);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = part;
  __syncthreads();
  int64_t off = 0;
  for (int w = 0; w < THREADS / 32; ++w) off += red[w];

  const int64_t row = p.rows[b];
  const int cnt = p.count[row];
  const int fr = p.frontier[row];
  const int64_t len = p.seq_lens[b];
  const int64_t units = (len + p.page - 1) / p.page;
  const int64_t tail = units - fr > 0 ? units - fr : 0;
  if (threadIdx.x == 0) {
    if (b == 0) p.indptr[0] = 0;
    p.indptr[b + 1] = static_cast<int32_t>(off + cnt + tail);
    if (p.tokens)
      p.tokens[b] = static_cast<int32_t>(static_cast<int64_t>(cnt) * p.page + len -
                                         static_cast<int64_t>(fr) * p.page);
    if (off + cnt + tail > p.capacity) flag_error(p.err, CE_EW_CAPACITY);
  }
  const int32_t* trow = p.table + row * p.table_stride;
  const int32_t* rrow = p.r2u + row * p.r2u_stride + fr;
  const int64_t total = cnt + tail;
  for (int64_t i = threadIdx.x; i < total; i += THREADS) {
    const int64_t dst = off + i;
    if (dst >= p.capacity) break;
    const int32_t v = (i < cnt) ? trow[i] : rrow[i - cnt];
    if (p.idx64)
      static_cast<int64_t*>(p.indices)[dst] = v;
    else
      static_cast<int32_t*>(p.indices)[dst] = v;
  }
}

}  // namespace fill
}  // namespace ce

int ce::host::fill_prepare_device() {
  cudaFuncAttributes a;
  if (cudaFuncGetAttributes(&a, ce::fill::fill_kernel) != cudaSuccess) return host::fail_cuda("fill kernel: set-up");
  return CE_OK;
}

extern "C" int ce_fill(const int32_t* table, int64_t table_stride, const int32_t* req_to_unit,
                       int64_t r2u_stride, const int32_t* frontier, const int32_t* count,
                       const int64_t* rows, const int64_t* seq_lens, int32_t bs,
                       int32_t page_size, int32_t* kv_indptr, void* kv_indices,
                       int32_t indices_i64, int64_t kv_capacity, int32_t* kv_tokens,
                       int32_t* err, void* stream) {
  using namespace ce;
  if (bs < 0 || page_size <= 0 || kv_capacity < 0) return host::fail(CE_ERR_ARG, "bad size");
  if (!kv_indptr) return host::fail(CE_ERR_ARG, "null kv_indptr");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (bs == 0) {
    if (cudaMemsetAsync(kv_indptr, 0, sizeof(int32_t), st) != cudaSuccess)
      return host::fail_cuda("ce_fill memset");
    return CE_OK;
  }
  if (!table || !req_to_unit || !frontier || !count || !rows || !seq_lens || !kv_indices)
    return host::fail(CE_ERR_ARG, "null pointer");
  fill::Params p{table, table_stride, req_to_unit, r2u_stride, frontier, count, rows, seq_lens,
                 bs, page_size, kv_indptr, kv_indices, indices_i64, kv_capacity, kv_tokens, err};
  fill::fill_kernel<<<bs, fill::THREADS, 0, st>>>(p);
  if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("fill_kernel launch");
  return CE_OK;
}

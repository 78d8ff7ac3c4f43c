// Batch-1 mixture-of-experts GEMVs for the gpt-oss-20b-shaped decoder of
// benchmark config 2 (a model harness around the eviction path, not part of
// the reference's overlay).  The router's top-k expert ids stay on the
// device, so a whole decode step can be one CUDA graph:
//
//   ce_moe_gate_up  g[k, i] = silu(W1[e_k, i] . x) * (W1[e_k, I + i] . x)
//   ce_moe_down     x[d]   += sum_k w_k (W2[e_k, d] . g[k])
//
// W1 [E, 2I, D] and W2 [E, D, I] are bf16, row-major (a row is one output
// feature).  One warp computes one output row (both halves for gate/up) with
// 16-byte loads: the kernels stream 4 experts' weights once and are bound by
// HBM bandwidth.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "../../include/ce_model.h"
#include "ce_common.cuh"
#include "ce_host.h"

namespace ce {
namespace moe {

constexpr int WARPS = 8;
constexpr int THREADS = WARPS * 32;
constexpr int MAX_DIM = 8192;   // shared-memory copy of the input vector

__device__ __forceinline__ float dot8(const uint4 w, const uint4 v) {
  const __nv_bfloat162* a = reinterpret_cast<const __nv_bfloat162*>(&w);
  const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&v);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 fa = __bfloat1622float2(a[j]);
    const float2 fb = __bfloat1622float2(b[j]);
    s = fmaf(fa.x, fb.x, s);
    s = fmaf(fa.y, fb.y, s);
  }
  return s;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// grid: (ceil(I / WARPS), K); warp w of block (bx, k) makes row i = bx*WARPS + w of expert k.
__global__ void __launch_bounds__(THREADS) gate_up_kernel(const __nv_bfloat16* __restrict__ x,
                                                         const __nv_bfloat16* __restrict__ w1,
                                                         const int32_t* __restrict__ ids, int E, int I,
                                                         int Dm, __nv_bfloat16* __restrict__ g,
                                                         int32_t* err) {
  __shared__ __align__(16) __nv_bfloat16 xs[MAX_DIM];
  const int k = blockIdx.y;
  const int chunks = Dm / 8;
  for (int c = threadIdx.x; c < chunks; c += THREADS)
    reinterpret_cast<uint4*>(xs)[c] = reinterpret_cast<const uint4*>(x)[c];
  __syncthreads();
  const int e = ids[k];
  if (e < 0 || e >= E) {
    if (threadIdx.x == 0) flag_error(err, CE_EW_INDEX);
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i = blockIdx.x * WARPS + warp;
  if (i >= I) return;
  const uint4* gate = reinterpret_cast<const uint4*>(w1 + (static_cast<int64_t>(e) * 2 * I + i) * Dm);
  const uint4* up = reinterpret_cast<const uint4*>(w1 + (static_cast<int64_t>(e) * 2 * I + I + i) * Dm);
  const uint4* xv = reinterpret_cast<const uint4*>(xs);
  float sg = 0.f, su = 0.f;
#pragma unroll 4
  for (int c = lane; c < chunks; c += 32) {
    const uint4 a = gate[c], b = up[c], v = xv[c];
    sg += dot8(a, v);
    su += dot8(b, v);
  }
  sg = warp_sum(sg);
  su = warp_sum(su);
  if (lane == 0) {
    const float act = sg / (1.f + __expf(-sg));
    g[static_cast<int64_t>(k) * I + i] = __float2bfloat16_rn(act * su);
  }
}

// grid: ceil(Dm / WARPS); warp w of block bx makes output d = bx*WARPS + w over all K experts.
__global__ void __launch_bounds__(THREADS) down_kernel(const __nv_bfloat16* __restrict__ g,
                                                      const __nv_bfloat16* __restrict__ w2,
                                                      const int32_t* __restrict__ ids,
                                                      const float* __restrict__ wk, int K, int E, int I,
                                                      int Dm, __nv_bfloat16* __restrict__ x, int32_t* err) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int d = blockIdx.x * WARPS + warp;
  if (d >= Dm) return;
  const int chunks = I / 8;
  float acc = 0.f;
  for (int k = 0; k < K; ++k) {
    const int e = ids[k];
    if (e < 0 || e >= E) {
      if (lane == 0 && d == 0) flag_error(err, CE_EW_INDEX);
      continue;
    }
    const uint4* row = reinterpret_cast<const uint4*>(w2 + (static_cast<int64_t>(e) * Dm + d) * I);
    const uint4* gv = reinterpret_cast<const uint4*>(g + static_cast<int64_t>(k) * I);
    float s = 0.f;
#pragma unroll 4
    for (int c = lane; c < chunks; c += 32) s += dot8(row[c], gv[c]);
    acc += wk[k] * warp_sum(s);
  }
  if (lane == 0) x[d] = __float2bfloat16_rn(__bfloat162float(x[d]) + acc);
}

}  // namespace moe
}  // namespace ce

using namespace ce;

extern "C" int ce_moe_gate_up(const void* x, const void* w1, const int32_t* ids, int32_t num_experts_chosen,
                              int32_t num_experts, int32_t inter, int32_t dim, void* g, int32_t* err,
                              void* stream) {
  if (num_experts_chosen <= 0 || num_experts <= 0 || inter <= 0 || dim <= 0)
    return host::fail(CE_ERR_ARG, "ce_moe_gate_up: bad sizes");
  if (dim % 8 || dim > moe::MAX_DIM) return host::fail(CE_ERR_UNSUPPORTED, "ce_moe_gate_up: dim must be a multiple of 8, <= 8192");
  if (!x || !w1 || !ids || !g) return host::fail(CE_ERR_ARG, "ce_moe_gate_up: null pointer");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w1)) & 15)
    return host::fail(CE_ERR_ARG, "ce_moe_gate_up: x and w1 must be 16-byte aligned");
  dim3 grid((inter + moe::WARPS - 1) / moe::WARPS, num_experts_chosen);
  moe::gate_up_kernel<<<grid, moe::THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w1), ids, num_experts, inter, dim,
      static_cast<__nv_bfloat16*>(g), err);
  if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("ce_moe_gate_up launch");
  return CE_OK;
}

extern "C" int ce_moe_down(const void* g, const void* w2, const int32_t* ids, const float* weights,
                           int32_t num_experts_chosen, int32_t num_experts, int32_t inter, int32_t dim, void* x,
                           int32_t* err, void* stream) {
  if (num_experts_chosen <= 0 || num_experts <= 0 || inter <= 0 || dim <= 0)
    return host::fail(CE_ERR_ARG, "ce_moe_down: bad sizes");
  if (inter % 8) return host::fail(CE_ERR_UNSUPPORTED, "ce_moe_down: inter must be a multiple of 8");
  if (!g || !w2 || !ids || !weights || !x) return host::fail(CE_ERR_ARG, "ce_moe_down: null pointer");
  if ((reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(w2)) & 15)
    return host::fail(CE_ERR_ARG, "ce_moe_down: g and w2 must be 16-byte aligned");
  moe::down_kernel<<<(dim + moe::WARPS - 1) / moe::WARPS, moe::THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(g), static_cast<const __nv_bfloat16*>(w2), ids, weights, num_experts_chosen,
      num_experts, inter, dim, static_cast<__nv_bfloat16*>(x), err);
  if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("ce_moe_down launch");
  return CE_OK;
}

// K5 (prefill / extend H2O scores) for sm_100a.
//
// Follows the reference's scoring of a prefill chunk: after_extend
// (code/cache_eviction/sglang_evict_runtime.py:277-311) calls _prefill_scores
// (:327-340), which builds the row's key list as prefix ++ new slots, masks
// causally by list index (key_pos = arange(total), query_pos = prefix + i,
// :334-336) and takes the exact softmax with the sink in the normalizer from
// _probabilities (:314-324):
//
//   p[g, j, i, t] = exp(scale * q_i,h . k_t - logaddexp(logsumexp_t(...), sink_h)),
//   h = g * 8 + j,
//   score[g, slot(t)] += sum_i (sum_j p  (mode 1)  or  max_j p  (mode 2)).
//
// At page granularity a unit's score is the sum over its tokens, which is the
// reference's token-slot score summed over the page.
//
// The work is two tensor-core passes over S = Q K^T per (batch entry, KV head)
// with mma.sync m16n8k16 (bf16 in, fp32 accumulate); rows of S are
// (query, head-in-group) pairs so the 8 query heads that share a KV head share
// every K fragment:
//   lse_kernel     CTA = 32 queries x 8 heads (256 rows), K streamed in
//                  64-key tiles through a cp.async double buffer; online
//                  log2-domain logsumexp per row, folded with the sink, into a
//                  [total_q, H] workspace.
//   colsum_kernel  CTA = 256 keys (64 per warp, held as B fragments in
//                  registers); Q streamed in 8-query blocks through a cp.async
//                  double buffer; p = exp2(s - lse) reduced over the group's
//                  heads (sum or max) and summed over queries in registers, so
//                  every column total is formed inside one warp and written
//                  once per unit without atomics.
// Both passes spend one exp2 per (row, key), so the kernel is bounded by the
// SFU exp2 rate as much as by the tensor pipe.

#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include "ce_common.cuh"
#include "ce_host.h"

namespace ce {
namespace prefill {

constexpr int D = 64;
constexpr int GROUP = 8;
constexpr float LOG2E = 1.4426950408889634f;

constexpr int KT = 64;            // keys per K tile (both passes)
constexpr int L_THREADS = 256;    // lse_kernel: 8 warps x 32 rows
constexpr int L_QT = 32;          // queries per lse CTA
constexpr int C_THREADS = 128;    // colsum_kernel: 4 warps x 64 keys
constexpr int C_KT = 256;         // keys per colsum CTA
constexpr int C_QB = 8;           // queries per Q block (4 m-tiles of 2 queries)
constexpr int TILE_BYTES = KT * D * 2;         // 8 KB: 64 rows of 128 B
constexpr int C_SMEM = 4 * TILE_BYTES + 2 * TILE_BYTES + 2 * C_QB * GROUP * 4;
constexpr int L_SMEM = L_QT * GROUP * 128 + 2 * TILE_BYTES;   // 48 KB

struct Params {
  const __nv_bfloat16* q;
  int64_t q_st, q_sh;
  const __nv_bfloat16* k;
  int64_t pool_units;
  const int32_t* qo_indptr;
  const int32_t* kv_indptr;
  const int32_t* kv_indices;
  const int32_t* kv_tokens;
  const float* sinks;
  const int32_t* mode_of_row;
  const int64_t* rows;
  float scale2;   // sm_scale * log2(e)
  int H, G, P, zero_new;
  float* scores;
  int64_t score_sg;
  float* lse2;    // [total_q, H] log2-domain normalizer incl. sink
  int total_q, max_q, max_tokens;
  int64_t kv_capacity;
  int32_t* err;
};

// Entry b's query range [qbeg, qbeg + nq) and key list (ntok tokens starting
// at kv_indices[list0]) must lie inside the arrays the caller sized; otherwise
// CE_EW_SHAPE and the entry is skipped.
__device__ __forceinline__ bool entry_ok(const Params& p, int b, int& qbeg, int& nq, int& ntok,
                                         int& list0) {
  qbeg = p.qo_indptr[b];
  nq = p.qo_indptr[b + 1] - qbeg;
  ntok = p.kv_tokens[b];
  list0 = p.kv_indptr[b];
  const int64_t units = (static_cast<int64_t>(ntok) + p.P - 1) / p.P;
  const bool ok = qbeg >= 0 && nq >= 0 && qbeg + static_cast<int64_t>(nq) <= p.total_q &&
                  nq <= p.max_q && ntok <= p.max_tokens &&
                  ntok >= nq && list0 >= 0 && list0 + units <= p.kv_capacity &&
                  units <= p.kv_indptr[b + 1] - list0;
  if (!ok && threadIdx.x == 0 && blockIdx.x == 0) flag_error(p.err, CE_EW_SHAPE);
  return ok;
}

__device__ __forceinline__ int entry_mode(const Params& p, int b) {
  if (!p.mode_of_row) return CE_MODE_NONE;
  return p.mode_of_row[p.rows ? p.rows[b] : b];
}

// 128-byte rows of eight 16-byte chunks; chunk c of row r lives at c ^ (r & 7)
// so the 8 rows an ldmatrix phase reads fall in 8 different bank groups.
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return static_cast<uint32_t>((r * 8 + (c ^ (r & 7))) * 16);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;  // 0: zero-fill, nothing read
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Address of chunk c (8 elements) of list token t of entry b, head g; nullptr
// (and CE_EW_INDEX) for a unit outside the pool.
__device__ __forceinline__ const __nv_bfloat16* key_chunk(const Params& p, int list0, int t, int g,
                                                          int c) {
  const int unit = p.kv_indices[list0 + t / p.P];
  if (unit < 0 || unit >= p.pool_units) {
    flag_error(p.err, CE_EW_INDEX);
    return nullptr;
  }
  return p.k + ((static_cast<int64_t>(unit) * p.G + g) * p.P + t % p.P) * D + c * 8;
}

// Stage keys [t0, t0 + rows) of (b, g) into a swizzled tile; tokens at or
// past ntok are zero-filled.  `nthreads` threads cooperate from `tid`.
__device__ __forceinline__ void load_keys(const Params& p, uint32_t tile, int list0, int ntok, int t0,
                                          int rows, int g, int tid, int nthreads) {
  for (int id = tid; id < rows * 8; id += nthreads) {
    const int r = id >> 3, c = id & 7;
    const int t = t0 + r;
    const __nv_bfloat16* src = (t < ntok) ? key_chunk(p, list0, t, g, c) : nullptr;
    cp_async16(tile + swz(r, c), src ? static_cast<const void*>(src) : static_cast<const void*>(p.k),
               src != nullptr);
  }
}

__device__ __forceinline__ uint32_t ld_u32(const __nv_bfloat16* a) {
  return *reinterpret_cast<const uint32_t*>(a);
}

// ---------------------------------------------------------------- pass 1
// Row r of m-tile mt of warp w: query q0 + 4w + 2mt + (r >> 3), head g*8 + (r & 7).
__global__ void __launch_bounds__(L_THREADS, 2) lse_kernel(const Params p) {
  const int b = blockIdx.z, g = blockIdx.y;
  const int mode = entry_mode(p, b);
  if (mode != CE_MODE_SUM && mode != CE_MODE_MAX) return;
  int qbeg, nq, ntok, list0;
  if (!entry_ok(p, b, qbeg, nq, ntok, list0)) return;
  const int q0 = blockIdx.x * L_QT;
  if (q0 >= nq) return;
  const int prefix = ntok - nq;
  const int kend = prefix + min(nq - 1, q0 + L_QT - 1) + 1;  // keys [0, kend) are visible to some row
  const int ntiles = (kend + KT - 1) / KT;

  // Q rows of the CTA (32 queries x 8 heads, row = 8 * query + head) and a
  // double-buffered K tile, all swizzled 128-byte rows.
  extern __shared__ __align__(128) uint8_t lsm_dyn[];
  const uint32_t qs = smem_addr(lsm_dyn);
  const uint32_t kb0 = qs + L_QT * GROUP * 128, kb1 = kb0 + TILE_BYTES;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int quad = lane >> 2, qc = lane & 3;

  for (int id = threadIdx.x; id < L_QT * GROUP * 8; id += L_THREADS) {
    const int r = id >> 3, c = id & 7;
    const int q = q0 + (r >> 3);
    const bool v = q < nq;
    cp_async16(qs + swz(r, c),
               p.q + (qbeg + (v ? q : 0)) * p.q_st + (g * GROUP + (r & 7)) * p.q_sh + c * 8, v);
  }
  int qrow[2][2];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) qrow[mt][hf] = q0 + warp * 4 + mt * 2 + hf;

  float m[2][2], l[2][2];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      m[mt][hf] = -INFINITY;
      l[mt][hf] = 0.f;
    }

  load_keys(p, kb0, list0, ntok, 0, KT, g, threadIdx.x, L_THREADS);
  cp_async_commit();  // group 0: Q rows + K tile 0
  for (int it = 0; it < ntiles; ++it) {
    if (it + 1 < ntiles) {
      load_keys(p, (it & 1) ? kb0 : kb1, list0, ntok, (it + 1) * KT, KT, g, threadIdx.x, L_THREADS);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint32_t kb = (it & 1) ? kb1 : kb0;
    float acc[2][8][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[mt][n][e] = 0.f;
#pragma unroll
    for (int k2 = 0; k2 < 2; ++k2) {
      // A fragments of both m-tiles for k-steps 2*k2 and 2*k2 + 1.
      uint32_t a[2][2][4];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int h = 0; h < 2; ++h)
          ldsm_x4(qs + swz(warp * 32 + mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8,
                           (2 * k2 + h) * 2 + (lane >> 4)),
                  a[mt][h][0], a[mt][h][1], a[mt][h][2], a[mt][h][3]);
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kb + swz(n * 8 + (lane & 7), k2 * 4 + (lane >> 3)), b0, b1, b2, b3);
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          mma_16816_full(acc[mt][n], a[mt][0][0], a[mt][0][1], a[mt][0][2], a[mt][0][3], b0, b1);
          mma_16816_full(acc[mt][n], a[mt][1][0], a[mt][1][1], a[mt][1][2], a[mt][1][3], b2, b3);
        }
      }
    }
    const int kbase = it * KT;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int lim = min(prefix + qrow[mt][hf], ntok - 1);  // last visible list token
        float mx = -INFINITY;
#pragma unroll
        for (int n = 0; n < 8; ++n)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int key = kbase + n * 8 + qc * 2 + e;
            float& v = acc[mt][n][hf * 2 + e];
            v = (key <= lim) ? v * p.scale2 : -INFINITY;
            mx = fmaxf(mx, v);
          }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mn = fmaxf(m[mt][hf], mx);
        if (mn == -INFINITY) continue;  // nothing visible yet (uniform over the quad)
        float sum = 0.f;
#pragma unroll
        for (int n = 0; n < 8; ++n)
#pragma unroll
          for (int e = 0; e < 2; ++e) sum += exp2f(acc[mt][n][hf * 2 + e] - mn);
        l[mt][hf] = l[mt][hf] * exp2f(m[mt][hf] - mn) + sum;
        m[mt][hf] = mn;
      }
    }
    __syncthreads();  // the next iteration refills the buffer just read
  }

#pragma unroll
  for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      float lt = l[mt][hf];
      lt += __shfl_xor_sync(0xffffffffu, lt, 1);
      lt += __shfl_xor_sync(0xffffffffu, lt, 2);
      const int q = qrow[mt][hf];
      if (qc != 0 || q >= nq) continue;
      const int h = g * GROUP + quad;
      float lse = m[mt][hf] + log2f(lt);
      if (p.sinks) {
        const float s2 = p.sinks[h] * LOG2E;
        const float mxs = fmaxf(lse, s2);
        lse = mxs + log2f(exp2f(lse - mxs) + exp2f(s2 - mxs));
      }
      p.lse2[static_cast<int64_t>(qbeg + q) * p.H + h] = lse;
    }
  }
}

// ---------------------------------------------------------------- pass 2
__global__ void __launch_bounds__(C_THREADS) colsum_kernel(const Params p) {
  const int b = blockIdx.z, g = blockIdx.y;
  const int mode = entry_mode(p, b);
  if (mode != CE_MODE_SUM && mode != CE_MODE_MAX) return;
  int qbeg, nq, ntok, list0;
  if (!entry_ok(p, b, qbeg, nq, ntok, list0)) return;
  const int prefix = ntok - nq;
  const int k0 = blockIdx.x * C_KT;
  if (nq <= 0 || k0 >= ntok) return;

  extern __shared__ __align__(128) uint8_t dyn[];
  uint8_t* ksm = dyn;                                  // 4 x 8 KB, one 64-key slice per warp
  uint8_t* qsm = dyn + 4 * TILE_BYTES;                 // 2 x 8 KB Q blocks (64 rows)
  float* lsm = reinterpret_cast<float*>(qsm + 2 * TILE_BYTES);  // 2 x 64 row normalizers
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int quad = lane >> 2, qc = lane & 3;
  const int kw = k0 + warp * KT;                       // this warp's first key

  const int qfirst = max(0, k0 - prefix);              // first query that sees key k0
  const int nblk = (nq - qfirst + C_QB - 1) / C_QB;
  const uint32_t kbase = smem_addr(ksm), qb0 = smem_addr(qsm), qb1 = qb0 + TILE_BYTES;

  auto load_q = [&](int blk, uint32_t dst, float* ldst) {
    const int qb = qfirst + blk * C_QB;
    for (int id = threadIdx.x; id < C_QB * GROUP * 8; id += C_THREADS) {
      const int r = id >> 3, c = id & 7;
      const int q = qb + (r >> 3);
      const bool v = q < nq;
      const __nv_bfloat16* src =
          p.q + (qbeg + (v ? q : 0)) * p.q_st + (g * GROUP + (r & 7)) * p.q_sh + c * 8;
      cp_async16(dst + swz(r, c), src, v);
    }
    if (threadIdx.x < C_QB * GROUP) {
      const int r = threadIdx.x, q = qb + (r >> 3);
      ldst[r] = (q < nq) ? p.lse2[static_cast<int64_t>(qbeg + q) * p.H + g * GROUP + (r & 7)]
                         : INFINITY;
    }
  };

  load_keys(p, kbase, list0, ntok, k0, C_KT, g, threadIdx.x, C_THREADS);
  load_q(0, qb0, lsm);
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();

  // B fragments of this warp's 64 keys: [n-tile][k-step][2].
  uint32_t bf[8][4][2];
  const uint32_t kt = kbase + warp * TILE_BYTES;
#pragma unroll
  for (int n = 0; n < 8; ++n)
#pragma unroll
    for (int k2 = 0; k2 < 2; ++k2)
      ldsm_x4(kt + swz(n * 8 + (lane & 7), k2 * 4 + (lane >> 3)), bf[n][2 * k2][0], bf[n][2 * k2][1],
              bf[n][2 * k2 + 1][0], bf[n][2 * k2 + 1][1]);

  float col[8][2];
#pragma unroll
  for (int n = 0; n < 8; ++n) col[n][0] = col[n][1] = 0.f;

  for (int blk = 0; blk < nblk; ++blk) {
    const uint32_t qcur = (blk & 1) ? qb1 : qb0;
    const float* lcur = lsm + (blk & 1) * C_QB * GROUP;
    if (blk + 1 < nblk) {
      load_q(blk + 1, (blk & 1) ? qb0 : qb1, lsm + ((blk + 1) & 1) * C_QB * GROUP);
      cp_async_commit();
    }
    const int qb = qfirst + blk * C_QB;
#pragma unroll 1
    for (int mt = 0; mt < 4; ++mt) {
      uint32_t a[4][4];
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        ldsm_x4(qcur + swz(mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, kk * 2 + (lane >> 4)),
                a[kk][0], a[kk][1], a[kk][2], a[kk][3]);
      float acc[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_16816_full(acc[n], a[kk][0], a[kk][1], a[kk][2], a[kk][3], bf[n][kk][0], bf[n][kk][1]);
      }
      const int qa = qb + mt * 2;
      const float l0 = lcur[mt * 16 + quad], l1 = lcur[mt * 16 + 8 + quad];
      const int lim0 = (qa < nq) ? min(prefix + qa, ntok - 1) : -1;
      const int lim1 = (qa + 1 < nq) ? min(prefix + qa + 1, ntok - 1) : -1;
      const bool full = kw + KT - 1 <= lim0;  // both rows see every key of the slice
#pragma unroll
      for (int n = 0; n < 8; ++n) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = kw + n * 8 + qc * 2 + e;
          float p0 = exp2f(fmaf(acc[n][e], p.scale2, -l0));
          float p1 = exp2f(fmaf(acc[n][2 + e], p.scale2, -l1));
          if (!full) {
            p0 = (key <= lim0) ? p0 : 0.f;
            p1 = (key <= lim1) ? p1 : 0.f;
          }
          if (mode == CE_MODE_SUM) {
            col[n][e] += p0 + p1;
          } else {
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
              p0 = fmaxf(p0, __shfl_xor_sync(0xffffffffu, p0, o));
              p1 = fmaxf(p1, __shfl_xor_sync(0xffffffffu, p1, o));
            }
            col[n][e] += p0 + p1;
          }
        }
      }
    }
    if (blk + 1 < nblk) cp_async_wait<0>();
    __syncthreads();  // next Q block landed; the block just read may be refilled
  }

  if (mode == CE_MODE_SUM) {
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 2; ++e)
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) col[n][e] += __shfl_xor_sync(0xffffffffu, col[n][e], o);
  }
  // Column totals of this warp's 64 keys -> its K slice's shared memory (no
  // longer needed), then per-unit sums.
  float* tot = reinterpret_cast<float*>(ksm + warp * TILE_BYTES);
  __syncwarp();
  if (quad == 0) {
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 2; ++e) tot[n * 8 + qc * 2 + e] = col[n][e];
  }
  __syncwarp();
  const int per = KT / p.P;  // units in this warp's slice
  for (int j = lane; j < per; j += 32) {
    const int t = kw + j * p.P;  // first token of the unit
    if (t >= ntok) continue;
    float s = 0.f;
    for (int x = 0; x < p.P; ++x) s += tot[j * p.P + x];
    const int unit = p.kv_indices[list0 + t / p.P];
    if (unit < 0 || unit >= p.pool_units) {
      flag_error(p.err, CE_EW_INDEX);
      continue;
    }
    float* sp = p.scores + static_cast<int64_t>(g) * p.score_sg + unit;
    *sp = (p.zero_new && t >= prefix) ? s : *sp + s;
  }
}

}  // namespace prefill
}  // namespace ce

using namespace ce;

extern "C" int64_t ce_prefill_workspace_bytes(int32_t total_q, int32_t num_q_heads) {
  if (total_q < 0 || num_q_heads <= 0) return -1;
  return static_cast<int64_t>(total_q > 0 ? total_q : 1) * num_q_heads * 4 + 256;
}

extern "C" int ce_prefill_scores(const void* q, int64_t q_st, int64_t q_sh, const void* k_pool,
                                 int64_t pool_units, const int32_t* qo_indptr,
                                 const int32_t* kv_indptr, const int32_t* kv_indices,
                                 const int32_t* kv_tokens, int64_t kv_capacity, const float* sinks,
                                 const int32_t* mode_of_row, const int64_t* rows, float sm_scale,
                                 int32_t bs, int32_t num_q_heads, int32_t num_kv_heads,
                                 int32_t head_dim, int32_t page_size, int32_t total_q,
                                 int32_t max_q, int32_t max_tokens, float* scores,
                                 int64_t score_sg, int32_t zero_new, void* workspace,
                                 int64_t workspace_bytes, int32_t* err, void* stream) {
  using namespace ce::prefill;
  if (bs < 0 || total_q < 0 || max_q < 0 || max_tokens < 0 || pool_units <= 0 || kv_capacity < 0)
    return host::fail(CE_ERR_ARG, "ce_prefill_scores: negative size");
  if (head_dim != D || num_kv_heads <= 0 || num_q_heads != GROUP * num_kv_heads)
    return host::fail(CE_ERR_UNSUPPORTED, "ce_prefill_scores: needs head_dim 64 and 8 query heads per KV head");
  if (page_size <= 0 || page_size > KT || KT % page_size != 0)
    return host::fail(CE_ERR_UNSUPPORTED, "ce_prefill_scores: page_size must divide 64");
  if (q_sh % 8 != 0 || q_st % 8 != 0 || q_sh < D || q_st < static_cast<int64_t>(num_q_heads) * q_sh)
    return host::fail(CE_ERR_ARG, "ce_prefill_scores: q strides must be multiples of 8 elements");
  if (bs == 0 || max_q == 0 || mode_of_row == nullptr || total_q == 0) return CE_OK;
  if (!q || !k_pool || !qo_indptr || !kv_indptr || !kv_indices || !kv_tokens || !scores)
    return host::fail(CE_ERR_ARG, "ce_prefill_scores: null pointer");
  if (score_sg < pool_units)
    return host::fail(CE_ERR_ARG, "ce_prefill_scores: score head stride below pool_units");
  if (bs > 65535) return host::fail(CE_ERR_UNSUPPORTED, "ce_prefill_scores: more than 65535 entries");
  const int64_t need = ce_prefill_workspace_bytes(total_q, num_q_heads);
  if (!workspace || workspace_bytes < need)
    return host::fail(CE_ERR_WORKSPACE, "ce_prefill_scores: workspace too small");
  if ((reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(k_pool) & 15) ||
      (reinterpret_cast<uintptr_t>(workspace) & 15))
    return host::fail(CE_ERR_ARG, "ce_prefill_scores: q, k_pool and workspace need 16-byte alignment");

  Params p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_st = q_st;
  p.q_sh = q_sh;
  p.k = static_cast<const __nv_bfloat16*>(k_pool);
  p.pool_units = pool_units;
  p.qo_indptr = qo_indptr;
  p.kv_indptr = kv_indptr;
  p.kv_indices = kv_indices;
  p.kv_tokens = kv_tokens;
  p.sinks = sinks;
  p.mode_of_row = mode_of_row;
  p.rows = rows;
  p.scale2 = sm_scale * LOG2E;
  p.H = num_q_heads;
  p.G = num_kv_heads;
  p.P = page_size;
  p.zero_new = zero_new ? 1 : 0;
  p.scores = scores;
  p.score_sg = score_sg;
  p.lse2 = static_cast<float*>(workspace);
  p.total_q = total_q;
  p.max_q = max_q;
  p.max_tokens = max_tokens;
  p.kv_capacity = kv_capacity;
  p.err = err;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 g1((max_q + L_QT - 1) / L_QT, num_kv_heads, bs);
  if (!host::set_smem(lse_kernel, L_SMEM)) return host::fail(CE_ERR_CUDA, "prefill smem attr");
  lse_kernel<<<g1, L_THREADS, L_SMEM, st>>>(p);
  if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("prefill lse_kernel");
  if (max_tokens == 0) return CE_OK;
  if (!host::set_smem(colsum_kernel, C_SMEM)) return host::fail(CE_ERR_CUDA, "prefill smem attr");
  const dim3 g2((max_tokens + C_KT - 1) / C_KT, num_kv_heads, bs);
  colsum_kernel<<<g2, C_THREADS, C_SMEM, st>>>(p);
  if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("prefill colsum_kernel");
  return CE_OK;
}

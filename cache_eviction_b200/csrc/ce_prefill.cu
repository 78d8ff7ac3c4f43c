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
// Two passes over S = Q K^T per (batch entry, KV head) on the 5th-generation
// tensor cores.  Each CTA has eight epilogue warps (one TMEM lane = one row of
// the accumulator per thread, two warps per row splitting its columns), a
// load warp and an MMA warp whose elected lane
// issues tcgen05.mma into one of two 128-column TMEM accumulators while the
// epilogue drains the other:
//   lse_kernel     M = 128 rows = 16 queries x the group's 8 query heads
//                  (Q tile by TMA), N = 128 keys per step streamed through a
//                  4-stage ring; each thread keeps its row's online log2
//                  logsumexp and writes it, folded with the sink, to a
//                  [total_q, H] workspace.
//   colsum_kernel  M = 128 keys (loaded once), N = 16 queries x 8 heads per
//                  step (Q block and its 128 normalizers by TMA through the
//                  ring): D = K Q^T, so each thread owns one key and sums
//                  p = exp2(s - lse) over its row -- over all 8 heads (SUM) or
//                  the max of each query's 8 adjacent columns (MAX) -- with no
//                  cross-thread reduction; unit sums are written once, no atomics.
// Key rows come from the paged pool one page per TMA load when a page is at
// least 8 rows (1 KB); smaller pages are gathered with cp.async and published
// to the tensor cores with a proxy fence.  Every wait is bounded;
// a wait that gives up flags CE_EW_TIMEOUT, tells the other roles to stop, and
// the CTA still drains its copies and frees its tensor memory.
// Both passes spend one exp2 per (row, key): three quarters on the SFU
// (ex2.approx) and a quarter as a polynomial on the FMA pipe, which together
// bound the kernel; the tensor cores run asynchronously beside them.

#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include "ce_common.cuh"
#include "ce_host.h"

namespace ce {
namespace prefill {

constexpr int D = 64;
constexpr int GROUP = 8;
constexpr float LOG2E = 1.4426950408889634f;

constexpr int BM = 128;                  // accumulator rows (TMEM lanes)
constexpr int BN = 128;                  // accumulator columns per step
constexpr int QT = BM / GROUP;           // 16 queries per pass-1 CTA / per pass-2 step
constexpr int TILE = 128 * 128;          // a 128-row K-major bf16 tile, 128 B per row
constexpr int NS = 5;                    // ring stages
constexpr int LAG = 3;                   // cp.async key tiles in flight before one is published
constexpr int EPI_WARPS = 8;             // two per TMEM lane quarter, 64 columns each
constexpr int THREADS = 32 * (EPI_WARPS + 2);   // warps 0-7 epilogue, 8 loads, 9 MMA
constexpr int LOAD_WARP = EPI_WARPS, MMA_WARP = EPI_WARPS + 1;
constexpr uint32_t TMEM_COLS = 2 * BN;
constexpr uint32_t IDESC = f16_idesc(BM, BN);
constexpr int LSE_BLOCK = QT * GROUP * 4;  // 512 B of normalizers per pass-2 step

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
  // lost-mass pass: evicted bits [S][G][lost_words] (bit set = key evicted by
  // spec s for KV head g), lost [S][lost_stride] accumulated per query
  const uint32_t* lost_bits;
  int64_t lost_words, lost_stride;
  int S;
  float lost_scale;
  float* lost;
  int all_entries;   // run every entry regardless of its score mode
  int32_t* err;
};

constexpr int MAX_SPECS = 8;

// Barriers and flags after the tiles in shared memory.
struct Sync {
  uint64_t full[NS], empty[NS];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t once;       // Q tile (pass 1) / key tile (pass 2)
  uint64_t mma_done;
  uint32_t tmem;
  int abort;
  float part[2][BM];   // the second column half's partial results, per row
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

// Unit holding list token t of the entry, or -1 past ntok / -2 outside the pool
// (flagged).
__device__ __forceinline__ int token_unit(const Params& p, int list0, int ntok, int t) {
  if (t >= ntok) return -1;
  const int unit = p.kv_indices[list0 + t / p.P];
  if (unit >= 0 && unit < p.pool_units) return unit;
  flag_error(p.err, CE_EW_INDEX);
  return -2;
}

// page_size >= 8: keys [t0, t0 + 128) of (b, g) as 128 / P page loads by TMA
// (pool viewed as [units * G * P, 64] rows; each page lands on a 1024-byte
// boundary of the tile), completing on `bar`.  Pages past ntok are not loaded
// (their rows are masked by every reader).
__device__ __forceinline__ void tma_key_tile(const Params& p, const CUtensorMap* kmap, uint8_t* tile,
                                             uint64_t* bar, int list0, int ntok, int t0, int g,
                                             int lane) {
  const int pages = BN / p.P;
  const int unit = lane < pages ? token_unit(p, list0, ntok, t0 + lane * p.P) : -1;
  const unsigned valid = __ballot_sync(0xffffffffu, unit >= 0);
  if (lane == 0) mbar_arrive_expect_tx(bar, __popc(valid) * p.P * 128);
  __syncwarp();
  if (unit >= 0) tma_load_2d(tile + lane * p.P * 128, kmap, 0, (unit * p.G + g) * p.P, bar);
}

// page_size < 8: one warp copies keys [t0, t0 + 128) into the tile with
// cp.async (tokens past ntok zero-filled).  The 128 unit indices are read in
// one batch (lane l: rows l, l+32, l+64, l+96) and passed around by shuffles;
// lanes 8i..8i+7 then copy the eight chunks of rows i, i+4, i+8, ...
__device__ __forceinline__ void copy_key_tile(const Params& p, uint32_t tile, int list0, int ntok,
                                              int t0, int g, int lane) {
  int u[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) u[k] = token_unit(p, list0, ntok, t0 + lane + 32 * k);
  const int c = lane & 7;
#pragma unroll
  for (int j = 0; j < BM / 4; ++j) {
    const int r = (lane >> 3) + 4 * j;
    const int unit = __shfl_sync(0xffffffffu, u[j >> 3], r & 31);
    const int t = t0 + r;
    const bool ok = unit >= 0;
    const __nv_bfloat16* src =
        ok ? p.k + ((static_cast<int64_t>(unit) * p.G + g) * p.P + t % p.P) * D + c * 8 : p.k;
    cp_async16(tile + swz(r, c), src, ok);
  }
}

// Barrier of the epilogue warps only (named barrier 1).
__device__ __forceinline__ void named_barrier_epi() {
  asm volatile("bar.sync 1, %0;" ::"n"(EPI_WARPS * 32) : "memory");
}

// Initialise the barriers and allocate the two TMEM accumulators; returns the
// TMEM base address (all threads).
__device__ __forceinline__ uint32_t setup(Sync* sy, uint32_t empty_count) {
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&sy->full[s], 1);
      mbar_init(&sy->empty[s], empty_count);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sy->acc_full[b], 1);
      mbar_init(&sy->acc_empty[b], EPI_WARPS);
    }
    mbar_init(&sy->once, 1);
    mbar_init(&sy->mma_done, 1);
    sy->abort = 0;
    fence_mbar_init();
  }
  if (warp == MMA_WARP) tmem_alloc(&sy->tmem, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  return sy->tmem;
}

// MMA warp epilogue of the role loop: every issued MMA completes before the
// accumulators may be freed.
__device__ __forceinline__ void mma_drain(Sync* sy, int32_t* err, bool issued) {
  if (!issued) return;
  tc_commit(&sy->mma_done);
  mbar_wait(&sy->mma_done, 0, err);
}

__device__ __forceinline__ void teardown(Sync* sy, uint32_t tmem) {
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if ((threadIdx.x >> 5) == MMA_WARP) tmem_dealloc(tmem, TMEM_COLS);
}

// ---------------------------------------------------------------- pass 1
// CTA (query tile x, KV head g, entry b); accumulator row r = query
// 16x + r / 8, head g*8 + r % 8.
// LOST = false: row normalisers into p.lse2.  LOST = true (the lost-mass
// diagnostic, runtime:587-613): the same S tiles again with the normalisers
// known; each row sums p over the keys every spec evicted, the 8 rows of a
// query are reduced, and lost[s][query] += that sum * lost_scale.
template <bool LOST>
__global__ void __launch_bounds__(THREADS, 2) lse_kernel(const Params p,
                                                          const __grid_constant__ CUtensorMap qmap,
                                                          const __grid_constant__ CUtensorMap kmap) {
  const int b = blockIdx.z, g = blockIdx.y;
  const int mode = entry_mode(p, b);
  if (!LOST && !p.all_entries && mode != CE_MODE_SUM && mode != CE_MODE_MAX) return;
  int qbeg, nq, ntok, list0;
  if (!entry_ok(p, b, qbeg, nq, ntok, list0)) return;
  const int q0 = blockIdx.x * QT;
  if (q0 >= nq) return;
  const int prefix = ntok - nq;
  const int kend = prefix + min(nq, q0 + QT);   // keys [0, kend) are visible to some row
  const int ntiles = (kend + BN - 1) / BN;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  const uint32_t qtile = smem_addr(sm);
  const uint32_t ring = qtile + TILE;
  Sync* sy = reinterpret_cast<Sync*>(sm + TILE + NS * TILE);
  volatile int* abort = &sy->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t tmem = setup(sy, 1);

  if (warp == LOAD_WARP) {
    // ------------------------------------------------------------ loads
    if (lane == 0) {
      mbar_arrive_expect_tx(&sy->once, TILE);
      tma_load_3d(sm, &qmap, 0, g * GROUP, qbeg + q0, &sy->once);
    }
    const bool tma = p.P >= 8;
    int t = 0;
    for (; t < ntiles; ++t) {
      const int s = t % NS;
      if (t >= NS && !warp_wait(&sy->empty[s], ((t / NS) & 1) ^ 1, p.err, abort, lane)) {
        *abort = 1;
        break;
      }
      if (tma) {
        tma_key_tile(p, &kmap, sm + TILE + s * TILE, &sy->full[s], list0, ntok, t * BN, g, lane);
        continue;
      }
      copy_key_tile(p, ring + s * TILE, list0, ntok, t * BN, g, lane);
      cp_async_commit();
      if (t >= LAG) {
        cp_async_wait<LAG>();
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sy->full[(t - LAG) % NS]);
      }
    }
    if (!tma) {
      cp_async_wait<0>();
      fence_proxy_async();
      __syncwarp();
      if (lane == 0 && !*abort)
        for (int u = max(0, t - LAG); u < t; ++u) mbar_arrive(&sy->full[u % NS]);
    }
    if (lane == 0) {
      // Every issued load lands before the CTA may exit.
      if (tma)
        for (int u = max(0, t - NS); u < t; ++u) mbar_wait(&sy->full[u % NS], (u / NS) & 1, p.err);
      mbar_wait(&sy->once, 0, p.err);
    }
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------------------- MMA
    bool issued = false;
    if (lane == 0 && mbar_wait_or_abort(&sy->once, 0, p.err, abort)) {
      tc_fence_after();
      const uint64_t adesc = sw128_desc(qtile);
      for (int t = 0; t < ntiles; ++t) {
        const int s = t % NS, buf = t & 1;
        if ((t >= 2 && !mbar_wait_or_abort(&sy->acc_empty[buf], ((t >> 1) & 1) ^ 1, p.err, abort)) ||
            !mbar_wait_or_abort(&sy->full[s], (t / NS) & 1, p.err, abort)) {
          *abort = 1;
          break;
        }
        tc_fence_after();
        const uint64_t bdesc = sw128_desc(ring + s * TILE);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          tc_mma(tmem + buf * BN, adesc + 2 * kk, bdesc + 2 * kk, IDESC, kk > 0);
        tc_commit(&sy->empty[s]);
        tc_commit(&sy->acc_full[buf]);
        issued = true;
      }
    } else if (lane == 0) {
      *abort = 1;
    }
    if (lane == 0) mma_drain(sy, p.err, issued);
    __syncwarp();
  } else {
    // -------------------------------------------------------- epilogue
    // Warp e reads TMEM lanes 32 (e % 4) .. +31 (its rows), columns
    // 64 (e / 4) .. +63 of each accumulator; the two halves of a row merge at
    // the end.
    const int quarter = warp & 3, half = warp >> 2;
    const int r = quarter * 32 + lane;         // accumulator row = TMEM lane
    const int q = q0 + r / GROUP;
    const int h = g * GROUP + r % GROUP;
    const int lim = prefix + min(q, nq - 1);   // last visible list token of this row
    float m = -INFINITY, l = 0.f;
    float lost[MAX_SPECS];
    float lse_row = INFINITY;
    if constexpr (LOST) {
#pragma unroll
      for (int x = 0; x < MAX_SPECS; ++x) lost[x] = 0.f;
      if (q < nq) lse_row = p.lse2[static_cast<int64_t>(qbeg + q) * p.H + h];
    }
    for (int t = 0; t < ntiles; ++t) {
      const int buf = t & 1;
      if (!warp_wait(&sy->acc_full[buf], (t >> 1) & 1, p.err, abort, lane)) {
        *abort = 1;
        break;
      }
      tc_fence_after();
      float v[64];
      __syncwarp();  // tcgen05.ld is warp-collective
      const uint32_t taddr = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + buf * BN + half * 64;
      tmem_ld32_async(taddr, v);
      tmem_ld32_async(taddr + 32, v + 32);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sy->acc_empty[buf]);  // the values are in registers
      const int kb = t * BN + half * 64;
      if constexpr (LOST) {
        // kb is a multiple of 64: the 64 keys are two whole mask words per spec
#pragma unroll
        for (int x = 0; x < MAX_SPECS; ++x) {
          if (x >= p.S) break;
          const uint32_t* w = p.lost_bits + (static_cast<int64_t>(x) * p.G + g) * p.lost_words + kb / 32;
          const uint32_t w0 = (kb / 32 < p.lost_words) ? w[0] : 0u;
          const uint32_t w1 = (kb / 32 + 1 < p.lost_words) ? w[1] : 0u;
          if (!(w0 | w1)) continue;
          float acc = 0.f;
#pragma unroll
          for (int i = 0; i < 64; ++i) {
            const bool ev = ((i < 32 ? w0 >> i : w1 >> (i - 32)) & 1u) && kb + i <= lim;
            acc += ev ? fast_exp2(fmaf(v[i], p.scale2, -lse_row)) : 0.f;
          }
          lost[x] += acc;
        }
        continue;
      }
      if (kb + 63 > lim) {
#pragma unroll
        for (int i = 0; i < 64; ++i) v[i] = (kb + i <= lim) ? v[i] : -INFINITY;
      }
      float mx[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx[i] = v[i];
#pragma unroll
      for (int i = 8; i < 64; ++i) mx[i & 7] = fmaxf(mx[i & 7], v[i]);
      const float mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                             fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
      const float mn = fmaxf(m, mt * p.scale2);  // scale2 > 0 keeps the order
      if (mn != -INFINITY) {
        float sm4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const float a = fmaf(v[i], p.scale2, -mn);
          sm4[i & 3] += (i & 3) == 3 ? poly_exp2(a) : fast_exp2(a);
        }
        l = l * fast_exp2(m - mn) + ((sm4[0] + sm4[1]) + (sm4[2] + sm4[3]));
        m = mn;
      }
    }
    if constexpr (LOST) {
      // The 8 rows of a query are 8 consecutive lanes of this warp.
#pragma unroll
      for (int x = 0; x < MAX_SPECS; ++x) {
        if (x >= p.S) break;
        float v = lost[x];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        if ((lane & 7) == 0 && q < nq && !*abort)
          atomicAdd(p.lost + static_cast<int64_t>(x) * p.lost_stride + q, v * p.lost_scale);
      }
    }
    if (LOST || half == 1) {
      sy->part[0][r] = m;
      sy->part[1][r] = l;
    }
    named_barrier_epi();
    if (!LOST && half == 0 && !*abort && q < nq) {
      const float m1 = sy->part[0][r], l1 = sy->part[1][r];
      const float M = fmaxf(m, m1);  // finite: key 0 is in every row's first half
      const float L = l * fast_exp2(m - M) + l1 * fast_exp2(m1 - M);
      float lse = M + log2f(L);
      if (p.sinks) {
        const float s2 = p.sinks[h] * LOG2E;
        const float mxs = fmaxf(lse, s2);
        lse = mxs + log2f(exp2f(lse - mxs) + exp2f(s2 - mxs));
      }
      p.lse2[static_cast<int64_t>(qbeg + q) * p.H + h] = lse;
    }
  }
  teardown(sy, tmem);
}

// ---------------------------------------------------------------- pass 2
// CTA (key tile x, KV head g, entry b); accumulator row r = key 128x + r,
// column c of step j = query qfirst + 16j + c / 8, head g*8 + c % 8.
__global__ void __launch_bounds__(THREADS, 2) colsum_kernel(const Params p,
                                                             const __grid_constant__ CUtensorMap qmap,
                                                             const __grid_constant__ CUtensorMap lmap,
                                                             const __grid_constant__ CUtensorMap kmap) {
  const int b = blockIdx.z, g = blockIdx.y;
  const int mode = entry_mode(p, b);
  if (mode != CE_MODE_SUM && mode != CE_MODE_MAX) return;
  int qbeg, nq, ntok, list0;
  if (!entry_ok(p, b, qbeg, nq, ntok, list0)) return;
  const int prefix = ntok - nq;
  const int k0 = blockIdx.x * BM;
  if (nq <= 0 || k0 >= ntok) return;
  const int qfirst = max(0, k0 - prefix);   // first query that sees key k0
  const int nblk = (nq - qfirst + QT - 1) / QT;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  const uint32_t ktile = smem_addr(sm);
  const uint32_t ring = ktile + TILE;
  float* lring = reinterpret_cast<float*>(sm + TILE + NS * TILE);           // NS x 128
  float* tot = lring + NS * QT * GROUP;                                     // 128
  Sync* sy = reinterpret_cast<Sync*>(tot + BM);
  volatile int* abort = &sy->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t tmem = setup(sy, 1 + EPI_WARPS);   // a stage is free after its MMA and the epilogue

  if (warp == LOAD_WARP) {
    // ------------------------------------------------------------ loads
    const bool tma = p.P >= 8;
    if (tma) {
      tma_key_tile(p, &kmap, sm, &sy->once, list0, ntok, k0, g, lane);
    } else {
      copy_key_tile(p, ktile, list0, ntok, k0, g, lane);
      cp_async_commit();
    }
    int j = 0;
    for (; j < nblk; ++j) {
      const int s = j % NS;
      if (j >= NS && !warp_wait(&sy->empty[s], ((j / NS) & 1) ^ 1, p.err, abort, lane)) {
        *abort = 1;
        break;
      }
      if (lane == 0) {
        const int z = qbeg + qfirst + j * QT;
        mbar_arrive_expect_tx(&sy->full[s], TILE + LSE_BLOCK);
        tma_load_3d(sm + TILE + s * TILE, &qmap, 0, g * GROUP, z, &sy->full[s]);
        tma_load_2d(lring + s * QT * GROUP, &lmap, g * GROUP, z, &sy->full[s]);
      }
      if (j == 0 && !tma) {
        cp_async_wait<0>();
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sy->once);
      }
    }
    if (j == 0 && !tma) {  // no step issued: still publish the key tile
      cp_async_wait<0>();
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sy->once);
    }
    // Every issued load lands before the CTA may exit.
    if (lane == 0) {
      for (int u = max(0, j - NS); u < j; ++u) mbar_wait(&sy->full[u % NS], (u / NS) & 1, p.err);
      if (tma) mbar_wait(&sy->once, 0, p.err);
    }
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------------------- MMA
    bool issued = false;
    if (lane == 0 && mbar_wait_or_abort(&sy->once, 0, p.err, abort)) {
      tc_fence_after();
      const uint64_t adesc = sw128_desc(ktile);
      for (int j = 0; j < nblk; ++j) {
        const int s = j % NS, buf = j & 1;
        if ((j >= 2 && !mbar_wait_or_abort(&sy->acc_empty[buf], ((j >> 1) & 1) ^ 1, p.err, abort)) ||
            !mbar_wait_or_abort(&sy->full[s], (j / NS) & 1, p.err, abort)) {
          *abort = 1;
          break;
        }
        tc_fence_after();
        const uint64_t bdesc = sw128_desc(ring + s * TILE);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          tc_mma(tmem + buf * BN, adesc + 2 * kk, bdesc + 2 * kk, IDESC, kk > 0);
        tc_commit(&sy->empty[s]);
        tc_commit(&sy->acc_full[buf]);
        issued = true;
      }
    } else if (lane == 0) {
      *abort = 1;
    }
    if (lane == 0) mma_drain(sy, p.err, issued);
    __syncwarp();
  } else {
    // -------------------------------------------------------- epilogue
    // Warp e: TMEM lanes 32 (e % 4) .. +31 (its keys), columns 64 (e / 4) ..
    // +63 = queries 8 (e / 4) .. +7 of each step; halves merge at the end.
    const int quarter = warp & 3, half = warp >> 2;
    const int r = quarter * 32 + lane;
    const int key = k0 + r;
    float acc[2] = {0.f, 0.f};
    for (int j = 0; j < nblk; ++j) {
      const int s = j % NS, buf = j & 1;
      // The stage's normalizers came by TMA: observe its completion here too
      // (already complete once the accumulator is).
      if (!warp_wait(&sy->acc_full[buf], (j >> 1) & 1, p.err, abort, lane) ||
          !warp_wait(&sy->full[s], (j / NS) & 1, p.err, abort, lane)) {
        *abort = 1;
        break;
      }
      tc_fence_after();
      float v[64];
      __syncwarp();  // tcgen05.ld is warp-collective
      const uint32_t taddr = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + buf * BN + half * 64;
      tmem_ld32_async(taddr, v);
      tmem_ld32_async(taddr + 32, v + 32);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sy->acc_empty[buf]);  // the values are in registers
      const float* lse = lring + s * QT * GROUP + half * 64;
      const int qb = qfirst + j * QT + half * 8;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int qq = qb + u;
        const bool vis = qq < nq && key <= prefix + qq;
        const float* lq = lse + u * GROUP;
        float e[GROUP];
#pragma unroll
        for (int x = 0; x < GROUP; ++x) {
          const float a = fmaf(v[u * 8 + x], p.scale2, -lq[x]);
          e[x] = x >= 6 ? poly_exp2(a) : fast_exp2(a);   // a quarter on the FMA pipe
        }
        float red;
        if (mode == CE_MODE_SUM)
          red = ((e[0] + e[1]) + (e[2] + e[3])) + ((e[4] + e[5]) + (e[6] + e[7]));
        else
          red = fmaxf(fmaxf(fmaxf(e[0], e[1]), fmaxf(e[2], e[3])),
                      fmaxf(fmaxf(e[4], e[5]), fmaxf(e[6], e[7])));
        acc[u & 1] += vis ? red : 0.f;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sy->empty[s]);  // done with this stage's normalizers
    }
    if (half == 1) sy->part[0][r] = acc[0] + acc[1];
    named_barrier_epi();
    if (half == 0) tot[r] = (key < ntok) ? (acc[0] + acc[1]) + sy->part[0][r] : 0.f;
  }
  teardown(sy, tmem);
  if (*abort) return;
  // Per-unit sums of the CTA's 128 keys (page_size divides 128).
  const int per = BM / p.P;
  for (int u = threadIdx.x; u < per; u += THREADS) {
    const int t = k0 + u * p.P;  // first token of the unit
    if (t >= ntok) continue;
    float s = 0.f;
    for (int x = 0; x < p.P; ++x) s += tot[u * p.P + x];
    const int unit = p.kv_indices[list0 + t / p.P];
    if (unit < 0 || unit >= p.pool_units) {
      flag_error(p.err, CE_EW_INDEX);
      continue;
    }
    float* sp = p.scores + static_cast<int64_t>(g) * p.score_sg + unit;
    *sp = (p.zero_new && t >= prefix) ? s : *sp + s;
  }
}

// Dynamic shared memory: 1 KB alignment slack + tiles + barriers.
constexpr int L_SMEM = 1024 + TILE + NS * TILE + static_cast<int>(sizeof(Sync));
constexpr int C_SMEM = 1024 + TILE + NS * TILE + NS * LSE_BLOCK + BM * 4 + static_cast<int>(sizeof(Sync));
// At most two CTAs fit on an SM (2 x 256 TMEM columns = all 512): tcgen05.alloc never waits.
static_assert(3 * L_SMEM > 227 * 1024 && 3 * C_SMEM > 227 * 1024, "a third CTA per SM would oversubscribe TMEM");
static_assert(2 * C_SMEM <= 227 * 1024, "two CTAs per SM");

}  // namespace prefill
}  // namespace ce

using namespace ce;

extern "C" int64_t ce_prefill_workspace_bytes(int32_t total_q, int32_t num_q_heads) {
  if (total_q < 0 || num_q_heads <= 0) return -1;
  return static_cast<int64_t>(total_q > 0 ? total_q : 1) * num_q_heads * 4 + 256;
}

namespace {

// Validation, tensor maps and parameters shared by the two entry points.
int prefill_prepare(const void* q, int64_t q_st, int64_t q_sh, const void* k_pool, int64_t pool_units,
                    const int32_t* qo_indptr, const int32_t* kv_indptr, const int32_t* kv_indices,
                    const int32_t* kv_tokens, int64_t kv_capacity, const float* sinks,
                    const int32_t* mode_of_row, const int64_t* rows, float sm_scale, int32_t bs,
                    int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, int32_t page_size,
                    int32_t total_q, int32_t max_q, int32_t max_tokens, float* scores, int64_t score_sg,
                    int32_t zero_new, void* workspace, int64_t workspace_bytes, int32_t* err,
                    ce::prefill::Params& p, CUtensorMap& qmap, CUtensorMap& lmap, CUtensorMap& kmap) {
  using namespace ce::prefill;
  if (bs < 0 || total_q < 0 || max_q < 0 || max_tokens < 0 || pool_units <= 0 || kv_capacity < 0)
    return host::fail(CE_ERR_ARG, "ce_prefill: negative size");
  if (!(sm_scale > 0.f)) return host::fail(CE_ERR_ARG, "ce_prefill: sm_scale must be positive");
  if (head_dim != D || num_kv_heads <= 0 || num_q_heads != GROUP * num_kv_heads)
    return host::fail(CE_ERR_UNSUPPORTED, "ce_prefill: needs head_dim 64 and 8 query heads per KV head");
  if (page_size <= 0 || page_size > 64 || 64 % page_size != 0)
    return host::fail(CE_ERR_UNSUPPORTED, "ce_prefill: page_size must divide 64");
  if (q_sh % 8 != 0 || q_st % 8 != 0 || q_sh < D || q_st < static_cast<int64_t>(num_q_heads) * q_sh)
    return host::fail(CE_ERR_ARG, "ce_prefill: q strides must be multiples of 8 elements");
  if (bs == 0 || max_q == 0 || total_q == 0) return 1;   // nothing to do
  if (!q || !k_pool || !qo_indptr || !kv_indptr || !kv_indices || !kv_tokens)
    return host::fail(CE_ERR_ARG, "ce_prefill: null pointer");
  if (bs > 65535) return host::fail(CE_ERR_UNSUPPORTED, "ce_prefill: more than 65535 entries");
  if (pool_units * num_kv_heads * page_size > INT32_MAX)
    return host::fail(CE_ERR_UNSUPPORTED, "ce_prefill: pool rows exceed 2^31");
  const int64_t need = ce_prefill_workspace_bytes(total_q, num_q_heads);
  if (!workspace || workspace_bytes < need)
    return host::fail(CE_ERR_WORKSPACE, "ce_prefill: workspace too small");
  if ((reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(k_pool) & 15) ||
      (reinterpret_cast<uintptr_t>(workspace) & 15))
    return host::fail(CE_ERR_ARG, "ce_prefill: q, k_pool and workspace need 16-byte alignment");
  {
    // Q as [total_q][H][64] with byte strides; box = 16 queries x 8 heads x 64.
    const uint64_t dims[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(num_q_heads),
                              static_cast<uint64_t>(total_q)};
    const uint64_t strides[2] = {static_cast<uint64_t>(q_sh) * 2, static_cast<uint64_t>(q_st) * 2};
    const uint32_t box[3] = {static_cast<uint32_t>(D), GROUP, QT};
    if (!host::encode_map(&qmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, q, dims, strides, box, true))
      return host::fail(CE_ERR_CUDA, "ce_prefill: query tensor map");
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(num_q_heads), static_cast<uint64_t>(total_q)};
    const uint64_t strides[1] = {static_cast<uint64_t>(num_q_heads) * 4};
    const uint32_t box[2] = {GROUP, QT};
    if (!host::encode_map(&lmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, workspace, dims, strides, box, false))
      return host::fail(CE_ERR_CUDA, "ce_prefill: normalizer tensor map");
  }
  // K pool as [units * G * page, 64] rows; box = one page of one head.
  if (!host::encode_rows_map(&kmap, k_pool, static_cast<uint64_t>(pool_units) * num_kv_heads * page_size,
                             D, static_cast<uint32_t>(page_size)))
    return host::fail(CE_ERR_CUDA, "ce_prefill: key tensor map");
  p = Params{};
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
  if (!host::set_smem(lse_kernel<false>, L_SMEM) || !host::set_smem(lse_kernel<true>, L_SMEM) ||
      !host::set_smem(colsum_kernel, C_SMEM))
    return host::fail(CE_ERR_CUDA, "ce_prefill: smem attr");
  return CE_OK;
}

}  // namespace

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
  Params p;
  CUtensorMap qmap, lmap, kmap;
  if (mode_of_row == nullptr) return CE_OK;
  if (scores == nullptr || score_sg < pool_units)
    return host::fail(CE_ERR_ARG, "ce_prefill_scores: scores missing or head stride below pool_units");
  const int st0 = prefill_prepare(q, q_st, q_sh, k_pool, pool_units, qo_indptr, kv_indptr, kv_indices,
                                  kv_tokens, kv_capacity, sinks, mode_of_row, rows, sm_scale, bs,
                                  num_q_heads, num_kv_heads, head_dim, page_size, total_q, max_q,
                                  max_tokens, scores, score_sg, zero_new, workspace, workspace_bytes,
                                  err, p, qmap, lmap, kmap);
  if (st0 != CE_OK) return st0 > 0 ? CE_OK : st0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 g1((max_q + QT - 1) / QT, num_kv_heads, bs);
  lse_kernel<false><<<g1, THREADS, L_SMEM, st>>>(p, qmap, kmap);
  if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("prefill lse_kernel");
  if (max_tokens == 0) return CE_OK;
  const dim3 g2((max_tokens + BM - 1) / BM, num_kv_heads, bs);
  colsum_kernel<<<g2, THREADS, C_SMEM, st>>>(p, qmap, lmap, kmap);
  if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("prefill colsum_kernel");
  return CE_OK;
}

extern "C" int ce_prefill_lost(const void* q, int64_t q_st, int64_t q_sh, const void* k_pool,
                               int64_t pool_units, const int32_t* qo_indptr, const int32_t* kv_indptr,
                               const int32_t* kv_indices, const int32_t* kv_tokens, int64_t kv_capacity,
                               const float* sinks, float sm_scale, int32_t num_q_heads,
                               int32_t num_kv_heads, int32_t head_dim, int32_t page_size,
                               int32_t total_q, int32_t max_q, int32_t max_tokens,
                               const uint32_t* evicted_bits, int32_t num_specs, int64_t bits_words,
                               float* lost, int64_t lost_stride, float lost_scale, void* workspace,
                               int64_t workspace_bytes, int32_t* err, void* stream) {
  using namespace ce::prefill;
  if (num_specs < 0 || num_specs > MAX_SPECS)
    return host::fail(CE_ERR_UNSUPPORTED, "ce_prefill_lost: at most 8 specs");
  if (num_specs == 0) return CE_OK;
  if (!evicted_bits || !lost || bits_words * 32 < max_tokens || lost_stride < max_q)
    return host::fail(CE_ERR_ARG, "ce_prefill_lost: evicted bits or lost buffer too small");
  Params p;
  CUtensorMap qmap, lmap, kmap;
  const int st0 = prefill_prepare(q, q_st, q_sh, k_pool, pool_units, qo_indptr, kv_indptr, kv_indices,
                                  kv_tokens, kv_capacity, sinks, nullptr, nullptr, sm_scale, 1,
                                  num_q_heads, num_kv_heads, head_dim, page_size, total_q, max_q,
                                  max_tokens, nullptr, 0, 0, workspace, workspace_bytes, err, p, qmap,
                                  lmap, kmap);
  if (st0 != CE_OK) return st0 > 0 ? CE_OK : st0;
  p.lost_bits = evicted_bits;
  p.lost_words = bits_words;
  p.lost_stride = lost_stride;
  p.S = num_specs;
  p.lost_scale = lost_scale;
  p.lost = lost;
  p.all_entries = 1;   // the normalisers pass runs for the entry whatever its score mode
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 g1((max_q + QT - 1) / QT, num_kv_heads, 1);
  lse_kernel<false><<<g1, THREADS, L_SMEM, st>>>(p, qmap, kmap);
  if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("prefill lse_kernel");
  lse_kernel<true><<<g1, THREADS, L_SMEM, st>>>(p, qmap, kmap);
  if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("prefill lost pass");
  return CE_OK;
}

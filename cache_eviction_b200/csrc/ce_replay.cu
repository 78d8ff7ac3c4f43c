// Replay layer error for sm_100a.
//
// The reference's static replay (code/cache_eviction/sglang_evict_runtime.py,
// _replay_layer_difference, :520-546) measures, for each prefill query of the
// first full layer, how far the evicted cache moves the attention output:
//
//   a_i = softmax_full(q_i K^T * scale, sink) V        (every causal key)
//   b_i = softmax_vis (q_i K^T * scale, sink) V        (each KV head's visible keys)
//   error_i = ||b_i - a_i|| / max(||a_i||, 1e-12)      (norms over all H x 64 values)
//
// with the unevicted keys and values kept by logical position (the shadow,
// :227-238) and visibility from _visible (:241-247).  Two tcgen05 passes per
// (16-query tile, KV head), M = 128 accumulator rows = 16 queries x the
// group's 8 query heads:
//
//   split_lse_kernel  S = Q K^T streamed over key tiles; each row keeps one
//                     running max and two online log2 sums under it, one over
//                     its visible keys and one over its evicted keys (each key
//                     is exactly one of the two, so one exp2 per element), and
//                     writes the full normaliser lse_a (with the sink) and
//                     r = (evicted mass) / (visible mass + sink), i.e.
//                     p_b = p_a (1 + r) on visible keys; r comes from two
//                     directly accumulated sums, not from the difference of
//                     two normalisers.
//   pv_kernel         S again; p_a = 2^(s - lse_a) and the difference
//                     d = p_b - p_a (p_a r on visible keys, -p_a on evicted
//                     ones), each split into a bf16 high part and a bf16
//                     residual, are stored into tensor memory (tcgen05.st) as
//                     the A operands of four MMAs per key tile that accumulate
//                     O_a = P_a V and O_d = P_d V in tensor memory (V is the
//                     MN-major B operand from shared memory).  b - a = O_d is
//                     formed directly, so a small eviction error is not the
//                     difference of two rounded outputs; each row's sums of
//                     squares are reduced over the query's 8 heads and added to
//                     a per-query pair.
//   finish_kernel     error = sqrt(sum d^2) / max(sqrt(sum a^2), 1e-12).
//
// The high + residual pair carries each probability to ~2^-17 relative (a
// single bf16 rounding, 2^-9, showed up at the 1e-3 level when attention is
// concentrated on a few keys).  Visible normalisers far below the full one
// (more than 2^126 apart) underflow; the reference's own fp32 path has the
// same range.
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include "ce_common.cuh"
#include "ce_host.h"

namespace ce {
namespace replay {

constexpr int D = 64;
constexpr int GROUP = 8;
constexpr float LOG2E = 1.4426950408889634f;
constexpr int BM = 128;                  // accumulator rows
constexpr int BN = 128;                  // keys per tile
constexpr int QT = BM / GROUP;           // 16 queries per CTA
constexpr int TILE = 128 * 128;          // 128 rows x 128 B
constexpr int EPI_WARPS = 8;
constexpr int THREADS = 32 * (EPI_WARPS + 2);
constexpr int LOAD_WARP = EPI_WARPS, MMA_WARP = EPI_WARPS + 1;
constexpr int NS1 = 5;                   // key-tile ring of pass 1
constexpr int NS2 = 4;                   // (key, value) tile ring of pass 2
constexpr uint32_t TMEM1 = 2 * BN;       // two S accumulators
// Pass 2 tensor memory (512 columns): S | O_a | O_d | P_a hi, lo | P_d hi, lo;
// a 128-key bf16 P tile takes 64 columns (two keys per 32-bit column).
constexpr uint32_t TMEM2 = 512;
constexpr uint32_t OA_COL = 128, OD_COL = 192;
constexpr uint32_t PAH_COL = 256, PAL_COL = 320, PDH_COL = 384, PDL_COL = 448;
// Pass 2 runs sixteen epilogue warps: four per TMEM lane quarter, 32 keys of
// each tile apiece.
constexpr int EPI2 = 16;
constexpr int THREADS2 = 32 * (EPI2 + 2);
constexpr int LOAD2 = EPI2, MMA2 = EPI2 + 1;
constexpr uint32_t IDESC_S = f16_idesc(BM, BN);
constexpr uint32_t IDESC_PV = f16_idesc(BM, D) | kIdescBMajorMN;

struct Params {
  float scale2;          // sm_scale * log2(e)
  int H, G, start, count;
  const float* sinks;
  const uint32_t* vis;   // [G][vis_words] or null (all visible)
  int64_t vis_words;
  float* lse2;           // [count, H]
  float* ratio;          // [count, H]
  float* sums;           // [count, 2]: sum d^2, sum a^2
  float* error;          // [count]
  float* out;            // [count, H, 64] masked output or null
  int32_t* err;
};

// 64 visibility bits of KV head g from key kb (a multiple of 64).
__device__ __forceinline__ void vis_words(const Params& p, int g, int kb, uint32_t& w0, uint32_t& w1) {
  if (!p.vis) {
    w0 = w1 = 0xffffffffu;
    return;
  }
  const int64_t w = kb / 32;
  const uint32_t* row = p.vis + static_cast<int64_t>(g) * p.vis_words;
  w0 = w < p.vis_words ? row[w] : 0u;
  w1 = w + 1 < p.vis_words ? row[w + 1] : 0u;
}

__device__ __forceinline__ bool bit_of(uint32_t w0, uint32_t w1, int i) {
  return ((i < 32 ? w0 >> i : w1 >> (i - 32)) & 1u) != 0u;
}

__device__ __forceinline__ void named_barrier_epi() {
  asm volatile("bar.sync 1, %0;" ::"n"(EPI_WARPS * 32) : "memory");
}

// ---------------------------------------------------------------- pass 1
struct Sync1 {
  uint64_t full[NS1], empty[NS1];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t once, mma_done;
  uint32_t tmem;
  int abort;
  float part[3][BM];
};

// CTA (16-query tile x, KV head g); accumulator row r = query 16x + r / 8,
// head g*8 + r % 8; keys of tile t are positions 128 t .. 128 t + 127.
__global__ void __launch_bounds__(THREADS, 2) split_lse_kernel(const Params p,
                                                                const __grid_constant__ CUtensorMap qmap,
                                                                const __grid_constant__ CUtensorMap kmap) {
  const int g = blockIdx.y;
  const int q0 = blockIdx.x * QT;
  if (q0 >= p.count) return;
  if (g == 0 && threadIdx.x < 2 * QT) {   // per-query sums for pass 2
    const int qi = q0 + threadIdx.x / 2;
    if (qi < p.count) p.sums[2 * qi + (threadIdx.x & 1)] = 0.f;
  }
  const int kend = p.start + min(p.count, q0 + QT);
  const int ntiles = (kend + BN - 1) / BN;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  const uint32_t qtile = smem_addr(sm);
  const uint32_t ring = qtile + TILE;
  Sync1* sy = reinterpret_cast<Sync1*>(sm + TILE + NS1 * TILE);
  volatile int* abort = &sy->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS1; ++s) {
      mbar_init(&sy->full[s], 1);
      mbar_init(&sy->empty[s], 1);
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
  if (warp == MMA_WARP) tmem_alloc(&sy->tmem, TMEM1);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sy->tmem;

  if (warp == LOAD_WARP) {
    int t = 0;
    if (lane == 0) {
      mbar_arrive_expect_tx(&sy->once, TILE);
      tma_load_3d(sm, &qmap, 0, g * GROUP, q0, &sy->once);
    }
    for (; t < ntiles; ++t) {
      const int s = t % NS1;
      if (t >= NS1 && !warp_wait(&sy->empty[s], ((t / NS1) & 1) ^ 1, p.err, abort, lane)) {
        *abort = 1;
        break;
      }
      if (lane == 0) {
        mbar_arrive_expect_tx(&sy->full[s], TILE);
        tma_load_3d(sm + TILE + s * TILE, &kmap, 0, g, t * BN, &sy->full[s]);
      }
    }
    if (lane == 0) {   // every issued load lands before the CTA may exit
      for (int u = max(0, t - NS1); u < t; ++u) mbar_wait(&sy->full[u % NS1], (u / NS1) & 1, p.err);
      mbar_wait(&sy->once, 0, p.err);
    }
  } else if (warp == MMA_WARP) {
    bool issued = false;
    if (lane == 0 && mbar_wait_or_abort(&sy->once, 0, p.err, abort)) {
      tc_fence_after();
      const uint64_t adesc = sw128_desc(qtile);
      for (int t = 0; t < ntiles; ++t) {
        const int s = t % NS1, buf = t & 1;
        if ((t >= 2 && !mbar_wait_or_abort(&sy->acc_empty[buf], ((t >> 1) & 1) ^ 1, p.err, abort)) ||
            !mbar_wait_or_abort(&sy->full[s], (t / NS1) & 1, p.err, abort)) {
          *abort = 1;
          break;
        }
        tc_fence_after();
        const uint64_t bdesc = sw128_desc(ring + s * TILE);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) tc_mma(tmem + buf * BN, adesc + 2 * kk, bdesc + 2 * kk, IDESC_S, kk > 0);
        tc_commit(&sy->empty[s]);
        tc_commit(&sy->acc_full[buf]);
        issued = true;
      }
    } else if (lane == 0) {
      *abort = 1;
    }
    if (lane == 0 && issued) {
      tc_commit(&sy->mma_done);
      mbar_wait(&sy->mma_done, 0, p.err);
    }
    __syncwarp();
  } else {
    // Warp e: TMEM lanes 32 (e % 4) .. +31, key columns 64 (e / 4) .. +63.
    const int quarter = warp & 3, half = warp >> 2;
    const int r = quarter * 32 + lane;
    const int q = q0 + r / GROUP;
    const int h = g * GROUP + r % GROUP;
    const int lim = p.start + min(q, p.count - 1);   // last causal key of this row
    // One running max over all causal keys; the visible and the evicted
    // sums share it, so each element costs one exponential whose value goes
    // to exactly one of the two sums (the bit as an integer mask).
    float m = -INFINITY, lv = 0.f, le = 0.f;
    for (int t = 0; t < ntiles; ++t) {
      const int buf = t & 1;
      if (!warp_wait(&sy->acc_full[buf], (t >> 1) & 1, p.err, abort, lane)) {
        *abort = 1;
        break;
      }
      tc_fence_after();
      float v[64];
      __syncwarp();
      const uint32_t taddr = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + buf * BN + half * 64;
      tmem_ld32_async(taddr, v);
      tmem_ld32_async(taddr + 32, v + 32);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sy->acc_empty[buf]);
      const int kb = t * BN + half * 64;
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
      const float mn = fmaxf(m, mt * p.scale2);
      if (mn == -INFINITY) continue;   // no causal key yet
      uint32_t w[2];
      vis_words(p, g, kb, w[0], w[1]);
      float sv[2] = {0.f, 0.f}, se[2] = {0.f, 0.f};
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        const float a = fmaf(v[i], p.scale2, -mn);
        const float e = (i & 3) == 3 ? poly_exp2(a) : fast_exp2(a);
        // all ones when bit i is set
        const uint32_t bm = static_cast<uint32_t>(static_cast<int32_t>(w[i >> 5] << (31 - (i & 31))) >> 31);
        const float ev = __uint_as_float(__float_as_uint(e) & bm);
        sv[i & 1] += ev;
        se[i & 1] += e - ev;
      }
      const float c = fast_exp2(m - mn);   // 0 while m is -inf
      lv = lv * c + (sv[0] + sv[1]);
      le = le * c + (se[0] + se[1]);
      m = mn;
    }
    if (half == 1) {
      sy->part[0][r] = m;
      sy->part[1][r] = lv;
      sy->part[2][r] = le;
    }
    named_barrier_epi();
    if (half == 0 && !*abort && q < p.count) {
      const float m1 = sy->part[0][r];
      const float M = fmaxf(m, m1);      // finite: key 0 is causal for every row
      const float c0 = exp2f(m - M), c1 = exp2f(m1 - M);
      float Lv = lv * c0 + sy->part[1][r] * c1;
      const float Le = le * c0 + sy->part[2][r] * c1;
      if (p.sinks) Lv += exp2f(p.sinks[h] * LOG2E - M);
      const int64_t o = static_cast<int64_t>(q) * p.H + h;
      p.lse2[o] = M + log2f(Lv + Le);
      // p_b = p_a (1 + r) on visible keys; a row with no visible mass left
      // (nothing visible, no sink) has no visible key to scale.
      p.ratio[o] = Lv > 0.f ? fminf(Le / Lv, 1e30f) : 0.f;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == MMA_WARP) tmem_dealloc(tmem, TMEM1);
}

// ---------------------------------------------------------------- pass 2
struct Sync2 {
  uint64_t full[NS2], empty[NS2];
  uint64_t sfull, sempty, pfull, pempty;
  uint64_t once, odone, mma_done;
  uint32_t tmem;
  int abort;
};

// Shared memory: Q tile | NS2 x (K tile, V tile) | barriers.  One CTA per SM
// (it holds all 512 TMEM columns).
constexpr int SMEM2 = 1024 + TILE + NS2 * 2 * TILE + static_cast<int>(sizeof(Sync2));
constexpr int SMEM1 = 1024 + TILE + NS1 * TILE + static_cast<int>(sizeof(Sync1));
static_assert(SMEM2 <= 227 * 1024 && 2 * SMEM2 > 228 * 1024, "pass 2: one CTA per SM");
static_assert(2 * SMEM1 <= 227 * 1024, "two pass-1 CTAs per SM");
static_assert(3 * SMEM1 > 227 * 1024, "a third pass-1 CTA would oversubscribe TMEM");

__global__ void __launch_bounds__(THREADS2, 1) pv_kernel(const Params p, const __grid_constant__ CUtensorMap qmap,
                                                         const __grid_constant__ CUtensorMap kmap,
                                                         const __grid_constant__ CUtensorMap vmap) {
  const int g = blockIdx.y;
  const int q0 = blockIdx.x * QT;
  if (q0 >= p.count) return;
  const int kend = p.start + min(p.count, q0 + QT);
  const int ntiles = (kend + BN - 1) / BN;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  const uint32_t qtile = smem_addr(sm);
  const uint32_t ring = qtile + TILE;                    // stage s: K at +2s TILE, V at +(2s+1) TILE
  Sync2* sy = reinterpret_cast<Sync2*>(sm + TILE + NS2 * 2 * TILE);
  volatile int* abort = &sy->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS2; ++s) {
      mbar_init(&sy->full[s], 1);
      mbar_init(&sy->empty[s], 1);
    }
    mbar_init(&sy->sfull, 1);
    mbar_init(&sy->sempty, EPI2);
    mbar_init(&sy->pfull, EPI2);
    mbar_init(&sy->pempty, 1);
    mbar_init(&sy->once, 1);
    mbar_init(&sy->odone, 1);
    mbar_init(&sy->mma_done, 1);
    sy->abort = 0;
    fence_mbar_init();
  }
  if (warp == MMA2) tmem_alloc(&sy->tmem, TMEM2);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sy->tmem;

  if (warp == LOAD2) {
    int t = 0;
    if (lane == 0) {
      mbar_arrive_expect_tx(&sy->once, TILE);
      tma_load_3d(sm, &qmap, 0, g * GROUP, q0, &sy->once);
    }
    for (; t < ntiles; ++t) {
      const int s = t % NS2;
      if (t >= NS2 && !warp_wait(&sy->empty[s], ((t / NS2) & 1) ^ 1, p.err, abort, lane)) {
        *abort = 1;
        break;
      }
      if (lane == 0) {
        uint8_t* st = sm + TILE + s * 2 * TILE;
        mbar_arrive_expect_tx(&sy->full[s], 2 * TILE);
        tma_load_3d(st, &kmap, 0, g, t * BN, &sy->full[s]);
        tma_load_3d(st + TILE, &vmap, 0, g, t * BN, &sy->full[s]);
      }
    }
    if (lane == 0) {
      for (int u = max(0, t - NS2); u < t; ++u) mbar_wait(&sy->full[u % NS2], (u / NS2) & 1, p.err);
      mbar_wait(&sy->once, 0, p.err);
    }
  } else if (warp == MMA2) {
    // Order: S(0), S(1), PV(0), S(2), PV(1), ... so the epilogue turns S(t+1)
    // into P while the tensor cores run PV(t).
    bool issued = false;
    if (lane == 0 && mbar_wait_or_abort(&sy->once, 0, p.err, abort)) {
      tc_fence_after();
      const uint64_t qdesc = sw128_desc(qtile);
      bool ok = true;
      for (int t = 0; t <= ntiles && ok; ++t) {
        if (t < ntiles) {
          const int s = t % NS2;
          if (!mbar_wait_or_abort(&sy->full[s], (t / NS2) & 1, p.err, abort) ||
              (t >= 1 && !mbar_wait_or_abort(&sy->sempty, (t - 1) & 1, p.err, abort))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t kdesc = sw128_desc(ring + s * 2 * TILE);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) tc_mma(tmem, qdesc + 2 * kk, kdesc + 2 * kk, IDESC_S, kk > 0);
          tc_commit(&sy->sfull);
          issued = true;
        }
        if (t >= 1) {
          const int u = t - 1, s = u % NS2;
          if (!mbar_wait_or_abort(&sy->pfull, u & 1, p.err, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t vt = ring + s * 2 * TILE + TILE;
          // K-step kk: keys 16 kk .. +15 = P columns 8 kk .. +7, V rows 16 kk .. +15.
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            const uint64_t vdesc = sw128_mn_desc(vt + kk * 2048);
            const uint32_t c = kk * 8;
            tc_mma_ts(tmem + OA_COL, tmem + PAH_COL + c, vdesc, IDESC_PV, u > 0 || kk > 0);
            tc_mma_ts(tmem + OA_COL, tmem + PAL_COL + c, vdesc, IDESC_PV, true);
            tc_mma_ts(tmem + OD_COL, tmem + PDH_COL + c, vdesc, IDESC_PV, u > 0 || kk > 0);
            tc_mma_ts(tmem + OD_COL, tmem + PDL_COL + c, vdesc, IDESC_PV, true);
          }
          tc_commit(&sy->pempty);
          tc_commit(&sy->empty[s]);
        }
      }
      if (ok) tc_commit(&sy->odone);
      else *abort = 1;
    } else if (lane == 0) {
      *abort = 1;
    }
    if (lane == 0 && issued) {
      tc_commit(&sy->mma_done);
      mbar_wait(&sy->mma_done, 0, p.err);
    }
    __syncwarp();
  } else {
    // Warp e: TMEM lanes 32 (e % 4) .. +31, keys 32 (e / 4) .. +31 of each
    // tile = columns 16 (e / 4) .. +15 of each P tile and of O.
    const int quarter = warp & 3, part = warp >> 2;
    const int r = quarter * 32 + lane;
    const int q = q0 + r / GROUP;
    const int h = g * GROUP + r % GROUP;
    const bool qv = q < p.count;
    const int lim = p.start + min(q, p.count - 1);
    const int64_t o = static_cast<int64_t>(qv ? q : 0) * p.H + h;
    const float lse = qv ? p.lse2[o] : 0.f;
    const float rr = qv ? p.ratio[o] : 0.f;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    bool ok = true;
    for (int t = 0; t < ntiles; ++t) {
      if (!warp_wait(&sy->sfull, t & 1, p.err, abort, lane)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float v[32];
      __syncwarp();
      tmem_ld32(tmem + lane_base + part * 32, v);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sy->sempty);
      const int kb = t * BN + part * 32;
      uint32_t w, w_unused;
      vis_words(p, g, kb, w, w_unused);
      if (t >= 1 && !warp_wait(&sy->pempty, (t - 1) & 1, p.err, abort, lane)) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {   // keys 16 hh .. +15 of this warp's 32
        uint32_t ah[8], al[8], dh[8], dl[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float e[2], d[2];
#pragma unroll
          for (int x = 0; x < 2; ++x) {
            const int i = hh * 16 + 2 * j + x;
            const bool in = qv && kb + i <= lim;
            const float y = in ? fast_exp2(fmaf(v[i], p.scale2, -lse)) : 0.f;
            e[x] = y;
            d[x] = ((w >> i) & 1u) ? y * rr : -y;
          }
          split_bf16x2(e[0], e[1], ah[j], al[j]);
          split_bf16x2(d[0], d[1], dh[j], dl[j]);
        }
        const uint32_t col = lane_base + part * 16 + hh * 8;
        tmem_st8_async(tmem + col + PAH_COL, ah);
        tmem_st8_async(tmem + col + PAL_COL, al);
        tmem_st8_async(tmem + col + PDH_COL, dh);
        tmem_st8_async(tmem + col + PDL_COL, dl);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sy->pfull);
    }
    if (!ok) *abort = 1;
    if (ok && warp_wait(&sy->odone, 0, p.err, abort, lane)) {
      tc_fence_after();
      float a[16], d[16];
      __syncwarp();
      tmem_ld16_async(tmem + lane_base + OA_COL + part * 16, a);
      tmem_ld16_async(tmem + lane_base + OD_COL + part * 16, d);
      tmem_ld_wait();
      float sa = 0.f, sd = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        sa = fmaf(a[i], a[i], sa);
        sd = fmaf(d[i], d[i], sd);
      }
      if (p.out && qv) {
        float4* dst = reinterpret_cast<float4*>(p.out + (o * D + part * 16));
#pragma unroll
        for (int i = 0; i < 4; ++i)
          dst[i] = make_float4(a[4 * i] + d[4 * i], a[4 * i + 1] + d[4 * i + 1], a[4 * i + 2] + d[4 * i + 2],
                               a[4 * i + 3] + d[4 * i + 3]);
      }
      // The query's 8 heads are 8 adjacent lanes.
#pragma unroll
      for (int m = 1; m < GROUP; m <<= 1) {
        sa += __shfl_xor_sync(0xffffffffu, sa, m);
        sd += __shfl_xor_sync(0xffffffffu, sd, m);
      }
      if ((lane & (GROUP - 1)) == 0 && qv) {
        atomicAdd(p.sums + 2 * q, sd);
        atomicAdd(p.sums + 2 * q + 1, sa);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == MMA2) tmem_dealloc(tmem, TMEM2);
}

__global__ void finish_kernel(const Params p) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < p.count) p.error[i] = sqrtf(p.sums[2 * i]) / fmaxf(sqrtf(p.sums[2 * i + 1]), 1e-12f);
}

}  // namespace replay
}  // namespace ce

using namespace ce;

namespace {
int64_t a256(int64_t x) { return (x + 255) & ~int64_t(255); }
}  // namespace

extern "C" int64_t ce_replay_workspace_bytes(int32_t count, int32_t num_q_heads) {
  if (count < 0 || num_q_heads <= 0) return -1;
  const int64_t c = count > 0 ? count : 1;
  return 2 * a256(c * num_q_heads * 4) + a256(c * 8);
}

extern "C" int ce_replay_error(const void* q, int64_t q_st, int64_t q_sh, const void* k, const void* v,
                               int64_t kv_rows, const uint32_t* visible, int64_t bits_words,
                               const float* sinks, float sm_scale, int32_t num_q_heads, int32_t num_kv_heads,
                               int32_t head_dim, int32_t start, int32_t count, float* error,
                               float* out_masked, void* workspace, int64_t workspace_bytes, int32_t* err,
                               void* stream) {
  using namespace ce::replay;
  if (start < 0 || count < 0 || kv_rows < 0) return host::fail(CE_ERR_ARG, "ce_replay_error: negative size");
  if (!(sm_scale > 0.f)) return host::fail(CE_ERR_ARG, "ce_replay_error: sm_scale must be positive");
  if (head_dim != D || num_kv_heads <= 0 || num_q_heads != GROUP * num_kv_heads)
    return host::fail(CE_ERR_UNSUPPORTED, "ce_replay_error: needs head_dim 64 and 8 query heads per KV head");
  if (count == 0) return CE_OK;
  if (!q || !k || !v || !error) return host::fail(CE_ERR_ARG, "ce_replay_error: null pointer");
  if (static_cast<int64_t>(start) + count > kv_rows)
    return host::fail(CE_ERR_ARG, "ce_replay_error: the shadow holds fewer than start + count positions");
  if (static_cast<int64_t>(start) + count > INT32_MAX - BN)
    return host::fail(CE_ERR_UNSUPPORTED, "ce_replay_error: too many positions");
  if (visible && bits_words * 32 < static_cast<int64_t>(start) + count)
    return host::fail(CE_ERR_ARG, "ce_replay_error: visibility bits shorter than start + count");
  if (q_sh % 8 != 0 || q_st % 8 != 0 || q_sh < D || q_st < static_cast<int64_t>(num_q_heads) * q_sh)
    return host::fail(CE_ERR_ARG, "ce_replay_error: q strides must be multiples of 8 elements");
  const int64_t need = ce_replay_workspace_bytes(count, num_q_heads);
  if (!workspace || workspace_bytes < need) return host::fail(CE_ERR_WORKSPACE, "ce_replay_error: workspace too small");
  if ((reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(k) & 15) ||
      (reinterpret_cast<uintptr_t>(v) & 15) || (reinterpret_cast<uintptr_t>(workspace) & 15) ||
      (reinterpret_cast<uintptr_t>(out_masked) & 15))
    return host::fail(CE_ERR_ARG, "ce_replay_error: q, k, v, out_masked and workspace need 16-byte alignment");
  CUtensorMap qmap, kmap, vmap;
  {
    // Q as [count][H][64] with byte strides; box = 16 queries x 8 heads x 64.
    const uint64_t dims[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(num_q_heads),
                              static_cast<uint64_t>(count)};
    const uint64_t strides[2] = {static_cast<uint64_t>(q_sh) * 2, static_cast<uint64_t>(q_st) * 2};
    const uint32_t box[3] = {static_cast<uint32_t>(D), GROUP, QT};
    if (!host::encode_map(&qmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, q, dims, strides, box, true))
      return host::fail(CE_ERR_CUDA, "ce_replay_error: query tensor map");
  }
  {
    // Shadow K and V as [positions][G][64]; box = 128 positions of one head.
    // Only the start + count positions the chunk can see are mapped, so the
    // rows past them read as zeros.
    const uint64_t dims[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(num_kv_heads),
                              static_cast<uint64_t>(start) + static_cast<uint64_t>(count)};
    const uint64_t strides[2] = {static_cast<uint64_t>(D) * 2, static_cast<uint64_t>(num_kv_heads) * D * 2};
    const uint32_t box[3] = {static_cast<uint32_t>(D), 1, BN};
    if (!host::encode_map(&kmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, k, dims, strides, box, true) ||
        !host::encode_map(&vmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, v, dims, strides, box, true))
      return host::fail(CE_ERR_CUDA, "ce_replay_error: shadow tensor maps");
  }
  Params p{};
  p.scale2 = sm_scale * LOG2E;
  p.H = num_q_heads;
  p.G = num_kv_heads;
  p.start = start;
  p.count = count;
  p.sinks = sinks;
  p.vis = visible;
  p.vis_words = bits_words;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const int64_t lse_bytes = a256(static_cast<int64_t>(count) * num_q_heads * 4);
  p.lse2 = reinterpret_cast<float*>(ws);
  p.ratio = reinterpret_cast<float*>(ws + lse_bytes);
  p.sums = reinterpret_cast<float*>(ws + 2 * lse_bytes);
  p.error = error;
  p.out = out_masked;
  p.err = err;
  if (!host::set_smem(split_lse_kernel, SMEM1) || !host::set_smem(pv_kernel, SMEM2))
    return host::fail(CE_ERR_CUDA, "ce_replay_error: smem attr");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid((count + QT - 1) / QT, num_kv_heads);
  split_lse_kernel<<<grid, THREADS, SMEM1, st>>>(p, qmap, kmap);
  if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("replay split_lse_kernel");
  pv_kernel<<<grid, THREADS2, SMEM2, st>>>(p, qmap, kmap, vmap);
  if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("replay pv_kernel");
  finish_kernel<<<(count + 255) / 256, 256, 0, st>>>(p);
  if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("replay finish_kernel");
  return CE_OK;
}

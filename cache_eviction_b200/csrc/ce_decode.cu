// K1: fused paged GQA decode attention + H2O score for sm_100a.
//
// Replaces, in one pass over the KV pool, what the reference does in two:
// SGLang's split-KV decode_attention_fwd (stage 1 + 2) followed by the
// overlay's _decode_scores Triton kernel that re-reads every resident key
// (code/cache_eviction/sglang_evict_runtime.py:155-224).
//
// Work split (stream-K over tokens): the concatenation of all sequences'
// 16-token-per-warp "stages" is cut into gridDim.x equal ranges, one per
// persistent CTA.  A CTA walks its range sequence by sequence and leaves one
// partial record (per-warp running max m, sum l and unnormalised O) for every
// sequence it touched.  Record (b, cta) lives at index b + cta, which is unique
// because both walks are monotone.
//
// Inside a CTA: warp 8 is the producer.  It issues one 2D bulk-tensor (TMA)
// load per KV page for K and one for V (box = the page's G*P rows of 128 B,
// 128-byte swizzle) into a ring of shared-memory stages guarded by mbarriers.
// Warps 0..7 consume: warp w owns KV head g = w % G and 16 tokens of the
// stage.  S = Q K^T and O += P V run on m16n8k16 bf16 tensor-core tiles with
// the group's 8 query heads in rows 0..7; P enters the PV product as a bf16
// hi/lo pair so the output keeps ~fp32 accuracy.
//
// Scores need the final normaliser, which only exists after the split
// combine.  For H2O rows the consumer therefore stores, per KV page and query
// head, log2 of the page's probability mass relative to the running max
// (CE_MODE_SUM), or every token's logit (CE_MODE_MAX, which needs a max over
// heads per token).  The finalize kernel rebuilds each head's normaliser from
// the records plus the sink -- the same normaliser as decode stage 2 and the
// reference score kernel (runtime:179-188) -- combines O, and adds
//   SUM: sum_h 2^(page_lse - LSE_h)   MAX: sum_t max_h 2^(s_t,h - LSE_h)
// into scores[g, unit] with a plain read-modify-write: a unit appears once in
// a batch, as in the reference kernel (runtime:199-200).
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "ce_common.cuh"
#include "ce_host.h"

namespace ce {
namespace decode {

constexpr int D = 64;
constexpr int GROUP = 8;
constexpr int NCW = 8;                    // consumer warps
constexpr int THREADS = (NCW + 1) * 32;   // + producer warp
constexpr int ROW_BYTES = D * 2;          // 128 B per (token, head) row
constexpr int HALF_STAGE = NCW * 16 * ROW_BYTES;  // 16 KB of K (or V) per stage
constexpr int STAGE_BYTES = 2 * HALF_STAGE;
constexpr int NSTAGES = 6;
constexpr int REC_ROWS = NCW * 8;         // virtual rows: warp w, head-row r
constexpr int REC_FLOATS = REC_ROWS * D + 2 * REC_ROWS;
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;
constexpr int SMEM_BYTES = NSTAGES * STAGE_BYTES + 1024 /*align*/ + 1024 /*barriers+misc*/;

struct Params {
  const __nv_bfloat16* q;
  int64_t q_sb, q_sh;
  const int32_t* kv_indptr;
  const int32_t* kv_indices;
  const int32_t* kv_tokens;
  int64_t kv_capacity;
  int64_t pool_units;
  const float* sinks;
  const int32_t* mode_of_row;
  const int64_t* rows;
  float scale_log2;
  int bs, H, G;
  float* scores;
  int64_t score_sg;
  int zero_new;
  void* out;
  int out_f32;
  int64_t o_sb, o_sh;
  float* lse_out;
  int32_t* prefix;   // [bs + 1] stage prefix (written by CTA 0)
  float* rec;        // [(bs + grid), REC_FLOATS]
  float* ul;         // [kv_capacity, H] unit log-mass (log2 units) or null
  float* tl;         // [kv_capacity * P, H] token logits (page_size > 1, MAX rows) or null
  int32_t* err;
};

__device__ __forceinline__ int stage_tokens(int G) { return 16 * (NCW / G); }

// Partitions actually used: at least MIN_STAGES_PER_CTA stages each, so a
// short batch is not spread thinner than the pipeline depth.
constexpr int64_t MIN_STAGES_PER_CTA = 4;
__device__ __forceinline__ int64_t eff_grid(int64_t S, int64_t launched) {
  const int64_t want = (S + MIN_STAGES_PER_CTA - 1) / MIN_STAGES_PER_CTA;
  return want < 1 ? 1 : (want < launched ? want : launched);
}

__device__ __forceinline__ int seq_tokens(const Params& p, int b, int P) {
  if (p.kv_tokens) return max(0, p.kv_tokens[b]);
  return max(0, (p.kv_indptr[b + 1] - p.kv_indptr[b]) * P);
}

__device__ __forceinline__ int seq_mode(const Params& p, int b) {
  if (!p.mode_of_row) return CE_MODE_NONE;
  const int64_t row = p.rows ? p.rows[b] : b;
  return p.mode_of_row[row];
}

// Block-wide exclusive scan of one int64 per thread (THREADS threads).
__device__ int64_t block_excl_scan(int64_t v, int64_t* sh, int64_t& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int64_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int64_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) sh[warp] = x;
  __syncthreads();
  if (threadIdx.x == 0) {
    int64_t run = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
      int64_t t = sh[w];
      sh[w] = run;
      run += t;
    }
    sh[31] = run;
  }
  __syncthreads();
  int64_t res = sh[warp] + x - v;
  total = sh[31];
  __syncthreads();
  return res;
}

template <int P>
__global__ void __launch_bounds__(THREADS, 1)
    attn_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NSTAGES * STAGE_BYTES);
  uint64_t* empty = full + NSTAGES;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + NSTAGES);
  int64_t* scan_sh = reinterpret_cast<int64_t*>(smem + NSTAGES * STAGE_BYTES + 128);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = p.G, H = p.H;
  const int ST = stage_tokens(G);
  const int UPS = ST / P;                 // pages per stage
  const int UNIT_ROWS = G * P;            // rows of one page (all local heads)
  const uint32_t UNIT_BYTES = UNIT_ROWS * ROW_BYTES;

  if (tid == 0) {
    for (int s = 0; s < NSTAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NCW);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");

  // ---- partition the global stage space --------------------------------------
  const int bs = p.bs;
  const int per = (bs + THREADS - 1) / THREADS;
  const int lo_b = min(bs, tid * per), hi_b = min(bs, lo_b + per);
  int64_t local = 0;
  for (int b = lo_b; b < hi_b; ++b) local += (seq_tokens(p, b, P) + ST - 1) / ST;
  int64_t S = 0;
  const int64_t excl = block_excl_scan(local, scan_sh, S);  // includes __syncthreads
  const int64_t k = blockIdx.x, grid = eff_grid(S, gridDim.x);
  const int64_t S_lo = k < grid ? k * S / grid : S, S_hi = k < grid ? (k + 1) * S / grid : S;
  if (blockIdx.x == 0) {
    int64_t run = excl;
    for (int b = lo_b; b < hi_b; ++b) {
      p.prefix[b] = static_cast<int32_t>(run);
      run += (seq_tokens(p, b, P) + ST - 1) / ST;
    }
    if (tid == 0) p.prefix[bs] = static_cast<int32_t>(S);
  }
  // Locate the sequence holding stage S_lo.
  int* start_sh = reinterpret_cast<int*>(scan_sh + 40);
  if (tid == 0) {
    start_sh[0] = bs;
    start_sh[1] = 0;
  }
  __syncthreads();
  if (S_lo < S_hi && excl <= S_lo && S_lo < excl + local) {
    int64_t run = excl;
    for (int b = lo_b; b < hi_b; ++b) {
      const int64_t n = (seq_tokens(p, b, P) + ST - 1) / ST;
      if (S_lo < run + n) {
        start_sh[0] = b;
        start_sh[1] = static_cast<int>(run);
        break;
      }
      run += n;
    }
  }
  __syncthreads();
  const int b_start = start_sh[0];
  const int base_start = start_sh[1];

  if (warp == NCW) {
    // ------------------------------- producer --------------------------------
    // Page indices are read in 32-entry windows one window ahead of use (the
    // CTA's CSR positions only move forward), so no TMA issue waits on a
    // dependent global load.
    int issued = 0;
    int b = b_start, base = base_start;
    int nst = 0, tok_b = 0;
    int64_t ip_b = 0;
    auto load_seq = [&](int bb) {
      tok_b = seq_tokens(p, bb, P);
      nst = (tok_b + ST - 1) / ST;
      ip_b = p.kv_indptr[bb];
    };
    if (b < bs) load_seq(b);
    auto fetch = [&](int64_t w0) -> int {
      const int64_t c = w0 + lane;
      return (c >= 0 && c < p.kv_capacity) ? p.kv_indices[c] : -2;
    };
    int64_t w0 = -1;
    int idx_cur = -2, idx_next = -2;
    for (int64_t x = S_lo; x < S_hi; ++x) {
      while (x >= base + nst) {
        base += nst;
        ++b;
        load_seq(b);
      }
      if (*abort_flag) break;
      const int j = static_cast<int>(x - base);
      const int ntok = min(ST, tok_b - j * ST);
      const int nunits = (ntok + P - 1) / P;
      const int64_t c0 = ip_b + static_cast<int64_t>(j) * UPS;
      if (w0 < 0 || c0 < w0 || c0 + nunits > w0 + 64) {
        w0 = c0;
        idx_cur = fetch(w0);
        idx_next = fetch(w0 + 32);
      } else if (c0 >= w0 + 32) {
        w0 += 32;
        idx_cur = idx_next;
        idx_next = fetch(w0 + 32);
      }
      const int s = issued % NSTAGES;
      const uint32_t ph = (issued / NSTAGES) & 1;
      if (issued >= NSTAGES) {
        bool ok = true;
        if (lane == 0) ok = mbar_wait(&empty[s], ph ^ 1, p.err);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
          *abort_flag = 1;
          break;
        }
      }
      // Unit of this lane's page: window slot (c0 - w0 + lane) of cur/next.
      const int slot = static_cast<int>(c0 - w0) + lane;
      const int a = __shfl_sync(0xffffffffu, idx_cur, slot & 31);
      const int bn = __shfl_sync(0xffffffffu, idx_next, slot & 31);
      int unit = -1;
      if (lane < nunits) {
        const int v = (slot < 32) ? a : bn;
        if (v == -2) {
          flag_error(p.err, CE_EW_CAPACITY);
        } else if (v < 0 || v >= p.pool_units) {
          flag_error(p.err, CE_EW_INDEX);
        } else {
          unit = v;
        }
      }
      const unsigned valid = __ballot_sync(0xffffffffu, unit >= 0);
      if (lane == 0) mbar_arrive_expect_tx(&full[s], __popc(valid) * UNIT_BYTES * 2);
      __syncwarp();
      if (unit >= 0) {
        uint8_t* kd = smem + s * STAGE_BYTES + lane * UNIT_BYTES;
        uint8_t* vd = kd + HALF_STAGE;
        const int32_t y = unit * UNIT_ROWS;
        tma_load_2d(kd, &kmap, 0, y, &full[s]);
        tma_load_2d(vd, &vmap, 0, y, &full[s]);
      }
      ++issued;
    }
    // Drain: every issued load must land before the CTA may exit.
    if (lane == 0) {
      for (int it = max(0, issued - NSTAGES); it < issued; ++it)
        mbar_wait(&full[it % NSTAGES], (it / NSTAGES) & 1, p.err);
    }
  } else {
    // ------------------------------- consumers -------------------------------
    const int g = warp % G;
    const int tb = warp / G;
    const int r = lane >> 2;   // query-head row within the group
    const int t = lane & 3;
    const int head = g * GROUP + r;
    float* rec_base = p.rec;

    // Row (in a stage) of token tau for this warp's KV head.
    auto row_of = [&](int tau) -> int { return (tau / P) * UNIT_ROWS + g * P + (tau % P); };

    uint32_t qa[4][2];
    float o[8][4];
    float m = -INFINITY, l = 0.f;
    int cur_b = -1, mode = CE_MODE_NONE;

    auto epilogue = [&](int bb) {
      float* rec = rec_base + static_cast<int64_t>(bb + blockIdx.x) * REC_FLOATS;
      const int vrow = warp * 8 + r;
#pragma unroll
      for (int dt = 0; dt < 8; ++dt) {
        float2 v = make_float2(o[dt][0], o[dt][1]);
        *reinterpret_cast<float2*>(rec + vrow * D + dt * 8 + 2 * t) = v;
      }
      if (t == 0) {
        rec[REC_ROWS * D + vrow] = m;
        rec[REC_ROWS * D + REC_ROWS + vrow] = l;
      }
    };

    int it = 0;
    int b = b_start, base = base_start;
    int nst = 0, tok_b = 0;
    int64_t ip_b = 0;
    auto load_seq = [&](int bb) {
      tok_b = seq_tokens(p, bb, P);
      nst = (tok_b + ST - 1) / ST;
      ip_b = p.kv_indptr[bb];
    };
    if (b < bs) load_seq(b);
    bool aborted = false;
    for (int64_t x = S_lo; x < S_hi; ++x, ++it) {
      while (x >= base + nst) {
        base += nst;
        ++b;
        load_seq(b);
      }
      if (b != cur_b) {
        if (cur_b >= 0) epilogue(cur_b);
        cur_b = b;
        const __nv_bfloat16* qrow = p.q + static_cast<int64_t>(b) * p.q_sb + static_cast<int64_t>(head) * p.q_sh;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          qa[ks][0] = *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 2 * t);
          qa[ks][1] = *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 8 + 2 * t);
        }
#pragma unroll
        for (int dt = 0; dt < 8; ++dt) o[dt][0] = o[dt][1] = o[dt][2] = o[dt][3] = 0.f;
        m = -INFINITY;
        l = 0.f;
        mode = seq_mode(p, b);
        if ((mode == CE_MODE_SUM || mode == CE_MODE_MAX) && !p.ul) {
          if (lane == 0 && warp == 0) flag_error(p.err, CE_EW_MODE);
          mode = CE_MODE_NONE;
        }
        if (mode == CE_MODE_MAX && P > 1 && !p.tl) {
          if (lane == 0 && warp == 0) flag_error(p.err, CE_EW_MODE);
          mode = CE_MODE_NONE;
        }
      }
      const int j = static_cast<int>(x - base);
      const int ntok = min(ST, tok_b - j * ST);
      const int s = it % NSTAGES;
      const uint32_t ph = (it / NSTAGES) & 1;
      if (!mbar_wait(&full[s], ph, p.err)) {
        *abort_flag = 1;
        aborted = true;
        break;
      }
      uint8_t* kst = smem + s * STAGE_BYTES;
      uint8_t* vst = kst + HALF_STAGE;
      const int tau0 = tb * 16;
      if (ntok < tau0 + 16) {
        // Zero V rows of tokens past the end so 0-probability * garbage stays 0.
        for (int idx = lane; idx < 16 * 8; idx += 32) {
          const int tau = tau0 + (idx >> 3);
          if (tau >= ntok)
            *reinterpret_cast<uint4*>(vst + row_of(tau) * ROW_BYTES + (idx & 7) * 16) =
                make_uint4(0, 0, 0, 0);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
      }
      if (tau0 < ntok) {
        // ---- S = Q K^T over the warp's 16 tokens -----------------------------
        float sacc[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.f;
#pragma unroll
          for (int kp = 0; kp < 2; ++kp) {
            const int mi = lane >> 3, rr = lane & 7;
            const int row = row_of(tau0 + nt * 8 + rr);
            const int chunk = kp * 4 + mi;
            const uint32_t addr = smem_addr(kst) + row * ROW_BYTES + ((chunk ^ (row & 7)) << 4);
            uint32_t b0, b1, b2, b3;
            ldsm_x4(addr, b0, b1, b2, b3);
            mma_16816(sacc[nt], qa[2 * kp][0], qa[2 * kp][1], b0, b1);
            mma_16816(sacc[nt], qa[2 * kp + 1][0], qa[2 * kp + 1][1], b2, b3);
          }
        }
        float sv[4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int tau = tau0 + nt * 8 + 2 * t + i;
            sv[nt * 2 + i] = (tau < ntok) ? sacc[nt][i] * p.scale_log2 : -INFINITY;
          }
        float mx = fmaxf(fmaxf(sv[0], sv[1]), fmaxf(sv[2], sv[3]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float m_new = fmaxf(m, mx);
        const float mu = (m_new == -INFINITY) ? 0.f : m_new;
        const float alpha = exp2f(m - mu);
        float pv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) pv[i] = exp2f(sv[i] - mu);
        float rs = (pv[0] + pv[1]) + (pv[2] + pv[3]);
        rs += __shfl_xor_sync(0xffffffffu, rs, 1);
        rs += __shfl_xor_sync(0xffffffffu, rs, 2);
        l = l * alpha + rs;
        m = m_new;
#pragma unroll
        for (int dt = 0; dt < 8; ++dt) {
          o[dt][0] *= alpha;
          o[dt][1] *= alpha;
        }
        // ---- O += P V (P as bf16 hi + lo) ------------------------------------
        uint32_t ph0, pl0, ph2, pl2;
        split_bf16x2(pv[0], pv[1], ph0, pl0);
        split_bf16x2(pv[2], pv[3], ph2, pl2);
#pragma unroll
        for (int dp = 0; dp < 4; ++dp) {
          const int mi = lane >> 3, rr = lane & 7;
          const int row = row_of(tau0 + (mi & 1) * 8 + rr);
          const int chunk = dp * 2 + (mi >> 1);
          const uint32_t addr = smem_addr(vst) + row * ROW_BYTES + ((chunk ^ (row & 7)) << 4);
          uint32_t v0, v1, v2, v3;
          ldsm_x4_trans(addr, v0, v1, v2, v3);
          mma_16816(o[2 * dp], ph0, ph2, v0, v1);
          mma_16816(o[2 * dp], pl0, pl2, v0, v1);
          mma_16816(o[2 * dp + 1], ph0, ph2, v2, v3);
          mma_16816(o[2 * dp + 1], pl0, pl2, v2, v3);
        }
        // ---- score side data ------------------------------------------------
        if (mode != CE_MODE_NONE) {
          const int64_t cbase = ip_b + static_cast<int64_t>(j) * UPS;
          if (P == 1) {
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
              for (int i = 0; i < 2; ++i) {
                const int tau = tau0 + nt * 8 + 2 * t + i;
                if (tau < ntok) {
                  const int64_t cpos = cbase + tau;
                  if (cpos < p.kv_capacity) p.ul[cpos * H + head] = sv[nt * 2 + i];
                }
              }
          } else if (mode == CE_MODE_SUM) {
            // P == 16: the warp's 16 tokens are exactly one page.
            if (t == 0) {
              const int64_t cpos = cbase + tb;
              if (cpos < p.kv_capacity) p.ul[cpos * H + head] = (rs > 0.f) ? mu + log2f(rs) : -INFINITY;
            }
          } else {
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
              for (int i = 0; i < 2; ++i) {
                const int tau = tau0 + nt * 8 + 2 * t + i;
                if (tau < ntok) {
                  const int64_t cpos = cbase + tau / P;
                  if (cpos < p.kv_capacity) p.tl[(cpos * P + tau % P) * H + head] = sv[nt * 2 + i];
                }
              }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (!aborted && cur_b >= 0) epilogue(cur_b);
  }
  __syncthreads();
}

// ---- finalize: split combine + scores ------------------------------------------
constexpr int FIN_THREADS = 256;
constexpr int FIN_WARPS = FIN_THREADS / 32;
constexpr int MAX_SLOTS = 160 * NCW;   // (record, sub-part) slots a sequence can span
constexpr int UNITS_PER_TASK = 128;

struct FinParams {
  Params a;
  int P;
  int grid;   // attention grid (partition count)
};

__device__ __forceinline__ int cta_of_stage(int64_t x, int64_t S, int64_t grid) {
  return static_cast<int>(((x + 1) * grid - 1) / S);
}

// When there are fewer stages than CTAs some partitions are empty and leave
// no record; a sequence's record range [k0, k1] may straddle them.
__device__ __forceinline__ bool cta_has_work(int64_t k, int64_t S, int64_t grid) {
  return (k * S) / grid < ((k + 1) * S) / grid;
}

__device__ __forceinline__ void seq_records(const Params& p, int b, int64_t S, int64_t grid,
                                            int& k0, int& k1) {
  const int64_t pre = p.prefix[b], n = p.prefix[b + 1] - pre;
  if (n <= 0) {
    k0 = 1;
    k1 = 0;
    return;
  }
  k0 = cta_of_stage(pre, S, grid);
  k1 = cta_of_stage(pre + n - 1, S, grid);
}

// Warp-cooperative log2 normaliser of query head h over its (record, sub)
// slots plus the sink.  Every lane returns M and L2 = log2 sum.
__device__ __forceinline__ void warp_head_norm(const Params& p, int b, int h, int k0, int k1,
                                               int64_t S, int64_t grid, float& M, float& L2) {
  const int lane = threadIdx.x & 31;
  const int G = p.G, g = h / GROUP, r = h % GROUP, subs = NCW / G;
  const int nslots = (k1 - k0 + 1) * subs;
  float m = -INFINITY;
  for (int i = lane; i < nslots; i += 32) {
    const int k = k0 + i / subs, sb = i % subs;
    if (!cta_has_work(k, S, grid)) continue;
    const float* rec = p.rec + static_cast<int64_t>(b + k) * REC_FLOATS;
    m = fmaxf(m, rec[REC_ROWS * D + (sb * G + g) * 8 + r]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float sink2 = p.sinks ? p.sinks[h] * LOG2E : -INFINITY;
  M = fmaxf(m, sink2);
  if (M == -INFINITY) {
    L2 = -INFINITY;
    return;
  }
  float den = 0.f;
  for (int i = lane; i < nslots; i += 32) {
    const int k = k0 + i / subs, sb = i % subs;
    if (!cta_has_work(k, S, grid)) continue;
    const float* rec = p.rec + static_cast<int64_t>(b + k) * REC_FLOATS;
    const int vrow = (sb * G + g) * 8 + r;
    const float mk = rec[REC_ROWS * D + vrow];
    if (mk != -INFINITY) den += rec[REC_ROWS * D + REC_ROWS + vrow] * exp2f(mk - M);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
  if (p.sinks) den += exp2f(sink2 - M);
  L2 = M + log2f(den);
}

__global__ void __launch_bounds__(FIN_THREADS)
    finalize_kernel(const FinParams f) {
  const Params& p = f.a;
  const int bs = p.bs, H = p.H, G = p.G, P = f.P;
  const int subs = NCW / G;
  const int64_t S = p.prefix[bs];
  const int64_t grid = eff_grid(S, f.grid);
  const int64_t total_units = min(static_cast<int64_t>(p.kv_indptr[bs]), p.kv_capacity);
  const int hgroups = H / GROUP;
  const int64_t combine_tasks = static_cast<int64_t>(bs) * hgroups;
  const bool scoring = p.mode_of_row && p.scores && p.ul;
  const int64_t unit_tasks = scoring ? (total_units + UNITS_PER_TASK - 1) / UNITS_PER_TASK : 0;
  const int64_t ntasks = combine_tasks + unit_tasks;
  __shared__ float wts[GROUP][MAX_SLOTS];
  __shared__ float sh_l2[64];
  __shared__ int sh_b;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  for (int64_t task = blockIdx.x; task < ntasks; task += gridDim.x) {
    if (task < combine_tasks) {
      // -------- combine sequence b, query heads hc*8 .. hc*8+7 ---------------
      const int b = static_cast<int>(task / hgroups), hc = static_cast<int>(task % hgroups);
      int k0, k1;
      seq_records(p, b, S, grid, k0, k1);
      const int nslots = (k1 - k0 + 1) * subs;
      const int h = hc * GROUP + warp;   // one warp per head
      float M, L2;
      warp_head_norm(p, b, h, k0, k1, S, grid, M, L2);
      const int g = h / GROUP, r = h % GROUP;
      const bool fits = nslots <= MAX_SLOTS;
      if (fits) {
        for (int i = lane; i < nslots; i += 32) {
          const int k = k0 + i / subs, sb = i % subs;
          float w = 0.f;
          if (L2 != -INFINITY && cta_has_work(k, S, grid)) {
            const float mk = p.rec[static_cast<int64_t>(b + k) * REC_FLOATS + REC_ROWS * D + (sb * G + g) * 8 + r];
            if (mk != -INFINITY) w = exp2f(mk - L2);
          }
          wts[warp][i] = w;
        }
      }
      if (lane == 0 && p.lse_out) p.lse_out[static_cast<int64_t>(b) * H + h] = L2 * LN2;
      __syncwarp();
      // Each warp writes its head's 64 outputs: O = sum_slots w_slot * O_slot.
      for (int d = lane; d < D; d += 32) {
        float acc = 0.f;
        for (int i = 0; i < nslots; ++i) {
          const int k = k0 + i / subs, sb = i % subs;
          float w;
          if (fits) {
            w = wts[warp][i];
          } else {
            w = 0.f;
            if (L2 != -INFINITY && cta_has_work(k, S, grid)) {
              const float mk = p.rec[static_cast<int64_t>(b + k) * REC_FLOATS + REC_ROWS * D + (sb * G + g) * 8 + r];
              if (mk != -INFINITY) w = exp2f(mk - L2);
            }
          }
          if (w != 0.f) acc += w * p.rec[static_cast<int64_t>(b + k) * REC_FLOATS + ((sb * G + g) * 8 + r) * D + d];
        }
        const int64_t off = static_cast<int64_t>(b) * p.o_sb + static_cast<int64_t>(h) * p.o_sh + d;
        if (p.out_f32)
          reinterpret_cast<float*>(p.out)[off] = acc;
        else
          reinterpret_cast<__nv_bfloat16*>(p.out)[off] = __float2bfloat16_rn(acc);
      }
      __syncwarp();
    } else {
      // -------- scores of UNITS_PER_TASK consecutive CSR units ----------------
      const int64_t u0 = (task - combine_tasks) * UNITS_PER_TASK;
      const int64_t u_end = min(u0 + UNITS_PER_TASK, total_units);
      if (threadIdx.x == 0) {
        int lo = 0, hi = bs - 1;
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (p.kv_indptr[mid] <= u0) lo = mid; else hi = mid - 1;
        }
        sh_b = lo;
      }
      __syncthreads();
      int b = sh_b;
      int64_t u = u0;
      while (u < u_end && b < bs) {
        const int64_t seg_end = min(u_end, static_cast<int64_t>(p.kv_indptr[b + 1]));
        int mode = seq_mode(p, b);
        if (mode == CE_MODE_MAX && P > 1 && !p.tl) mode = CE_MODE_NONE;
        if ((mode == CE_MODE_SUM || mode == CE_MODE_MAX) && seg_end > u) {
          int k0, k1;
          seq_records(p, b, S, grid, k0, k1);
          for (int h = warp; h < H; h += FIN_WARPS) {
            float M, L2;
            warp_head_norm(p, b, h, k0, k1, S, grid, M, L2);
            if (lane == 0) sh_l2[h] = L2;
          }
          __syncthreads();
          const int tokens = seq_tokens(p, b, P);
          const int npages = (tokens + P - 1) / P;
          const int64_t npairs = (seg_end - u) * G;
          for (int64_t pr = threadIdx.x; pr < npairs; pr += FIN_THREADS) {
            const int64_t cpos = u + pr / G;
            const int g = static_cast<int>(pr % G);
            const int64_t jj = cpos - p.kv_indptr[b];
            if (jj >= npages) continue;
            const int unit = p.kv_indices[cpos];
            if (unit < 0 || unit >= p.pool_units) {
              flag_error(p.err, CE_EW_INDEX);
              continue;
            }
            const float* L2 = sh_l2 + g * GROUP;
            float contrib = 0.f;
            if (mode == CE_MODE_SUM) {
              const float* uv = p.ul + cpos * H + g * GROUP;
#pragma unroll
              for (int rr = 0; rr < GROUP; ++rr)
                if (uv[rr] != -INFINITY) contrib += exp2f(uv[rr] - L2[rr]);
            } else if (P == 1) {
              const float* uv = p.ul + cpos * H + g * GROUP;
              float mx = 0.f;
#pragma unroll
              for (int rr = 0; rr < GROUP; ++rr) mx = fmaxf(mx, exp2f(uv[rr] - L2[rr]));
              contrib = mx;
            } else {
              const int vt = (jj == npages - 1) ? tokens - static_cast<int>(jj) * P : P;
              for (int tt = 0; tt < vt; ++tt) {
                const float* uv = p.tl + (cpos * P + tt) * H + g * GROUP;
                float mx = 0.f;
#pragma unroll
                for (int rr = 0; rr < GROUP; ++rr) mx = fmaxf(mx, exp2f(uv[rr] - L2[rr]));
                contrib += mx;
              }
            }
            float* sp = p.scores + g * p.score_sg + unit;
            const bool fresh = p.zero_new && jj == npages - 1 && ((tokens - 1) % P) == 0;
            *sp = fresh ? contrib : *sp + contrib;
          }
        }
        __syncthreads();
        u = max(u, seg_end);
        ++b;
      }
      __syncthreads();
    }
  }
}

}  // namespace decode
}  // namespace ce

using namespace ce;
using namespace ce::decode;

namespace {

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct DecodeLayout {
  size_t prefix, rec, ul, tl, total;
};

DecodeLayout decode_layout(int bs, int64_t cap, int H, int P, int flags, int grid) {
  DecodeLayout L{};
  size_t off = 0;
  L.prefix = off;
  off += align256(sizeof(int32_t) * (bs + 1));
  L.rec = off;
  off += align256(sizeof(float) * (size_t)(bs + grid) * REC_FLOATS);
  L.ul = off;
  if (flags & 3) off += align256(sizeof(float) * (size_t)cap * H);
  L.tl = off;
  if ((flags & 2) && P > 1) off += align256(sizeof(float) * (size_t)cap * P * H);
  L.total = off;
  return L;
}

}  // namespace

extern "C" int64_t ce_decode_workspace_bytes(int32_t bs, int64_t kv_capacity, int32_t num_q_heads,
                                             int32_t num_kv_heads, int32_t page_size,
                                             int32_t score_flags) {
  (void)num_kv_heads;
  if (bs < 0 || kv_capacity < 0 || num_q_heads <= 0 || page_size <= 0) return -1;
  const int grid = host::sm_count();
  if (grid <= 0) return -1;
  return (int64_t)decode_layout(bs, kv_capacity, num_q_heads, page_size, score_flags, grid).total;
}

extern "C" int ce_decode_attn_score(const void* q, int64_t q_sb, int64_t q_sh, const void* k_pool,
                                    const void* v_pool, int64_t pool_units,
                                    const int32_t* kv_indptr, const int32_t* kv_indices,
                                    const int32_t* kv_tokens, int64_t kv_capacity,
                                    const float* sinks, const int32_t* mode_of_row,
                                    const int64_t* rows, float sm_scale, int32_t bs,
                                    int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                    int32_t page_size, float* scores, int64_t score_sg,
                                    int32_t zero_new, void* out, int32_t out_f32, int64_t o_sb,
                                    int64_t o_sh, float* lse_out, int32_t score_flags,
                                    void* workspace, int64_t workspace_bytes, int32_t* err,
                                    void* stream) {
  if (bs < 0 || pool_units < 0 || kv_capacity < 0) return host::fail(CE_ERR_ARG, "negative size");
  if (head_dim != D) return host::fail(CE_ERR_UNSUPPORTED, "head_dim must be 64");
  if (num_kv_heads <= 0 || num_q_heads != GROUP * num_kv_heads || NCW % num_kv_heads != 0)
    return host::fail(CE_ERR_UNSUPPORTED, "need 8 query heads per KV head and 1/2/4/8 KV heads");
  if (!(page_size == 16 || (page_size == 1 && num_kv_heads == 8)))
    return host::fail(CE_ERR_UNSUPPORTED, "page_size must be 16 (or 1 with 8 KV heads)");
  if (bs == 0) return CE_OK;
  if (!q || !k_pool || !v_pool || !kv_indptr || !kv_indices || !out || !workspace)
    return host::fail(CE_ERR_ARG, "null pointer");
  if (page_size > 1 && !kv_tokens) return host::fail(CE_ERR_ARG, "kv_tokens required for page_size > 1");
  if (pool_units * num_kv_heads * (int64_t)page_size >= (int64_t(1) << 31))
    return host::fail(CE_ERR_UNSUPPORTED, "pool too large for 32-bit TMA rows");
  if ((reinterpret_cast<uintptr_t>(k_pool) | reinterpret_cast<uintptr_t>(v_pool)) & 15)
    return host::fail(CE_ERR_ARG, "pools must be 16-byte aligned");
  if ((q_sh | q_sb) & 1) return host::fail(CE_ERR_ARG, "q strides must be even");
  const int grid = host::sm_count();
  if (grid <= 0) return host::fail(CE_ERR_CUDA, "no device");
  DecodeLayout L = decode_layout(bs, kv_capacity, num_q_heads, page_size, score_flags, grid);
  if (workspace_bytes < (int64_t)L.total) return host::fail(CE_ERR_WORKSPACE, "decode workspace too small");

  CUtensorMap kmap, vmap;
  const uint64_t rows_total = (uint64_t)pool_units * num_kv_heads * page_size;
  const uint32_t box_rows = num_kv_heads * page_size;
  if (pool_units == 0) return host::fail(CE_ERR_ARG, "empty pool");
  if (!host::encode_rows_map(&kmap, k_pool, rows_total, D, box_rows) ||
      !host::encode_rows_map(&vmap, v_pool, rows_total, D, box_rows))
    return host::fail(CE_ERR_CUDA, "cuTensorMapEncodeTiled failed");

  Params p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_sb = q_sb;
  p.q_sh = q_sh;
  p.kv_indptr = kv_indptr;
  p.kv_indices = kv_indices;
  p.kv_tokens = kv_tokens;
  p.kv_capacity = kv_capacity;
  p.pool_units = pool_units;
  p.sinks = sinks;
  p.mode_of_row = mode_of_row;
  p.rows = rows;
  p.scale_log2 = sm_scale * LOG2E;
  p.bs = bs;
  p.H = num_q_heads;
  p.G = num_kv_heads;
  p.scores = scores;
  p.score_sg = score_sg;
  p.zero_new = zero_new;
  p.out = out;
  p.out_f32 = out_f32;
  p.o_sb = o_sb;
  p.o_sh = o_sh;
  p.lse_out = lse_out;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.prefix = reinterpret_cast<int32_t*>(ws + L.prefix);
  p.rec = reinterpret_cast<float*>(ws + L.rec);
  p.ul = (score_flags & 3) ? reinterpret_cast<float*>(ws + L.ul) : nullptr;
  p.tl = ((score_flags & 2) && page_size > 1) ? reinterpret_cast<float*>(ws + L.tl) : nullptr;
  p.err = err;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (page_size == 16) {
    if (!host::set_smem(attn_kernel<16>, SMEM_BYTES)) return host::fail(CE_ERR_CUDA, "smem attr");
    attn_kernel<16><<<grid, THREADS, SMEM_BYTES, st>>>(kmap, vmap, p);
  } else {
    if (!host::set_smem(attn_kernel<1>, SMEM_BYTES)) return host::fail(CE_ERR_CUDA, "smem attr");
    attn_kernel<1><<<grid, THREADS, SMEM_BYTES, st>>>(kmap, vmap, p);
  }
  if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("attn_kernel launch");
  FinParams f{p, page_size, grid};
  finalize_kernel<<<2 * grid, FIN_THREADS, 0, st>>>(f);
  if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("finalize_kernel launch");
  return CE_OK;
}

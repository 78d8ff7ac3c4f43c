// K1: fused paged GQA decode attention + H2O score for sm_100a.
//
// Replaces, in one pass over the KV pool, what the reference does in two:
// SGLang's split-KV decode_attention_fwd (stage 1 + 2) followed by the
// overlay's _decode_scores Triton kernel that re-reads every resident key
// (code/cache_eviction/sglang_evict_runtime.py:155-224).
//
// Work split (stream-K over tokens): the concatenation of all sequences'
// 16-token-per-warp "stages" is cut into equal contiguous ranges, one per
// persistent CTA.  A CTA walks its range sequence by sequence and leaves one
// partial record (per-warp running max m, sum l and unnormalised O) for every
// sequence it touched.  Record (b, cta) lives at index b + cta, which is unique
// because both walks are monotone.  combine_kernel then merges each
// sequence's records with the sink into the output and the log-sum-exp.
//
// Inside a CTA: warps 8..11 are the producers (stage k is issued by warp
// 8 + k % 4).  They issue one 2D bulk-tensor (TMA) load per KV page for K and
// one for V (box = the page's G*P rows of 128 B, 128-byte swizzle) into a
// ring of shared-memory stages guarded by mbarriers.
// Warps 0..7 consume: warp w owns KV head g = w % G and 16 tokens of the
// stage; they copy their K and V fragments to registers and release the stage
// before doing any math.  S^T = K Q^T and O^T += V^T P^T run on m16n8k16 bf16
// tensor-core tiles (tokens, then head dims, as the 16-row operand; the group's
// 8 query heads as the 8 columns); P^T is formed in registers by movmatrix and
// enters as a bf16 hi/lo pair so the output keeps ~fp32 accuracy.
//
// Scores need the final normaliser.  For H2O rows the consumer stores, per KV
// page and query head, log2 of the page's probability mass relative to the
// running max (CE_MODE_SUM), or every token's logit (CE_MODE_MAX, which needs a
// max over heads per token).  combine_kernel, after merging a sequence, adds
//   SUM: sum_h 2^(page_lse - LSE_h)   MAX: sum_t max_h 2^(s_t,h - LSE_h)
// into scores[g, unit] with a plain read-modify-write: a unit appears once in
// a batch, as in the reference kernel (runtime:199-200).  LSE_h is the same
// normaliser as decode stage 2 and the reference score kernel
// (runtime:179-188): every key's logit plus the sink.
#include <algorithm>
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
constexpr int NPW = 4;                    // producer warps (stage k is issued by warp NCW + k % NPW)
constexpr int THREADS = (NCW + NPW) * 32;
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
  float* lse2;       // [bs, H] log2 normaliser per query head (for scores)
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

__device__ __forceinline__ int cta_of_stage(int64_t x, int64_t S, int64_t grid) {
  return static_cast<int>(((x + 1) * grid - 1) / S);
}

// When there are fewer stages than CTAs some partitions are empty and leave
// no record; a sequence's record range [k0, k1] may straddle them.
__device__ __forceinline__ bool cta_has_work(int64_t k, int64_t S, int64_t grid) {
  return (k * S) / grid < ((k + 1) * S) / grid;
}

__device__ __forceinline__ void store_out(const Params& p, int b, int h, int d, float v) {
  const int64_t off = static_cast<int64_t>(b) * p.o_sb + static_cast<int64_t>(h) * p.o_sh + d;
  if (p.out_f32)
    reinterpret_cast<float*>(p.out)[off] = v;
  else
    reinterpret_cast<__nv_bfloat16*>(p.out)[off] = __float2bfloat16_rn(v);
}

// A sequence with no tokens attends only to the sink: zero output.
__device__ void empty_sequence(const Params& p, int b) {
  for (int h = 0; h < p.H; ++h) {
    for (int d = 0; d < D; ++d) store_out(p, b, h, d, 0.f);
    const float s2 = p.sinks ? p.sinks[h] * LOG2E : -INFINITY;
    p.lse2[static_cast<int64_t>(b) * p.H + h] = s2;
    if (p.lse_out) p.lse_out[static_cast<int64_t>(b) * p.H + h] = s2 * LN2;
  }
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
      const int64_t n = (seq_tokens(p, b, P) + ST - 1) / ST;
      run += n;
      if (n == 0) empty_sequence(p, b);   // no CTA will touch it
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

  if (warp >= NCW) {
    // ------------------------------- producers -------------------------------
    // Every producer warp walks every stage (sequence and page-index window
    // state stay warp-uniform); stage k's loads are issued by warp NCW + k % NPW,
    // so consecutive stages' TMA issue overlaps.  At one KV head per GPU a stage
    // is 8 pages, 16 boxes of 2 KB, and one issuing warp capped the kernel at
    // ~4.1 TB/s; with four, every head count streams ~5.9-6.0 TB/s.
    const int pw = warp - NCW;
    // Page indices are read in 32-entry windows (the CTA's CSR positions only
    // move forward): the two windows in use and a third one in flight, so a
    // window is loaded a whole window of stages before any lookup reads it
    // and no TMA issue waits on a dependent global load.  (With one window
    // ahead, a stage of 8 pages -- one KV head per GPU -- waited for a load
    // every 4 stages.)
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
    int idx_cur = -2, idx_next = -2, idx_ahead = -2;
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
        idx_ahead = fetch(w0 + 64);
      } else if (c0 >= w0 + 32) {
        w0 += 32;
        idx_cur = idx_next;
        idx_next = idx_ahead;
        idx_ahead = fetch(w0 + 64);
      }
      const int s = issued % NSTAGES;
      const uint32_t ph = (issued / NSTAGES) & 1;
      if (issued % NPW != pw) {
        ++issued;
        continue;
      }
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
    // Drain: every load this warp issued must land before the CTA may exit.
    if (lane == 0) {
      for (int it = max(0, issued - NSTAGES); it < issued; ++it)
        if (it % NPW == pw) mbar_wait(&full[it % NSTAGES], (it / NSTAGES) & 1, p.err);
    }
  } else {
    // ------------------------------- consumers -------------------------------
    // Warp w owns KV head g = w % G and tokens [16*tb, 16*tb+16) of each stage.
    // S^T = K Q^T: the 16 tokens are the MMA rows (no padding), the group's 8
    // query heads the columns.  Thread (r = lane/4, t = lane%4) holds tokens r
    // and r+8 for heads 2t and 2t+1, and keeps the running max/sum of those two
    // heads.  O^T = V^T P^T: 4 tiles of 16 dims x 8 heads; P^T comes from the
    // S^T fragments by an in-register 8x8 transpose (movmatrix).
    const int g = warp % G;
    const int tb = warp / G;
    const int r = lane >> 2;
    const int t = lane & 3;
    const int head = g * GROUP + r;     // head whose q row this lane loads
    const int tau0 = tb * 16;

    auto row_of = [&](int tau) -> int { return (tau / P) * UNIT_ROWS + g * P + (tau % P); };

    // Swizzled shared-memory offsets of this lane's ldmatrix rows: the same in
    // every stage, so they are computed once.
    uint32_t koff[4], voff[4];
    {
      const int mi = lane >> 3, rr = lane & 7;
      const int krow = row_of(tau0 + (mi & 1) * 8 + rr);
      const int vrow = row_of(tau0 + (mi >> 1) * 8 + rr);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        koff[c] = krow * ROW_BYTES + (((c * 2 + (mi >> 1)) ^ (krow & 7)) << 4);
        voff[c] = HALF_STAGE + vrow * ROW_BYTES + (((c * 2 + (mi & 1)) ^ (vrow & 7)) << 4);
      }
    }
    const uint32_t ring = smem_addr(smem);

    uint32_t qb[4][2];                  // B operand (Q^T) per k-step
    float o[4][4];                      // O^T accumulators
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
    int cur_b = -1, mode = CE_MODE_NONE;

    auto leave = [&](int bb) {
      float* rec = p.rec + static_cast<int64_t>(bb + blockIdx.x) * REC_FLOATS;
      const int v0 = warp * 8 + 2 * t;   // virtual rows of heads 2t, 2t+1
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        rec[v0 * D + mt * 16 + r] = o[mt][0];
        rec[(v0 + 1) * D + mt * 16 + r] = o[mt][1];
        rec[v0 * D + mt * 16 + r + 8] = o[mt][2];
        rec[(v0 + 1) * D + mt * 16 + r + 8] = o[mt][3];
      }
      if (r == 0) {
        rec[REC_ROWS * D + v0] = m[0];
        rec[REC_ROWS * D + v0 + 1] = m[1];
        rec[REC_ROWS * D + REC_ROWS + v0] = l[0];
        rec[REC_ROWS * D + REC_ROWS + v0 + 1] = l[1];
      }
    };

    int s = 0;
    uint32_t ph = 0;
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
    for (int64_t x = S_lo; x < S_hi; ++x) {
      while (x >= base + nst) {
        base += nst;
        ++b;
        load_seq(b);
      }
      if (b != cur_b) {
        if (cur_b >= 0) leave(cur_b);
        cur_b = b;
        const __nv_bfloat16* qrow = p.q + static_cast<int64_t>(b) * p.q_sb + static_cast<int64_t>(head) * p.q_sh;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          qb[ks][0] = *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 2 * t);
          qb[ks][1] = *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 8 + 2 * t);
        }
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
        m[0] = m[1] = -INFINITY;
        l[0] = l[1] = 0.f;
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
      const int cs = s;
      const uint32_t cph = ph;
      if (++s == NSTAGES) {
        s = 0;
        ph ^= 1u;
      }
      // After a timeout the warp keeps walking (so the record writes stay in
      // step) but waits for and computes nothing more.
      if (!aborted && !mbar_wait_or_abort(&full[cs], cph, p.err, abort_flag)) {
        *abort_flag = 1;
        aborted = true;
      }
      if (aborted) continue;
      uint8_t* kst = smem + cs * STAGE_BYTES;
      uint8_t* vst = kst + HALF_STAGE;
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
      if (tau0 >= ntok) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[cs]);
        continue;
      }
      // ---- copy the warp's K and V fragments out, then release the stage -----
      const uint32_t sbase = ring + cs * STAGE_BYTES;
      uint32_t kf[4][4], vf[4][4];
#pragma unroll
      for (int c = 0; c < 4; ++c) ldsm_x4(sbase + koff[c], kf[c][0], kf[c][1], kf[c][2], kf[c][3]);
#pragma unroll
      for (int c = 0; c < 4; ++c)
        ldsm_x4_trans(sbase + voff[c], vf[c][0], vf[c][1], vf[c][2], vf[c][3]);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[cs]);   // release orders the reads above
      // ---- S^T = K Q^T over the warp's 16 tokens: 4 MMAs ----------------------
      float sacc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        mma_16816_full(sacc, kf[ks][0], kf[ks][1], kf[ks][2], kf[ks][3], qb[ks][0], qb[ks][1]);
      const bool v_lo = tau0 + r < ntok, v_hi = tau0 + r + 8 < ntok;
      float sv[4];
      sv[0] = v_lo ? sacc[0] * p.scale_log2 : -INFINITY;
      sv[1] = v_lo ? sacc[1] * p.scale_log2 : -INFINITY;
      sv[2] = v_hi ? sacc[2] * p.scale_log2 : -INFINITY;
      sv[3] = v_hi ? sacc[3] * p.scale_log2 : -INFINITY;
      float mx0 = fmaxf(sv[0], sv[2]), mx1 = fmaxf(sv[1], sv[3]);
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
      }
      const float mn0 = fmaxf(m[0], mx0), mn1 = fmaxf(m[1], mx1);
      const float mu0 = (mn0 == -INFINITY) ? 0.f : mn0;
      const float mu1 = (mn1 == -INFINITY) ? 0.f : mn1;
      float pv[4];
      pv[0] = exp2f(sv[0] - mu0);
      pv[1] = exp2f(sv[1] - mu1);
      pv[2] = exp2f(sv[2] - mu0);
      pv[3] = exp2f(sv[3] - mu1);
      float rs0 = pv[0] + pv[2], rs1 = pv[1] + pv[3];
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        rs0 += __shfl_xor_sync(0xffffffffu, rs0, off);
        rs1 += __shfl_xor_sync(0xffffffffu, rs1, off);
      }
      // Rescale the running state only when some head's max moved.
      if (__any_sync(0xffffffffu, (mn0 != m[0]) || (mn1 != m[1]))) {
        const float al0 = exp2f(m[0] - mu0), al1 = exp2f(m[1] - mu1);
        l[0] *= al0;
        l[1] *= al1;
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) {
          o[mt][0] *= al0;
          o[mt][1] *= al1;
          o[mt][2] *= al0;
          o[mt][3] *= al1;
        }
        m[0] = mn0;
        m[1] = mn1;
      }
      l[0] += rs0;
      l[1] += rs1;
      // ---- O^T += V^T P^T, P^T as bf16 hi + lo via movmatrix ------------------
      uint32_t h01, l01, h23, l23;
      split_bf16x2(pv[0], pv[1], h01, l01);
      split_bf16x2(pv[2], pv[3], h23, l23);
      const uint32_t bh0 = movmatrix_trans(h01), bh1 = movmatrix_trans(h23);
      const uint32_t bl0 = movmatrix_trans(l01), bl1 = movmatrix_trans(l23);
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        mma_16816_full(o[mt], vf[mt][0], vf[mt][1], vf[mt][2], vf[mt][3], bh0, bh1);
        mma_16816_full(o[mt], vf[mt][0], vf[mt][1], vf[mt][2], vf[mt][3], bl0, bl1);
      }
      // ---- score side data --------------------------------------------------
      if (mode != CE_MODE_NONE) {
        const int64_t cbase = ip_b + static_cast<int64_t>(j) * UPS;
        const int hcol = g * GROUP + 2 * t;
        if (P == 1) {
          if (v_lo) {
            const int64_t cpos = cbase + tau0 + r;
            if (cpos < p.kv_capacity)
              *reinterpret_cast<float2*>(p.ul + cpos * H + hcol) = make_float2(sv[0], sv[1]);
          }
          if (v_hi) {
            const int64_t cpos = cbase + tau0 + r + 8;
            if (cpos < p.kv_capacity)
              *reinterpret_cast<float2*>(p.ul + cpos * H + hcol) = make_float2(sv[2], sv[3]);
          }
        } else if (mode == CE_MODE_SUM) {
          // P == 16: the warp's 16 tokens are exactly one page.
          if (r == 0) {
            const int64_t cpos = cbase + tb;
            if (cpos < p.kv_capacity)
              *reinterpret_cast<float2*>(p.ul + cpos * H + hcol) =
                  make_float2(rs0 > 0.f ? mu0 + __log2f(rs0) : -INFINITY,
                              rs1 > 0.f ? mu1 + __log2f(rs1) : -INFINITY);
          }
        } else {
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            const int tau = tau0 + r + 8 * half;
            if (tau < ntok) {
              const int64_t cpos = cbase + tau / P;
              if (cpos < p.kv_capacity)
                *reinterpret_cast<float2*>(p.tl + (cpos * P + tau % P) * H + hcol) =
                    make_float2(sv[2 * half], sv[2 * half + 1]);
            }
          }
        }
      }
    }
    if (cur_b >= 0) leave(cur_b);
  }
  __syncthreads();
}

// ---- combine: records of a sequence + sink -> output, lse, page scores --------
//
// One task per (sequence b, KV head g, chunk c): the chunks of a (b, g) split
// its eight query heads' output merges and its page scoring between them, so
// a small batch (one sequence spread over every attention CTA) still fills the
// GPU.  Every task first rebuilds the eight heads' normalisers from the
// sequence's record slots: one pass in which thread t merges slots t, t+256,
// ... (each slot's eight maxima and sums are two pairs of 16-byte loads), then
// a shared-memory reduction per head, with the sink folded in (the normaliser
// of SGLang's stage 2 and of runtime:179-188).
constexpr int CB_THREADS = 256;
// Record slots a thread loads before merging them.  In a large batch a head
// has few slots (its sequence spans few attention CTAs): a batch of one keeps
// the kernel at 64 registers, so four blocks share an SM and a 64-sequence
// batch's 512 tasks run in one wave.  A small batch (a head's slots come from
// up to every attention CTA) takes a batch of four.
constexpr int CB_SLOT_BATCH_WIDE = 4;
constexpr int CB_MAX_CHUNKS = 64;

struct CombineParams {
  Params a;
  int grid;     // CTAs the attention kernel was launched with
  int P;
  int defer;    // CE_SCORE_DEFER: keep the normalisers in lse2, add no scores here
  int chunks;   // tasks per (sequence, KV head)
};

__device__ __forceinline__ void merge_ml(float& m, float& l, float m2, float l2) {
  if (m2 == -INFINITY) return;
  const float mn = fmaxf(m, m2);
  l = l * exp2f(m - mn) + l2 * exp2f(m2 - mn);
  m = mn;
}

// Record slots of sequence b for KV head g: slot i is sub-part i % subs of
// record k0 + i / subs (an attention CTA's warps over G heads: NCW / G of them
// per head).
struct SeqSlots {
  int b, g, subs, k0, nslots;
  int64_t S, grid;
  __device__ const float* rec(const Params& p, int i) const {
    return p.rec + static_cast<int64_t>(b + k0 + i / subs) * REC_FLOATS;
  }
  __device__ int vrow(int i, int G) const { return ((i % subs) * G + g) * GROUP; }  // + head row r
  __device__ bool live(int i) const { return cta_has_work(k0 + i / subs, S, grid); }
};

// sh_l2[r] = log2 normaliser of query head g*8 + r (record maxima, sums and
// the sink).  sh_m / sh_l: [GROUP][CB_THREADS] scratch.
template <int SB>
__device__ void group_normalisers(const Params& p, const SeqSlots& q, float* sh_m, float* sh_l,
                                  float* sh_l2) {
  const int tid = threadIdx.x, G = p.G;
  float m[GROUP], l[GROUP];
#pragma unroll
  for (int r = 0; r < GROUP; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
  }
  for (int i0 = tid; i0 < q.nslots; i0 += CB_THREADS * SB) {
    float4 ma[SB], mb[SB], la[SB], lb[SB];
#pragma unroll
    for (int u = 0; u < SB; ++u) {
      const int i = i0 + u * CB_THREADS;
      ma[u] = mb[u] = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      la[u] = lb[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i < q.nslots && q.live(i)) {
        const float4* st = reinterpret_cast<const float4*>(q.rec(p, i) + REC_ROWS * D + q.vrow(i, G));
        ma[u] = st[0];
        mb[u] = st[1];
        la[u] = st[REC_ROWS / 4];
        lb[u] = st[REC_ROWS / 4 + 1];
      }
    }
#pragma unroll
    for (int u = 0; u < SB; ++u) {
      merge_ml(m[0], l[0], ma[u].x, la[u].x);
      merge_ml(m[1], l[1], ma[u].y, la[u].y);
      merge_ml(m[2], l[2], ma[u].z, la[u].z);
      merge_ml(m[3], l[3], ma[u].w, la[u].w);
      merge_ml(m[4], l[4], mb[u].x, lb[u].x);
      merge_ml(m[5], l[5], mb[u].y, lb[u].y);
      merge_ml(m[6], l[6], mb[u].z, lb[u].z);
      merge_ml(m[7], l[7], mb[u].w, lb[u].w);
    }
  }
#pragma unroll
  for (int r = 0; r < GROUP; ++r) {
    sh_m[r * CB_THREADS + tid] = m[r];
    sh_l[r * CB_THREADS + tid] = l[r];
  }
  __syncthreads();
  // warp r reduces head r over the 256 partial states
  const int warp = tid >> 5, lane = tid & 31;
  float mw = -INFINITY, lw = 0.f;
#pragma unroll
  for (int k = 0; k < CB_THREADS / 32; ++k)
    merge_ml(mw, lw, sh_m[warp * CB_THREADS + k * 32 + lane], sh_l[warp * CB_THREADS + k * 32 + lane]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, mw, o), l2 = __shfl_xor_sync(0xffffffffu, lw, o);
    merge_ml(mw, lw, m2, l2);
  }
  if (lane == 0) {
    const int h = q.g * GROUP + warp;
    const float sink2 = p.sinks ? p.sinks[h] * LOG2E : -INFINITY;
    const float M = fmaxf(mw, sink2);
    float den = 0.f;
    if (M != -INFINITY) {
      den = (mw == -INFINITY) ? 0.f : lw * exp2f(mw - M);
      if (p.sinks) den += exp2f(sink2 - M);
    }
    sh_l2[warp] = (M == -INFINITY) ? -INFINITY : M + log2f(den);
  }
  __syncthreads();
}

// Outputs of the query heads r = c, c + C, ... (r < 8) of KV head g: each a
// sum over the slots of 2^(m_i - L2) O_i.  The block's threads split as heads
// x 16 dimension quads x slot groups; partial sums meet in shared memory.
template <int AB>
__device__ void group_outputs(const Params& p, const SeqSlots& q, int c, int C, const float* sh_l2,
                              float4* red) {
  const int nh = (c < GROUP) ? (GROUP - 1 - c) / C + 1 : 0;
  if (nh == 0) return;
  const int nhr = nh <= 1 ? 1 : nh <= 2 ? 2 : nh <= 4 ? 4 : 8;
  const int tph = CB_THREADS / nhr;        // threads per head
  const int sgn = tph / 16;                // slot groups per head
  const int tid = threadIdx.x, hh = tid / tph, lt = tid % tph, dq = lt & 15, sg = lt >> 4;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (hh < nh) {
    const int r = c + hh * C;
    const float L2 = sh_l2[r];
    for (int i0 = sg; i0 < q.nslots; i0 += sgn * AB) {
      float w[AB];
      float4 o[AB];
#pragma unroll
      for (int u = 0; u < AB; ++u) {
        const int i = i0 + u * sgn;
        w[u] = 0.f;
        o[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i < q.nslots && q.live(i) && L2 != -INFINITY) {
          // the slot's maximum and its output row are loaded together
          const float* rc = q.rec(p, i);
          const int v = q.vrow(i, p.G) + r;
          w[u] = rc[REC_ROWS * D + v];
          o[u] = reinterpret_cast<const float4*>(rc + v * D)[dq];
        } else {
          w[u] = -INFINITY;
        }
      }
#pragma unroll
      for (int u = 0; u < AB; ++u) w[u] = w[u] == -INFINITY ? 0.f : exp2f(w[u] - L2);
#pragma unroll
      for (int u = 0; u < AB; ++u) {
        if (w[u] != 0.f) {
          acc.x += w[u] * o[u].x;
          acc.y += w[u] * o[u].y;
          acc.z += w[u] * o[u].z;
          acc.w += w[u] * o[u].w;
        }
      }
    }
  }
  red[tid] = acc;
  __syncthreads();
  if (tid < nh * 16) {
    const int h2 = tid >> 4, d2 = tid & 15;
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < sgn; ++k) {
      const float4 v = red[h2 * tph + k * 16 + d2];
      s.x += v.x;
      s.y += v.y;
      s.z += v.z;
      s.w += v.w;
    }
    const int h = q.g * GROUP + c + h2 * C;
    store_out(p, q.b, h, d2 * 4 + 0, s.x);
    store_out(p, q.b, h, d2 * 4 + 1, s.y);
    store_out(p, q.b, h, d2 * 4 + 2, s.z);
    store_out(p, q.b, h, d2 * 4 + 3, s.w);
  }
}

// Add pages [lo, hi) of sequence b's page masses for KV head g into scores[g, unit]:
//   SUM: sum_h 2^(page_lse - LSE_h)   MAX: sum_t max_h 2^(s_t,h - LSE_h)
// L2s holds the group's 8 log2 normalisers.  Each thread takes 4 pages per
// round and issues all their loads before any store.
__device__ void score_pages(const Params& p, int b, int g, int mode, int P, const float* L2s, int lo,
                            int hi) {
  const int H = p.H;
  const int tokens = seq_tokens(p, b, P);
  const int npages = (tokens + P - 1) / P;
  hi = min(hi, npages);
  const int64_t ip = p.kv_indptr[b];
  float L2[GROUP];
#pragma unroll
  for (int rr = 0; rr < GROUP; ++rr) L2[rr] = L2s[rr];
  const bool fresh_tail = p.zero_new && ((tokens - 1) % P) == 0;
  const int32_t* __restrict__ kvi = p.kv_indices;
  const float* __restrict__ ul = p.ul;
  float* __restrict__ sc = p.scores + g * p.score_sg;
  constexpr int BATCH = 4;
  for (int j0 = lo + threadIdx.x * BATCH; j0 < hi; j0 += CB_THREADS * BATCH) {
    int unit[BATCH];
    float contrib[BATCH], old[BATCH];
#pragma unroll
    for (int q = 0; q < BATCH; ++q) {
      const int jj = j0 + q;
      unit[q] = -1;
      if (jj < hi && ip + jj < p.kv_capacity) unit[q] = kvi[ip + jj];
    }
#pragma unroll
    for (int q = 0; q < BATCH; ++q) {
      const int jj = j0 + q;
      contrib[q] = 0.f;
      old[q] = 0.f;
      if (unit[q] < 0 || unit[q] >= p.pool_units) continue;
      old[q] = sc[unit[q]];
      const int64_t cpos = ip + jj;
      if (mode == CE_MODE_SUM) {
        const float4* u4 = reinterpret_cast<const float4*>(ul + cpos * H + g * GROUP);
        const float4 a = u4[0], c = u4[1];
        const float uv[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
#pragma unroll
        for (int rr = 0; rr < GROUP; ++rr)
          if (uv[rr] != -INFINITY) contrib[q] += exp2f(uv[rr] - L2[rr]);
      } else if (P == 1) {
        const float* uv = ul + cpos * H + g * GROUP;
        float mx = 0.f;
#pragma unroll
        for (int rr = 0; rr < GROUP; ++rr) mx = fmaxf(mx, exp2f(uv[rr] - L2[rr]));
        contrib[q] = mx;
      } else {
        const int vt = (jj == npages - 1) ? tokens - jj * P : P;
        for (int tt = 0; tt < vt; ++tt) {
          const float* uv = p.tl + (cpos * P + tt) * H + g * GROUP;
          float mx = 0.f;
#pragma unroll
          for (int rr = 0; rr < GROUP; ++rr) mx = fmaxf(mx, exp2f(uv[rr] - L2[rr]));
          contrib[q] += mx;
        }
      }
    }
#pragma unroll
    for (int q = 0; q < BATCH; ++q) {
      const int jj = j0 + q;
      if (jj >= hi) continue;
      if (unit[q] < 0 || unit[q] >= p.pool_units) {
        if (ip + jj < p.kv_capacity) flag_error(p.err, CE_EW_INDEX);
        continue;
      }
      const bool fresh = fresh_tail && jj == npages - 1;
      sc[unit[q]] = fresh ? contrib[q] : old[q] + contrib[q];
    }
  }
}

__device__ __forceinline__ int score_mode_of(const Params& p, int b, int P) {
  int mode = (p.mode_of_row && p.scores && p.ul) ? seq_mode(p, b) : CE_MODE_NONE;
  if (mode == CE_MODE_MAX && P > 1 && !p.tl) mode = CE_MODE_NONE;
  return (mode == CE_MODE_SUM || mode == CE_MODE_MAX) ? mode : CE_MODE_NONE;
}

// Chunk c of C of sequence b's pages.
__device__ __forceinline__ void chunk_pages(const Params& p, int b, int P, int c, int C, int& lo, int& hi) {
  const int npages = (seq_tokens(p, b, P) + P - 1) / P;
  const int per = (npages + C - 1) / C;
  lo = min(npages, c * per);
  hi = min(npages, lo + per);
}

template <int SB>
__global__ void __launch_bounds__(CB_THREADS, SB == 1 ? 4 : 2) combine_kernel(const CombineParams cp) {
  const Params& p = cp.a;
  const int bs = p.bs, H = p.H, G = p.G, C = cp.chunks;
  const int64_t S = p.prefix[bs];
  const int64_t grid = eff_grid(S, cp.grid);
  const int hgroups = H / GROUP;
  const int64_t ntasks = static_cast<int64_t>(bs) * hgroups * C;
  __shared__ float sh_m[GROUP * CB_THREADS], sh_l[GROUP * CB_THREADS];
  __shared__ float4 red[CB_THREADS];
  __shared__ float sh_l2[GROUP];
  for (int64_t task = blockIdx.x; task < ntasks; task += gridDim.x) {
    const int c = static_cast<int>(task % C);
    const int64_t bg = task / C;
    const int b = static_cast<int>(bg / hgroups), hc = static_cast<int>(bg % hgroups);
    const int64_t pre = p.prefix[b], n = p.prefix[b + 1] - pre;
    if (n <= 0) continue;   // empty sequences were written by the attention kernel
    SeqSlots q;
    q.b = b;
    q.g = hc;
    q.subs = NCW / G;
    q.S = S;
    q.grid = grid;
    q.k0 = cta_of_stage(pre, S, grid);
    q.nslots = (cta_of_stage(pre + n - 1, S, grid) - q.k0 + 1) * q.subs;
    // Page scoring (else score_kernel adds the page masses later).  A chunk of
    // at most one page per thread (small batches) issues its page's index and
    // log-masses before the normaliser merge, which they do not depend on, so
    // their latency hides behind it; only the old score's load (which needs
    // the index) and the store follow the merge.
    const int mode = cp.defer ? CE_MODE_NONE : score_mode_of(p, b, cp.P);
    int lo = 0, hi = 0;
    if (mode != CE_MODE_NONE) chunk_pages(p, b, cp.P, c, C, lo, hi);
    const bool early = mode != CE_MODE_NONE && hi - lo <= CB_THREADS && (mode == CE_MODE_SUM || cp.P == 1);
    const int jj = lo + threadIdx.x;
    const int64_t cpos = p.kv_indptr[b] + jj;
    int unit = -1;
    float4 ua = make_float4(0.f, 0.f, 0.f, 0.f), ub = ua;
    if (early && jj < hi && cpos < p.kv_capacity) {
      unit = p.kv_indices[cpos];
      const float4* u4 = reinterpret_cast<const float4*>(p.ul + cpos * H + hc * GROUP);
      ua = u4[0];
      ub = u4[1];
    }
    group_normalisers<SB>(p, q, sh_m, sh_l, sh_l2);
    group_outputs<SB == 1 ? 2 : 4>(p, q, c, C, sh_l2, red);
    if (c == 0 && threadIdx.x < GROUP) {
      const int h = hc * GROUP + threadIdx.x;
      const float L2 = sh_l2[threadIdx.x];
      if (p.lse_out) p.lse_out[static_cast<int64_t>(b) * H + h] = L2 * LN2;
      if (cp.defer) p.lse2[static_cast<int64_t>(b) * H + h] = L2;
    }
    if (early) {
      if (jj < hi && cpos < p.kv_capacity) {
        if (unit < 0 || unit >= p.pool_units) {
          flag_error(p.err, CE_EW_INDEX);
        } else {
          float* sc = p.scores + hc * p.score_sg;
          const float old = sc[unit];
          const float uv[8] = {ua.x, ua.y, ua.z, ua.w, ub.x, ub.y, ub.z, ub.w};
          float contrib = 0.f;
          if (mode == CE_MODE_SUM) {
#pragma unroll
            for (int rr = 0; rr < GROUP; ++rr)
              if (uv[rr] != -INFINITY) contrib += exp2f(uv[rr] - sh_l2[rr]);
          } else {   // MAX at page size 1: the page is one token
#pragma unroll
            for (int rr = 0; rr < GROUP; ++rr) contrib = fmaxf(contrib, exp2f(uv[rr] - sh_l2[rr]));
          }
          const int tokens = seq_tokens(p, b, cp.P);
          const int npages = (tokens + cp.P - 1) / cp.P;
          const bool fresh = p.zero_new && ((tokens - 1) % cp.P) == 0 && jj == npages - 1;
          sc[unit] = fresh ? contrib : old + contrib;
        }
      }
    } else if (mode != CE_MODE_NONE) {
      score_pages(p, b, hc, mode, cp.P, sh_l2, lo, hi);
    }
    __syncthreads();
  }
}

// The page masses of a deferred decode (CE_SCORE_DEFER): the same work as
// the tail of combine_kernel, one task per (sequence, KV head, chunk), from
// the normalisers combine_kernel left in lse2.  Small enough to run beside
// the next layer's attention kernel on another stream.
__global__ void __launch_bounds__(CB_THREADS) score_kernel(const CombineParams cp) {
  const Params& p = cp.a;
  const int hgroups = p.H / GROUP, C = cp.chunks;
  const int64_t ntasks = static_cast<int64_t>(p.bs) * hgroups * C;
  __shared__ float sh_l2[GROUP];
  for (int64_t task = blockIdx.x; task < ntasks; task += gridDim.x) {
    const int c = static_cast<int>(task % C);
    const int64_t bg = task / C;
    const int b = static_cast<int>(bg / hgroups), hc = static_cast<int>(bg % hgroups);
    const int mode = score_mode_of(p, b, cp.P);
    if (seq_tokens(p, b, cp.P) <= 0 || mode == CE_MODE_NONE) continue;
    if (threadIdx.x < GROUP) sh_l2[threadIdx.x] = p.lse2[static_cast<int64_t>(b) * p.H + hc * GROUP + threadIdx.x];
    __syncthreads();
    int lo, hi;
    chunk_pages(p, b, cp.P, c, C, lo, hi);
    score_pages(p, b, hc, mode, cp.P, sh_l2, lo, hi);
    __syncthreads();
  }
}

}  // namespace decode
}  // namespace ce

using namespace ce;
using namespace ce::decode;

namespace {

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Tasks per (sequence, KV head) of the combine and score kernels: enough for
// about two blocks per SM when the batch alone would leave SMs idle (a
// batch-1 decode has one task per KV head otherwise).
int combine_chunks(int bs, int H, int sms) {
  const int64_t base = static_cast<int64_t>(bs) * (H / GROUP);
  if (base <= 0) return 1;
  const int64_t c = (2LL * sms + base - 1) / base;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(c, CB_MAX_CHUNKS)));
}

struct DecodeLayout {
  size_t prefix, lse2, rec, ul, tl, total;
};

DecodeLayout decode_layout(int bs, int64_t cap, int H, int P, int flags, int grid) {
  DecodeLayout L{};
  size_t off = 0;
  L.prefix = off;
  off += align256(sizeof(int32_t) * (bs + 1));
  L.lse2 = off;
  off += align256(sizeof(float) * (size_t)bs * H);
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
  p.lse2 = reinterpret_cast<float*>(ws + L.lse2);
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
  const bool defer = (score_flags & CE_SCORE_DEFER) != 0;
  CombineParams cp{p, grid, page_size, defer ? 1 : 0, combine_chunks(bs, num_q_heads, grid)};
  // A deferred decode's page scores run beside the next layer's attention
  // kernel (195 KB of shared memory per CTA): keep SMs at the largest carveout.
  const int64_t tasks = static_cast<int64_t>(bs) * (num_q_heads / GROUP) * cp.chunks;
  const int cb_grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(tasks, 4LL * grid)));
  // Fewer (sequence, KV head) pairs than attention CTAs: each head has many
  // record slots (up to one per CTA and warp group) and the tasks are chunks
  // of few sequences -- the wide variant's batched loads win.
  const bool wide = static_cast<int64_t>(bs) * (num_q_heads / GROUP) < grid;
  if (wide) {
    if (defer && !host::set_max_shared_carveout(combine_kernel<CB_SLOT_BATCH_WIDE>))
      return host::fail(CE_ERR_CUDA, "carveout attr");
    combine_kernel<CB_SLOT_BATCH_WIDE><<<cb_grid, CB_THREADS, 0, st>>>(cp);
  } else {
    if (defer && !host::set_max_shared_carveout(combine_kernel<1>)) return host::fail(CE_ERR_CUDA, "carveout attr");
    combine_kernel<1><<<cb_grid, CB_THREADS, 0, st>>>(cp);
  }
  if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("combine_kernel launch");
  return CE_OK;
}

int ce::host::decode_prepare_device() {
  // cudaFuncGetAttributes loads a kernel under lazy module loading; the
  // shared-memory attribute is the one the first launch would set.
  cudaFuncAttributes a;
  if (!host::set_smem(attn_kernel<16>, SMEM_BYTES) || !host::set_smem(attn_kernel<1>, SMEM_BYTES) ||
      cudaFuncGetAttributes(&a, combine_kernel<1>) != cudaSuccess ||
      cudaFuncGetAttributes(&a, combine_kernel<CB_SLOT_BATCH_WIDE>) != cudaSuccess)
    return host::fail_cuda("decode kernels: set-up");
  return CE_OK;
}

extern "C" int ce_decode_scores(const int32_t* kv_indptr, const int32_t* kv_indices,
                                const int32_t* kv_tokens, int64_t kv_capacity, int64_t pool_units,
                                const int32_t* mode_of_row, const int64_t* rows, int32_t bs,
                                int32_t num_q_heads, int32_t num_kv_heads, int32_t page_size,
                                float* scores, int64_t score_sg, int32_t zero_new, int32_t score_flags,
                                const void* workspace, int64_t workspace_bytes, int32_t* err,
                                void* stream) {
  if (bs < 0 || pool_units < 0 || kv_capacity < 0) return host::fail(CE_ERR_ARG, "negative size");
  if (num_kv_heads <= 0 || num_q_heads != GROUP * num_kv_heads || NCW % num_kv_heads != 0)
    return host::fail(CE_ERR_UNSUPPORTED, "need 8 query heads per KV head and 1/2/4/8 KV heads");
  if (!(page_size == 16 || (page_size == 1 && num_kv_heads == 8)))
    return host::fail(CE_ERR_UNSUPPORTED, "page_size must be 16 (or 1 with 8 KV heads)");
  if (bs == 0 || !mode_of_row || !scores || !(score_flags & 3)) return CE_OK;
  if (!kv_indptr || !kv_indices || !workspace) return host::fail(CE_ERR_ARG, "null pointer");
  if (page_size > 1 && !kv_tokens) return host::fail(CE_ERR_ARG, "kv_tokens required for page_size > 1");
  const int grid = host::sm_count();
  if (grid <= 0) return host::fail(CE_ERR_CUDA, "no device");
  DecodeLayout L = decode_layout(bs, kv_capacity, num_q_heads, page_size, score_flags, grid);
  if (workspace_bytes < (int64_t)L.total) return host::fail(CE_ERR_WORKSPACE, "decode workspace too small");
  Params p{};
  p.kv_indptr = kv_indptr;
  p.kv_indices = kv_indices;
  p.kv_tokens = kv_tokens;
  p.kv_capacity = kv_capacity;
  p.pool_units = pool_units;
  p.mode_of_row = mode_of_row;
  p.rows = rows;
  p.bs = bs;
  p.H = num_q_heads;
  p.G = num_kv_heads;
  p.scores = scores;
  p.score_sg = score_sg;
  p.zero_new = zero_new;
  uint8_t* ws = static_cast<uint8_t*>(const_cast<void*>(workspace));
  p.lse2 = reinterpret_cast<float*>(ws + L.lse2);
  p.ul = reinterpret_cast<float*>(ws + L.ul);
  p.tl = ((score_flags & 2) && page_size > 1) ? reinterpret_cast<float*>(ws + L.tl) : nullptr;
  p.err = err;
  CombineParams cp{p, grid, page_size, 1, combine_chunks(bs, num_q_heads, grid)};
  if (!host::set_max_shared_carveout(score_kernel)) return host::fail(CE_ERR_CUDA, "carveout attr");
  const int sc_grid = static_cast<int>(std::max<int64_t>(
      1, std::min<int64_t>(static_cast<int64_t>(bs) * (num_q_heads / GROUP) * cp.chunks, 2LL * grid)));
  score_kernel<<<sc_grid, CB_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(cp);
  if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("score_kernel launch");
  return CE_OK;
}

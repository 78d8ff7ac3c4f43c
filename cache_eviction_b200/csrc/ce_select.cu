// K2 (selection) and K3 (compaction) for sm_100a.
//
// Selection follows the reference's choose (code/cache_eviction/sglang_evict_runtime.py:376-397):
// positions below the prefix, in the recent window or at/after the
// sliding-window cursor are protected; the rest of the budget goes to the
// largest keys, ties to the newer (larger) position; prefix_sliding keeps only
// the protected set.  Instead of two argsorts per (layer, KV head) each CTA runs
// an MSB-first 8-bit radix select on order-preserving integer keys (fp32 scores,
// fp64 uniforms and 53-bit reservoir draws all map to unsigned integers with the
// same order, and -0.0 folds onto +0.0 as in the reference's double compare),
// then breaks the remaining tie with a second radix select on position.  The
// kept set is written in ascending position order by ranking positions in a
// shared-memory bitmap (rank = popcount prefix), which is the order _boundary
// needs (runtime:442-446).
//
// Compaction follows _boundary (runtime:415-507): every head's j-th middle
// survivor moves to the j-th non-protected candidate unit (column order).  A
// source unit that is also some other item's target is a hazard; those sources
// are staged in a scratch buffer by one launch and every item is written by the
// next launch, which reproduces the reference's "gather all sources, then
// scatter" semantics without copying the non-hazard items twice.
#include <algorithm>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include "ce_common.cuh"
#include "ce_host.h"

namespace ce {
namespace sel {

constexpr int T = 512;
constexpr int NW = T / 32;

struct Sh {
  int hist[256];
  int red[NW];
  int bc[8];
};

__device__ __forceinline__ int warp_sum(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ int block_sum(int v, Sh& sh) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) sh.red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    int x = (threadIdx.x < NW) ? sh.red[threadIdx.x] : 0;
    x = warp_sum(x);
    if (threadIdx.x == 0) sh.bc[7] = x;
  }
  __syncthreads();
  const int r = sh.bc[7];
  __syncthreads();
  return r;
}

// Exclusive block scan; `total` receives the block sum.
__device__ int block_excl(int v, Sh& sh, int& total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) sh.red[w] = x;
  __syncthreads();
  if (threadIdx.x < 32) {
    const int a = (threadIdx.x < NW) ? sh.red[threadIdx.x] : 0;
    int s = a;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, s, o);
      if (threadIdx.x >= o) s += y;
    }
    if (threadIdx.x < NW) sh.red[threadIdx.x] = s - a;
    if (threadIdx.x == 31) sh.bc[6] = s;
  }
  __syncthreads();
  const int r = sh.red[w] + x - v;
  total = sh.bc[6];
  __syncthreads();
  return r;
}

// hist[256] holds digit counts.  Find d with sum(hist[>d]) < krem <= sum(hist[>=d]);
// sh.bc[0] = d, bc[1] = sum(hist[>d]), bc[2] = hist[d].
__device__ void find_digit(Sh& sh, int krem) {
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    int c[8];
    int s = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      c[q] = sh.hist[255 - 8 * lane - q];
      s += c[q];
    }
    int incl = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const int excl = incl - s;
    if (excl < krem && krem <= incl) {
      int run = excl;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        if (run + c[q] >= krem) {
          sh.bc[0] = 255 - 8 * lane - q;
          sh.bc[1] = run;
          sh.bc[2] = c[q];
          break;
        }
        run += c[q];
      }
    }
  }
  __syncthreads();
}

struct Thresh {
  uint64_t key;
  int pos;
  bool none;  // k == 0: nothing selected
};

// Column sets a CTA selects over.  pv < 0 marks a protected column (position
// in the low 31 bits); pv == -1 marks a slot past the end (no column).
//
// RegCols: up to ITEMS columns per thread held in registers (column
// c = threadIdx.x + i*T) -- every pass of the select is then register work.
// MemCols: any number of columns in a global workspace (L2-resident).
constexpr int32_t kAbsent = -1;

template <int ITEMS>
struct RegCols {
  uint64_t key[ITEMS];
  int32_t pv[ITEMS];
  template <class F>
  __device__ __forceinline__ void each(F f) const {
#pragma unroll
    for (int i = 0; i < ITEMS; ++i)
      if (pv[i] != kAbsent) f(static_cast<int>(threadIdx.x) + i * T, key[i], pv[i]);
  }
};

struct MemCols {
  const uint64_t* kv;
  const int32_t* pv;
  int N;
  template <class F>
  __device__ __forceinline__ void each(F f) const {
    for (int c = threadIdx.x; c < N; c += T) f(c, kv[c], pv[c]);
  }
};

// Plain column range [0, N) for ranks that do not need keys.
struct RangeCols {
  int N;
  template <class F>
  __device__ __forceinline__ void each(F f) const {
    for (int c = threadIdx.x; c < N; c += T) f(c, 0ull, 0);
  }
};

// Column range [0, N) whose per-column loads (load(c, key, pv): loads only)
// are issued for B columns of a thread before any of them is used, so a pass
// over a long range costs one load latency per B columns of a thread.
template <class LoadF>
struct LoadedRange {
  int N;
  LoadF load;
  static constexpr int B = 8;
  template <class F>
  __device__ __forceinline__ void each(F f) const {
    for (int c0 = threadIdx.x; c0 < N; c0 += B * T) {
      uint64_t k[B];
      int32_t v[B];
#pragma unroll
      for (int b = 0; b < B; ++b) {
        k[b] = 0ull;
        v[b] = 0;
        if (c0 + b * T < N) load(c0 + b * T, k[b], v[b]);
      }
#pragma unroll
      for (int b = 0; b < B; ++b)
        if (c0 + b * T < N) f(c0 + b * T, k[b], v[b]);
    }
  }
};
template <class LoadF>
__device__ __forceinline__ LoadedRange<LoadF> loaded_range(int N, LoadF load) {
  return LoadedRange<LoadF>{N, load};
}

// for (k = threadIdx.x; k < n; k += T) with the loads of B iterations in
// flight together: a = l1(k), then b = l2(k, a) (a load that needs a), then
// use(k, a, b), each stage for all B iterations before the next.
template <int B, class L1, class L2, class U>
__device__ __forceinline__ void batched(int n, L1 l1, L2 l2, U use) {
  using A = decltype(l1(0));
  using V = decltype(l2(0, A{}));
  for (int k0 = threadIdx.x; k0 < n; k0 += B * T) {
    A a[B];
    V v[B];
#pragma unroll
    for (int b = 0; b < B; ++b) a[b] = (k0 + b * T < n) ? l1(k0 + b * T) : A{};
#pragma unroll
    for (int b = 0; b < B; ++b) v[b] = (k0 + b * T < n) ? l2(k0 + b * T, a[b]) : V{};
#pragma unroll
    for (int b = 0; b < B; ++b)
      if (k0 + b * T < n) use(k0 + b * T, a[b], v[b]);
  }
}

// Threshold of the k largest (key, pos) pairs among unprotected columns:
// MSB-first 8-bit radix select on the key, then on the position among the
// columns equal to the threshold key (newer wins).
template <class Cols>
__device__ Thresh radix_threshold(const Cols& cols, int k, int nonprot, int key_bits, Sh& sh) {
  Thresh th{0ull, 0, false};
  if (k <= 0) {
    th.none = true;
    return th;
  }
  if (k >= nonprot) return th;  // everything unprotected is kept
  uint64_t prefix = 0, mask = 0;
  int krem = k, eq = 0;
  for (int shift = key_bits - 8; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += T) sh.hist[i] = 0;
    __syncthreads();
    cols.each([&](int, uint64_t key, int32_t pc) {
      if (pc >= 0 && (key & mask) == prefix) atomicAdd(&sh.hist[(key >> shift) & 255], 1);
    });
    __syncthreads();
    find_digit(sh, krem);
    const int d = sh.bc[0];
    krem -= sh.bc[1];
    eq = sh.bc[2];
    prefix |= static_cast<uint64_t>(d) << shift;
    mask |= static_cast<uint64_t>(255) << shift;
  }
  th.key = prefix;
  if (krem < eq) {
    // Among equal keys keep the krem newest positions.
    int pp = 0, pm = 0, kr = krem;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int i = threadIdx.x; i < 256; i += T) sh.hist[i] = 0;
      __syncthreads();
      cols.each([&](int, uint64_t key, int32_t pc) {
        if (pc >= 0 && key == prefix && (pc & pm) == pp) atomicAdd(&sh.hist[(pc >> shift) & 255], 1);
      });
      __syncthreads();
      find_digit(sh, kr);
      kr -= sh.bc[1];
      pp |= sh.bc[0] << shift;
      pm |= 255 << shift;
    }
    th.pos = pp;
  }
  __syncthreads();
  return th;
}

__device__ __forceinline__ bool selected(const Thresh& th, uint64_t key, int pc) {
  if (th.none || pc < 0) return false;
  return key > th.key || (key == th.key && pc >= th.pos);
}

// Rank every column whose posf(c, key, pv) >= 0 by ascending position using a
// bitmap of nw words, then call emit(rank, c, pos, key).  Positions must be
// < 32*nw.  Returns the number of ranked columns.
template <class Cols, class PosF, class EmitF>
__device__ int emit_sorted(const Cols& cols, int nw, uint32_t* bits, int* pre, PosF posf, EmitF emit,
                           Sh& sh, int32_t* err) {
  for (int w = threadIdx.x; w < nw; w += T) bits[w] = 0u;
  __syncthreads();
  cols.each([&](int c, uint64_t key, int32_t pc) {
    const int p = posf(c, key, pc);
    if (p < 0) return;
    if (p >= 32 * nw) {
      flag_error(err, CE_EW_SHAPE);
      return;
    }
    atomicOr(&bits[p >> 5], 1u << (p & 31));
  });
  __syncthreads();
  int carry = 0;
  for (int base = 0; base < nw; base += T) {
    const int w = base + threadIdx.x;
    const int v = (w < nw) ? __popc(bits[w]) : 0;
    int tot;
    const int ex = block_excl(v, sh, tot);
    if (w < nw) pre[w] = carry + ex;
    carry += tot;
  }
  __syncthreads();
  cols.each([&](int c, uint64_t key, int32_t pc) {
    const int p = posf(c, key, pc);
    if (p < 0 || p >= 32 * nw) return;
    const int rank = pre[p >> 5] + __popc(bits[p >> 5] & ((1u << (p & 31)) - 1u));
    emit(rank, c, p, key);
  });
  __syncthreads();
  return carry;
}

// Ranks by ascending position of the items a thread holds in a register
// layout (item it = column threadIdx.x + it * T): posv[it] is the position to
// rank, or -1 for an item that is not in the set; rank[it] receives its rank
// (-1 when not in the set).  Same bitmap method as emit_sorted, without
// calling back per column, so the caller can batch its loads afterwards.
template <int ITEMS>
__device__ void rank_sorted(const int32_t (&posv)[ITEMS], int nw, uint32_t* bits, int* pre, int (&rank)[ITEMS],
                            Sh& sh, int32_t* err) {
  for (int w = threadIdx.x; w < nw; w += T) bits[w] = 0u;
  __syncthreads();
#pragma unroll
  for (int it = 0; it < ITEMS; ++it) {
    const int q = posv[it];
    if (q < 0) continue;
    if (q >= 32 * nw) {
      flag_error(err, CE_EW_SHAPE);
      continue;
    }
    atomicOr(&bits[q >> 5], 1u << (q & 31));
  }
  __syncthreads();
  int carry = 0;
  for (int base = 0; base < nw; base += T) {
    const int w = base + threadIdx.x;
    const int v = (w < nw) ? __popc(bits[w]) : 0;
    int tot;
    const int ex = block_excl(v, sh, tot);
    if (w < nw) pre[w] = carry + ex;
    carry += tot;
  }
  __syncthreads();
#pragma unroll
  for (int it = 0; it < ITEMS; ++it) {
    const int q = posv[it];
    rank[it] = (q < 0 || q >= 32 * nw) ? -1 : pre[q >> 5] + __popc(bits[q >> 5] & ((1u << (q & 31)) - 1u));
  }
  __syncthreads();
}

// Register path for segments of up to REG_ITEMS * T columns.
// Eight columns per thread keep the register path at <= 64 registers, so two
// 512-thread blocks fit on an SM and a 256-segment select runs in one wave.
constexpr int REG_ITEMS = 8;

__device__ __forceinline__ bool is_prot(int pos, const ce_row_params& q) {
  return pos < q.prefix || pos >= q.n - q.recent || (q.cursor >= 0 && pos >= q.cursor);
}

__device__ __forceinline__ int key_bits_of(int policy, int score_dtype) {
  if (policy == CE_POLICY_RESERVOIR) return 64;
  if (policy == CE_POLICY_RANDOM) return score_dtype == CE_DTYPE_F64 ? 64 : 32;
  return 32;
}

// ---- large segments: REG_ITEMS*T+1 .. LARGE_MAX columns ------------------------
// One pass over the inputs keeps a 16-bit monotone prefix of every unprotected
// key in shared memory and a 4,096-bin histogram of its top 12 bits.  The
// k-th largest key's prefix is then found in shared memory (the 12-bit bin,
// then its 16 sub-bins), and only the columns sharing that prefix -- the
// candidates, typically tens -- have their full keys computed again to settle
// the exact threshold (key, then newer position) with the radix select above.
// Positions are read once more, for kept columns only, when the kept set is
// ranked.  So the inputs cross HBM about once, instead of once per radix pass.
// A segment whose candidates overflow the buffer (e.g. thousands of equal
// scores) returns false and takes the general path.
constexpr int LARGE_MAX = 65536;
constexpr int LHIST = 4096;
constexpr int LCAND = 2048;
constexpr int LARGE_BYTES = LARGE_MAX * 2 + 2 * (LARGE_MAX / 8) + LCAND * 16;  // 176 KB
// Columns per thread whose loads are in flight together.  Large segments run
// one CTA per SM (shared memory), so their kernel instance may use 128
// registers and deep batches.
constexpr int LARGE_LB = 16;
static_assert(LHIST == 8 * T, "one thread scans 8 bins");
enum BinKind { BIN_K32 = 0, BIN_K64 = 1, BIN_R53 = 2, BIN_U64 = 3 };

__device__ __forceinline__ double f64_from_key(uint64_t k) {
  const uint64_t u = (k & 0x8000000000000000ull) ? (k & 0x7fffffffffffffffull) : ~k;
  return __longlong_as_double(static_cast<long long>(u));
}

// 16-bit prefix, non-decreasing in the key: the top 16 bits of 32-bit, 64-bit
// and 53-bit keys; f64 uniforms map linearly from [0, 1) (their top bits are
// nearly all exponent).
__device__ __forceinline__ uint32_t bin16_of(uint64_t key, int kind) {
  switch (kind) {
    case BIN_K32:
      return static_cast<uint32_t>(key >> 16) & 0xFFFFu;
    case BIN_K64:
      return static_cast<uint32_t>(key >> 48);
    case BIN_R53:
      return static_cast<uint32_t>(key >> 37) & 0xFFFFu;
    default: {
      const double d = f64_from_key(key);
      if (!(d == d) || d >= 1.0) return 0xFFFFu;
      if (d <= 0.0) return 0u;
      return min(0xFFFFu, static_cast<uint32_t>(d * 65536.0));
    }
  }
}

// bin16_of with the key kind fixed at compile time, for the scan loops (a
// runtime switch there repeats every kind's code once per unrolled column).
template <int KIND>
__device__ __forceinline__ uint32_t bin16_k(uint64_t key) {
  if constexpr (KIND == BIN_K32) return static_cast<uint32_t>(key >> 16) & 0xFFFFu;
  else if constexpr (KIND == BIN_K64) return static_cast<uint32_t>(key >> 48);
  else if constexpr (KIND == BIN_R53) return static_cast<uint32_t>(key >> 37) & 0xFFFFu;
  else return bin16_of(key, BIN_U64);
}

struct LargeBuf {
  uint16_t* bin;   // [LARGE_MAX] key prefix of unprotected columns
  uint32_t* prot;  // [LARGE_MAX / 32] protected columns
  uint32_t* pick;  // [LARGE_MAX / 32] candidates that made the cut
  int* hist;       // [LHIST], shares storage with the candidate arrays
  uint64_t* ckey;  // [LCAND]
  int* ccol;       // [LCAND]
  int32_t* cpv;    // [LCAND]
};

__device__ __forceinline__ LargeBuf large_buf(uint32_t* base) {
  LargeBuf b;
  uint8_t* q = reinterpret_cast<uint8_t*>(base);
  b.bin = reinterpret_cast<uint16_t*>(q);
  q += LARGE_MAX * 2;
  b.prot = reinterpret_cast<uint32_t*>(q);
  q += LARGE_MAX / 8;
  b.pick = reinterpret_cast<uint32_t*>(q);
  q += LARGE_MAX / 8;
  b.hist = reinterpret_cast<int*>(q);
  b.ckey = reinterpret_cast<uint64_t*>(q);
  q += LCAND * 8;
  b.ccol = reinterpret_cast<int*>(q);
  q += LCAND * 4;
  b.cpv = reinterpret_cast<int32_t*>(q);
  return b;
}

struct LargeSel {
  int t16;      // unprotected columns with a larger prefix are kept
  bool all_eq;  // every column with prefix t16 is kept (no candidate round)
  bool none;    // no unprotected column is kept
  bool all;     // every unprotected column is kept
};

__device__ __forceinline__ bool is_bit(const uint32_t* m, int c) { return (m[c >> 5] >> (c & 31)) & 1u; }

// Pass over the inputs: prefixes, protected bits, histogram.  large_init
// clears the buffers; scan_quads takes four consecutive columns per 16-byte
// load (a quarter of the memory requests of per-column loads, which is what
// bounds this pass), issuing a whole batch of loads before it computes any
// key so that many loads are in flight per thread; large_tail takes single
// columns (the tail of a quad scan, or every column) through colfn.  Both
// return this thread's protected count (the caller reduces it).
__device__ __forceinline__ void large_init(int N, const LargeBuf& lb) {
  for (int i = threadIdx.x; i < LHIST; i += T) lb.hist[i] = 0;
  for (int i = threadIdx.x; i < (N + 31) / 32; i += T) {
    lb.prot[i] = 0u;
    lb.pick[i] = 0u;
  }
  __syncthreads();
}

// Bins, histogram and protected bits of one quad (columns 4q .. 4q + 3).
template <int KIND>
__device__ __forceinline__ int large_quad(int q, const uint64_t (&key)[4], const bool (&pr)[4],
                                          const LargeBuf& lb) {
  int np = 0;
  uint32_t pm = 0u;
  uint64_t packed = 0ull;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    if (pr[e]) {
      ++np;
      pm |= 1u << e;
    } else {
      const uint32_t b = bin16_k<KIND>(key[e]);
      packed |= static_cast<uint64_t>(b) << (16 * e);
      atomicAdd(&lb.hist[b >> 4], 1);
    }
  }
  *reinterpret_cast<uint64_t*>(lb.bin + 4 * q) = packed;
  if (pm) atomicOr(&lb.prot[q >> 3], pm << (4 * (q & 7)));
  return np;
}

// Qd supplies Raw (the loaded words of a quad, raw.pos its four positions),
// load(c, raw) (loads only), make(raw, key, pr) (keys and protection from the
// loaded words) and pos_at(c).  On the way, the scan checks whether the
// positions ascend strictly with the column index (each quad in itself, and
// against the previous quad's last position: lane - 1's quad, or one load for
// a warp's first lane); `ascending` is the block's verdict.
template <int LQN, int KIND, class Qd>
__device__ int scan_quads(const Qd& qd, int nq, const LargeBuf& lb, bool& ascending) {
  int np = 0;
  bool ok = true;
  const int lane = threadIdx.x & 31;
  // the loop bound is the warp's first quad, so every lane takes every
  // iteration and each shuffle below has the whole warp
  for (int qw = threadIdx.x - lane; qw < nq; qw += LQN * T) {
    const int q0 = qw + lane;
    typename Qd::Raw raw[LQN];
#pragma unroll
    for (int u = 0; u < LQN; ++u)
      if (q0 + u * T < nq) qd.load(4 * (q0 + u * T), raw[u]);
#pragma unroll
    for (int u = 0; u < LQN; ++u) {
      const int q = q0 + u * T;
      const bool live = q < nq;
      // lanes of a warp hold consecutive quads, and a live lane's lower
      // neighbours are live: the previous quad's last position comes from
      // lane - 1, or from memory for lane 0 (whose previous quad is the last
      // one of the warp below)
      const int last = live ? raw[u].pos.w : 0;
      int prev = __shfl_up_sync(0xffffffffu, last, 1);
      if (!live) continue;
      if (lane == 0) prev = q > 0 ? qd.pos_at(4 * q - 1) : -1;
      ok = ok && prev < raw[u].pos.x && raw[u].pos.x < raw[u].pos.y && raw[u].pos.y < raw[u].pos.z &&
           raw[u].pos.z < raw[u].pos.w;
      uint64_t key[4];
      bool pr[4];
      qd.make(raw[u], key, pr);
      np += large_quad<KIND>(q, key, pr, lb);
    }
  }
  ascending = __syncthreads_and(ok) != 0;
  return np;
}

template <int KIND, class ColFn>
__device__ int large_tail(ColFn colfn, int cstart, int N, const LargeBuf& lb) {
  int np = 0;
  constexpr int LB = LARGE_LB;
  for (int c0 = cstart + threadIdx.x; c0 < N; c0 += LB * T) {
    uint64_t key[LB];
    int32_t pv[LB];
    bool pr[LB];
#pragma unroll
    for (int u = 0; u < LB; ++u) {
      const int c = c0 + u * T;
      pr[u] = c < N ? colfn(c, key[u], pv[u]) : false;
    }
#pragma unroll
    for (int u = 0; u < LB; ++u) {
      const int c = c0 + u * T;
      if (c >= N) continue;
      if (pr[u]) {
        ++np;
        atomicOr(&lb.prot[c >> 5], 1u << (c & 31));
        lb.bin[c] = 0;
      } else {
        const uint32_t b = bin16_k<KIND>(key[u]);
        lb.bin[c] = static_cast<uint16_t>(b);
        atomicAdd(&lb.hist[b >> 4], 1);
      }
    }
  }
  return np;
}

// Columns 32 w .. 32 w + 31 that exist (w < (N + 31) / 32).
__device__ __forceinline__ uint32_t valid_bits(int w, int N) {
  const int n = N - 32 * w;
  return n >= 32 ? ~0u : ((1u << n) - 1u);
}

// The 16-bit prefixes of columns 32 w .. 32 w + 31 as eight 8-byte shared
// loads: element 4 j + e of the word is bits 16 (e & 1) of bb[j][e >> 1].
__device__ __forceinline__ void bins32(const LargeBuf& lb, int w, uint2 (&bb)[8]) {
  const uint2* b2 = reinterpret_cast<const uint2*>(lb.bin + 32 * w);   // 8-byte aligned
#pragma unroll
  for (int j = 0; j < 8; ++j) bb[j] = b2[j];
}
__device__ __forceinline__ uint32_t bin_at(const uint2 (&bb)[8], int i) {
  const uint32_t v = (i & 2) ? bb[i >> 2].y : bb[i >> 2].x;
  return (i & 1) ? (v >> 16) : (v & 0xFFFFu);
}

// The k largest of the nonprot unprotected columns (0 < k < nonprot handled
// here; the caller covers k <= 0 and k >= nonprot).  Returns false on
// candidate overflow.
template <class ColFn>
__device__ bool large_select(ColFn colfn, int N, int k, int nonprot, int kind, const LargeBuf& lb,
                             Sh& sh, LargeSel& r) {
  r = LargeSel{0, false, false, false};
  if (k <= 0) {
    r.none = true;
    return true;
  }
  if (k >= nonprot) {
    r.all = true;
    return true;
  }
  // 12-bit bin from the top: thread t owns bins 4095-8t .. 4088-8t.
  int c8[8];
  int s8 = 0;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    c8[q] = lb.hist[LHIST - 1 - 8 * threadIdx.x - q];
    s8 += c8[q];
  }
  int total;
  const int ex = block_excl(s8, sh, total);
  if (ex < k && k <= ex + s8) {
    int run = ex;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      if (run + c8[q] >= k) {
        sh.bc[0] = LHIST - 1 - 8 * threadIdx.x - q;
        sh.bc[1] = run;
        break;
      }
      run += c8[q];
    }
  }
  __syncthreads();
  const int t12 = sh.bc[0], above12 = sh.bc[1];
  __syncthreads();
  // Its 16 sub-bins.
  if (threadIdx.x < 16) lb.hist[threadIdx.x] = 0;
  __syncthreads();
  const int nw = (N + 31) / 32;
  for (int w = threadIdx.x; w < nw; w += T) {
    const uint32_t unprot = ~lb.prot[w] & valid_bits(w, N);
    uint2 bb[8];
    bins32(lb, w, bb);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const uint32_t b = bin_at(bb, i);
      if (((unprot >> i) & 1u) && (b >> 4) == static_cast<uint32_t>(t12)) atomicAdd(&lb.hist[b & 15], 1);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = above12;
    for (int d = 15; d >= 0; --d) {
      if (run + lb.hist[d] >= k) {
        sh.bc[0] = (t12 << 4) | d;
        sh.bc[1] = run;
        sh.bc[2] = lb.hist[d];
        break;
      }
      run += lb.hist[d];
    }
    sh.bc[5] = 0;
  }
  __syncthreads();
  const int t16 = sh.bc[0], above16 = sh.bc[1], eq16 = sh.bc[2];
  r.t16 = t16;
  const int krem = k - above16;
  if (krem >= eq16) {
    r.all_eq = true;
    return true;
  }
  if (eq16 > LCAND) return false;
  // Candidates: full keys of the columns with prefix t16 (hist is dead now).
  for (int w = threadIdx.x; w < nw; w += T) {
    const uint32_t unprot = ~lb.prot[w] & valid_bits(w, N);
    uint2 bb[8];
    bins32(lb, w, bb);
    uint32_t hit = 0u;
#pragma unroll
    for (int i = 0; i < 32; ++i) hit |= (bin_at(bb, i) == static_cast<uint32_t>(t16)) ? (1u << i) : 0u;
    hit &= unprot;
    while (hit) {
      const int c = 32 * w + __ffs(hit) - 1;
      hit &= hit - 1;
      uint64_t key;
      int32_t pv;
      colfn(c, key, pv);
      const int idx = atomicAdd(&sh.bc[5], 1);
      if (idx < LCAND) {
        lb.ckey[idx] = key;
        lb.cpv[idx] = pv;
        lb.ccol[idx] = c;
      }
    }
  }
  __syncthreads();
  if (eq16 <= T) {
    // One candidate per thread: its rank is the number of candidates before it
    // in the selection order (larger key first, then the newer position --
    // positions are distinct), and the krem first are kept.  One pass instead
    // of a radix select's 4-12 (each with three block barriers).
    if (threadIdx.x < eq16) {
      const uint64_t kj = lb.ckey[threadIdx.x];
      const int32_t pj = lb.cpv[threadIdx.x];
      int rank = 0;
      for (int m = 0; m < eq16; ++m) {
        const uint64_t km = lb.ckey[m];
        rank += (km > kj || (km == kj && lb.cpv[m] > pj)) ? 1 : 0;
      }
      const int c = lb.ccol[threadIdx.x];
      if (rank < krem) atomicOr(&lb.pick[c >> 5], 1u << (c & 31));
    }
    __syncthreads();
    return true;
  }
  const int bits = (kind == BIN_K32) ? 32 : 64;
  const Thresh th = radix_threshold(MemCols{lb.ckey, lb.cpv, eq16}, krem, eq16, bits, sh);
  for (int i = threadIdx.x; i < eq16; i += T)
    if (selected(th, lb.ckey[i], lb.cpv[i])) atomicOr(&lb.pick[lb.ccol[i] >> 5], 1u << (lb.ccol[i] & 31));
  __syncthreads();
  return true;
}

// Kept columns of a large segment as a bitmap kb[(N + 31) / 32] (shared
// memory), one pass of 8-byte prefix loads: the chosen unprotected columns
// (prefix above the threshold's, or equal to it and picked), plus the
// protected ones when WITH_PROT.
template <bool WITH_PROT>
__device__ void large_kept_bits(const LargeBuf& lb, const LargeSel& r, int N, uint32_t* kb) {
  const int nw = (N + 31) / 32;
  for (int w = threadIdx.x; w < nw; w += T) {
    const uint32_t prot = lb.prot[w];
    uint32_t sel = 0u;
    if (r.all) {
      sel = ~0u;
    } else if (!r.none) {
      const uint32_t pick = r.all_eq ? ~0u : lb.pick[w];
      uint2 bb[8];
      bins32(lb, w, bb);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const uint32_t b = bin_at(bb, i);
        const bool k = b > static_cast<uint32_t>(r.t16) || (b == static_cast<uint32_t>(r.t16) && ((pick >> i) & 1u));
        sel |= k ? (1u << i) : 0u;
      }
    }
    sel &= ~prot & valid_bits(w, N);
    kb[w] = WITH_PROT ? (sel | prot) : sel;
  }
  __syncthreads();
}

// The columns set in kb, each with its position pos(c) (read only for kept
// columns), as emit_sorted's column set.  With pos4 (vec), positions of four
// consecutive columns come from one 16-byte load.  Each thread marks which of
// its next 32 quads (columns) hold a kept column, then loads the positions of
// the marked ones eight at a time, so a pass costs one load latency per eight
// kept quads of a thread.
template <class PosF, class Pos4F>
struct KeptBits {
  int N;
  const uint32_t* kb;
  PosF pos;
  Pos4F pos4;
  bool vec;
  static constexpr int B = 8;
  template <class F>
  __device__ __forceinline__ void each(F f) const {
    int cstart = 0;
    if (vec) {
      const int nq = N / 4;
      for (int j0 = 0; j0 * T < nq; j0 += 32) {
        uint32_t m = 0u;   // bit jj: quad threadIdx.x + (j0 + jj) T holds a kept column
#pragma unroll 4
        for (int jj = 0; jj < 32; ++jj) {
          const int q = threadIdx.x + (j0 + jj) * T;
          if (q < nq && ((kb[q >> 3] >> (4 * (q & 7))) & 15u)) m |= 1u << jj;
        }
        while (m) {
          int qs[B];
          int4 ps[B];
#pragma unroll
          for (int b = 0; b < B; ++b) {
            qs[b] = -1;
            ps[b] = make_int4(0, 0, 0, 0);
            if (m) {
              qs[b] = threadIdx.x + (j0 + __ffs(m) - 1) * T;
              m &= m - 1;
              ps[b] = pos4(4 * qs[b]);
            }
          }
#pragma unroll
          for (int b = 0; b < B; ++b) {
            if (qs[b] < 0) continue;
            const int c = 4 * qs[b];
            const uint32_t km = (kb[qs[b] >> 3] >> (4 * (qs[b] & 7))) & 15u;
            if (km & 1u) f(c, 0ull, ps[b].x);
            if (km & 2u) f(c + 1, 0ull, ps[b].y);
            if (km & 4u) f(c + 2, 0ull, ps[b].z);
            if (km & 8u) f(c + 3, 0ull, ps[b].w);
          }
        }
      }
      cstart = 4 * nq;
    }
    for (int j0 = 0; cstart + j0 * T < N; j0 += 32) {
      uint32_t m = 0u;     // bit jj: column cstart + threadIdx.x + (j0 + jj) T is kept
#pragma unroll 4
      for (int jj = 0; jj < 32; ++jj) {
        const int c = cstart + threadIdx.x + (j0 + jj) * T;
        if (c < N && ((kb[c >> 5] >> (c & 31)) & 1u)) m |= 1u << jj;
      }
      while (m) {
        int cs[B];
        int32_t ps[B];
#pragma unroll
        for (int b = 0; b < B; ++b) {
          cs[b] = -1;
          ps[b] = 0;
          if (m) {
            cs[b] = cstart + threadIdx.x + (j0 + __ffs(m) - 1) * T;
            m &= m - 1;
            ps[b] = pos(cs[b]);
          }
        }
#pragma unroll
        for (int b = 0; b < B; ++b)
          if (cs[b] >= 0) f(cs[b], 0ull, ps[b]);
      }
    }
  }
};
template <class PosF, class Pos4F>
__device__ __forceinline__ KeptBits<PosF, Pos4F> kept_bits(int N, const uint32_t* kb, PosF pos, Pos4F pos4,
                                                           bool vec) {
  return KeptBits<PosF, Pos4F>{N, kb, pos, pos4, vec};
}

// ============================== ce_choose ========================================
struct ChooseParams {
  const int32_t* pos;
  const int32_t* ncols;
  int n_cols;
  const void* score;
  int sdt;
  const ce_row_params* params;
  int problems, layers, heads, head_offset, nw;
  int vec4;   // pos and score rows allow 16-byte loads of 4 columns
  int32_t* kept;
  int kept_stride;
  int32_t* status;
  int32_t* pcount;
  uint64_t* kv;
  int32_t* pv;
  int32_t* seg_info;
  int32_t* err;
};

__device__ __forceinline__ float score_f(const void* s, int dt, int64_t idx) {
  return dt == CE_DTYPE_F64 ? static_cast<float>(static_cast<const double*>(s)[idx])
                            : static_cast<const float*>(s)[idx];
}

// Key of column c for ce_choose; returns whether the column is protected.
__device__ __forceinline__ bool choose_column(const ChooseParams& p, int i, int l, int g, int64_t base,
                                              const ce_row_params& q, int c, uint64_t& key,
                                              int32_t& pv) {
  const int segs = p.layers * p.heads;
  const int pos = p.pos[base + c];
  // The score loads do not wait for the protection test, so a batch of
  // columns has all its loads in flight at once.
  uint64_t k = 0;
  switch (q.policy) {
    case CE_POLICY_RESERVOIR:
      k = reservoir53(q.seed, l, p.head_offset + g, static_cast<uint64_t>(pos));
      break;
    case CE_POLICY_H2O_GLOBAL:
      if (p.sdt == CE_DTYPE_F64) {
        double acc = 0.0;
        for (int gg = 0; gg < p.heads; ++gg)
          acc += static_cast<const double*>(p.score)[(static_cast<int64_t>(i) * segs + l * p.heads + gg) * p.n_cols + c];
        k = key_from_f64(acc);
      } else {
        float acc = 0.f;
        for (int gg = 0; gg < p.heads; ++gg)
          acc += static_cast<const float*>(p.score)[(static_cast<int64_t>(i) * segs + l * p.heads + gg) * p.n_cols + c];
        k = key_from_f32(acc);
      }
      break;
    case CE_POLICY_PREFIX_SLIDING:
      break;
    default:
      k = (p.sdt == CE_DTYPE_F64) ? key_from_f64(static_cast<const double*>(p.score)[base + c])
                                  : key_from_f32(static_cast<const float*>(p.score)[base + c]);
  }
  const bool pr = is_prot(pos, q);
  pv = pos | (pr ? static_cast<int>(0x80000000u) : 0);
  key = pr ? 0 : k;
  return pr;
}

// Columns c..c+3 of a ce_choose segment from 16-byte loads (c % 4 == 0; the
// host checked alignment), for scan_quads: the same keys as choose_column.
// SRC fixes where the key comes from, so load() is straight-line loads.
enum QuadSrc { QS_POS = 0, QS_F32 = 1, QS_F64 = 2, QS_H2O_F32 = 3, QS_H2O_F64 = 4 };
template <int SRC>
struct ChooseQuads {
  const ChooseParams* p;
  int64_t base, hbase;   // this segment's columns; head 0 of its layer (H2O global)
  ce_row_params q;
  uint64_t head;          // global KV head index (reservoir draws)
  int l;
  struct Raw {
    int4 pos;
    float4 f;
    double2 d0, d1;
  };
  __device__ __forceinline__ void load(int c, Raw& r) const {
    r.pos = *reinterpret_cast<const int4*>(p->pos + base + c);
    if constexpr (SRC == QS_F32) {
      r.f = *reinterpret_cast<const float4*>(static_cast<const float*>(p->score) + base + c);
    } else if constexpr (SRC == QS_F64) {
      const double2* s2 = reinterpret_cast<const double2*>(static_cast<const double*>(p->score) + base + c);
      r.d0 = s2[0];
      r.d1 = s2[1];
    } else if constexpr (SRC == QS_H2O_F32) {
      // fp32 sum over the layer's heads in ascending head order
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int gg = 0; gg < p->heads; ++gg) {
        const float4 x = *reinterpret_cast<const float4*>(static_cast<const float*>(p->score) + hbase +
                                                           static_cast<int64_t>(gg) * p->n_cols + c);
        a.x += x.x; a.y += x.y; a.z += x.z; a.w += x.w;
      }
      r.f = a;
    } else if constexpr (SRC == QS_H2O_F64) {
      double2 a0 = make_double2(0.0, 0.0), a1 = make_double2(0.0, 0.0);
      for (int gg = 0; gg < p->heads; ++gg) {
        const double2* s2 = reinterpret_cast<const double2*>(static_cast<const double*>(p->score) + hbase +
                                                             static_cast<int64_t>(gg) * p->n_cols + c);
        const double2 x = s2[0], y = s2[1];
        a0.x += x.x; a0.y += x.y; a1.x += y.x; a1.y += y.y;
      }
      r.d0 = a0;
      r.d1 = a1;
    }
  }
  __device__ __forceinline__ int pos_at(int c) const { return p->pos[base + c]; }
  __device__ __forceinline__ void make(const Raw& r, uint64_t (&key)[4], bool (&pr)[4]) const {
    const int pos[4] = {r.pos.x, r.pos.y, r.pos.z, r.pos.w};
    uint64_t k[4] = {0ull, 0ull, 0ull, 0ull};
    if constexpr (SRC == QS_POS) {
      if (q.policy == CE_POLICY_RESERVOIR)
#pragma unroll
        for (int e = 0; e < 4; ++e) k[e] = reservoir53(q.seed, l, head, static_cast<uint64_t>(pos[e]));
    } else if constexpr (SRC == QS_F32 || SRC == QS_H2O_F32) {
      k[0] = key_from_f32(r.f.x); k[1] = key_from_f32(r.f.y); k[2] = key_from_f32(r.f.z); k[3] = key_from_f32(r.f.w);
    } else {
      k[0] = key_from_f64(r.d0.x); k[1] = key_from_f64(r.d0.y); k[2] = key_from_f64(r.d1.x); k[3] = key_from_f64(r.d1.y);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      pr[e] = is_prot(pos[e], q);
      key[e] = pr[e] ? 0 : k[e];
    }
  }
};

template <class Cols>
__device__ void choose_body(const ChooseParams& p, const Cols& cols, int np, int i, int s, int N,
                            const ce_row_params& q, Sh& sh, uint32_t* dyn) {
  const int segs = p.layers * p.heads;
  const int nprot = block_sum(np, sh);
  if (threadIdx.x == 0) p.seg_info[static_cast<int64_t>(i) * segs + s] = nprot;
  if (nprot > q.budget) return;
  const int k = (q.policy == CE_POLICY_PREFIX_SLIDING) ? 0 : q.budget - nprot;
  const int bits = (q.policy == CE_POLICY_RESERVOIR) ? 64 : (p.sdt == CE_DTYPE_F64 ? 64 : 32);
  const Thresh th = radix_threshold(cols, k, N - nprot, bits, sh);
  int32_t* out = p.kept + (static_cast<int64_t>(i) * segs + s) * p.kept_stride;
  const int stride = p.kept_stride;
  int32_t* err = p.err;
  emit_sorted(
      cols, p.nw, dyn, reinterpret_cast<int*>(dyn + p.nw),
      [&](int, uint64_t key, int32_t pc) -> int {
        if (pc < 0) return pc & 0x7fffffff;
        return selected(th, key, pc) ? pc : -1;
      },
      [&](int rank, int c, int, uint64_t) {
        if (rank < stride) out[rank] = c;
        else flag_error(err, CE_EW_CAPACITY);
      },
      sh, p.err);
}

// The kept columns of a large segment (bitmap kb over its N columns) into
// out[0 .. stride), ranked by position.  When the positions ascend with the
// column (`ascending`, verified by the scan), a kept column's rank is the
// number of kept columns before it, a prefix popcount over kb, and no
// position is read; otherwise emit_sorted ranks by a position bitmap.
__device__ void choose_emit(const ChooseParams& p, int32_t* out, int stride, const int32_t* pos, int N,
                            const uint32_t* kb, bool ascending, Sh& sh, uint32_t* dyn) {
  int32_t* err = p.err;
  if (ascending) {
    const int nwc = (N + 31) / 32;
    int carry = 0;
    for (int b0 = 0; b0 < nwc; b0 += T) {
      const int w = b0 + threadIdx.x;
      const uint32_t m0 = w < nwc ? kb[w] : 0u;
      int tot;
      const int ex = block_excl(__popc(m0), sh, tot);
      int rank = carry + ex;
      for (uint32_t m = m0; m; m &= m - 1, ++rank) {
        if (rank < stride) out[rank] = 32 * w + __ffs(m) - 1;
        else flag_error(err, CE_EW_CAPACITY);
      }
      carry += tot;
    }
    __syncthreads();
    return;
  }
  emit_sorted(
      kept_bits(N, kb, [&](int c) { return pos[c]; },
                [&](int c) { return *reinterpret_cast<const int4*>(pos + c); }, p.vec4 != 0),
      p.nw, dyn, reinterpret_cast<int*>(dyn + p.nw), [](int, uint64_t, int32_t pc) -> int { return pc; },
      [&](int rank, int c, int, uint64_t) {
        if (rank < stride) out[rank] = c;
        else flag_error(err, CE_EW_CAPACITY);
      },
      sh, p.err);
}

// Large segments (see large_select); false = candidate overflow, nothing emitted.
__device__ bool choose_large(const ChooseParams& p, int i, int l, int g, int s, int64_t base,
                             const ce_row_params& q, int N, Sh& sh, uint32_t* dyn) {
  const int segs = p.layers * p.heads;
  const LargeBuf lb = large_buf(dyn + 2 * p.nw);
  const int kind = q.policy == CE_POLICY_RESERVOIR ? BIN_R53
                   : p.sdt == CE_DTYPE_F64 ? (q.policy == CE_POLICY_RANDOM ? BIN_U64 : BIN_K64)
                                           : BIN_K32;
  auto colfn = [&](int c, uint64_t& key, int32_t& pv) -> bool {
    return choose_column(p, i, l, g, base, q, c, key, pv);
  };
  large_init(N, lb);
  int np = 0, cstart = 0;
  bool ascending = false;
  if (p.vec4) {
    // Quads per thread per batch, by the registers a quad's loaded words take.
    const int nq = N / 4;
    const int64_t hbase = (static_cast<int64_t>(i) * segs + l * p.heads) * p.n_cols;
    const uint64_t head = static_cast<uint64_t>(p.head_offset + g);
    // (loader, key kind) pairs; prefix_sliding keys are all 0, whose bin is 0 in every kind
    if (q.policy == CE_POLICY_RESERVOIR)
      np = scan_quads<16, BIN_R53>(ChooseQuads<QS_POS>{&p, base, hbase, q, head, l}, nq, lb, ascending);
    else if (q.policy == CE_POLICY_PREFIX_SLIDING)
      np = scan_quads<16, BIN_K32>(ChooseQuads<QS_POS>{&p, base, hbase, q, head, l}, nq, lb, ascending);
    else if (q.policy == CE_POLICY_H2O_GLOBAL)
      np = p.sdt == CE_DTYPE_F64
               ? scan_quads<2, BIN_K64>(ChooseQuads<QS_H2O_F64>{&p, base, hbase, q, head, l}, nq, lb, ascending)
               : scan_quads<4, BIN_K32>(ChooseQuads<QS_H2O_F32>{&p, base, hbase, q, head, l}, nq, lb, ascending);
    else if (p.sdt == CE_DTYPE_F64)
      np = kind == BIN_U64 ? scan_quads<6, BIN_U64>(ChooseQuads<QS_F64>{&p, base, hbase, q, head, l}, nq, lb, ascending)
                           : scan_quads<6, BIN_K64>(ChooseQuads<QS_F64>{&p, base, hbase, q, head, l}, nq, lb, ascending);
    else
      np = scan_quads<8, BIN_K32>(ChooseQuads<QS_F32>{&p, base, hbase, q, head, l}, nq, lb, ascending);
    cstart = 4 * nq;
  }
  if (cstart < N) ascending = false;   // tail columns are not checked
  np += kind == BIN_K32   ? large_tail<BIN_K32>(colfn, cstart, N, lb)
        : kind == BIN_K64 ? large_tail<BIN_K64>(colfn, cstart, N, lb)
        : kind == BIN_R53 ? large_tail<BIN_R53>(colfn, cstart, N, lb)
                          : large_tail<BIN_U64>(colfn, cstart, N, lb);
  const int nprot = block_sum(np, sh);
  if (threadIdx.x == 0) p.seg_info[static_cast<int64_t>(i) * segs + s] = nprot;
  if (nprot > q.budget) return true;
  const int k = (q.policy == CE_POLICY_PREFIX_SLIDING) ? 0 : q.budget - nprot;
  LargeSel sel;
  if (!large_select(colfn, N, k, N - nprot, kind, lb, sh, sel)) return false;
  int32_t* out = p.kept + (static_cast<int64_t>(i) * segs + s) * p.kept_stride;
  const int stride = p.kept_stride;
  const int32_t* pos = p.pos + base;
  // kept bitmap in the histogram's storage (dead once the threshold is known)
  uint32_t* kb = reinterpret_cast<uint32_t*>(lb.hist);
  large_kept_bits<true>(lb, sel, N, kb);
  choose_emit(p, out, stride, pos, N, kb, ascending, sh, dyn);
  return true;
}


// LARGE: the launch carries the large-segment shared-memory buffer (one CTA
// per SM); otherwise two CTAs share an SM and large segments take the
// general path.
template <bool LARGE>
__global__ void __launch_bounds__(T, LARGE ? 1 : 2) choose_seg_kernel(const ChooseParams p) {
  extern __shared__ uint32_t dyn[];
  __shared__ Sh sh;
  const int segs = p.layers * p.heads;
  const int i = blockIdx.x / segs, s = blockIdx.x % segs;
  const int l = s / p.heads, g = s % p.heads;
  const ce_row_params q = p.params[i];
  const int N = p.ncols ? min(p.ncols[i], p.n_cols) : p.n_cols;
  const int64_t base = (static_cast<int64_t>(i) * segs + s) * p.n_cols;
  int np = 0;
  if (N <= REG_ITEMS * T) {
    RegCols<REG_ITEMS> cols;
#pragma unroll
    for (int it = 0; it < REG_ITEMS; ++it) {
      const int c = threadIdx.x + it * T;
      cols.pv[it] = kAbsent;
      cols.key[it] = 0;
      if (c < N) np += choose_column(p, i, l, g, base, q, c, cols.key[it], cols.pv[it]);
    }
    choose_body(p, cols, np, i, s, N, q, sh, dyn);
    return;
  }
  if constexpr (LARGE) {
    if (N <= LARGE_MAX && choose_large(p, i, l, g, s, base, q, N, sh, dyn)) return;
  }
  {
    uint64_t* kv = p.kv + base;
    int32_t* pv = p.pv + base;
    for (int c = threadIdx.x; c < N; c += T) np += choose_column(p, i, l, g, base, q, c, kv[c], pv[c]);
    __syncthreads();
    choose_body(p, MemCols{kv, pv, N}, np, i, s, N, q, sh, dyn);
  }
}

__global__ void choose_status_kernel(const ChooseParams p) {
  const int i = blockIdx.x;
  const int segs = p.layers * p.heads;
  if (threadIdx.x != 0) return;
  const ce_row_params q = p.params[i];
  const int n0 = p.seg_info[static_cast<int64_t>(i) * segs];
  int st = 0;
  for (int s = 1; s < segs; ++s)
    if (p.seg_info[static_cast<int64_t>(i) * segs + s] != n0) st = 3;
  if (st == 0 && n0 > q.budget) st = 2;
  if (st == 3) flag_error(p.err, CE_EW_PROTECTED);
  p.status[i] = st;
  if (p.pcount) p.pcount[i] = n0;
}

// ============================== ce_boundary ======================================
// Per-row record the selection leaves for the later kernels (row_info).
constexpr int RI = 16;

struct BParams {
  int32_t* table;
  int64_t ts;
  int table_width;
  int32_t* r2u;
  int64_t rs;
  int r2u_width;
  int32_t* frontier;
  int32_t* count;
  int32_t* pos;
  int64_t prs;
  int pos_cap;
  float* scores;
  int64_t sls, shs, pool_units;
  const uint64_t* k_layers;
  const uint64_t* v_layers;
  int L, G, P, head_offset;
  int32_t* marks;
  int epoch;
  const int64_t* swa;
  const int32_t* rows;
  const ce_row_params* params;
  int R;
  const void* uniforms;
  int udt;
  const float* gscores;
  int GH;
  int live, max_cols, max_width, nw;
  int ch;   // middle survivors per compaction chunk (chunk_items)
  // workspace
  uint64_t* kv;
  int32_t* pv;
  int32_t* seg_info;   // [R*L*G]
  int32_t* mid_col;    // [R*L*G*max_cols]
  int32_t* src_unit;
  int32_t* new_pos;
  float* score_scr;
  uint8_t* hflag;      // [R*L*G*max_cols] middle survivor whose source is staged (bgather)
  int32_t* row_info;   // [R*RI]: N, nprot, W, after, true_u, nleft, count, status, swa_bad, npacked
  int32_t* cand_rank;  // [R*max_cols]
  int32_t* new_table;  // [R*max_cols]
  int32_t* prot_col;   // [R*max_cols] the (0,0) head's protected columns in its position order
  int32_t* pack;       // [R*max_cols] the row's packed req_to_unit prefix (live)
  uint8_t* hazard;
  int32_t* freed;
  int64_t freed_stride;
  int32_t* result;
  uint32_t* rec_delta;   // retention record or NULL
  int64_t rec_stride;
  int32_t* rec_counts;
  int32_t* err;
};

struct RowCtx {
  int row, cnt, fr, N;
  ce_row_params q;
};

__device__ __forceinline__ RowCtx row_ctx(const BParams& p, int i) {
  RowCtx r;
  r.row = p.rows[i];
  r.q = p.params[i];
  r.cnt = p.count[r.row];
  r.fr = p.frontier[r.row];
  r.N = r.cnt + (r.q.n - r.fr);
  return r;
}

// Row sizes within the arguments, and the uniforms a random row draws from present.
__device__ __forceinline__ bool row_shape_ok(const BParams& p, const RowCtx& r) {
  return r.cnt >= 0 && r.fr >= 0 && r.fr <= r.q.n && r.N >= 0 && r.N <= p.max_cols &&
         r.q.n <= 32 * p.nw && r.q.n <= p.r2u_width && r.cnt <= p.pos_cap &&
         (r.q.policy != CE_POLICY_RANDOM || p.uniforms != nullptr);
}

__device__ __forceinline__ int col_unit(const BParams& p, const RowCtx& r, int c) {
  return c < r.cnt ? p.table[r.row * p.ts + c] : p.r2u[r.row * p.rs + r.fr + (c - r.cnt)];
}

__device__ __forceinline__ int col_pos(const BParams& p, const RowCtx& r, int lg, int c) {
  return c < r.cnt ? p.pos[r.row * p.prs + static_cast<int64_t>(lg) * p.pos_cap + c]
                   : r.fr + (c - r.cnt);
}

__device__ __forceinline__ float unit_score(const BParams& p, int l, int g, int unit) {
  if (unit < 0 || unit >= p.pool_units) return 0.f;
  return p.scores[l * p.sls + g * p.shs + unit];
}

// Key of boundary column c for segment (i, lg); returns whether the column is
// protected.  Keys follow _scores (runtime:400-412).
__device__ __forceinline__ bool bsel_column(const BParams& p, const RowCtx& r, int i, int lg, int c,
                                            uint64_t& key, int32_t& pv) {
  const int LG = p.L * p.G;
  const int l = lg / p.G, g = lg % p.G;
  const int pos = col_pos(p, r, lg, c);
  // Score loads are issued before the protection test (see choose_column).
  uint64_t k = 0;
  switch (r.q.policy) {
    case CE_POLICY_RANDOM: {
      const int64_t ui = (static_cast<int64_t>(i) * LG + lg) * p.max_cols + c;
      k = (p.udt == CE_DTYPE_F64) ? key_from_f64(static_cast<const double*>(p.uniforms)[ui])
                                  : key_from_f32(static_cast<const float*>(p.uniforms)[ui]);
      break;
    }
    case CE_POLICY_RESERVOIR:
      k = reservoir53(r.q.seed, l, p.head_offset + g, static_cast<uint64_t>(pos));
      break;
    case CE_POLICY_HEAD_SUM:
    case CE_POLICY_HEAD_MAX:
      k = key_from_f32(unit_score(p, l, g, col_unit(p, r, c)));
      break;
    case CE_POLICY_H2O_GLOBAL: {
      float acc = 0.f;
      if (p.gscores) {
        for (int gg = 0; gg < p.GH; ++gg)
          acc += p.gscores[((static_cast<int64_t>(i) * p.L + l) * p.GH + gg) * p.max_cols + c];
      } else {
        const int u = col_unit(p, r, c);
        for (int gg = 0; gg < p.G; ++gg) acc += unit_score(p, l, gg, u);
      }
      k = key_from_f32(acc);
      break;
    }
    default:
      break;
  }
  const bool pr = is_prot(pos, r.q);
  pv = pos | (pr ? static_cast<int>(0x80000000u) : 0);
  key = pr ? 0 : k;
  return pr;
}

// The register path's columns (item it = column threadIdx.x + it * T) with
// the keys of bsel_column, loaded in phases so that each phase's loads for
// all of a thread's columns are in flight together: positions and units,
// then the scores the policy needs, then keys and protection.  Returns this
// thread's protected count.
__device__ int bsel_reg_columns(const BParams& p, const RowCtx& r, int i, int lg, RegCols<REG_ITEMS>& cols) {
  const int LG = p.L * p.G;
  const int l = lg / p.G, g = lg % p.G;
  int pos[REG_ITEMS], unit[REG_ITEMS];
  bool in[REG_ITEMS];
#pragma unroll
  for (int it = 0; it < REG_ITEMS; ++it) {
    const int c = static_cast<int>(threadIdx.x) + it * T;
    in[it] = c < r.N;
    pos[it] = in[it] ? col_pos(p, r, lg, c) : 0;
    unit[it] = in[it] ? col_unit(p, r, c) : -1;
  }
  float f[REG_ITEMS];
  uint64_t k[REG_ITEMS];
  const int policy = r.q.policy;
  if (policy == CE_POLICY_HEAD_SUM || policy == CE_POLICY_HEAD_MAX) {
#pragma unroll
    for (int it = 0; it < REG_ITEMS; ++it) f[it] = in[it] ? unit_score(p, l, g, unit[it]) : 0.f;
#pragma unroll
    for (int it = 0; it < REG_ITEMS; ++it) k[it] = key_from_f32(f[it]);
  } else if (policy == CE_POLICY_H2O_GLOBAL) {
    // fp32 sum over the layer's heads in ascending head order
#pragma unroll
    for (int it = 0; it < REG_ITEMS; ++it) f[it] = 0.f;
    if (p.gscores) {
      const float* gs = p.gscores + (static_cast<int64_t>(i) * p.L + l) * p.GH * p.max_cols;
      for (int gg = 0; gg < p.GH; ++gg)
#pragma unroll
        for (int it = 0; it < REG_ITEMS; ++it)
          if (in[it]) f[it] += gs[static_cast<int64_t>(gg) * p.max_cols + threadIdx.x + it * T];
    } else {
      for (int gg = 0; gg < p.G; ++gg)
#pragma unroll
        for (int it = 0; it < REG_ITEMS; ++it)
          if (in[it]) f[it] += unit_score(p, l, gg, unit[it]);
    }
#pragma unroll
    for (int it = 0; it < REG_ITEMS; ++it) k[it] = key_from_f32(f[it]);
  } else if (policy == CE_POLICY_RANDOM) {
    const int64_t ub = (static_cast<int64_t>(i) * LG + lg) * p.max_cols + threadIdx.x;
#pragma unroll
    for (int it = 0; it < REG_ITEMS; ++it) {
      const int64_t ui = ub + it * T;
      k[it] = !in[it] ? 0ull
              : (p.udt == CE_DTYPE_F64) ? key_from_f64(static_cast<const double*>(p.uniforms)[ui])
                                        : key_from_f32(static_cast<const float*>(p.uniforms)[ui]);
    }
  } else if (policy == CE_POLICY_RESERVOIR) {
#pragma unroll
    for (int it = 0; it < REG_ITEMS; ++it)
      k[it] = reservoir53(r.q.seed, l, p.head_offset + g, static_cast<uint64_t>(pos[it]));
  } else {
#pragma unroll
    for (int it = 0; it < REG_ITEMS; ++it) k[it] = 0ull;
  }
  int np = 0;
#pragma unroll
  for (int it = 0; it < REG_ITEMS; ++it) {
    cols.pv[it] = kAbsent;
    cols.key[it] = 0;
    if (!in[it]) continue;
    const bool pr = is_prot(pos[it], r.q);
    cols.pv[it] = pos[it] | (pr ? static_cast<int>(0x80000000u) : 0);
    cols.key[it] = pr ? 0 : k[it];
    np += pr;
  }
  return np;
}

// Middle survivors (cols with posf(c, key, pv) >= 0) in ascending position
// after the nprot protected slots (runtime:444-446); their units and scores
// are loaded after the ranking, eight survivors of a thread at a time.  The
// protected slots are filled by bfinish_kernel.
template <class Cols, class PosF>
__device__ void bsel_emit(const BParams& p, const RowCtx& r, const Cols& cols, PosF posf, int nprot,
                          int i, int lg, int64_t base, Sh& sh, uint32_t* bitsm, int* pre) {
  const int l = lg / p.G, g = lg % p.G;
  int32_t* mid = p.mid_col + base;
  int32_t* npos = p.new_pos + base;
  int32_t* srcu = p.src_unit + base;
  float* ssc = p.score_scr + base;
  const int max_cols = p.max_cols;
  const int nmid = emit_sorted(
      cols, p.nw, bitsm, pre, posf,
      [&](int rank, int c, int pos, uint64_t) {
        if (nprot + rank >= max_cols) return;
        mid[rank] = c;
        npos[nprot + rank] = pos;
      },
      sh, p.err);
  batched<8>(
      min(nmid, max_cols - nprot), [&](int j) { return col_unit(p, r, mid[j]); },
      [&](int, int u) { return unit_score(p, l, g, u); },
      [&](int j, int u, float sc) {
        srcu[j] = u;
        ssc[j] = sc;
      });
}

template <class Cols>
__device__ void bsel_body(const BParams& p, const RowCtx& r, const Cols& cols, int np, int i, int lg,
                          int64_t base, Sh& sh, uint32_t* bitsm, int* pre) {
  const int LG = p.L * p.G;
  const int nprot = block_sum(np, sh);
  if (threadIdx.x == 0) p.seg_info[static_cast<int64_t>(i) * LG + lg] = nprot;
  if (nprot > r.q.budget) return;
  const int k = (r.q.policy == CE_POLICY_PREFIX_SLIDING) ? 0 : r.q.budget - nprot;
  const int bits = key_bits_of(r.q.policy, p.udt);
  const Thresh th = radix_threshold(cols, k, r.N - nprot, bits, sh);
  bsel_emit(p, r, cols, [&](int, uint64_t key, int32_t pc) -> int { return selected(th, key, pc) ? pc : -1; },
            nprot, i, lg, base, sh, bitsm, pre);
}

// Register path of the boundary selection: the same outputs as bsel_emit,
// with ranks computed first and every global load (units, scores) issued for
// all of a thread's columns at once.
__device__ void bsel_body(const BParams& p, const RowCtx& r, const RegCols<REG_ITEMS>& cols, int np, int i,
                          int lg, int64_t base, Sh& sh, uint32_t* bitsm, int* pre) {
  const int LG = p.L * p.G;
  const int nprot = block_sum(np, sh);
  if (threadIdx.x == 0) p.seg_info[static_cast<int64_t>(i) * LG + lg] = nprot;
  if (nprot > r.q.budget) return;
  const int k = (r.q.policy == CE_POLICY_PREFIX_SLIDING) ? 0 : r.q.budget - nprot;
  const int bits = key_bits_of(r.q.policy, p.udt);
  const Thresh th = radix_threshold(cols, k, r.N - nprot, bits, sh);
  const int l = lg / p.G, g = lg % p.G;
  const int max_cols = p.max_cols;
  // middle survivors, ranked by position (runtime:444-446)
  int32_t posv[REG_ITEMS];
  int rank[REG_ITEMS];
#pragma unroll
  for (int it = 0; it < REG_ITEMS; ++it)
    posv[it] = (cols.pv[it] != kAbsent && selected(th, cols.key[it], cols.pv[it])) ? cols.pv[it] : -1;
  rank_sorted(posv, p.nw, bitsm, pre, rank, sh, p.err);
  int unit[REG_ITEMS];
#pragma unroll
  for (int it = 0; it < REG_ITEMS; ++it)
    unit[it] = rank[it] >= 0 ? col_unit(p, r, static_cast<int>(threadIdx.x) + it * T) : -1;
  float sc[REG_ITEMS];
#pragma unroll
  for (int it = 0; it < REG_ITEMS; ++it) sc[it] = rank[it] >= 0 ? unit_score(p, l, g, unit[it]) : 0.f;
#pragma unroll
  for (int it = 0; it < REG_ITEMS; ++it) {
    const int rk = rank[it];
    if (rk < 0 || nprot + rk >= max_cols) continue;
    p.mid_col[base + rk] = static_cast<int>(threadIdx.x) + it * T;
    p.new_pos[base + nprot + rk] = posv[it];
    p.src_unit[base + rk] = unit[it];
    p.score_scr[base + rk] = sc[it];
  }
}

// Pass over a large boundary segment (large_tail's outputs) with the key
// source fixed at compile time, so that each batch of LARGE_LB columns of a
// thread is straight-line code: positions and units of the batch, then the
// scores or uniforms they select, then keys, bins and protection.  Keys are
// those of bsel_column.  The kept columns [0, count) and the new ones
// [count, N) run as two ranges (KEPT), so neither tests which one a column
// is in, and a new column's position is arithmetic.
enum BselSrc { BS_NONE = 0, BS_SCORE = 1, BS_H2O = 2, BS_U32 = 3, BS_U64 = 4, BS_RES = 5 };
template <int SRC, int KIND, bool KEPT>
__device__ int bsel_scan_range(const BParams& p, const RowCtx& r, int i, int lg, int cb, int ce,
                               const LargeBuf& lb) {
  constexpr int B = LARGE_LB;
  const int LG = p.L * p.G;
  const int l = lg / p.G, g = lg % p.G;
  // row-relative bases: column c's position, unit, uniform and H2O sum
  const int32_t* posr = p.pos + r.row * p.prs + static_cast<int64_t>(lg) * p.pos_cap;
  const int32_t* unitr = KEPT ? p.table + r.row * p.ts : p.r2u + r.row * p.rs + (r.fr - r.cnt);
  const float* sc = p.scores + l * p.sls + g * p.shs;
  const int64_t ub = (static_cast<int64_t>(i) * LG + lg) * p.max_cols;
  const float* gs = p.gscores + (static_cast<int64_t>(i) * p.L + l) * p.GH * p.max_cols;
  const int pos0 = r.fr - r.cnt;   // position of new column c: pos0 + c
  const int64_t pool = p.pool_units;
  int np = 0;
  for (int c0 = cb + static_cast<int>(threadIdx.x); c0 < ce; c0 += B * T) {
    int pos[B];
    uint64_t key[B];
#pragma unroll
    for (int b = 0; b < B; ++b) {
      const int c = c0 + b * T;
      pos[b] = KEPT ? (c < ce ? posr[c] : 0) : pos0 + c;
    }
    if constexpr (SRC == BS_SCORE) {
      int unit[B];
#pragma unroll
      for (int b = 0; b < B; ++b) unit[b] = c0 + b * T < ce ? unitr[c0 + b * T] : -1;
#pragma unroll
      for (int b = 0; b < B; ++b)
        key[b] = key_from_f32((unit[b] >= 0 && unit[b] < pool) ? sc[unit[b]] : 0.f);
    } else if constexpr (SRC == BS_H2O) {
      float f[B];
#pragma unroll
      for (int b = 0; b < B; ++b) f[b] = 0.f;
      for (int gg = 0; gg < p.GH; ++gg)
#pragma unroll
        for (int b = 0; b < B; ++b)
          if (c0 + b * T < ce) f[b] += gs[static_cast<int64_t>(gg) * p.max_cols + c0 + b * T];
#pragma unroll
      for (int b = 0; b < B; ++b) key[b] = key_from_f32(f[b]);
    } else if constexpr (SRC == BS_U32) {
      const float* u = static_cast<const float*>(p.uniforms) + ub;
#pragma unroll
      for (int b = 0; b < B; ++b) key[b] = c0 + b * T < ce ? key_from_f32(u[c0 + b * T]) : 0ull;
    } else if constexpr (SRC == BS_U64) {
      const double* u = static_cast<const double*>(p.uniforms) + ub;
#pragma unroll
      for (int b = 0; b < B; ++b) key[b] = c0 + b * T < ce ? key_from_f64(u[c0 + b * T]) : 0ull;
    } else if constexpr (SRC == BS_RES) {
#pragma unroll
      for (int b = 0; b < B; ++b)
        key[b] = reservoir53(r.q.seed, l, p.head_offset + g, static_cast<uint64_t>(pos[b]));
    } else {
#pragma unroll
      for (int b = 0; b < B; ++b) key[b] = 0ull;
    }
#pragma unroll
    for (int b = 0; b < B; ++b) {
      const int c = c0 + b * T;
      if (c >= ce) continue;
      if (is_prot(pos[b], r.q)) {
        ++np;
        atomicOr(&lb.prot[c >> 5], 1u << (c & 31));
        lb.bin[c] = 0;
      } else {
        const uint32_t bn = bin16_k<KIND>(key[b]);
        lb.bin[c] = static_cast<uint16_t>(bn);
        atomicAdd(&lb.hist[bn >> 4], 1);
      }
    }
  }
  return np;
}

template <int SRC, int KIND>
__device__ int bsel_scan(const BParams& p, const RowCtx& r, int i, int lg, const LargeBuf& lb) {
  return bsel_scan_range<SRC, KIND, true>(p, r, i, lg, 0, r.cnt, lb) +
         bsel_scan_range<SRC, KIND, false>(p, r, i, lg, r.cnt, r.N, lb);
}

// The columns set in kb[0 .. nwc) (shared memory) with their positions
// pos(c), as emit_sorted's column set: each thread takes whole words and
// loads the positions of their set bits eight at a time, so a pass costs a
// few shared loads per thread plus one load latency per eight kept columns.
template <class PosF>
struct KeptWords {
  int nwc;
  const uint32_t* kb;
  PosF pos;
  static constexpr int B = 8;
  template <class F>
  __device__ __forceinline__ void each(F f) const {
    for (int w = threadIdx.x; w < nwc; w += T) {
      uint32_t m = kb[w];
      while (m) {
        int cs[B];
        int32_t ps[B];
#pragma unroll
        for (int b = 0; b < B; ++b) {
          cs[b] = -1;
          ps[b] = 0;
          if (m) {
            cs[b] = 32 * w + __ffs(m) - 1;
            m &= m - 1;
            ps[b] = pos(cs[b]);
          }
        }
#pragma unroll
        for (int b = 0; b < B; ++b)
          if (cs[b] >= 0) f(cs[b], 0ull, ps[b]);
      }
    }
  }
};
template <class PosF>
__device__ __forceinline__ KeptWords<PosF> kept_words(int N, const uint32_t* kb, PosF pos) {
  return KeptWords<PosF>{(N + 31) / 32, kb, pos};
}

// Large segments (see large_select); false = candidate overflow, nothing emitted.
__device__ bool bsel_large(const BParams& p, const RowCtx& r, int i, int lg, int64_t base, Sh& sh,
                           uint32_t* bitsm, int* pre) {
  const int LG = p.L * p.G;
  const LargeBuf lb = large_buf(bitsm + 2 * p.nw);
  const int kind = r.q.policy == CE_POLICY_RESERVOIR ? BIN_R53
                   : (r.q.policy == CE_POLICY_RANDOM && p.udt == CE_DTYPE_F64) ? BIN_U64
                                                                              : BIN_K32;
  auto colfn = [&](int c, uint64_t& key, int32_t& pv) -> bool { return bsel_column(p, r, i, lg, c, key, pv); };
  large_init(r.N, lb);
  int np;
  switch (r.q.policy) {
    case CE_POLICY_HEAD_SUM:
    case CE_POLICY_HEAD_MAX:
      np = bsel_scan<BS_SCORE, BIN_K32>(p, r, i, lg, lb);
      break;
    case CE_POLICY_H2O_GLOBAL:
      np = p.gscores ? bsel_scan<BS_H2O, BIN_K32>(p, r, i, lg, lb) : large_tail<BIN_K32>(colfn, 0, r.N, lb);
      break;
    case CE_POLICY_RANDOM:
      np = p.udt == CE_DTYPE_F64 ? bsel_scan<BS_U64, BIN_U64>(p, r, i, lg, lb)
                                 : bsel_scan<BS_U32, BIN_K32>(p, r, i, lg, lb);
      break;
    case CE_POLICY_RESERVOIR:
      np = bsel_scan<BS_RES, BIN_R53>(p, r, i, lg, lb);
      break;
    default:
      np = bsel_scan<BS_NONE, BIN_K32>(p, r, i, lg, lb);
  }
  const int nprot = block_sum(np, sh);
  if (threadIdx.x == 0) p.seg_info[static_cast<int64_t>(i) * LG + lg] = nprot;
  if (nprot > r.q.budget) return true;
  const int k = (r.q.policy == CE_POLICY_PREFIX_SLIDING) ? 0 : r.q.budget - nprot;
  LargeSel sel;
  if (!large_select(colfn, r.N, k, r.N - nprot, kind, lb, sh, sel)) return false;
  uint32_t* kb = reinterpret_cast<uint32_t*>(lb.hist);
  large_kept_bits<false>(lb, sel, r.N, kb);
  bsel_emit(p, r, kept_words(r.N, kb, [&](int c) { return col_pos(p, r, lg, c); }),
            [](int, uint64_t, int32_t pc) -> int { return pc; }, nprot, i, lg, base, sh, bitsm, pre);
  return true;
}

// A row's new columns [cnt, N) hold the consecutive positions [fr, n)
// (column c: pos0 + c).  By is_prot, the protected ones are [fr, a1) (under
// the prefix) and [b0, n) (the recent window and the cursor guard), and the
// candidates are [a1, b0).
struct RowSplit {
  int pos0, a1, b0;
};
__device__ __forceinline__ RowSplit row_split(const RowCtx& r) {
  const int n = r.q.n;
  const int lo = r.q.cursor >= 0 ? min(n - r.q.recent, r.q.cursor) : n - r.q.recent;
  RowSplit s;
  s.pos0 = r.fr - r.cnt;
  s.a1 = min(max(r.q.prefix, r.fr), n);
  s.b0 = min(max(lo, s.a1), n);
  return s;
}

// The (0,0) head's protected columns of a row as emit_sorted's column set
// (key = unit, pv = position): the kept columns through their loaded
// positions, then the new columns at positions [fr, a1) and [b0, n).
struct RowProtCols {
  const BParams* p;
  RowCtx r;
  RowSplit sp;
  template <class F>
  __device__ __forceinline__ void each(F f) const {
    const BParams& pp = *p;
    const RowCtx& rr = r;
    loaded_range(rr.cnt, [&](int c, uint64_t& key, int32_t& pv) {
      pv = col_pos(pp, rr, 0, c);
      key = static_cast<uint32_t>(pp.table[rr.row * pp.ts + c]);
    }).each(f);
    const int32_t* r2u_row = pp.r2u + rr.row * pp.rs;
    const int pos0 = sp.pos0;
    auto fresh = [&](int x0, int x1) {
      batched<8>(
          x1 - x0, [&](int k) { return r2u_row[x0 + k]; }, [](int, int) { return 0; },
          [&](int k, int u, int) { f(x0 + k - pos0, static_cast<uint64_t>(static_cast<uint32_t>(u)), x0 + k); });
    };
    fresh(rr.fr, sp.a1);
    fresh(sp.b0, rr.q.n);
  }
};

// R row blocks, then R*L*G segment blocks.  Row blocks come first so that
// when the segments take more than one wave, the row blocks (a full pass
// over each row's columns) run beside the first wave instead of after it.
template <bool LARGE>
__global__ void __launch_bounds__(T, LARGE ? 1 : 2) bsel_kernel(const BParams p) {
  extern __shared__ uint32_t dyn[];
  __shared__ Sh sh;
  uint32_t* bitsm = dyn;
  int* pre = reinterpret_cast<int*>(dyn + p.nw);
  const int LG = p.L * p.G;
  if (static_cast<int>(blockIdx.x) >= p.R) {
    const int sb = static_cast<int>(blockIdx.x) - p.R;
    const int i = sb / LG, lg = sb % LG;
    const RowCtx r = row_ctx(p, i);
    if (!row_shape_ok(p, r) || r.N <= r.q.budget) return;
    const int64_t base = (static_cast<int64_t>(i) * LG + lg) * p.max_cols;
    int np = 0;
    if (r.N <= REG_ITEMS * T) {
      RegCols<REG_ITEMS> cols;
      np = bsel_reg_columns(p, r, i, lg, cols);
      bsel_body(p, r, cols, np, i, lg, base, sh, bitsm, pre);
      return;
    }
    if constexpr (LARGE) {
      if (r.N <= LARGE_MAX && bsel_large(p, r, i, lg, base, sh, bitsm, pre)) return;
    }
    {
      uint64_t* kv = p.kv + base;
      int32_t* pv = p.pv + base;
      for (int c = threadIdx.x; c < r.N; c += T) np += bsel_column(p, r, i, lg, c, kv[c], pv[c]);
      __syncthreads();
      bsel_body(p, r, MemCols{kv, pv, r.N}, np, i, lg, base, sh, bitsm, pre);
    }
  } else {
    // ---------------- row block: table, candidates, leftovers, marks -----------
    const int i = blockIdx.x;
    const RowCtx r = row_ctx(p, i);
    int32_t* info = p.row_info + i * RI;
    if (!row_shape_ok(p, r) || r.N <= r.q.budget) return;
    // Kept columns [0, cnt) are counted and ranked through the (0,0) head's
    // loaded positions; new columns hold consecutive positions, so theirs
    // follow from the split (row_split) without loads.
    const RowSplit sp = row_split(r);
    int np = 0;
    loaded_range(r.cnt, [&](int c, uint64_t&, int32_t& pos) { pos = col_pos(p, r, 0, c); })
        .each([&](int, uint64_t, int32_t pos) { np += is_prot(pos, r.q); });
    const int nprot = block_sum(np, sh) + (sp.a1 - r.fr) + (r.q.n - sp.b0);
    if (nprot > r.q.budget) {
      if (threadIdx.x == 0) info[1] = nprot;
      return;
    }
    const int W = (r.q.policy == CE_POLICY_PREFIX_SLIDING) ? 0 : r.q.budget - nprot;
    int32_t* ntab = p.new_table + static_cast<int64_t>(i) * p.max_cols;
    int32_t* crank = p.cand_rank + static_cast<int64_t>(i) * p.max_cols;
    int32_t* pcol = p.prot_col + static_cast<int64_t>(i) * p.max_cols;
    const int32_t* r2u_row = p.r2u + r.row * p.rs;
    // protected units first, in (0,0) position order (key = unit, pv = position),
    // and their columns for the protected slots of every head (bfinish_kernel)
    emit_sorted(
        RowProtCols{&p, r, sp}, p.nw, bitsm, pre,
        [&](int, uint64_t, int32_t p00) -> int { return is_prot(p00, r.q) ? p00 : -1; },
        [&](int rank, int c, int, uint64_t key) {
          ntab[rank] = static_cast<int32_t>(key);
          pcol[rank] = c;
        },
        sh, p.err);
    // Candidates (columns the (0,0) head does not protect) ranked in column
    // order.  Kept columns: tiles of 8 words of 32 columns per warp, each lane
    // loading its column of every word; the ballots give the candidate words
    // and one block scan per tile offsets the warps.
    int carry = 0;
    int swa_bad = 0;   // a freed unit still maps to a sliding-window slot (runtime:477-479)
    auto swa_of = [&](int u) -> int64_t { return (p.swa && u >= 0 && u < p.pool_units) ? p.swa[u] : 0; };
    {
      constexpr int WW = 8;
      const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
      const uint32_t below = (1u << lane) - 1u;
      for (int t0 = 0; t0 < r.cnt; t0 += NW * WW * 32) {
        const int cw = t0 + warp * WW * 32 + lane;
        int pos[WW], unit[WW];
#pragma unroll
        for (int j = 0; j < WW; ++j) {
          const int c = cw + 32 * j;
          pos[j] = c < r.cnt ? col_pos(p, r, 0, c) : 0;
          unit[j] = c < r.cnt ? col_unit(p, r, c) : 0;
        }
        uint32_t word[WW];
        int wtot = 0;
#pragma unroll
        for (int j = 0; j < WW; ++j) {
          word[j] = __ballot_sync(0xffffffffu, cw + 32 * j < r.cnt && !is_prot(pos[j], r.q));
          wtot += __popc(word[j]);
        }
        int tot;
        const int ex = block_excl(lane == 0 ? wtot : 0, sh, tot);
        int run = carry + __shfl_sync(0xffffffffu, ex, 0);
        int cr[WW];   // candidate rank, -1 for a protected column
#pragma unroll
        for (int j = 0; j < WW; ++j) {
          cr[j] = ((word[j] >> lane) & 1u) ? run + __popc(word[j] & below) : -1;
          run += __popc(word[j]);
        }
        if (p.live && p.swa) {
#pragma unroll
          for (int j = 0; j < WW; ++j) swa_bad |= cr[j] >= W && swa_of(unit[j]) != 0;
        }
#pragma unroll
        for (int j = 0; j < WW; ++j) {
          const int c = cw + 32 * j;
          if (c >= r.cnt) continue;
          crank[c] = cr[j];
          if (cr[j] < 0) continue;
          if (cr[j] < W)
            ntab[nprot + cr[j]] = unit[j];
          else if (p.live)
            p.freed[i * p.freed_stride + (cr[j] - W)] = unit[j];
        }
        carry += tot;
      }
    }
    // New columns: the candidates are the positions [a1, b0), after the kept ones.
    batched<8>(
        r.N - r.cnt,
        [&](int k) {
          const int x = r.fr + k;
          return (x >= sp.a1 && x < sp.b0) ? r2u_row[x] : 0;
        },
        [&](int k, int u) -> int64_t {
          const int x = r.fr + k;
          return (p.live && x >= sp.a1 && x < sp.b0 && carry + (x - sp.a1) >= W) ? swa_of(u) : 0;
        },
        [&](int k, int u, int64_t m) {
          const int x = r.fr + k, c = r.cnt + k;
          swa_bad |= m != 0;
          if (x >= sp.a1 && x < sp.b0) {
            const int cr = carry + (x - sp.a1);
            crank[c] = cr;
            if (cr < W)
              ntab[nprot + cr] = u;
            else if (p.live)
              p.freed[i * p.freed_stride + (cr - W)] = u;
          } else {
            crank[c] = -1;
          }
        });
    swa_bad = block_sum(swa_bad, sh);
    const int true_u = min(r.q.n - r.q.recent, r.q.cursor >= 0 ? r.q.cursor : r.q.n);
    if (p.live) {
      const int x0 = max(true_u, 0);
      batched<8>(
          r.q.n - x0, [&](int k) { return p.r2u[r.row * p.rs + x0 + k]; }, [](int, int) { return 0; },
          [&](int, int u, int) {
            if (u >= 0 && u < p.pool_units) p.marks[u] = p.epoch;
          });
    }
    // The packed req_to_unit prefix (runtime:484-491): every unit of the new
    // table that is not a real slot of [true_u, n), in table order.  The table
    // and the marks are this block's own writes; bfinish_kernel copies the
    // list into the row once the other blocks no longer read it.
    int npacked = 0;
    if (p.live) {
      __syncthreads();
      const int after = nprot + W;
      int32_t* plist = p.pack + static_cast<int64_t>(i) * p.max_cols;
      constexpr int WW = 8;
      const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
      const uint32_t below = (1u << lane) - 1u;
      for (int t0 = 0; t0 < after; t0 += NW * WW * 32) {
        const int kw = t0 + warp * WW * 32 + lane;
        int u[WW], m[WW];
#pragma unroll
        for (int j = 0; j < WW; ++j) u[j] = kw + 32 * j < after ? ntab[kw + 32 * j] : -1;
#pragma unroll
        for (int j = 0; j < WW; ++j) m[j] = (u[j] >= 0 && u[j] < p.pool_units) ? p.marks[u[j]] : 0;
        uint32_t word[WW];
        int wtot = 0;
#pragma unroll
        for (int j = 0; j < WW; ++j) {
          const bool real = u[j] >= 0 && u[j] < p.pool_units && m[j] == p.epoch;
          word[j] = __ballot_sync(0xffffffffu, kw + 32 * j < after && !real);
          wtot += __popc(word[j]);
        }
        int tot;
        const int ex = block_excl(lane == 0 ? wtot : 0, sh, tot);
        int run = npacked + __shfl_sync(0xffffffffu, ex, 0);
#pragma unroll
        for (int j = 0; j < WW; ++j) {
          if ((word[j] >> lane) & 1u) plist[run + __popc(word[j] & below)] = u[j];
          run += __popc(word[j]);
        }
        npacked += tot;
      }
    }
    if (threadIdx.x == 0) {
      info[9] = npacked;
      info[0] = r.N;
      info[1] = nprot;
      info[2] = W;
      info[3] = nprot + W;
      info[4] = true_u;
      info[5] = r.N - nprot - W;
      info[6] = r.cnt;
      info[8] = swa_bad > 0;
    }
  }
}

// H2O global keys of every boundary column, once per (row, layer) instead of
// once per KV-head segment: the fp32 sum of the layer's KV heads' unit
// scores in ascending head order (the same additions the selection would
// make).  Grid (column blocks, rows); rows of other policies are skipped.
// With usum (unit_sum_kernel's per-unit sums) a column reads its unit's sum
// instead of gathering the G head scores itself.
__global__ void hsum_kernel(const BParams p, float* gsum, const float* usum) {
  const int i = blockIdx.y;
  const RowCtx r = row_ctx(p, i);
  if (r.q.policy != CE_POLICY_H2O_GLOBAL || !row_shape_ok(p, r) || r.N <= r.q.budget) return;
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < r.N; c += gridDim.x * blockDim.x) {
    const int u = col_unit(p, r, c);
    const bool ok = u >= 0 && u < p.pool_units;
    for (int l = 0; l < p.L; ++l) {
      float acc = 0.f;
      if (usum) {
        acc = ok ? usum[static_cast<int64_t>(l) * p.pool_units + u] : 0.f;
      } else {
        for (int gg = 0; gg < p.G; ++gg) acc += unit_score(p, l, gg, u);
      }
      gsum[(static_cast<int64_t>(i) * p.L + l) * p.max_cols + c] = acc;
    }
  }
}

// Per-unit sums over the layer's KV heads (ascending head order, starting
// from 0 as hsum_kernel does) for every pool unit, in one coalesced pass over
// the score rows.  Used when the batch's rows own most of the pool, where it
// replaces G scattered loads per column by one; returns at once when no row
// of the batch is H2O global.
__global__ void unit_sum_kernel(const BParams p, float* usum) {
  __shared__ int any;
  if (threadIdx.x == 0) {
    any = 0;
    for (int i = 0; i < p.R; ++i) any |= p.params[i].policy == CE_POLICY_H2O_GLOBAL;
  }
  __syncthreads();
  if (!any) return;
  for (int64_t u = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; u < p.pool_units;
       u += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    for (int l = 0; l < p.L; ++l) {
      float acc = 0.f;
      for (int gg = 0; gg < p.G; ++gg) acc += p.scores[l * p.sls + gg * p.shs + u];
      usum[static_cast<int64_t>(l) * p.pool_units + u] = acc;
    }
  }
}

__global__ void bvalidate_kernel(const BParams p) {
  const int i = blockIdx.x;
  if (threadIdx.x != 0) return;
  const RowCtx r = row_ctx(p, i);
  const int LG = p.L * p.G;
  int32_t* info = p.row_info + i * RI;
  int st;
  int after = r.N;
  if (!row_shape_ok(p, r)) {
    st = 6;
    flag_error(p.err, CE_EW_SHAPE);
  } else if (r.N <= r.q.budget) {
    st = 1;
  } else {
    const int n0 = info[1];
    st = 0;
    for (int s = 0; s < LG; ++s)
      if (p.seg_info[static_cast<int64_t>(i) * LG + s] != n0) st = 3;
    if (st == 3) {
      flag_error(p.err, CE_EW_PROTECTED);
    } else if (n0 > r.q.budget) {
      st = 2;
    } else {
      after = info[3];
      if (after > p.table_width || after > p.pos_cap || info[2] > p.max_width) {
        st = 6;
        flag_error(p.err, CE_EW_CAPACITY);
      }
    }
  }
  info[7] = st;
  int32_t* res = p.result + i * 4;
  res[0] = st;
  res[1] = r.N;
  res[2] = (st == 0) ? after : (st == 2 ? info[1] : r.N);
  res[3] = 0;
}

// Retention record (runtime:465-467, 500-507): per (row, layer, KV head) the
// positions of the columns this boundary evicts -- neither protected for this
// head nor among its middle survivors -- in ascending order and delta-coded
// (the first value is the position itself).  Runs after selection and before
// bfinish rewrites the positions.  One block per segment.
__global__ void __launch_bounds__(T) brecord_kernel(const BParams p) {
  extern __shared__ uint32_t dyn[];
  __shared__ Sh sh;
  const int LG = p.L * p.G;
  const int i = blockIdx.x / LG, lg = blockIdx.x % LG;
  const int32_t* info = p.row_info + i * RI;
  int32_t* cnt_out = p.rec_counts + static_cast<int64_t>(i) * LG + lg;
  if (info[7] != 0) {
    if (threadIdx.x == 0) *cnt_out = 0;
    return;
  }
  const RowCtx r = row_ctx(p, i);
  const int nprot = info[1], W = info[2];
  const int64_t base = (static_cast<int64_t>(i) * LG + lg) * p.max_cols;
  uint32_t* bits = dyn;
  int* pre = reinterpret_cast<int*>(dyn + p.nw);
  uint32_t* kept = dyn + 2 * p.nw;
  for (int w = threadIdx.x; w < (r.N + 31) / 32; w += T) kept[w] = 0u;
  __syncthreads();
  for (int c = threadIdx.x; c < r.N; c += T)
    if (is_prot(col_pos(p, r, lg, c), r.q)) atomicOr(&kept[c >> 5], 1u << (c & 31));
  for (int j = threadIdx.x; j < W; j += T) {
    const int c = p.mid_col[base + j];
    if (c >= 0 && c < r.N) atomicOr(&kept[c >> 5], 1u << (c & 31));
  }
  __syncthreads();
  uint32_t* out = p.rec_delta + (static_cast<int64_t>(i) * LG + lg) * p.rec_stride;
  const int64_t stride = p.rec_stride;
  int32_t* err = p.err;
  emit_sorted(
      RangeCols{r.N}, p.nw, bits, pre,
      [&](int c, uint64_t, int32_t) -> int { return is_bit(kept, c) ? -1 : col_pos(p, r, lg, c); },
      [&](int rank, int, int pos, uint64_t) {
        if (rank < stride) out[rank] = static_cast<uint32_t>(pos);
        else flag_error(err, CE_EW_CAPACITY);
      },
      sh, p.err);
  const int64_t nv64 = static_cast<int64_t>(r.N - nprot - W);
  const int nv = static_cast<int>(nv64 < stride ? nv64 : stride);
  if (threadIdx.x == 0) *cnt_out = nv;
  // Delta-code in place, top chunk first, so every out[j - 1] is read before
  // its own chunk is rewritten.
  for (int top = nv; top > 0; top -= T) {
    const int j = top - T + static_cast<int>(threadIdx.x);
    uint32_t cur = 0u, prev = 0u;
    if (j >= 0) {
      cur = out[j];
      prev = j ? out[j - 1] : 0u;
    }
    __syncthreads();
    if (j >= 0) out[j] = cur - prev;
    __syncthreads();
  }
}

// One warp per chunk of p.ch consecutive middle survivors j of one (row,
// layer-in-group, head): lane k < p.ch holds item j0 + k.  The chunk index is
// decoded once with 32-bit arithmetic (the host checks that the count fits)
// and the lanes load their items' metadata in parallel.  Slices of 2 KB and
// more (page size >= 16) take chunks of 8 items copied one after another,
// each a 4 KB K + V pair in flight; smaller slices take chunks of 32 items
// copied together (copy_items).
constexpr int CH_PAGED = 8;
constexpr int CH_SMALL = 32;
__host__ __device__ __forceinline__ int chunk_items(int P) { return P * 128 >= 2048 ? CH_PAGED : CH_SMALL; }

struct Chunk {
  int i, l, g, j;         // this lane's item
  int W, nprot;
  int64_t base;           // segment base in the [R, L, G, max_cols] arrays
  int64_t item;           // flat item index within the launch (hazard scratch slot)
  bool valid;
};

__device__ __forceinline__ int chunks_per_seg(const BParams& p) { return (p.max_width + p.ch - 1) / p.ch; }

__device__ __forceinline__ Chunk decode_chunk(const BParams& p, uint32_t wi, int r0, int l0, int nl, int lane) {
  Chunk c;
  const uint32_t cps = static_cast<uint32_t>(chunks_per_seg(p));
  const uint32_t seg = wi / cps, jc = wi - seg * cps;
  const uint32_t lg = static_cast<uint32_t>(nl * p.G);
  const int ir = static_cast<int>(seg / lg);   // row within the launch
  c.i = r0 + ir;
  const uint32_t rem = seg - static_cast<uint32_t>(ir) * lg;
  const int ll = static_cast<int>(rem / static_cast<uint32_t>(p.G));
  c.g = static_cast<int>(rem) - ll * p.G;
  c.l = l0 + ll;
  c.j = static_cast<int>(jc) * p.ch + lane;
  const int32_t* info = p.row_info + c.i * RI;
  c.W = info[2];
  c.nprot = info[1];
  c.valid = lane < p.ch && info[7] == 0 && c.j < c.W;
  c.base = (static_cast<int64_t>(c.i) * p.L * p.G + static_cast<int64_t>(c.l) * p.G + c.g) * p.max_cols;
  c.item = ((static_cast<int64_t>(ir) * nl + ll) * p.G + c.g) * p.max_width + c.j;
  return c;
}

__device__ __forceinline__ bool chunk_hazard(const BParams& p, const Chunk& c) {
  const int col = p.mid_col[c.base + c.j];
  const int cr = p.cand_rank[static_cast<int64_t>(c.i) * p.max_cols + col];
  return cr >= 0 && cr < c.W && cr != c.j;
}

__device__ __forceinline__ uint8_t* unit_ptr(const uint64_t* layers, int l, int unit, int g, int G,
                                             int P) {
  return reinterpret_cast<uint8_t*>(layers[l]) +
         (static_cast<int64_t>(unit) * G + g) * static_cast<int64_t>(P) * 128;
}

// Copy one head slice of K and of V (bytes each) with the warp: every lane
// issues all of its loads (up to 4 x 16 B of K and of V) before its first
// store, so a warp keeps a whole 2 KB + 2 KB page pair in flight.  Sources are
// never written by the launch that reads them (hazard sources are staged by
// the previous launch), so the loads take the non-coherent path.
__device__ __forceinline__ void copy_pair(uint8_t* dk, uint8_t* dv, const uint8_t* sk, const uint8_t* sv,
                                          int bytes, int lane) {
  for (int o = lane * 16; o < bytes; o += 4 * 32 * 16) {
    uint4 a[4], b[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int x = o + u * 32 * 16;
      if (x < bytes) {
        a[u] = __ldg(reinterpret_cast<const uint4*>(sk + x));
        b[u] = __ldg(reinterpret_cast<const uint4*>(sv + x));
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int x = o + u * 32 * 16;
      if (x < bytes) {
        *reinterpret_cast<uint4*>(dk + x) = a[u];
        *reinterpret_cast<uint4*>(dv + x) = b[u];
      }
    }
  }
}

// Copy the K and V slices (bytes each, under 2 KB) of every item whose bit is
// set in todo (warp-uniform, from a ballot) with the whole warp at once: the
// (item, 16-byte vector) pairs are spread over the lanes, two per lane in
// flight (few registers, so that many warps fit an SM), so a chunk costs
// about one load latency instead of one per item.  addr(k, sk, sv, dk, dv)
// gives item k's addresses; it shuffles from lane k, so every lane calls it,
// for items that are skipped too.
template <class AddrF>
__device__ __forceinline__ void copy_items(unsigned todo, int bytes, int lane, AddrF addr) {
  if (!todo) return;
  constexpr int DEPTH = 2;
  const int vecs = bytes >> 4;
  const int total = (32 - __clz(static_cast<int>(todo))) * vecs;
  for (int f0 = 0; f0 < total; f0 += DEPTH * 32) {
    uint4 a[DEPTH], b[DEPTH];
    uint8_t* dk[DEPTH];
    uint8_t* dv[DEPTH];
    bool ok[DEPTH];
#pragma unroll
    for (int u = 0; u < DEPTH; ++u) {
      const int f = f0 + u * 32 + lane;
      const int k = min(f / vecs, 31);
      const uint8_t* sk;
      const uint8_t* sv;
      addr(k, sk, sv, dk[u], dv[u]);
      ok[u] = f < total && ((todo >> k) & 1u);
      if (ok[u]) {
        const int x = (f - k * vecs) * 16;
        a[u] = __ldg(reinterpret_cast<const uint4*>(sk + x));
        b[u] = __ldg(reinterpret_cast<const uint4*>(sv + x));
        dk[u] += x;
        dv[u] += x;
      }
    }
#pragma unroll
    for (int u = 0; u < DEPTH; ++u) {
      if (ok[u]) {
        *reinterpret_cast<uint4*>(dk[u]) = a[u];
        *reinterpret_cast<uint4*>(dv[u]) = b[u];
      }
    }
  }
}

__device__ __forceinline__ uint32_t launch_chunks(const BParams& p, int nr, int nl) {
  return static_cast<uint32_t>(nr) * static_cast<uint32_t>(nl * p.G) * static_cast<uint32_t>(chunks_per_seg(p));
}

// Stage every hazard source of the group's layers (a unit that some other
// item of its row overwrites) in the scratch buffer.
// SMALL: slices under 2 KB (copy_items); otherwise one page pair at a time.
template <bool SMALL>
__global__ void __launch_bounds__(256, SMALL ? 4 : 2) bgather_kernel(const BParams p, int r0, int nr, int l0,
                                                                     int nl) {
  const int lane = threadIdx.x & 31;
  const uint32_t nchunks = launch_chunks(p, nr, nl);
  const uint32_t nwarps = gridDim.x * (blockDim.x >> 5);
  const int bytes = p.P * 128;
  for (uint32_t wi = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); wi < nchunks; wi += nwarps) {
    const Chunk c = decode_chunk(p, wi, r0, l0, nl, lane);
    int src = -1;
    bool hz = false;
    if (c.valid) {
      hz = chunk_hazard(p, c);
      src = p.src_unit[c.base + c.j];
      if (hz && (src < 0 || src >= p.pool_units)) {
        flag_error(p.err, CE_EW_INDEX);
        hz = false;
      }
      p.hflag[c.base + c.j] = hz;
    }
    const unsigned hmask = __ballot_sync(0xffffffffu, hz);
    if constexpr (SMALL) {
      // c.l, c.g and c.item - lane are the same on every lane of the chunk
      const int64_t item0 = c.item - lane;
      copy_items(hmask, bytes, lane,
                 [&](int k, const uint8_t*& sk, const uint8_t*& sv, uint8_t*& dk, uint8_t*& dv) {
                   const int s = max(__shfl_sync(0xffffffffu, src, k), 0);
                   sk = unit_ptr(p.k_layers, c.l, s, c.g, p.G, p.P);
                   sv = unit_ptr(p.v_layers, c.l, s, c.g, p.G, p.P);
                   dk = p.hazard + (item0 + k) * 2 * bytes;
                   dv = dk + bytes;
                 });
      continue;
    }
    for (unsigned todo = hmask; todo; todo &= todo - 1) {
      const int k = __ffs(todo) - 1;
      const int s = __shfl_sync(0xffffffffu, src, k);
      const int64_t it = __shfl_sync(0xffffffffu, c.item, k);
      uint8_t* scr = p.hazard + it * 2 * bytes;
      copy_pair(scr, scr + bytes, unit_ptr(p.k_layers, c.l, s, c.g, p.G, p.P),
                unit_ptr(p.v_layers, c.l, s, c.g, p.G, p.P), bytes, lane);
    }
  }
}

// Write every middle survivor of the group's layers to its target unit (from
// the scratch copy when its source is a hazard) and move its score.
template <bool SMALL>
__global__ void __launch_bounds__(256, SMALL ? 4 : 2) bscatter_kernel(const BParams p, int r0, int nr, int l0,
                                                                      int nl) {
  const int lane = threadIdx.x & 31;
  const uint32_t nchunks = launch_chunks(p, nr, nl);
  const uint32_t nwarps = gridDim.x * (blockDim.x >> 5);
  const int bytes = p.P * 128;
  for (uint32_t wi = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); wi < nchunks; wi += nwarps) {
    const Chunk c = decode_chunk(p, wi, r0, l0, nl, lane);
    int src = -1, dst = -1;
    bool move = false, hz = false;
    if (c.valid) {
      dst = p.new_table[static_cast<int64_t>(c.i) * p.max_cols + c.nprot + c.j];
      src = p.src_unit[c.base + c.j];
      const float sc = p.score_scr[c.base + c.j];
      const bool staged = p.hflag[c.base + c.j] != 0;
      if (dst < 0 || dst >= p.pool_units || src < 0 || src >= p.pool_units) {
        flag_error(p.err, CE_EW_INDEX);
      } else {
        p.scores[c.l * p.sls + c.g * p.shs + dst] = sc;
        move = src != dst;
        hz = move && staged;
      }
    }
    const unsigned mmask = __ballot_sync(0xffffffffu, move);
    if constexpr (SMALL) {
      const int64_t item0 = c.item - lane;
      copy_items(mmask, bytes, lane,
                 [&](int k, const uint8_t*& sk, const uint8_t*& sv, uint8_t*& dk, uint8_t*& dv) {
                   const int s = max(__shfl_sync(0xffffffffu, src, k), 0);
                   const int d = max(__shfl_sync(0xffffffffu, dst, k), 0);
                   const bool h = __shfl_sync(0xffffffffu, hz, k);
                   const uint8_t* scr = p.hazard + (item0 + k) * 2 * bytes;
                   sk = h ? scr : unit_ptr(p.k_layers, c.l, s, c.g, p.G, p.P);
                   sv = h ? scr + bytes : unit_ptr(p.v_layers, c.l, s, c.g, p.G, p.P);
                   dk = unit_ptr(p.k_layers, c.l, d, c.g, p.G, p.P);
                   dv = unit_ptr(p.v_layers, c.l, d, c.g, p.G, p.P);
                 });
      continue;
    }
    for (unsigned todo = mmask; todo; todo &= todo - 1) {
      const int k = __ffs(todo) - 1;
      const int s = __shfl_sync(0xffffffffu, src, k);
      const int d = __shfl_sync(0xffffffffu, dst, k);
      const bool h = __shfl_sync(0xffffffffu, hz, k);
      const int64_t it = __shfl_sync(0xffffffffu, c.item, k);
      const uint8_t* ks = h ? p.hazard + it * 2 * bytes : unit_ptr(p.k_layers, c.l, s, c.g, p.G, p.P);
      const uint8_t* vs = h ? p.hazard + it * 2 * bytes + bytes : unit_ptr(p.v_layers, c.l, s, c.g, p.G, p.P);
      copy_pair(unit_ptr(p.k_layers, c.l, d, c.g, p.G, p.P), unit_ptr(p.v_layers, c.l, d, c.g, p.G, p.P), ks, vs,
                bytes, lane);
    }
  }
}

// Grid (rows, 1 + L * G).  Block (i, 0): table, count, frontier, the
// req_to_unit packing of row i and, for a live boundary that passed the
// sliding-window guard, the tag -epoch in marks[] on every freed unit of the
// row (bzero_kernel then zeroes their scores).  Block (i, 1 + s): the new
// positions of segment s = (layer, head) -- its protected slots gathered
// here, its middle survivors from the selection.
__global__ void __launch_bounds__(T) bfinish_kernel(const BParams p) {
  const int i = blockIdx.x;
  const int32_t* info = p.row_info + i * RI;
  if (info[7] != 0) return;
  // The row as the selection saw it (block (i, 0) rewrites count and frontier).
  RowCtx r;
  r.row = p.rows[i];
  r.q = p.params[i];
  r.N = info[0];
  r.cnt = info[6];
  r.fr = r.cnt + r.q.n - r.N;
  const int after = info[3], true_u = info[4], nleft = info[5];
  const bool bad = info[8] != 0;   // guard of runtime:477-479, checked by the row block
  const int LG = p.L * p.G;
  const int32_t* ntab = p.new_table + static_cast<int64_t>(i) * p.max_cols;
  const int32_t* left = p.freed + i * p.freed_stride;
  if (blockIdx.y > 0) {
    const int lg = static_cast<int>(blockIdx.y) - 1;
    if (lg >= LG) return;
    int32_t* src = p.new_pos + (static_cast<int64_t>(i) * LG + lg) * p.max_cols;
    int32_t* dst = p.pos + r.row * p.prs + static_cast<int64_t>(lg) * p.pos_cap;
    // Protected slots: this head's positions at the (0,0) head's protected
    // columns, in (0,0) position order (runtime:442-443, 469).  Every read
    // of the old positions ends before the copy below overwrites them.
    const int32_t* pcol = p.prot_col + static_cast<int64_t>(i) * p.max_cols;
    batched<8>(
        info[1], [&](int k) { return pcol[k]; }, [&](int, int c) { return col_pos(p, r, lg, c); },
        [&](int k, int, int v) { src[k] = v; });
    __syncthreads();
    batched<8>(
        after, [&](int k) { return src[k]; }, [](int, int) { return 0; },
        [&](int k, int v, int) { dst[k] = v; });
    return;
  }
  batched<8>(
      after, [&](int k) { return ntab[k]; }, [](int, int) { return 0; },
      [&](int k, int u, int) { p.table[r.row * p.ts + k] = u; });
  int32_t* res = p.result + i * 4;
  if (threadIdx.x == 0) {
    p.count[r.row] = after;
    p.frontier[r.row] = r.q.n;
  }
  if (!p.live) {
    if (threadIdx.x == 0) res[3] = 0;
    return;
  }
  if (bad) {
    if (threadIdx.x == 0) {
      res[0] = 5;
      flag_error(p.err, CE_EW_SWA);
    }
    return;
  }
  if (threadIdx.x == 0) res[3] = nleft;
  // Freed units: their scores are zeroed at every (layer, head) (runtime:481)
  // by bzero_kernel, which finds them by this tag.  A freed unit is never a
  // real slot of [true_u, n) (those are protected), so the tags do not meet.
  batched<8>(
      nleft, [&](int k) { return left[k]; }, [](int, int) { return 0; },
      [&](int, int u, int) {
        if (u >= 0 && u < p.pool_units) p.marks[u] = -p.epoch;
      });
  // The packed prefix the row block listed (runtime:484-491), then zeros up to true_u.
  const int npacked = info[9];
  if (npacked > true_u) {
    if (threadIdx.x == 0) {
      res[0] = 4;
      flag_error(p.err, CE_EW_PACK);
    }
    return;
  }
  int32_t* rrow = p.r2u + r.row * p.rs;
  const int32_t* plist = p.pack + static_cast<int64_t>(i) * p.max_cols;
  batched<8>(
      npacked, [&](int k) { return plist[k]; }, [](int, int) { return 0; },
      [&](int k, int u, int) { rrow[k] = u; });
  for (int x = npacked + threadIdx.x; x < min(true_u, p.r2u_width); x += T) rrow[x] = 0;
}

// Zero the scores of every unit bfinish_kernel tagged as freed, at every
// (layer, head): one thread per pool unit, so each warp's stores cover 32
// consecutive units of one (layer, head) row -- coalesced, where zeroing
// from the rows' freed lists would scatter one 4-byte store per (unit,
// layer, head).
__global__ void bzero_kernel(const BParams p) {
  const int64_t u = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (u >= p.pool_units || p.marks[u] != -p.epoch) return;
  for (int l = 0; l < p.L; ++l)
    for (int g = 0; g < p.G; ++g) p.scores[l * p.sls + g * p.shs + u] = 0.f;
}

__global__ void gather_scores_kernel(const BParams p, float* out) {
  const int LG = p.L * p.G;
  const int i = blockIdx.x / LG, lg = blockIdx.x % LG;
  const int l = lg / p.G, g = lg % p.G;
  const RowCtx r = row_ctx(p, i);
  float* o = out + (static_cast<int64_t>(i) * LG + lg) * p.max_cols;
  const int N = (r.N >= 0 && r.N <= p.max_cols) ? r.N : 0;
  for (int c = threadIdx.x; c < p.max_cols; c += blockDim.x)
    o[c] = (c < N) ? unit_score(p, l, g, col_unit(p, r, c)) : 0.f;
}

__global__ void reservoir_kernel(const int32_t* pos, int layers, int heads, int n_cols,
                                 int head_offset, uint64_t seed, uint64_t* out) {
  const int64_t total = static_cast<int64_t>(layers) * heads * n_cols;
  for (int64_t x = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; x < total;
       x += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int l = static_cast<int>(x / (static_cast<int64_t>(heads) * n_cols));
    const int g = static_cast<int>((x / n_cols) % heads);
    out[x] = reservoir53(seed, l, head_offset + g, static_cast<uint64_t>(pos[x]));
  }
}

}  // namespace sel
}  // namespace ce

using namespace ce;
using namespace ce::sel;

int ce::host::select_prepare_device() {
  // cudaFuncGetAttributes loads a kernel under lazy module loading.
  cudaFuncAttributes a;
  const void* fns[] = {
      reinterpret_cast<const void*>(bsel_kernel<true>), reinterpret_cast<const void*>(bsel_kernel<false>),
      reinterpret_cast<const void*>(bvalidate_kernel), reinterpret_cast<const void*>(bgather_kernel<true>),
      reinterpret_cast<const void*>(bgather_kernel<false>), reinterpret_cast<const void*>(bscatter_kernel<true>),
      reinterpret_cast<const void*>(bscatter_kernel<false>), reinterpret_cast<const void*>(bfinish_kernel),
      reinterpret_cast<const void*>(bzero_kernel), reinterpret_cast<const void*>(hsum_kernel),
      reinterpret_cast<const void*>(unit_sum_kernel), reinterpret_cast<const void*>(brecord_kernel),
      reinterpret_cast<const void*>(choose_seg_kernel<true>), reinterpret_cast<const void*>(choose_seg_kernel<false>),
      reinterpret_cast<const void*>(choose_status_kernel), reinterpret_cast<const void*>(gather_scores_kernel),
      reinterpret_cast<const void*>(reservoir_kernel)};
  for (const void* f : fns)
    if (cudaFuncGetAttributes(&a, f) != cudaSuccess) return host::fail_cuda("selection kernels: set-up");
  return CE_OK;
}

namespace {
size_t a256(size_t x) { return (x + 255) & ~size_t(255); }

struct BLayout {
  size_t kv, pv, seg, mid, src, npos, ssc, hflag, info, crank, ntab, pcol, pack, hsum, hazard, total;
};

BLayout boundary_layout(int R, int L, int G, int max_cols, int64_t hazard_bytes) {
  BLayout b{};
  const size_t cells = static_cast<size_t>(R) * L * G * max_cols;
  size_t o = 0;
  b.kv = o; o += a256(cells * 8);
  b.pv = o; o += a256(cells * 4);
  b.seg = o; o += a256(static_cast<size_t>(R) * L * G * 4);
  b.mid = o; o += a256(cells * 4);
  b.src = o; o += a256(cells * 4);
  b.npos = o; o += a256(cells * 4);
  b.ssc = o; o += a256(cells * 4);
  b.hflag = o; o += a256(cells);
  b.info = o; o += a256(static_cast<size_t>(R) * RI * 4);
  b.crank = o; o += a256(static_cast<size_t>(R) * max_cols * 4);
  b.ntab = o; o += a256(static_cast<size_t>(R) * max_cols * 4);
  b.pcol = o; o += a256(static_cast<size_t>(R) * max_cols * 4);
  b.pack = o; o += a256(static_cast<size_t>(R) * max_cols * 4);
  b.hsum = o; o += a256(static_cast<size_t>(R) * L * max_cols * 4);
  b.hazard = o; o += a256(static_cast<size_t>(hazard_bytes));
  b.total = o;
  return b;
}

int64_t hazard_per_layer(int R, int G, int max_width, int P) {
  return static_cast<int64_t>(R) * G * max_width * 2 * P * 128;
}

int sel_smem(int nw) { return nw * 8; }
constexpr int kLargeSmemMax = 220 * 1024;   // dynamic shared memory a large-segment launch may use
}  // namespace

extern "C" int64_t ce_choose_workspace_bytes(int32_t problems, int32_t segs, int32_t n_cols) {
  if (problems < 0 || segs <= 0 || n_cols < 0) return -1;
  const size_t cells = static_cast<size_t>(problems) * segs * n_cols;
  return static_cast<int64_t>(a256(cells * 8) + a256(cells * 4) +
                              a256(static_cast<size_t>(problems) * segs * 4));
}

extern "C" int ce_choose(const int32_t* pos, const int32_t* ncols, int32_t n_cols, const void* score,
                         int32_t score_dtype, const ce_row_params* params, int32_t problems,
                         int32_t max_n, int32_t layers, int32_t heads, int32_t head_offset,
                         int32_t* kept, int32_t kept_stride, int32_t* status,
                         int32_t* protected_count, void* workspace, int64_t workspace_bytes,
                         int32_t* err, void* stream) {
  if (problems < 0 || n_cols < 0 || layers <= 0 || heads <= 0 || max_n < 0 || kept_stride < 0)
    return host::fail(CE_ERR_ARG, "bad size");
  if (problems == 0) return CE_OK;
  if (!pos || !params || !kept || !status || !workspace) return host::fail(CE_ERR_ARG, "null pointer");
  if (score && score_dtype != CE_DTYPE_F32 && score_dtype != CE_DTYPE_F64)
    return host::fail(CE_ERR_ARG, "score dtype must be f32 or f64");
  const int segs = layers * heads;
  const int64_t need = ce_choose_workspace_bytes(problems, segs, n_cols);
  if (workspace_bytes < need) return host::fail(CE_ERR_WORKSPACE, "choose workspace too small");
  const int nw = (max_n + 31) / 32;
  if (sel_smem(nw) > 200 * 1024) return host::fail(CE_ERR_UNSUPPORTED, "max_n too large");
  const size_t cells = static_cast<size_t>(problems) * segs * n_cols;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  ChooseParams p{};
  p.pos = pos;
  p.ncols = ncols;
  p.n_cols = n_cols;
  p.score = score;
  p.sdt = score ? score_dtype : CE_DTYPE_F32;
  p.params = params;
  p.problems = problems;
  p.layers = layers;
  p.heads = heads;
  p.head_offset = head_offset;
  p.nw = nw;
  p.kept = kept;
  p.kept_stride = kept_stride;
  p.status = status;
  p.pcount = protected_count;
  p.kv = reinterpret_cast<uint64_t*>(ws);
  p.pv = reinterpret_cast<int32_t*>(ws + a256(cells * 8));
  p.seg_info = reinterpret_cast<int32_t*>(ws + a256(cells * 8) + a256(cells * 4));
  p.err = err;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  p.vec4 = (n_cols % 4 == 0) && (reinterpret_cast<uintptr_t>(pos) % 16 == 0) &&
           (reinterpret_cast<uintptr_t>(score) % 16 == 0);
  const bool large = n_cols > REG_ITEMS * T && sel_smem(nw) + LARGE_BYTES <= kLargeSmemMax;
  const int smem = sel_smem(nw) + (large ? LARGE_BYTES : 0);
  if (large) {
    if (!host::set_smem(choose_seg_kernel<true>, smem)) return host::fail(CE_ERR_CUDA, "smem attr");
    choose_seg_kernel<true><<<problems * segs, T, smem, st>>>(p);
  } else {
    if (!host::set_smem(choose_seg_kernel<false>, smem)) return host::fail(CE_ERR_CUDA, "smem attr");
    choose_seg_kernel<false><<<problems * segs, T, smem, st>>>(p);
  }
  if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("choose_seg_kernel");
  choose_status_kernel<<<problems, 32, 0, st>>>(p);
  if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("choose_status_kernel");
  return CE_OK;
}

extern "C" int64_t ce_boundary_workspace_bytes(int32_t num_rows, int32_t layers, int32_t kv_heads,
                                               int32_t head_dim, int32_t page_size,
                                               int32_t max_cols, int32_t max_width,
                                               int32_t global_heads, int64_t hazard_bytes) {
  (void)global_heads;
  if (num_rows < 0 || layers <= 0 || kv_heads <= 0 || head_dim != 64 || page_size <= 0 ||
      max_cols < 0)
    return -1;
  const int width = (max_width > 0 && max_width < max_cols) ? max_width : max_cols;
  const int64_t one = hazard_per_layer(1, kv_heads, width, page_size);   // one row of one layer
  const int64_t hz = hazard_bytes < one ? one : hazard_bytes;
  return static_cast<int64_t>(boundary_layout(num_rows, layers, kv_heads, max_cols, hz).total);
}

static int boundary_params(BParams& p, int32_t* table, int64_t table_stride, int32_t table_width,
                           int32_t* req_to_unit, int64_t r2u_stride, int32_t r2u_width,
                           int32_t* frontier, int32_t* count, int32_t* pos,
                           int64_t pos_row_stride, int32_t pos_cap, float* scores,
                           int64_t sls, int64_t shs, int64_t pool_units, int32_t layers,
                           int32_t kv_heads, int32_t page_size, const int32_t* rows,
                           const ce_row_params* params, int32_t num_rows, int32_t max_cols,
                           int32_t max_n) {
  p.table = table;
  p.ts = table_stride;
  p.table_width = table_width;
  p.r2u = req_to_unit;
  p.rs = r2u_stride;
  p.r2u_width = r2u_width;
  p.frontier = frontier;
  p.count = count;
  p.pos = pos;
  p.prs = pos_row_stride;
  p.pos_cap = pos_cap;
  p.scores = scores;
  p.sls = sls;
  p.shs = shs;
  p.pool_units = pool_units;
  p.L = layers;
  p.G = kv_heads;
  p.P = page_size;
  p.rows = rows;
  p.params = params;
  p.R = num_rows;
  p.max_cols = max_cols;
  p.nw = (max_n + 31) / 32;
  return CE_OK;
}

extern "C" int ce_gather_row_scores(const int32_t* table, int64_t table_stride,
                                    const int32_t* req_to_unit, int64_t r2u_stride,
                                    const int32_t* frontier, const int32_t* count,
                                    const float* scores, int64_t score_layer_stride,
                                    int64_t score_head_stride, int64_t pool_units, int32_t layers,
                                    int32_t kv_heads, const int32_t* rows,
                                    const ce_row_params* params, int32_t num_rows,
                                    int32_t max_cols, float* out, int32_t* err, void* stream) {
  if (num_rows < 0 || layers <= 0 || kv_heads <= 0 || max_cols < 0)
    return host::fail(CE_ERR_ARG, "bad size");
  if (num_rows == 0 || max_cols == 0) return CE_OK;
  BParams p{};
  boundary_params(p, const_cast<int32_t*>(table), table_stride, 0,
                  const_cast<int32_t*>(req_to_unit), r2u_stride, 0, const_cast<int32_t*>(frontier),
                  const_cast<int32_t*>(count), nullptr, 0, 0, const_cast<float*>(scores),
                  score_layer_stride, score_head_stride, pool_units, layers, kv_heads, 1, rows,
                  params, num_rows, max_cols, 0);
  p.err = err;
  gather_scores_kernel<<<num_rows * layers * kv_heads, 256, 0, static_cast<cudaStream_t>(stream)>>>(p, out);
  if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("gather_scores_kernel");
  return CE_OK;
}

extern "C" int ce_boundary(int32_t* table, int64_t table_stride, int32_t table_width,
                           int32_t* req_to_unit, int64_t r2u_stride, int32_t r2u_width,
                           int32_t* frontier, int32_t* count, int32_t* pos,
                           int64_t pos_row_stride, int32_t pos_cap, float* scores,
                           int64_t score_layer_stride, int64_t score_head_stride,
                           int64_t pool_units, const uint64_t* k_layers,
                           const uint64_t* v_layers, int32_t layers, int32_t kv_heads,
                           int32_t head_dim, int32_t page_size, int32_t head_offset,
                           int32_t* marks, int32_t epoch, const int64_t* swa_mapping,
                           const int32_t* rows, const ce_row_params* params, int32_t num_rows,
                           const void* uniforms, int32_t uniform_dtype,
                           const float* global_scores, int32_t global_heads, int32_t live,
                           int32_t max_cols, int32_t max_width, int32_t max_n, int32_t* result,
                           int32_t* freed_units, int64_t freed_stride, void* workspace,
                           int64_t workspace_bytes, int64_t hazard_bytes, uint32_t* record_delta,
                           int64_t record_stride, int32_t* record_counts, int32_t* err,
                           void* stream) {
  if (num_rows < 0 || layers <= 0 || kv_heads <= 0 || max_cols < 0 || max_n < 0 || page_size <= 0)
    return host::fail(CE_ERR_ARG, "bad size");
  if (record_delta && (!record_counts || record_stride < max_cols))
    return host::fail(CE_ERR_ARG, "retention record needs counts and a row stride >= max_cols");
  if (head_dim != 64) return host::fail(CE_ERR_UNSUPPORTED, "head_dim must be 64");
  if (num_rows == 0) return CE_OK;
  if (!table || !req_to_unit || !frontier || !count || !pos || !scores || !k_layers || !v_layers ||
      !rows || !params || !result || !workspace)
    return host::fail(CE_ERR_ARG, "null pointer");
  if (live && (!marks || !freed_units)) return host::fail(CE_ERR_ARG, "live needs marks and freed_units");
  if (live && epoch <= 0) return host::fail(CE_ERR_ARG, "live needs epoch >= 1");
  if (uniforms && uniform_dtype != CE_DTYPE_F32 && uniform_dtype != CE_DTYPE_F64)
    return host::fail(CE_ERR_ARG, "uniform dtype must be f32 or f64");
  const int nw = (max_n + 31) / 32;
  if (sel_smem(nw) > 200 * 1024) return host::fail(CE_ERR_UNSUPPORTED, "max_n too large");
  const int width = (max_width > 0 && max_width < max_cols) ? max_width : max_cols;
  const int64_t one = hazard_per_layer(1, kv_heads, width, page_size);   // one row of one layer
  const int64_t hz = hazard_bytes < one ? one : hazard_bytes;
  const BLayout Lo = boundary_layout(num_rows, layers, kv_heads, max_cols, hz);
  if (workspace_bytes < static_cast<int64_t>(Lo.total))
    return host::fail(CE_ERR_WORKSPACE, "boundary workspace too small");
  BParams p{};
  boundary_params(p, table, table_stride, table_width, req_to_unit, r2u_stride, r2u_width,
                  frontier, count, pos, pos_row_stride, pos_cap, scores, score_layer_stride,
                  score_head_stride, pool_units, layers, kv_heads, page_size, rows, params,
                  num_rows, max_cols, max_n);
  p.max_width = width;
  p.ch = chunk_items(page_size);
  p.k_layers = k_layers;
  p.v_layers = v_layers;
  p.head_offset = head_offset;
  p.marks = marks;
  p.epoch = epoch;
  p.swa = swa_mapping;
  p.uniforms = uniforms;
  p.udt = uniform_dtype;
  p.gscores = global_scores;
  p.GH = global_heads;
  p.live = live;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.kv = reinterpret_cast<uint64_t*>(ws + Lo.kv);
  p.pv = reinterpret_cast<int32_t*>(ws + Lo.pv);
  p.seg_info = reinterpret_cast<int32_t*>(ws + Lo.seg);
  p.mid_col = reinterpret_cast<int32_t*>(ws + Lo.mid);
  p.src_unit = reinterpret_cast<int32_t*>(ws + Lo.src);
  p.new_pos = reinterpret_cast<int32_t*>(ws + Lo.npos);
  p.score_scr = reinterpret_cast<float*>(ws + Lo.ssc);
  p.hflag = ws + Lo.hflag;
  p.row_info = reinterpret_cast<int32_t*>(ws + Lo.info);
  p.cand_rank = reinterpret_cast<int32_t*>(ws + Lo.crank);
  p.new_table = reinterpret_cast<int32_t*>(ws + Lo.ntab);
  p.prot_col = reinterpret_cast<int32_t*>(ws + Lo.pcol);
  p.pack = reinterpret_cast<int32_t*>(ws + Lo.pack);
  p.hazard = ws + Lo.hazard;
  if (!global_scores) {   // H2O global rows sum their heads once, in hsum_kernel
    p.gscores = reinterpret_cast<float*>(ws + Lo.hsum);
    p.GH = 1;
  }
  p.freed = freed_units;
  p.freed_stride = freed_stride;
  p.result = result;
  p.rec_delta = record_delta;
  p.rec_stride = record_stride;
  p.rec_counts = record_counts;
  p.err = err;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool large = max_cols > REG_ITEMS * T && sel_smem(nw) + LARGE_BYTES <= kLargeSmemMax;
  const int smem = sel_smem(nw) + (large ? LARGE_BYTES : 0);
  if (!host::set_smem(bsel_kernel<false>, smem) || !host::set_smem(bsel_kernel<true>, smem))
    return host::fail(CE_ERR_CUDA, "smem attr");
  if (cudaMemsetAsync(p.row_info, 0, sizeof(int32_t) * RI * num_rows, st) != cudaSuccess)
    return host::fail_cuda("row_info memset");
  if (!global_scores) {
    // Long rows (more than 4,096 columns) that own most of the pool
    // (pool_units <= 2 x rows x columns): per-unit head sums in the kv region
    // (free until the selection, and at least 8 x rows x layers x max_cols
    // bytes) save G - 1 gathers per column.  Shorter rows gather cheaply and
    // would only pay the extra launch.
    float* usum = nullptr;
    if (max_cols > REG_ITEMS * T && pool_units > 0 && pool_units <= 2LL * num_rows * max_cols) {
      usum = reinterpret_cast<float*>(p.kv);
      const int64_t ublocks = std::min<int64_t>((pool_units + 255) / 256, 8LL * host::sm_count());
      unit_sum_kernel<<<static_cast<unsigned>(std::max<int64_t>(1, ublocks)), 256, 0, st>>>(p, usum);
      if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("unit_sum_kernel");
    }
    hsum_kernel<<<dim3((max_cols + 255) / 256, num_rows), 256, 0, st>>>(p, const_cast<float*>(p.gscores), usum);
    if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("hsum_kernel");
  }
  if (large)
    bsel_kernel<true><<<num_rows * layers * kv_heads + num_rows, T, smem, st>>>(p);
  else
    bsel_kernel<false><<<num_rows * layers * kv_heads + num_rows, T, smem, st>>>(p);
  if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("bsel_kernel");
  bvalidate_kernel<<<num_rows, 32, 0, st>>>(p);
  if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("bvalidate_kernel");
  if (record_delta) {
    const int rsmem = sel_smem(nw) + ((max_cols + 31) / 32) * 4;
    if (!host::set_smem(brecord_kernel, rsmem)) return host::fail(CE_ERR_CUDA, "smem attr");
    brecord_kernel<<<num_rows * layers * kv_heads, T, rsmem, st>>>(p);
    if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("brecord_kernel");
  }
  // Launch groups of rows x layers that fit the hazard workspace (all rows
  // of as many layers as fit, or fewer rows of one layer).  Splitting further
  // to keep the staged copies in L2 was measured slower: the extra launches
  // cost more than the DRAM round trip they save.
  const int64_t row_layer = hazard_per_layer(1, kv_heads, width, page_size);
  const int rows_per = static_cast<int>(std::min<int64_t>(num_rows, std::max<int64_t>(1, hz / row_layer)));
  const int group = static_cast<int>(
      std::min<int64_t>(layers, std::max<int64_t>(1, hz / (static_cast<int64_t>(rows_per) * row_layer))));
  const int nsm = host::sm_count();
  const bool small = chunk_items(page_size) == CH_SMALL;   // matches the kernels' copy path
  for (int r0 = 0; r0 < num_rows; r0 += rows_per) {
    const int nr = std::min(rows_per, num_rows - r0);
    for (int l0 = 0; l0 < layers; l0 += group) {
      const int nl = std::min(group, layers - l0);
      // one warp per chunk of p.ch middle survivors of a (row, layer, head)
      const int64_t chunks = static_cast<int64_t>(nr) * nl * kv_heads * ((width + p.ch - 1) / p.ch);
      if (chunks > INT32_MAX) return host::fail(CE_ERR_UNSUPPORTED, "ce_boundary: too many rows x layers x heads");
      const int64_t want = (chunks * 32 + 255) / 256;
      const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, 8LL * nsm)));
      if (small) {
        bgather_kernel<true><<<blocks, 256, 0, st>>>(p, r0, nr, l0, nl);
      } else {
        bgather_kernel<false><<<blocks, 256, 0, st>>>(p, r0, nr, l0, nl);
      }
      if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("bgather_kernel");
      if (small) {
        bscatter_kernel<true><<<blocks, 256, 0, st>>>(p, r0, nr, l0, nl);
      } else {
        bscatter_kernel<false><<<blocks, 256, 0, st>>>(p, r0, nr, l0, nl);
      }
      if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("bscatter_kernel");
    }
  }
  bfinish_kernel<<<dim3(num_rows, 1 + layers * kv_heads), T, 0, st>>>(p);
  if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("bfinish_kernel");
  if (live && pool_units > 0) {
    bzero_kernel<<<static_cast<unsigned>((pool_units + 255) / 256), 256, 0, st>>>(p);
    if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("bzero_kernel");
  }
  return CE_OK;
}

extern "C" int ce_reservoir_scores(const int32_t* pos, int32_t layers, int32_t heads, int32_t n_cols,
                                   int32_t head_offset, uint64_t seed, uint64_t* out,
                                   void* stream) {
  if (layers < 0 || heads < 0 || n_cols < 0) return host::fail(CE_ERR_ARG, "bad size");
  const int64_t total = static_cast<int64_t>(layers) * heads * n_cols;
  if (total == 0) return CE_OK;
  if (!pos || !out) return host::fail(CE_ERR_ARG, "null pointer");
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 4096));
  reservoir_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(pos, layers, heads, n_cols,
                                                                            head_offset, seed, out);
  if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("reservoir_kernel");
  return CE_OK;
}

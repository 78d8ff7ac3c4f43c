// Shared device helpers for the sm_100a eviction kernels: error words,
// bounded mbarrier waits, bulk-tensor (TMA) loads, ldmatrix and the
// m16n8k16 bf16 tensor-core step used by the decode kernel.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include "../../include/ce_api.h"

namespace ce {

// A device wait that has not completed after this many nanoseconds of
// %globaltimer gives up, flags CE_EW_TIMEOUT and lets the kernel return.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ void flag_error(int32_t* err, int bits) {
  if (err) atomicOr(err, bits);
}

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ---------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and flags the error
// word) when the phase did not complete within limit_ns (kWaitLimitNs for
// every kernel; the self-test passes a shorter one).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int32_t* err,
                                          unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > limit_ns) {
      flag_error(err, CE_EW_TIMEOUT);
      return false;
    }
  }
}

// Bounded wait that also gives up as soon as another warp of the CTA has set
// *abort (polled only on the slow path, so a ready stage costs one try_wait).
__device__ __forceinline__ bool mbar_wait_or_abort(uint64_t* bar, uint32_t parity, int32_t* err,
                                                   volatile int* abort,
                                                   unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (global_timer_ns() - t0 > limit_ns) {
      flag_error(err, CE_EW_TIMEOUT);
      return false;
    }
  }
}

// ---- TMA: 2D tiled bulk-tensor load into shared memory, no multicast --------
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, int32_t x,
                                            int32_t y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

// ---- warp-level tensor-core helpers ------------------------------------------
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                              uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D += A(16x16, rows 8..15 zero) * B(16x8); a1/a3 (the zero rows) are passed
// as 0 so only the upper half of the tile carries query heads.
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0,
                                          uint32_t b1) {
  const uint32_t z = 0u;
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(z), "r"(a2), "r"(z), "r"(b0), "r"(b1));
}

// D += A(16x16) * B(16x8), all four A registers live.
__device__ __forceinline__ void mma_16816_full(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// In-register transpose of an 8x8 b16 matrix held one row-pair per thread in
// the MMA fragment layout (thread i: row i/4, columns 2(i%4), 2(i%4)+1).
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// Split two fp32 values into bf16 hi parts and bf16 residuals so that
// hi + lo reproduces each value to ~2^-17 relative.
__device__ __forceinline__ void split_bf16x2(float a, float b, uint32_t& hi, uint32_t& lo) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  float2 hf = __bfloat1622float2(h);
  __nv_bfloat162 l = __floats2bfloat162_rn(a - hf.x, b - hf.y);
  hi = *reinterpret_cast<uint32_t*>(&h);
  lo = *reinterpret_cast<uint32_t*>(&l);
}

// ---- order-preserving integer keys for fp scores ------------------------------
// Larger float -> larger unsigned key.  -0.0 is folded onto +0.0 (the reference
// compares doubles, where they are equal) and NaN maps to the largest key.
__device__ __forceinline__ uint64_t key_from_f32(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7fffffffu) == 0u) u = 0u;
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return 0xffffffffull;
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return static_cast<uint64_t>(u);
}

__device__ __forceinline__ uint64_t key_from_f64(double d) {
  uint64_t u = static_cast<uint64_t>(__double_as_longlong(d));
  if ((u & 0x7fffffffffffffffull) == 0ull) u = 0ull;
  if ((u & 0x7ff0000000000000ull) == 0x7ff0000000000000ull && (u & 0x000fffffffffffffull))
    return 0xffffffffffffffffull;
  return (u & 0x8000000000000000ull) ? ~u : (u | 0x8000000000000000ull);
}

// splitmix64 of (seed, layer, kv head, position) as in the reference's
// reservoir_scores (runtime:358-373) and core.reservoir_score (core.py:23-30);
// returns the top 53 bits (the double is this integer / 2^53).
__device__ __forceinline__ uint64_t reservoir53(uint64_t seed, uint64_t layer, uint64_t head,
                                                uint64_t pos) {
  uint64_t x = pos * 0x9E3779B97F4A7C15ull + layer * 0xBF58476D1CE4E5B9ull +
               head * 0x94D049BB133111EBull + seed * 0xD1B54A32D192ED03ull +
               0x632BE59BD9B4E019ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  x = x ^ (x >> 31);
  return x >> 11;
}


// ---- TMA: 3D tiled bulk-tensor load, no multicast -----------------------------
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const void* tmap, int32_t x, int32_t y,
                                            int32_t z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_addr(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
      : "memory");
}

// ---- 5th-generation tensor cores (tcgen05) and tensor memory ------------------
// Allocation by one full warp; the TMEM address lands in *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_addr(dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Shared-memory matrix descriptor of a K-major bf16 tile whose 128-byte rows
// are laid out in 1024-byte, 8-row atoms with the 128-byte swizzle (chunk c of
// row r at chunk c ^ (r & 7)): start address >> 4, leading offset 16 B
// (unused by swizzled K-major), stride 1024 B between 8-row atoms,
// descriptor version 1, layout SWIZZLE_128B.  The tile base must be
// 1024-byte aligned; K-steps of 16 elements advance the start by 32 bytes.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) |
         (1ull << 46) | (2ull << 61);
}
// Instruction descriptor of kind::f16: bf16 A and B (K-major), fp32 D, M x N.
__host__ __device__ constexpr uint32_t f16_idesc(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}
// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate ? 1u : 0u)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]^T, issued by one thread: A (M x K, K-major)
// lives in tensor memory, row m in lane m, two 16-bit K elements per 32-bit
// column (the lower K index in the low half).
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                          bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate ? 1u : 0u)
      : "memory");
}
// Arrive on *bar once every tcgen05.mma this thread issued so far has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_addr(bar))
      : "memory");
}
// 32 consecutive fp32 columns of this thread's TMEM lane (32x32b shape, x32);
// the registers are valid after tmem_ld_wait().
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// 32 consecutive fp32 columns of this thread's TMEM lane, waited for.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  tmem_ld32_async(taddr, v);
  tmem_ld_wait();
}
// Store 8 consecutive 32-bit columns of this thread's TMEM lane (32x32b
// shape, x8); complete after tmem_st_wait().
__device__ __forceinline__ void tmem_st8_async(uint32_t taddr, const uint32_t* r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
// 16 consecutive fp32 columns of this thread's TMEM lane (valid after tmem_ld_wait()).
__device__ __forceinline__ void tmem_ld16_async(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor of an MN-major bf16 operand in the same
// 128-byte-swizzled 1024-byte atoms: each 128-byte row holds 64 consecutive
// MN elements of one K index, 8 K indices per atom.  Atoms follow each other
// along K every 1024 B (stride offset); an operand of at most 64 MN elements
// has a single column of atoms, and the leading offset (the step between
// 64-element MN blocks) is given the same 1024 B so that it stays inside the
// tile either way.  K-steps of 16 elements advance the start by 2048 bytes.
__device__ __forceinline__ uint64_t sw128_mn_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (64ull << 16) | (64ull << 32) |
         (1ull << 46) | (2ull << 61);
}
// The instruction descriptor's B-operand major-ness bit: B is MN-major.
constexpr uint32_t kIdescBMajorMN = 1u << 16;

// ---- tiles shared by the tcgen05 kernels -----------------------------------------
// 128-byte rows of eight 16-byte chunks in 1024-byte atoms; chunk c of row r
// lives at c ^ (r & 7) (the layout TMA's 128-byte swizzle writes and the
// tcgen05 SWIZZLE_128B descriptors read).
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
// Generic-proxy writes to shared memory become visible to the async proxy
// (TMA, tcgen05.mma operand reads).
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Wait by one lane of a warp, result broadcast to the warp.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int32_t* err,
                                          volatile int* abort, int lane) {
  bool ok = true;
  if (lane == 0) ok = mbar_wait_or_abort(bar, parity, err, abort);
  return __shfl_sync(0xffffffffu, ok, 0);
}

// ---- exponentials ------------------------------------------------------------------
// 2^x with the SFU's approximate exp2 (PTX ex2.approx.ftz.f32): relative
// error near 2^-22, -inf -> +0, results below the normal range flush to 0.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA/ALU pipes, for a share of the exponentials so the SFU is not
// the only unit doing them: x = n + f with n = round(x) (adding 1.5 * 2^23
// leaves round(x) in the low mantissa bits), f in [-0.5, 0.5]; 2^f from a
// degree-3 polynomial (coefficients fitted for minimal relative error on
// [-0.5, 0.5], max relative error 7.6e-5) and 2^n added to the exponent
// field ((bits(t) << 23) == n << 23 because bits(1.5 * 2^23) end in 23 zero
// bits).  Arguments are clamped at -126 (the result is then a denormal
// near 0, like ex2.approx.ftz's 0); the callers' arguments are <= ~0.
__device__ __forceinline__ float poly_exp2(float x) {
  x = fmaxf(x, -126.f);
  const float t = x + 12582912.f;
  const float f = x - (t - 12582912.f);
  const float p = fmaf(fmaf(fmaf(0.055174146f, f, 0.24261758f), f, 0.69326109f), f, 0.99992758f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

}  // namespace ce

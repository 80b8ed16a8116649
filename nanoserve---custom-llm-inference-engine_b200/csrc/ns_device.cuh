// ns_device.cuh -- device helpers for the sm_100a sampling kernel.
//
// Inline-PTX wrappers for thread-block-cluster distributed shared memory
// (mapa / ld / st / red / atom on .shared::cluster), the split cluster
// barrier, mbarrier-tracked bulk copies (cp.async.bulk, global -> own
// shared memory, no multicast), plus the scalar arithmetic the sampler
// needs: correctly rounded division by a per-row constant, an order-
// preserving float key, and the Philox4x32-10 counter-based generator.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/nanoserve_sampler.h"

namespace ns {

// ----------------------------------------------------------------- smem / DSMEM
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Address of the same shared-memory offset in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t dsmem_map(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

__device__ __forceinline__ void dsmem_st_u32(uint32_t a, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}
__device__ __forceinline__ void dsmem_st_f32(uint32_t a, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(a), "f"(v) : "memory");
}
__device__ __forceinline__ void dsmem_st_u64(uint32_t a, uint64_t v) {
  asm volatile("st.shared::cluster.u64 [%0], %1;" ::"r"(a), "l"(v) : "memory");
}
__device__ __forceinline__ void dsmem_st_f64(uint32_t a, double v) {
  asm volatile("st.shared::cluster.f64 [%0], %1;" ::"r"(a), "d"(v) : "memory");
}
__device__ __forceinline__ uint32_t dsmem_ld_u32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t dsmem_ld_u64(uint32_t a) {
  uint64_t v;
  asm volatile("ld.shared::cluster.u64 %0, [%1];" : "=l"(v) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ float dsmem_ld_f32(uint32_t a) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ double dsmem_ld_f64(uint32_t a) {
  double v;
  asm volatile("ld.shared::cluster.f64 %0, [%1];" : "=d"(v) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ void dsmem_red_add_u32(uint32_t a, uint32_t v) {
  asm volatile("red.shared::cluster.add.u32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t dsmem_atom_add_u32(uint32_t a, uint32_t v) {
  uint32_t old;
  asm volatile("atom.shared::cluster.add.u32 %0, [%1], %2;" : "=r"(old) : "r"(a), "r"(v) : "memory");
  return old;
}

// Split cluster barrier.  Every thread of every CTA must take part, with
// warp-uniform control flow (the .aligned forms).
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_sync() {
  cluster_arrive();
  cluster_wait();
}
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// ----------------------------------------------------------------- mbarrier + bulk copy
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
// Non-blocking probe of phase `parity`; returns true once it completed.
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
// Asynchronous global -> shared copies of 8 / 16 bytes (cp.async, no
// mbarrier): used to fetch the next row's small parameters while the current
// row is being sampled.
__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_all;" ::: "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Orders this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (bulk copy) accesses to the same shared memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned) from
// global memory into this CTA's shared memory; completion is counted on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// ----------------------------------------------------------------- float helpers
// Order-preserving map float -> uint32 (larger float => larger key; -0 < +0).
__device__ __forceinline__ uint32_t f2key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}

// 2^x with the SFU (ex2.approx.ftz.f32: no subnormal results).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

constexpr float kLog2e = 1.4426950408889634f;

// e = exp(s - m) for s <= m; the only exponential used anywhere in the
// kernel, so every path sees identical values for the same (s, m).
__device__ __forceinline__ float exp_shifted(float s, float m) {
  return ex2_approx(__fmul_rn(__fsub_rn(s, m), kLog2e));
}

// Correctly rounded x / t given r = RN(1/t) (Markstein's division by a
// constant: q0 = RN(x r), rem = x - q0 t exactly via FMA, q = RN(q0 + rem r)).
// The remainder is exact only when neither x nor q0 is near the underflow
// range, so operands with min(|x|,|q0|) < 2^-60 or max(|x|,|q0|) > 2^100
// (zero, tiny, huge, non-finite) take the IEEE division instruction.  With
// that guard the result equals x / t bit for bit for every fp32 x; this was
// checked exhaustively over all 2^32 inputs for ten divisors from 1e-6 to
// 1e30 (tests/test_division_identity.py re-checks a sample on the CPU).
// The IEEE division, out of line: streaming loops that may need it (rarely)
// keep only a call, so their hot code stays small.
static __device__ __noinline__ float div_rn_out_of_line(float x, float t) { return __fdiv_rn(x, t); }

__device__ __forceinline__ float div_by_const(float x, float t, float r) {
  float q0 = __fmul_rn(x, r);
  float rem = __fmaf_rn(-q0, t, x);
  float q = __fmaf_rn(rem, r, q0);
  float ax = fabsf(x), aq = fabsf(q0);
  if (!(fminf(ax, aq) >= 0x1p-60f && fmaxf(ax, aq) <= 0x1p+100f)) q = div_rn_out_of_line(x, t);
  return q;
}

// Repetition penalty on one logit (HF rule, nanoserve/scheduler/sampler.py:37):
// negative scores are multiplied by rp, others divided by rp (IEEE fp32).
__device__ __forceinline__ float penalize(float x, float rp) {
  return (x < 0.0f) ? __fmul_rn(x, rp) : div_rn_out_of_line(x, rp);
}
// x / rp rounded to fp32 as IEEE division rounds it, for every x and rp,
// with no branch and no call (so that it can sit in unrolled streaming loops):
// given inv = RN64(1/rp), q0 = RN64(x inv) and one FMA correction give q1
// within an fp64 ulp of x / rp.  A quotient of two 24-bit significands is
// never that close to a midpoint of two fp32 neighbours (nor exactly on one),
// so RN32(q1) = RN32(x / rp); fp64 holds every such quotient without overflow
// or underflow.  When q0 is zero, infinite or NaN (x = 0, x = +-inf or NaN,
// rp = 0, +-inf or NaN) the correction would turn it into NaN, and q0 itself
// is already the IEEE result.
__device__ __forceinline__ float div_by_row_const(float x, float rp, double inv) {
  const double xd = (double)x;
  const double q0 = xd * inv;
  const double q1 = fma(fma(-q0, (double)rp, xd), inv, q0);
  return (float)((q0 != 0.0 && fabs(q0) <= 1.7976931348623157e308) ? q1 : q0);
}

// The same with inv = RN64(1/rp) (the row's constant): no out-of-line
// division path.
__device__ __forceinline__ float penalize(float x, float rp, double inv) {
  return (x < 0.0f) ? __fmul_rn(x, rp) : div_by_row_const(x, rp, inv);
}

// Approximate mass of one positive normal float for the top-p locator
// histogram: the top 16 of its 24 significand bits.  Every element of one
// histogram bucket shares its binary exponent, so a bucket's sum of these
// values, scaled by 2^(exponent - 142), under-estimates the bucket's true mass
// by less than a factor (1 - 2^-15).
__device__ __forceinline__ uint32_t approx_mass16(uint32_t bits) {
  return ((bits >> 8) & 0x7fffu) | 0x8000u;
}
// Scale a sum of approx_mass16 values of one binade (biased exponent ex) to
// 2^-44 fixed point (truncating).
__device__ __forceinline__ uint64_t mass16_to_fixed(uint64_t sum, int ex) {
  const int sh = ex - 98;  // value = sum * 2^(ex-142); fixed = value * 2^44
  if (sh >= 0) return sum << sh;
  if (sh <= -64) return 0ull;
  return sum >> (-sh);
}
constexpr double kFixedToReal = 1.0 / 17592186044416.0;  // 2^-44

// max that propagates NaN (any NaN operand gives NaN), used so that one pass
// both finds the row maximum and detects NaN logits.
__device__ __forceinline__ float fmax_nan(float a, float b) {
  float d;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}

// ----------------------------------------------------------------- warp helpers
__device__ __forceinline__ double warp_dsum(double v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ uint32_t warp_incl_u32(uint32_t v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    uint32_t t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  return v;
}
__device__ __forceinline__ double warp_incl_f64(double v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    double t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

// The reference keeps sorted rank j of the top-p pass iff j == 0 or
// float32(cum[j-1]) <= top_p (sampler.py:66-70); the first rank whose
// inclusive mass passes this test is the last one kept.
__device__ __forceinline__ bool topp_crossed(double cum, double z, float p) {
  return (float)(cum / z) > p;
}

// The same test without a division: fp32(cum / z) > p exactly when cum / z
// lies above the midpoint between p and the next float up, so with
// thr = topp_threshold(z, p) the test is cum > thr (the two differ only
// where cum / z is within a double rounding of that midpoint).
__device__ __forceinline__ double topp_threshold(double z, float p) {
  const float up = __uint_as_float(__float_as_uint(p) + (p >= 0.0f ? 1u : -1u));
  return 0.5 * ((double)p + (double)up) * z;
}

// Sort key: ascending keys give (value descending, index ascending).
__device__ __forceinline__ unsigned long long rank_key(float s, int idx) {
  return ((unsigned long long)(~f2key(s)) << 32) | (uint32_t)idx;
}
__device__ __forceinline__ float key_value(unsigned long long k) { return key2f(~(uint32_t)(k >> 32)); }
__device__ __forceinline__ int key_index(unsigned long long k) { return (int)(uint32_t)k; }

__device__ __forceinline__ void write_token(void* out, bool i32, int row, int tok) {
  if (i32) reinterpret_cast<int32_t*>(out)[row] = tok;
  else reinterpret_cast<int64_t*>(out)[row] = tok;
}

// ----------------------------------------------------------------- Philox4x32-10
// Counter-based generator of Salmon, Moraes, Dror and Shaw, "Parallel random
// numbers: as easy as 1, 2, 3" (SC'11): 10 rounds of the 4x32 Philox
// S-box with multipliers 0xD2511F53 / 0xCD9E8D57 and Weyl key increments
// 0x9E3779B9 / 0xBB67AE85.
struct U4 {
  uint32_t x, y, z, w;
};
__host__ __device__ __forceinline__ U4 philox4x32_10(U4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int i = 0; i < 10; ++i) {
    uint64_t p0 = (uint64_t)0xD2511F53u * c.x;
    uint64_t p1 = (uint64_t)0xCD9E8D57u * c.z;
    uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    c = U4{hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c;
}
// Uniform double in [0,1) with 53 random bits, for one (key, offset, row).
__host__ __device__ __forceinline__ double philox_uniform(uint64_t key, uint64_t offset, uint64_t row) {
  U4 c{(uint32_t)offset, (uint32_t)(offset >> 32), (uint32_t)row, (uint32_t)(row >> 32)};
  U4 o = philox4x32_10(c, (uint32_t)key, (uint32_t)(key >> 32));
  uint64_t a = o.x >> 5, b = o.y >> 6;  // 27 + 26 bits
  return (double)((a << 26) | b) * (1.0 / 9007199254740992.0);
}

// The uniform that drives row `row` of a call, clamped to [0, 1): the
// caller's uniforms[row] when given; else Philox4x32-10.  A row with
// NS_ROW_SEED uses its own key (the request's seed) and counter (seed_step,
// 0), so a seeded request draws the same numbers whatever batch it is in,
// wherever it sits in it and however many steps the sampler has run; other
// rows use key philox_seed and counter (philox_offset, row_offset + row).
__device__ __forceinline__ double row_uniform(const NsSampleArgs& a, const NsRowParams& P, int row) {
  double u;
  if (a.uniforms) {
    u = (double)a.uniforms[row];
  } else if (P.flags & NS_ROW_SEED) {
    u = philox_uniform(P.seed, (uint64_t)P.seed_step, 0ull);
  } else {
    u = philox_uniform(a.philox_seed, a.philox_offset, (uint64_t)(a.row_offset + row));
  }
  if (!(u >= 0.0)) u = 0.0;
  if (u >= 1.0) u = 0x1.fffffffffffffp-1;
  return u;
}

}  // namespace ns

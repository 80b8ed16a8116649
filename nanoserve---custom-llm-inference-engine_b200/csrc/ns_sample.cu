// ns_sample.cu -- B200 (sm_100a) token sampling: one kernel launch per step.
//
// Replaces nanoserve/scheduler/sampler.py:21-89 (Sampler.sample).  Design:
//
//  * One thread-block cluster of kCluster (8) CTAs per sampled row.  CTA r
//    owns the contiguous vocabulary slice [r*W, r*W+W) and keeps it in its
//    shared memory for the whole step, so the row crosses HBM exactly once.
//    Each warp pulls its own contiguous piece of the slice with one
//    mbarrier-tracked bulk copy (cp.async.bulk, no multicast) and starts
//    working on it as soon as it lands.
//  * Row statistics, histograms and candidate lists are exchanged through
//    distributed shared memory (st/ld/red/atom .shared::cluster) between
//    split cluster barriers.  No global scratch memory is used.
//  * Three row paths, chosen per row (uniformly across the cluster):
//      GREEDY   temperature == 0 and no debug output: first-index argmax
//               (sampler.py:82-83), one exchange.
//      TOPK     0 < top_k <= kTopkSmall: a per-thread-maximum histogram gives
//               a lower bound for the k-th largest logit, every element above
//               it is sent to the leader CTA, which finishes top-k
//               (sampler.py:53-58), top-p (sampler.py:60-73), softmax and the
//               inverse-CDF draw on that short list.
//      GENERAL  anything else: exp(s - max) is computed once per element and
//               kept in place; top-p uses a mass histogram keyed on the bits
//               of exp(s - max) (log-spaced buckets), refined until the
//               crossing bucket fits a candidate list, which the leader sorts
//               and scans.  Large top-k runs an exact 3-level radix select
//               first.  The draw scans per-warp masses in vocabulary order.
//  * Masses that decide filters are 2^-44 fixed point in 64-bit integers,
//    so every decision is order-independent and bit-reproducible.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <climits>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/nanoserve_sampler.h"
#include "ns_device.cuh"

namespace ns {

constexpr int kCluster = 8;
constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kBins = 2048;          // fine histogram buckets
constexpr int kCoarse = 32;          // coarse buckets (kBins / kCoarse fine each)
constexpr int kFinePerCoarse = kBins / kCoarse;
constexpr int kCap = 512;            // leader candidate list capacity
constexpr int kTopkSmall = 128;      // largest top_k served by the TOPK path
constexpr int kTmBins = 4096;        // per-thread-maximum histogram (u16 counts)
constexpr int kMaxSlice = 24576;     // largest slice (elements) one CTA holds
constexpr uint32_t kOne = 0x3F800000u;  // bits of 1.0f
constexpr uint64_t kCountOne = 1ull << 40;
constexpr uint64_t kMassMask = kCountOne - 1ull;

enum : uint32_t { kFlagNonFinite = 1u };

// Fixed-size control block at the start of dynamic shared memory.
struct __align__(16) Ctl {
  uint64_t mbar[kWarps];
  // per-peer records (slot = peer rank), written by the peers
  float rec_max[kCluster];
  float rec_minf[kCluster];
  uint32_t rec_flags[kCluster];
  int32_t rec_amax[kCluster];
  int32_t rec_nan[kCluster];
  int32_t rec_pinf[kCluster];
  double rec_mass[kCluster];
  // own coarse histogram, double-buffered (peers read it)
  uint64_t cmass[2][kCoarse];
  uint32_t ccnt[2][kCoarse];
  // leader candidate counter (peers add to it)
  uint32_t cand_n;
  // leader broadcast
  float bc_thr;
  int32_t bc_thr_idx;
  float bc_m;
  uint32_t bc_flag;
  double bc_z;
  // crossing search result (CTA-local broadcast)
  int32_t sel_b;
  int32_t sel_found;
  uint32_t sel_cnt;
  uint32_t sel_before_cnt;
  uint64_t sel_before_mass;
  uint64_t sel_z;
  // reductions
  float red_a[kWarps];
  float red_b[kWarps];
  int32_t red_i[kWarps];
  uint32_t red_u[kWarps];
  int32_t red_j[kWarps];
  double wmass[kWarps];
  uint64_t red_q[kWarps];
  int32_t misc_i;
  uint32_t mem_n;
  int32_t token;
};

struct Layout {
  size_t ctl, hist, bitmap, cand_s, cand_i, cand_e, perm, mem_s, mem_i, vals, total;
};

__host__ __device__ inline size_t align16(size_t x) { return (x + 15) & ~size_t(15); }

__host__ __device__ inline Layout make_layout(int W) {
  Layout L;
  size_t o = 0;
  L.ctl = o;    o = align16(o + sizeof(Ctl));
  L.hist = o;   o = align16(o + sizeof(uint64_t) * kBins);
  L.bitmap = o; o = align16(o + sizeof(uint32_t) * ((W + 31) / 32));
  L.cand_s = o; o = align16(o + sizeof(float) * kCap);
  L.cand_i = o; o = align16(o + sizeof(int32_t) * kCap);
  L.cand_e = o; o = align16(o + sizeof(float) * kCap);
  L.perm = o;   o = align16(o + sizeof(int32_t) * kCap);
  L.mem_s = o;  o = align16(o + sizeof(float) * kCap);
  L.mem_i = o;  o = align16(o + sizeof(int32_t) * kCap);
  L.vals = o;   o = align16(o + sizeof(float) * W);
  L.total = o;
  return L;
}

// ---------------------------------------------------------------- reductions
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ uint32_t warp_or(uint32_t v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v |= __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ int warp_imin(int v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ double warp_dsum(double v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ uint64_t warp_u64_sum(uint64_t v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
// (value, index) argmax with first-index tie break; NaN-free inputs.
__device__ __forceinline__ void warp_argmax(float& v, int& i) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, v, o);
    int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
  }
}
// inclusive scan over lanes (lane 0 first)
__device__ __forceinline__ uint64_t warp_incl_u64(uint64_t v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    uint64_t t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
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
__device__ __forceinline__ bool topp_crossed(uint64_t cum, uint64_t z, float p) {
  return (float)((double)cum / (double)z) > p;
}

// ---------------------------------------------------------------- per-row context
struct Row {
  const NsSampleArgs* a;
  int row, V, W, base, len, nf4, full4;
  int f_begin, f_end;
  uint32_t rank;
  const float* src32;
  const __nv_bfloat16* src16;
  bool tma, vec16;
  float T, rT;
  bool t_one, greedy, topp, pen;
  int k;
  float p;
  float rp;
  int64_t h0, h1;
};

__device__ __forceinline__ void set_status(const NsSampleArgs& a, uint32_t bits) {
  if (a.status) atomicOr(a.status, bits);
}

__device__ __forceinline__ float load_scalar(const Row& R, int local) {
  if (R.src16) return __bfloat162float(R.src16[R.base + local]);
  return R.src32[R.base + local];
}

// Logit after the repetition penalty for one element, from global memory
// (used for candidate re-computation and debug outputs).
__device__ __forceinline__ float penalized_from_global(const Row& R, const uint32_t* bitmap, int local) {
  float x = load_scalar(R, local);
  if (R.pen && ((bitmap[local >> 5] >> (local & 31)) & 1u)) x = penalize(x, R.rp);
  return x;
}
__device__ __forceinline__ float scaled(const Row& R, float x) {
  return R.t_one ? x : div_by_const(x, R.T, R.rT);
}

// Load float4 slot f (4 logits) of this CTA's slice with the penalty applied,
// store it to shared memory when it did not arrive there by bulk copy or was
// changed, and emit the penalized debug output.  Elements past the slice
// end read as -inf.
__device__ __forceinline__ float4 load_slot(const Row& R, float* vals, const uint32_t* bitmap, int f) {
  float4 v;
  const int e0 = f * 4;
  bool dirty = false;
  if (R.tma && f < R.full4) {
    v = reinterpret_cast<const float4*>(vals)[f];
  } else if (R.vec16 && e0 + 3 < R.len) {
    uint2 raw = *reinterpret_cast<const uint2*>(R.src16 + R.base + e0);
    __nv_bfloat162 lo = *reinterpret_cast<__nv_bfloat162*>(&raw.x);
    __nv_bfloat162 hi = *reinterpret_cast<__nv_bfloat162*>(&raw.y);
    float2 a = __bfloat1622float2(lo), b = __bfloat1622float2(hi);
    v = make_float4(a.x, a.y, b.x, b.y);
    dirty = true;
  } else {
    float t[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) t[c] = (e0 + c < R.len) ? load_scalar(R, e0 + c) : -INFINITY;
    v = make_float4(t[0], t[1], t[2], t[3]);
    dirty = true;
  }
  if (R.pen) {
    uint32_t nib = (bitmap[f >> 3] >> ((f & 7) << 2)) & 0xFu;
    if (nib) {
      if (nib & 1u) v.x = penalize(v.x, R.rp);
      if (nib & 2u) v.y = penalize(v.y, R.rp);
      if (nib & 4u) v.z = penalize(v.z, R.rp);
      if (nib & 8u) v.w = penalize(v.w, R.rp);
      dirty = true;
    }
  }
  if (dirty) reinterpret_cast<float4*>(vals)[f] = v;
  if (R.a->out_penalized) {
    float* o = R.a->out_penalized + (int64_t)R.row * R.V + R.base + e0;
    float t[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int c = 0; c < 4; ++c)
      if (e0 + c < R.len) o[c] = t[c];
  }
  return v;
}

// Wait for this warp's bulk copy (bounded; on give-up the status word is set
// and the kernel carries on so that no cluster barrier is left waiting).
__device__ __forceinline__ void wait_my_copy(const Row& R, Ctl& ctl, int warp) {
  if (!R.tma || R.f_begin >= min(R.f_end, R.full4)) return;
  uint32_t spins = 0;
  while (!mbar_try_wait(&ctl.mbar[warp], 0)) {
    if (++spins > (1u << 22)) {
      set_status(*R.a, NS_STATUS_WAIT_TIMEOUT);
      break;
    }
    if (spins > 64) __nanosleep(128);
  }
}

// Smallest float c <= b with RN(c/T) == RN(b/T): the lower end of the set of
// logits whose scaled value is at least RN(b/T).
__device__ float lower_preimage(const Row& R, float b) {
  if (R.t_one || !(b > -INFINITY) || !(b < INFINITY)) return b;
  float target = div_by_const(b, R.T, R.rT);
  float c = b;
  for (int i = 0; i < 64; ++i) {
    float d = nextafterf(c, -INFINITY);
    if (div_by_const(d, R.T, R.rT) == target) c = d; else return c;
  }
  return -INFINITY;
}

// ---------------------------------------------------------------- CTA-level helpers
// Block-wide exclusive scan of one u32 per thread (thread 0 first).
__device__ uint32_t block_excl_u32(Ctl& ctl, uint32_t v, uint32_t& total, int tid) {
  const int lane = tid & 31, warp = tid >> 5;
  uint32_t inc = warp_incl_u32(v, lane);
  if (lane == 31) ctl.red_u[warp] = inc;
  __syncthreads();
  uint32_t wpre = 0, tot = 0;
  for (int w = 0; w < kWarps; ++w) {
    uint32_t x = ctl.red_u[w];
    if (w < warp) wpre += x;
    tot += x;
  }
  __syncthreads();
  total = tot;
  return wpre + inc - v;
}

// Cluster-wide crossing search over the fine histogram `hist` (packed
// count<<40 | m24-sum, kBins buckets, bucket 0 = largest values).
//   count mode: first bucket whose inclusive count reaches `kneed`;
//   mass mode:  first bucket whose inclusive mass passes topp_crossed().
// Bucket b's elements share the biased exponent exps(b) (mass mode only).
// All CTAs compute the same answer from the peers' coarse sums and the fine
// buckets of the chosen coarse bucket.  Contains one cluster barrier; the
// caller must not overwrite `hist` or ctl.c*[buf] until after the next
// cluster barrier.
struct BucketExp {
  uint32_t top;  // key of bucket 0's top element
  int sh;        // log2 bucket width in keys
  __device__ __forceinline__ int exp_of(int b) const {
    uint32_t lo = top - (uint32_t)(b + 1) * (1u << sh) + 1u;
    return (int)(lo >> 23);
  }
};

__device__ void cluster_crossing(Ctl& ctl, const uint64_t* hist, int buf, bool mass_mode, uint32_t kneed,
                                 uint64_t base_mass, uint64_t zmass, float p, BucketExp be, bool mass_last_valid,
                                 int tid) {
  const int lane = tid & 31, warp = tid >> 5;
  // 1) own coarse sums: 16 threads per coarse bucket, 4 fine buckets each
  {
    const int c = tid >> 4;  // 0..31
    const int f0 = tid * 4;
    uint32_t cnt = 0;
    uint64_t ms = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int b = f0 + j;
      uint64_t h = hist[b];
      cnt += (uint32_t)(h >> 40);
      if (mass_mode && (mass_last_valid || b != kBins - 1)) ms += m24_to_fixed(h & kMassMask, be.exp_of(b));
    }
#pragma unroll
    for (int o = 8; o; o >>= 1) {
      cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
      ms += __shfl_xor_sync(0xffffffffu, ms, o);
    }
    if ((tid & 15) == 0) {
      ctl.ccnt[buf][c] = cnt;
      ctl.cmass[buf][c] = ms;
    }
  }
  cluster_sync();
  if (warp == 0) {
    // 2) pull every CTA's coarse sums (lane = coarse bucket)
    uint32_t cnt = 0;
    uint64_t ms = 0;
    const uint32_t acnt = smem_addr(&ctl.ccnt[buf][lane]);
    const uint32_t ams = smem_addr(&ctl.cmass[buf][lane]);
#pragma unroll
    for (int r = 0; r < kCluster; ++r) {
      cnt += dsmem_ld_u32(dsmem_map(acnt, r));
      ms += dsmem_ld_u64(dsmem_map(ams, r));
    }
    uint32_t icnt = warp_incl_u32(cnt, lane);
    uint64_t ims = warp_incl_u64(ms, lane);
    uint64_t z = zmass;
    if (z == 0ull) z = __shfl_sync(0xffffffffu, ims, 31);
    bool hit = mass_mode ? (ms > 0 && topp_crossed(base_mass + ims, z, p)) : (icnt >= kneed);
    uint32_t bal = __ballot_sync(0xffffffffu, hit);
    int found = bal != 0u;
    int cb = found ? __ffs(bal) - 1 : 0;
    uint32_t before_cnt = __shfl_sync(0xffffffffu, icnt - cnt, cb);
    uint64_t before_ms = __shfl_sync(0xffffffffu, ims - ms, cb);
    int b_sel = 0;
    uint32_t b_cnt = 0, b_before_cnt = 0;
    uint64_t b_before_ms = 0;
    if (found) {
      // 3) pull the fine buckets of coarse bucket cb (2 per lane)
      uint32_t fc[2];
      uint64_t fm[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int b = cb * kFinePerCoarse + h * 32 + lane;
        const uint32_t ah = smem_addr(&hist[b]);
        uint32_t c2 = 0;
        uint64_t m2 = 0;
#pragma unroll
        for (int r = 0; r < kCluster; ++r) {
          uint64_t x = dsmem_ld_u64(dsmem_map(ah, r));
          c2 += (uint32_t)(x >> 40);
          m2 += x & kMassMask;
        }
        fc[h] = c2;
        fm[h] = (mass_mode && (mass_last_valid || b != kBins - 1)) ? m24_to_fixed(m2, be.exp_of(b)) : 0ull;
      }
      uint32_t run_c = before_cnt;
      uint64_t run_m = before_ms;
      bool done = false;
#pragma unroll
      for (int h = 0; h < 2 && !done; ++h) {
        uint32_t ic = warp_incl_u32(fc[h], lane);
        uint64_t im = warp_incl_u64(fm[h], lane);
        bool hit2 = mass_mode ? (fm[h] > 0 && topp_crossed(base_mass + run_m + im, z, p)) : (run_c + ic >= kneed);
        uint32_t bal2 = __ballot_sync(0xffffffffu, hit2);
        if (bal2) {
          int l = __ffs(bal2) - 1;
          b_sel = cb * kFinePerCoarse + h * 32 + l;
          b_cnt = __shfl_sync(0xffffffffu, fc[h], l);
          b_before_cnt = run_c + __shfl_sync(0xffffffffu, ic - fc[h], l);
          b_before_ms = run_m + __shfl_sync(0xffffffffu, im - fm[h], l);
          done = true;
        } else {
          run_c += __shfl_sync(0xffffffffu, ic, 31);
          run_m += __shfl_sync(0xffffffffu, im, 31);
        }
      }
      if (!done) found = 0;  // only possible through rounding at the coarse level
    }
    if (lane == 0) {
      ctl.sel_found = found;
      ctl.sel_b = b_sel;
      ctl.sel_cnt = b_cnt;
      ctl.sel_before_cnt = b_before_cnt;
      ctl.sel_before_mass = b_before_ms;
      ctl.sel_z = z;
    }
  }
  __syncthreads();
}

// Rank-by-counting sort of the leader's n candidates: perm[rank] = i with
// order (s descending, index ascending).  n <= kCap.
__device__ void leader_sort(int n, const float* cs, const int32_t* ci, int32_t* perm, int tid) {
  for (int i = tid; i < n; i += kThreads) {
    const float si = cs[i];
    const int ii = ci[i];
    int r = 0;
    for (int j = 0; j < n; ++j) {
      const float sj = cs[j];
      r += (sj > si) || (sj == si && ci[j] < ii);
    }
    perm[r] = i;
  }
  __syncthreads();
}

// ---------------------------------------------------------------- the kernel
__global__ void __launch_bounds__(kThreads, 2) sample_kernel(const NsSampleArgs a, int W, int tma_ok, int vec16_ok) {
  extern __shared__ __align__(128) unsigned char smem[];
  const Layout L = make_layout(W);
  Ctl& ctl = *reinterpret_cast<Ctl*>(smem + L.ctl);
  uint64_t* hist = reinterpret_cast<uint64_t*>(smem + L.hist);
  uint32_t* bitmap = reinterpret_cast<uint32_t*>(smem + L.bitmap);
  float* cand_s = reinterpret_cast<float*>(smem + L.cand_s);
  int32_t* cand_i = reinterpret_cast<int32_t*>(smem + L.cand_i);
  float* cand_e = reinterpret_cast<float*>(smem + L.cand_e);
  int32_t* perm = reinterpret_cast<int32_t*>(smem + L.perm);
  float* mem_s = reinterpret_cast<float*>(smem + L.mem_s);
  int32_t* mem_i = reinterpret_cast<int32_t*>(smem + L.mem_i);
  float* vals = reinterpret_cast<float*>(smem + L.vals);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  Row R;
  R.a = &a;
  R.rank = cluster_ctarank();
  R.row = blockIdx.x / kCluster;
  R.V = a.vocab_size;
  R.W = W;
  R.base = (int)R.rank * W;
  R.len = max(0, min(W, R.V - R.base));
  R.nf4 = (R.len + 3) >> 2;
  R.full4 = R.len >> 2;
  {
    const int chunk = (R.nf4 + kWarps - 1) / kWarps;
    R.f_begin = min(R.nf4, warp * chunk);
    R.f_end = min(R.nf4, R.f_begin + chunk);
  }
  const bool leader = (R.rank == 0);

  // source row (fused gather of sample_indices)
  int64_t src = R.row;
  bool bad_row = false;
  if (a.sample_indices) {
    src = a.sample_indices[R.row];
    if (src < 0 || src >= a.num_logit_rows) { bad_row = true; src = 0; }
  } else if (src >= a.num_logit_rows) {
    bad_row = true;
    src = 0;
  }
  if (a.logits_dtype == NS_DTYPE_BF16) {
    R.src16 = reinterpret_cast<const __nv_bfloat16*>(a.logits) + src * a.logits_row_stride;
    R.src32 = nullptr;
  } else {
    R.src32 = reinterpret_cast<const float*>(a.logits) + src * a.logits_row_stride;
    R.src16 = nullptr;
  }
  R.tma = tma_ok && R.src32 != nullptr;
  R.vec16 = vec16_ok && R.src16 != nullptr;

  const NsRowParams P = a.row_params[R.row];
  R.greedy = (P.flags & NS_ROW_GREEDY) != 0u;
  R.T = R.greedy ? 1.0f : P.temperature;
  R.rT = __frcp_rn(R.T);
  R.t_one = (R.T == 1.0f);
  R.topp = (P.flags & NS_ROW_TOP_P) != 0u;
  R.p = P.top_p;
  R.k = (P.top_k > 0 && P.top_k < R.V) ? P.top_k : 0;
  R.rp = P.repetition_penalty;
  R.h0 = R.h1 = 0;
  if (a.history_offsets && (P.flags & NS_ROW_PENALTY)) {
    R.h0 = a.history_offsets[R.row];
    R.h1 = a.history_offsets[R.row + 1];
  }
  R.pen = (P.flags & NS_ROW_PENALTY) != 0u && R.h1 > R.h0;
  const bool debug = (a.out_filtered != nullptr) || (a.out_probs != nullptr);

  enum { kGreedy, kTopk, kGeneral };
  int mode = (R.greedy && !debug) ? kGreedy : (R.k > 0 && R.k <= kTopkSmall) ? kTopk : kGeneral;

  // ---------------- setup: barriers, zeroed histograms, penalty bitmap
  if (tid == 0) {
    for (int w = 0; w < kWarps; ++w) mbar_init(&ctl.mbar[w], 1);
    fence_mbar_init();
    ctl.cand_n = 0u;
    ctl.mem_n = 0u;
    ctl.bc_flag = 0u;
  }
  for (int i = tid; i < kBins; i += kThreads) hist[i] = 0ull;
  if (R.pen)
    for (int i = tid; i < (W + 31) / 32; i += kThreads) bitmap[i] = 0u;
  __syncthreads();
  cluster_arrive();  // barrier 0: every CTA's shared memory is initialised

  // each warp fetches its own piece of the slice
  if (R.tma && lane == 0) {
    const int fe = min(R.f_end, R.full4);
    if (fe > R.f_begin) {
      const uint32_t bytes = (uint32_t)(fe - R.f_begin) * 16u;
      mbar_arrive_expect_tx(&ctl.mbar[warp], bytes);
      bulk_g2s(vals + 4 * R.f_begin, R.src32 + R.base + 4 * R.f_begin, bytes, &ctl.mbar[warp]);
    }
  }
  if (R.pen) {
    uint32_t bad = 0;
    for (int64_t i = R.h0 + tid; i < R.h1; i += kThreads) {
      const int id = a.history_ids[i];
      if (id < 0 || id >= R.V) { bad = 1; continue; }
      const int local = id - R.base;
      if (local >= 0 && local < R.len) atomicOr(&bitmap[local >> 5], 1u << (local & 31));
    }
    if (bad && R.rank == 0) set_status(a, NS_STATUS_BAD_HISTORY_ID);
    __syncthreads();
  }
  if (bad_row && leader && tid == 0) set_status(a, NS_STATUS_BAD_SAMPLE_INDEX);

  wait_my_copy(R, ctl, warp);

  // row uniform
  double u;
  if (a.uniforms) {
    u = (double)a.uniforms[R.row];
  } else {
    const uint64_t key = (P.flags & NS_ROW_SEED) ? P.seed : a.philox_seed;
    u = philox_uniform(key, a.philox_offset, (uint64_t)(a.row_offset + R.row));
  }
  if (!(u >= 0.0)) u = 0.0;
  if (u >= 1.0) u = 0x1.fffffffffffffp-1;

  float4* vals4 = reinterpret_cast<float4*>(vals);
  const int64_t out_row_off = (int64_t)R.row * R.V;

  // ---------------- pass 1 (mode-specific statistics)
  float st_max = -INFINITY, st_minf = INFINITY, nfacc = 0.0f;
  int st_amax = INT_MAX;
  if (mode == kGreedy || mode == kGeneral) {
    for (int f = R.f_begin + lane; f < R.f_end; f += 32) {
      float4 v = load_slot(R, vals, bitmap, f);
      float m4 = fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w));
      nfacc = __fmaf_rn(__fadd_rn(__fadd_rn(v.x, v.y), __fadd_rn(v.z, v.w)), 0.0f, nfacc);
      if (m4 > st_max) {
        st_max = m4;
        const int c = (v.x == m4) ? 0 : (v.y == m4) ? 1 : (v.z == m4) ? 2 : 3;
        st_amax = R.base + 4 * f + c;
      }
      if (mode == kGeneral) {
        float a0 = v.x > -INFINITY ? v.x : INFINITY;
        float a1 = v.y > -INFINITY ? v.y : INFINITY;
        float a2 = v.z > -INFINITY ? v.z : INFINITY;
        float a3 = v.w > -INFINITY ? v.w : INFINITY;
        st_minf = fminf(st_minf, fminf(fminf(a0, a1), fminf(a2, a3)));
      }
    }
  } else {  // kTopk: per-thread maxima (with the argmax for greedy rows)
    for (int f = R.f_begin + lane; f < R.f_end; f += 32) {
      float4 v = load_slot(R, vals, bitmap, f);
      float m4 = fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w));
      nfacc = __fmaf_rn(__fadd_rn(__fadd_rn(v.x, v.y), __fadd_rn(v.z, v.w)), 0.0f, nfacc);
      if (m4 > st_max) {
        st_max = m4;
        const int c = (v.x == m4) ? 0 : (v.y == m4) ? 1 : (v.z == m4) ? 2 : 3;
        st_amax = R.base + 4 * f + c;
      }
    }
    // local histogram of thread maxima (u16 counts packed in u32 words)
    uint32_t* tm_local = reinterpret_cast<uint32_t*>(hist);
    const uint32_t b = f2key(st_max) >> 20;
    atomicAdd(&tm_local[b >> 1], 1u << ((b & 1u) << 4));
  }
  uint32_t my_flags = (nfacc == nfacc) ? 0u : kFlagNonFinite;

  // CTA reduction of (max, argmax, minf, flags)
  {
    float vmax = st_max;
    int vi = st_amax;
    warp_argmax(vmax, vi);
    float vminf = warp_min(st_minf);
    uint32_t fl = warp_or(my_flags);
    if (lane == 0) {
      ctl.red_a[warp] = vmax;
      ctl.red_i[warp] = vi;
      ctl.red_b[warp] = vminf;
      ctl.red_u[warp] = fl;
    }
    __syncthreads();
    if (tid == 0) {
      float m = -INFINITY, mf = INFINITY;
      int mi = INT_MAX;
      uint32_t f = 0;
      for (int w = 0; w < kWarps; ++w) {
        float x = ctl.red_a[w];
        int xi = ctl.red_i[w];
        if (x > m || (x == m && xi < mi)) { m = x; mi = xi; }
        mf = fminf(mf, ctl.red_b[w]);
        f |= ctl.red_u[w];
      }
      ctl.red_a[0] = m;
      ctl.red_i[0] = mi;
      ctl.red_b[0] = mf;
      ctl.red_u[0] = f;
    }
    __syncthreads();
  }
  const float cta_max = ctl.red_a[0];
  const int cta_amax = ctl.red_i[0];
  const float cta_minf = ctl.red_b[0];
  const uint32_t cta_flags = ctl.red_u[0];
  __syncthreads();

  cluster_wait();  // barrier 0 complete: peers may now be written

  // push this CTA's record to every CTA; TOPK also pushes its maxima histogram
  if (tid < kCluster) {
    const uint32_t r = (uint32_t)tid;
    dsmem_st_f32(dsmem_map(smem_addr(&ctl.rec_max[R.rank]), r), cta_max);
    dsmem_st_f32(dsmem_map(smem_addr(&ctl.rec_minf[R.rank]), r), cta_minf);
    dsmem_st_u32(dsmem_map(smem_addr(&ctl.rec_flags[R.rank]), r), cta_flags);
    dsmem_st_u32(dsmem_map(smem_addr(&ctl.rec_amax[R.rank]), r), (uint32_t)cta_amax);
  }
  if (mode == kTopk) {
    const uint32_t* tm_local = reinterpret_cast<const uint32_t*>(hist);
    uint32_t* tm_global = reinterpret_cast<uint32_t*>(hist) + kTmBins / 2;
    for (int w = tid; w < kTmBins / 2; w += kThreads) {
      const uint32_t v = tm_local[w];
      if (v) {
        const uint32_t ad = smem_addr(&tm_global[w]);
#pragma unroll
        for (int r = 0; r < kCluster; ++r) dsmem_red_add_u32(dsmem_map(ad, r), v);
      }
    }
  }
  cluster_sync();  // barrier 1: records (and maxima histograms) delivered

  // ---------------- non-finite rows: classify on a rescan
  uint32_t any_nf = 0;
  float gmax = -INFINITY, gminf = INFINITY;
  int gamax = INT_MAX;
  for (int r = 0; r < kCluster; ++r) {
    any_nf |= ctl.rec_flags[r];
    const float x = ctl.rec_max[r];
    if (x > gmax) { gmax = x; gamax = ctl.rec_amax[r]; }
    gminf = fminf(gminf, ctl.rec_minf[r]);
  }
  if (gmax == -INFINITY) gamax = 0;  // all -inf (or empty): torch.argmax -> 0

  if (any_nf) {
    int my_nan = INT_MAX, my_pinf = INT_MAX;
    for (int f = R.f_begin + lane; f < R.f_end; f += 32) {
      const float4 v = vals4[f];
      const float t[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int idx = R.base + 4 * f + c;
        if (4 * f + c < R.len) {
          if (t[c] != t[c]) my_nan = min(my_nan, idx);
          if (t[c] == INFINITY) my_pinf = min(my_pinf, idx);
        }
      }
    }
    my_nan = warp_imin(my_nan);
    my_pinf = warp_imin(my_pinf);
    if (lane == 0) { ctl.red_i[warp] = my_nan; ctl.red_j[warp] = my_pinf; }
    __syncthreads();
    if (tid < kCluster) {
      int n = INT_MAX, q = INT_MAX;
      for (int w = 0; w < kWarps; ++w) { n = min(n, ctl.red_i[w]); q = min(q, ctl.red_j[w]); }
      dsmem_st_u32(dsmem_map(smem_addr(&ctl.rec_nan[R.rank]), tid), (uint32_t)n);
      dsmem_st_u32(dsmem_map(smem_addr(&ctl.rec_pinf[R.rank]), tid), (uint32_t)q);
    }
    cluster_sync();
    int gnan = INT_MAX, gpinf = INT_MAX;
    for (int r = 0; r < kCluster; ++r) {
      gnan = min(gnan, ctl.rec_nan[r]);
      gpinf = min(gpinf, ctl.rec_pinf[r]);
    }
    if (gnan != INT_MAX || gpinf != INT_MAX || gmax == -INFINITY) {
      // softmax of this row is NaN -> uniform 1/V (sampler.py:76-80)
      if (leader && tid == 0) {
        int tok;
        if (R.greedy) tok = (gnan != INT_MAX) ? gnan : (gpinf != INT_MAX) ? gpinf : 0;
        else tok = min(R.V - 1, (int)(u * (double)R.V));
        if (a.out_dtype == NS_OUT_I32) reinterpret_cast<int32_t*>(a.out_tokens)[R.row] = tok;
        else reinterpret_cast<int64_t*>(a.out_tokens)[R.row] = tok;
      }
      if (debug) {
        const float pu = 1.0f / (float)R.V;
        for (int i = tid; i < R.len; i += kThreads) {
          if (a.out_probs) a.out_probs[out_row_off + R.base + i] = pu;
          if (a.out_filtered) a.out_filtered[out_row_off + R.base + i] = scaled(R, vals[i]);
        }
      }
      return;
    }
    // only -inf entries: a regular row
  }

  // ================================================================ GREEDY
  if (mode == kGreedy) {
    if (leader && tid == 0) {
      if (a.out_dtype == NS_OUT_I32) reinterpret_cast<int32_t*>(a.out_tokens)[R.row] = gamax;
      else reinterpret_cast<int64_t*>(a.out_tokens)[R.row] = gamax;
    }
    return;
  }

  const uint32_t cand_n_addr0 = dsmem_map(smem_addr(&ctl.cand_n), 0);

  // ================================================================ TOPK
  if (mode == kTopk) {
    // bound: lowest key of the bucket holding the k-th largest thread maximum
    const uint32_t* tm_global = reinterpret_cast<const uint32_t*>(hist) + kTmBins / 2;
    {
      // thread t owns buckets [kTmBins-8(t+1), kTmBins-8t), scanned from the top
      uint32_t cnt[8];
      uint32_t s = 0;
      const int bhi = kTmBins - 1 - 8 * tid;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int b = bhi - j;
        cnt[j] = (tm_global[b >> 1] >> ((b & 1) << 4)) & 0xFFFFu;
        s += cnt[j];
      }
      uint32_t tot;
      uint32_t pre = block_excl_u32(ctl, s, tot, tid);
      if (pre < (uint32_t)R.k && pre + s >= (uint32_t)R.k) {
        uint32_t run = pre;
        for (int j = 0; j < 8; ++j) {
          run += cnt[j];
          if (run >= (uint32_t)R.k) { ctl.misc_i = bhi - j; break; }
        }
      }
      if (tot < (uint32_t)R.k && tid == 0) ctl.misc_i = 0;
      __syncthreads();
    }
    const uint32_t bkey = (uint32_t)ctl.misc_i << 20;
    float bound = (bkey < 0x00800000u) ? -INFINITY : key2f(bkey);
    bound = lower_preimage(R, bound);

    // send every element >= bound to the leader (warp-aggregated slots)
    for (int f = R.f_begin + lane; f - lane < R.f_end; f += 32) {
      float4 v = (f < R.f_end) ? vals4[f] : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      const float t[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const bool take = (f < R.f_end) && (4 * f + c < R.len) && (t[c] >= bound);
        const uint32_t bal = __ballot_sync(0xffffffffu, take);
        if (bal) {
          uint32_t slot0 = 0;
          const int first = __ffs(bal) - 1;
          if (lane == first) slot0 = dsmem_atom_add_u32(cand_n_addr0, (uint32_t)__popc(bal));
          slot0 = __shfl_sync(0xffffffffu, slot0, first);
          if (take) {
            const uint32_t slot = slot0 + (uint32_t)__popc(bal & ((1u << lane) - 1u));
            if (slot < (uint32_t)kCap) {
              dsmem_st_f32(dsmem_map(smem_addr(&cand_s[slot]), 0), scaled(R, t[c]));
              dsmem_st_u32(dsmem_map(smem_addr(&cand_i[slot]), 0), (uint32_t)(R.base + 4 * f + c));
            }
          }
        }
      }
    }
    cluster_sync();  // barrier 2: candidates delivered
    const uint32_t ncand = dsmem_ld_u32(cand_n_addr0);
    cluster_arrive();  // barrier 3 (arrive): nobody needs the leader's counter afterwards
    if (ncand <= (uint32_t)kCap) {
      if (leader) {
        const int n = (int)ncand;
        leader_sort(n, cand_s, cand_i, perm, tid);
        // top-k threshold and survivors (ties at the threshold are kept)
        const float s0 = cand_s[perm[0]];
        const int kk = min(R.k, n);
        const float thr = cand_s[perm[kk - 1]];
        if (tid == 0) ctl.misc_i = n;
        __syncthreads();
        for (int r = tid; r < n; r += kThreads) {
          const bool in = cand_s[perm[r]] >= thr;
          const bool nxt = (r + 1 < n) && (cand_s[perm[r + 1]] >= thr);
          if (in && !nxt) ctl.misc_i = r + 1;
        }
        __syncthreads();
        const int n1 = ctl.misc_i;
        for (int r = tid; r < n1; r += kThreads) cand_e[r] = exp_shifted(cand_s[perm[r]], s0);  // e by rank
        __syncthreads();
        int n2 = n1;
        if (R.topp) {
          if (warp == 0) {
            uint64_t z = 0;
            for (int c0 = 0; c0 < n1; c0 += 32) {
              const int r = c0 + lane;
              z += warp_u64_sum(r < n1 ? f2fixed(cand_e[r]) : 0ull);
            }
            uint64_t run = 0;
            int j0 = -1;
            for (int c0 = 0; c0 < n1 && j0 < 0; c0 += 32) {
              const int r = c0 + lane;
              const uint64_t fx = r < n1 ? f2fixed(cand_e[r]) : 0ull;
              const uint64_t inc = warp_incl_u64(fx, lane) + run;
              const uint32_t bal = __ballot_sync(0xffffffffu, r < n1 && topp_crossed(inc, z, R.p));
              if (bal) j0 = c0 + __ffs(bal) - 1;
              run = __shfl_sync(0xffffffffu, inc, 31);
            }
            // keep exactly ranks 0..j0 in (value desc, index asc) order
            if (lane == 0) ctl.misc_i = (j0 >= 0) ? j0 + 1 : n1;
          }
          __syncthreads();
          n2 = ctl.misc_i;
        }
        // total kept mass and the inverse-CDF draw in vocabulary order
        if (warp == 0) {
          uint64_t z = 0;
          for (int c0 = 0; c0 < n2; c0 += 32) {
            const int r = c0 + lane;
            z += warp_u64_sum(r < n2 ? f2fixed(cand_e[r]) : 0ull);
          }
          if (lane == 0) { ctl.sel_z = z; ctl.token = -1; }
        }
        __syncthreads();
        const uint64_t z2 = ctl.sel_z;
        const double target = u * (double)z2;
        for (int r = tid; r < n2; r += kThreads) {
          const int ir = cand_i[perm[r]];
          const uint64_t fr = f2fixed(cand_e[r]);
          uint64_t before = 0;
          for (int q = 0; q < n2; ++q)
            if (cand_i[perm[q]] < ir) before += f2fixed(cand_e[q]);
          if (fr > 0 && (double)before <= target && target < (double)(before + fr)) ctl.token = ir;
        }
        __syncthreads();
        if (tid == 0) {
          int tok = ctl.token;
          if (tok < 0) {
            // target at the very top (rounding): last kept element with mass
            int last = -1;
            for (int r = 0; r < n2; ++r)
              if (f2fixed(cand_e[r]) > 0 && cand_i[perm[r]] > last) last = cand_i[perm[r]];
            tok = last >= 0 ? last : cand_i[perm[0]];
          }
          if (R.greedy) tok = cand_i[perm[0]];
          if (a.out_dtype == NS_OUT_I32) reinterpret_cast<int32_t*>(a.out_tokens)[R.row] = tok;
          else reinterpret_cast<int64_t*>(a.out_tokens)[R.row] = tok;
          if (debug) {
            const float thr2 = cand_s[perm[n2 - 1]];
            const int thr_idx = cand_i[perm[n2 - 1]];
            for (int r = 0; r < kCluster; ++r) {
              dsmem_st_f32(dsmem_map(smem_addr(&ctl.bc_thr), r), thr2);
              dsmem_st_u32(dsmem_map(smem_addr(&ctl.bc_thr_idx), r), (uint32_t)thr_idx);
              dsmem_st_f32(dsmem_map(smem_addr(&ctl.bc_m), r), s0);
              dsmem_st_f64(dsmem_map(smem_addr(&ctl.bc_z), r), (double)z2 * kFixedToReal);
            }
          }
        }
      }
      cluster_wait();  // barrier 3
      if (debug) {
        cluster_sync();  // barrier 4: leader's broadcast delivered
        const float thr2 = ctl.bc_thr, m = ctl.bc_m;
        const int thr_idx = ctl.bc_thr_idx;
        const double z = ctl.bc_z;
        for (int i = tid; i < R.len; i += kThreads) {
          const float s = scaled(R, vals[i]);
          const bool kept = s > thr2 || (s == thr2 && R.base + i <= thr_idx);
          if (a.out_filtered) a.out_filtered[out_row_off + R.base + i] = kept ? s : -INFINITY;
          if (a.out_probs) a.out_probs[out_row_off + R.base + i] = kept ? (float)((double)exp_shifted(s, m) / z) : 0.0f;
        }
      }
      return;
    }
    // candidate list overflowed: fall back to the general path for this row
    cluster_wait();  // barrier 3
    if (leader && tid == 0) set_status(a, NS_STATUS_CAP_OVERFLOW);
    mode = kGeneral;
    // the general path needs min-finite; recompute it from the slice
    float mf = INFINITY;
    for (int f = R.f_begin + lane; f < R.f_end; f += 32) {
      const float4 v = vals4[f];
      float a0 = v.x > -INFINITY ? v.x : INFINITY, a1 = v.y > -INFINITY ? v.y : INFINITY;
      float a2 = v.z > -INFINITY ? v.z : INFINITY, a3 = v.w > -INFINITY ? v.w : INFINITY;
      mf = fminf(mf, fminf(fminf(a0, a1), fminf(a2, a3)));
    }
    mf = warp_min(mf);
    if (lane == 0) ctl.red_b[warp] = mf;
    __syncthreads();
    if (tid < kCluster) {
      float m2 = INFINITY;
      for (int w = 0; w < kWarps; ++w) m2 = fminf(m2, ctl.red_b[w]);
      dsmem_st_f32(dsmem_map(smem_addr(&ctl.rec_minf[R.rank]), tid), m2);
    }
    cluster_sync();
    gminf = INFINITY;
    for (int r = 0; r < kCluster; ++r) gminf = fminf(gminf, ctl.rec_minf[r]);
    if (tid == 0) ctl.cand_n = 0u;
    __syncthreads();
    cluster_sync();  // counter reset visible before reuse
  }

  // ================================================================ GENERAL
  const float m = R.t_one ? gmax : __fdiv_rn(gmax, R.T);            // max scaled logit
  const float minf_s = (gminf < INFINITY) ? (R.t_one ? gminf : __fdiv_rn(gminf, R.T)) : m;
  int hbuf = 0;  // histogram double-buffer index (for the coarse arrays)

  // ---- large top-k: exact radix select of the k-th largest penalized logit
  bool have_thr_k = false;
  float thr_k_s = -INFINITY;
  if (R.k > 0) {
    uint32_t prefix = 0, krem = (uint32_t)R.k;
    const int shifts[3] = {21, 10, 0};
    const int widths[3] = {11, 11, 10};
    bool ok = true;
    for (int lvl = 0; lvl < 3; ++lvl) {
      const int sh = shifts[lvl], wd = widths[lvl];
      const uint32_t nbm = (1u << wd) - 1u;
      for (int i = tid; i < kBins; i += kThreads) hist[i] = 0ull;
      __syncthreads();
      for (int f = R.f_begin + lane; f < R.f_end; f += 32) {
        const float4 v = vals4[f];
        const float t[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if (4 * f + c >= R.len) continue;
          const uint32_t key = f2key(t[c]);
          if (lvl > 0 && (key >> (sh + wd)) != prefix) continue;
          const uint32_t b = nbm - ((key >> sh) & nbm);
          atomicAdd(reinterpret_cast<unsigned long long*>(&hist[b]), (unsigned long long)kCountOne);
        }
      }
      __syncthreads();
      BucketExp be{0u, 0};
      cluster_crossing(ctl, hist, hbuf, false, krem, 0ull, 0ull, 0.0f, be, true, tid);
      hbuf ^= 1;
      if (!ctl.sel_found) { ok = false; break; }
      krem -= ctl.sel_before_cnt;
      prefix = (prefix << wd) | (nbm - (uint32_t)ctl.sel_b);
      cluster_sync();  // peers done reading this level's histogram
    }
    if (ok) {
      have_thr_k = true;
      thr_k_s = scaled(R, key2f(prefix));
    }
  }

  // ---- pass 2: e = exp(s - m) in place; top-p mass histogram or draw masses
  float e_lo_src = have_thr_k ? fmaxf(minf_s, thr_k_s) : minf_s;
  const float e_lo = exp_shifted(e_lo_src, m);
  int SH = 0;
  {
    const uint32_t D = (e_lo > 0.0f) ? (kOne - __float_as_uint(e_lo)) : kOne;
    while (SH < 18 && (int64_t)(((D + (1u << SH) - 1u) >> SH)) + 1 > kBins - 2) ++SH;
  }
  uint32_t KC = kOne - 1u + (1u << SH);
  if (R.topp) {
    for (int i = tid; i < kBins; i += kThreads) hist[i] = 0ull;
    __syncthreads();
  }
  float lane_mass = 0.0f;
  for (int f = R.f_begin + lane; f < R.f_end; f += 32) {
    const float4 v = vals4[f];
    float t[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float e = 0.0f;
      if (4 * f + c < R.len) {
        const float s = scaled(R, t[c]);
        if (!have_thr_k || s >= thr_k_s) e = exp_shifted(s, m);
      }
      t[c] = e;
      if (R.topp) {
        if (e > 0.0f) {
          const uint32_t bits = __float_as_uint(e);
          const uint32_t b = min((uint32_t)(kBins - 1), (KC - bits) >> SH);
          atomicAdd(reinterpret_cast<unsigned long long*>(&hist[b]),
                    (unsigned long long)(kCountOne | (uint64_t)((bits & 0x7fffffu) | 0x800000u)));
        }
      } else {
        lane_mass = __fadd_rn(lane_mass, e);
      }
    }
    vals4[f] = make_float4(t[0], t[1], t[2], t[3]);
  }
  __syncthreads();

  // ---- top-p: find the crossing bucket, refine, collect, decide
  float keep_lo = 0.0f;  // kept <=> e >= keep_lo && e > 0
  if (R.topp) {
    BucketExp be{KC, SH};
    uint32_t lo_key = 0, hi_key = 0;
    uint64_t before = 0, z = 0;
    bool crossed = false;
    int lvl = 0;
    int sh_cur = SH;
    uint32_t top_cur = KC;
    for (;;) {
      cluster_crossing(ctl, hist, hbuf, true, 0u, before, z, R.p, be, lvl > 0, tid);
      hbuf ^= 1;
      if (lvl == 0) z = ctl.sel_z;
      if (!ctl.sel_found) break;
      const int B = ctl.sel_b;
      before += ctl.sel_before_mass;
      lo_key = top_cur - (uint32_t)(B + 1) * (1u << sh_cur) + 1u;
      hi_key = top_cur - (uint32_t)B * (1u << sh_cur);
      crossed = true;
      const uint32_t cnt = ctl.sel_cnt;
      if (cnt <= (uint32_t)kCap || sh_cur == 0 || lvl >= 3) break;
      // refine inside [lo_key, hi_key]
      cluster_sync();  // peers done reading this level's histogram
      const int sh_next = max(0, sh_cur - 11);
      for (int i = tid; i < kBins; i += kThreads) hist[i] = 0ull;
      __syncthreads();
      for (int f = R.f_begin + lane; f < R.f_end; f += 32) {
        const float4 v = vals4[f];
        const float t[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t bits = __float_as_uint(t[c]);
          if (t[c] > 0.0f && bits >= lo_key && bits <= hi_key) {
            const uint32_t b = (hi_key - bits) >> sh_next;
            atomicAdd(reinterpret_cast<unsigned long long*>(&hist[b]),
                      (unsigned long long)(kCountOne | (uint64_t)((bits & 0x7fffffu) | 0x800000u)));
          }
        }
      }
      __syncthreads();
      sh_cur = sh_next;
      top_cur = hi_key;
      be = BucketExp{hi_key, sh_next};
      ++lvl;
    }
    if (!crossed) {
      keep_lo = 0.0f;  // the mass never passes top_p: keep everything
      cluster_sync();
    } else {
      cluster_sync();  // peers done reading the last histogram; leader counter is zero
      const uint32_t total_cnt = ctl.sel_cnt;
      const bool collect = total_cnt <= (uint32_t)kCap;
      if (collect) {
        // members of the crossing bucket -> leader (exact s recomputed from global)
        for (int f = R.f_begin + lane; f - lane < R.f_end; f += 32) {
          const float4 v = (f < R.f_end) ? vals4[f] : make_float4(0.f, 0.f, 0.f, 0.f);
          const float t[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint32_t bits = __float_as_uint(t[c]);
            const bool take = (f < R.f_end) && t[c] > 0.0f && bits >= lo_key && bits <= hi_key;
            const uint32_t bal = __ballot_sync(0xffffffffu, take);
            if (bal) {
              uint32_t slot0 = 0;
              const int first = __ffs(bal) - 1;
              if (lane == first) slot0 = dsmem_atom_add_u32(cand_n_addr0, (uint32_t)__popc(bal));
              slot0 = __shfl_sync(0xffffffffu, slot0, first);
              if (take) {
                const uint32_t slot = slot0 + (uint32_t)__popc(bal & ((1u << lane) - 1u));
                const int local = 4 * f + c;
                const float s = scaled(R, penalized_from_global(R, bitmap, local));
                if (slot < (uint32_t)kCap) {
                  dsmem_st_f32(dsmem_map(smem_addr(&cand_s[slot]), 0), s);
                  dsmem_st_u32(dsmem_map(smem_addr(&cand_i[slot]), 0), (uint32_t)(R.base + local));
                  dsmem_st_f32(dsmem_map(smem_addr(&cand_e[slot]), 0), t[c]);
                }
                const uint32_t ms = atomicAdd(&ctl.mem_n, 1u);
                if (ms < (uint32_t)kCap) { mem_s[ms] = s; mem_i[ms] = local; }
              }
            }
          }
        }
      }
      cluster_sync();  // barrier: members delivered
      if (leader && collect) {
        const int n = (int)min(ctl.cand_n, (uint32_t)kCap);
        leader_sort(n, cand_s, cand_i, perm, tid);
        if (warp == 0) {
          uint64_t run = before;
          int j0 = -1;
          for (int c0 = 0; c0 < n && j0 < 0; c0 += 32) {
            const int r = c0 + lane;
            const uint64_t fx = r < n ? f2fixed(cand_e[perm[r]]) : 0ull;
            const uint64_t inc = warp_incl_u64(fx, lane) + run;
            const uint32_t bal = __ballot_sync(0xffffffffu, r < n && fx > 0 && topp_crossed(inc, z, R.p));
            if (bal) j0 = c0 + __ffs(bal) - 1;
            run = __shfl_sync(0xffffffffu, inc, 31);
          }
          if (lane == 0) {
            // rank j0 in (value desc, index asc) order is the last one kept
            const float thr = (j0 >= 0) ? cand_s[perm[j0]] : -INFINITY;
            const int thr_idx = (j0 >= 0) ? cand_i[perm[j0]] : INT_MAX;
            for (int r = 0; r < kCluster; ++r) {
              dsmem_st_f32(dsmem_map(smem_addr(&ctl.bc_thr), r), thr);
              dsmem_st_u32(dsmem_map(smem_addr(&ctl.bc_thr_idx), r), (uint32_t)thr_idx);
              dsmem_st_u32(dsmem_map(smem_addr(&ctl.bc_flag), r), 1u);
            }
          }
        }
      }
      if (!collect && leader && tid == 0) set_status(a, NS_STATUS_CAP_OVERFLOW);
      cluster_sync();  // barrier: decision delivered
      if (collect && ctl.bc_flag) {
        // drop this CTA's members ranked after the threshold element
        const float thr = ctl.bc_thr;
        const int thr_idx = ctl.bc_thr_idx;
        const int nm = (int)min(ctl.mem_n, (uint32_t)kCap);
        for (int i = tid; i < nm; i += kThreads) {
          const float sm = mem_s[i];
          if (sm < thr || (sm == thr && R.base + mem_i[i] > thr_idx)) vals[mem_i[i]] = 0.0f;
        }
        __syncthreads();
      }
      keep_lo = __uint_as_float(lo_key);
    }
    // per-lane kept mass
    lane_mass = 0.0f;
    for (int f = R.f_begin + lane; f < R.f_end; f += 32) {
      const float4 v = vals4[f];
      lane_mass = __fadd_rn(lane_mass, (v.x >= keep_lo && v.x > 0.f) ? v.x : 0.f);
      lane_mass = __fadd_rn(lane_mass, (v.y >= keep_lo && v.y > 0.f) ? v.y : 0.f);
      lane_mass = __fadd_rn(lane_mass, (v.z >= keep_lo && v.z > 0.f) ? v.z : 0.f);
      lane_mass = __fadd_rn(lane_mass, (v.w >= keep_lo && v.w > 0.f) ? v.w : 0.f);
    }
  }

  // ---- CTA masses -> every CTA
  {
    const double wm = warp_dsum((double)lane_mass);
    if (lane == 0) ctl.wmass[warp] = wm;
    __syncthreads();
    if (tid < kCluster) {
      double cm = 0.0;
      for (int w = 0; w < kWarps; ++w) cm += ctl.wmass[w];
      dsmem_st_f64(dsmem_map(smem_addr(&ctl.rec_mass[R.rank]), tid), cm);
    }
  }
  cluster_sync();  // barrier: masses delivered

  double ztot = 0.0;
  for (int r = 0; r < kCluster; ++r) ztot += ctl.rec_mass[r];
  const double target = u * ztot;
  int owner = -1;
  double pre_owner = 0.0;
  {
    double run = 0.0;
    int last_pos = -1;
    double last_pre = 0.0;
    for (int r = 0; r < kCluster; ++r) {
      const double mr = ctl.rec_mass[r];
      if (mr > 0.0) { last_pos = r; last_pre = run; }
      if (owner < 0 && mr > 0.0 && run + mr > target) { owner = r; pre_owner = run; }
      run += mr;
    }
    if (owner < 0) { owner = last_pos; pre_owner = last_pre; }
  }
  if (R.greedy) {
    if (leader && tid == 0) {
      if (a.out_dtype == NS_OUT_I32) reinterpret_cast<int32_t*>(a.out_tokens)[R.row] = gamax;
      else reinterpret_cast<int64_t*>(a.out_tokens)[R.row] = gamax;
    }
  } else if ((int)R.rank == owner) {
    // owning warp
    double tloc = target - pre_owner;
    int wsel = -1;
    double wpre = 0.0;
    {
      double run = 0.0;
      int lastw = -1;
      double lastpre = 0.0;
      for (int w = 0; w < kWarps; ++w) {
        const double x = ctl.wmass[w];
        if (x > 0.0) { lastw = w; lastpre = run; }
        if (wsel < 0 && x > 0.0 && run + x > tloc) { wsel = w; wpre = run; }
        run += x;
      }
      if (wsel < 0) { wsel = lastw; wpre = lastpre; }
    }
    if (warp == wsel) {
      const double tw = tloc - wpre;
      double run = 0.0;
      int tok = -1, last_kept = -1;
      for (int f0 = R.f_begin; f0 < R.f_end && tok < 0; f0 += 32) {
        const int f = f0 + lane;
        float q[4] = {0.f, 0.f, 0.f, 0.f};
        if (f < R.f_end) {
          const float4 v = vals4[f];
          const float t[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int c = 0; c < 4; ++c) q[c] = (t[c] >= keep_lo && t[c] > 0.f) ? t[c] : 0.f;
        }
        const float ls = __fadd_rn(__fadd_rn(__fadd_rn(q[0], q[1]), q[2]), q[3]);
        const double inc = warp_incl_f64((double)ls, lane);
        const double rowtot = __shfl_sync(0xffffffffu, inc, 31);
        // last kept element seen so far (for the clamp)
        int lk = -1;
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if (q[c] > 0.f) lk = R.base + 4 * f + c;
        for (int o = 16; o; o >>= 1) lk = max(lk, __shfl_xor_sync(0xffffffffu, lk, o));
        if (lk >= 0) last_kept = lk;
        if (run + rowtot > tw) {
          const uint32_t bal = __ballot_sync(0xffffffffu, run + inc > tw && ls > 0.f);
          if (bal) {
            const int l = __ffs(bal) - 1;
            if (lane == l) {
              double cum = run + inc - (double)ls;
              int pick = -1, lastc = -1;
              for (int c = 0; c < 4; ++c) {
                if (q[c] > 0.f) {
                  lastc = c;
                  cum += (double)q[c];
                  if (pick < 0 && cum > tw) pick = c;
                }
              }
              if (pick < 0) pick = lastc;
              tok = R.base + 4 * f + pick;
            }
            tok = __shfl_sync(0xffffffffu, tok, l);
          }
        }
        run += rowtot;
      }
      if (tok < 0) tok = last_kept;
      if (tok < 0) tok = gamax;  // no kept mass at all (cannot happen for a regular row)
      if (lane == 0) {
        if (a.out_dtype == NS_OUT_I32) reinterpret_cast<int32_t*>(a.out_tokens)[R.row] = tok;
        else reinterpret_cast<int64_t*>(a.out_tokens)[R.row] = tok;
      }
    }
  }
  if (debug) {
    for (int i = tid; i < R.len; i += kThreads) {
      const float e = vals[i];
      const bool kept = (e >= keep_lo && e > 0.f);
      if (a.out_probs) a.out_probs[out_row_off + R.base + i] = kept ? (float)((double)e / ztot) : 0.0f;
      if (a.out_filtered) {
        float sv = -INFINITY;
        if (kept) sv = scaled(R, penalized_from_global(R, bitmap, i));
        a.out_filtered[out_row_off + R.base + i] = sv;
      }
    }
  }
}

// ---------------------------------------------------------------- host side
thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

struct DeviceState {
  size_t smem_set = 0;
};
std::mutex g_mu;
DeviceState g_dev[64];

int slice_width(int V) {
  int W = (V + kCluster - 1) / kCluster;
  return (W + 7) & ~7;
}

}  // namespace ns

extern "C" {

int ns_abi_version(void) { return NS_ABI_VERSION; }

const char* ns_last_error(void) { return ns::g_last_error.c_str(); }

int32_t ns_max_vocab(int32_t logits_dtype) {
  (void)logits_dtype;
  return ns::kMaxSlice * ns::kCluster;
}

int ns_sample(const NsSampleArgs* args, void* stream) {
  using namespace ns;
  if (!args) return fail(NS_ERR_INVALID_ARG, "ns_sample: args is NULL");
  const NsSampleArgs& a = *args;
  if (a.num_rows < 0) return fail(NS_ERR_INVALID_ARG, "ns_sample: num_rows < 0");
  if (a.num_rows == 0) return NS_OK;
  if (!a.logits || !a.row_params || !a.out_tokens)
    return fail(NS_ERR_INVALID_ARG, "ns_sample: logits, row_params and out_tokens are required");
  if (a.logits_dtype != NS_DTYPE_F32 && a.logits_dtype != NS_DTYPE_BF16)
    return fail(NS_ERR_INVALID_ARG, "ns_sample: logits_dtype must be NS_DTYPE_F32 or NS_DTYPE_BF16");
  if (a.out_dtype != NS_OUT_I64 && a.out_dtype != NS_OUT_I32)
    return fail(NS_ERR_INVALID_ARG, "ns_sample: out_dtype must be NS_OUT_I64 or NS_OUT_I32");
  if (a.vocab_size <= 0) return fail(NS_ERR_INVALID_ARG, "ns_sample: vocab_size must be positive");
  if (a.vocab_size > ns_max_vocab(a.logits_dtype))
    return fail(NS_ERR_UNSUPPORTED, "ns_sample: vocab_size " + std::to_string(a.vocab_size) +
                                        " exceeds the supported maximum " +
                                        std::to_string(ns_max_vocab(a.logits_dtype)));
  if (a.logits_row_stride < a.vocab_size)
    return fail(NS_ERR_INVALID_ARG, "ns_sample: logits_row_stride < vocab_size");
  if (a.num_logit_rows <= 0) return fail(NS_ERR_INVALID_ARG, "ns_sample: num_logit_rows must be positive");
  if (!a.sample_indices && a.num_logit_rows < a.num_rows)
    return fail(NS_ERR_INVALID_ARG, "ns_sample: fewer logits rows than num_rows and no sample_indices");
  if (a.history_offsets && !a.history_ids)
    return fail(NS_ERR_INVALID_ARG, "ns_sample: history_offsets given without history_ids");
  if ((int64_t)a.num_rows * kCluster > INT_MAX)
    return fail(NS_ERR_UNSUPPORTED, "ns_sample: too many rows for one launch");

  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return fail(NS_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(err));
  const int W = slice_width(a.vocab_size);
  const Layout L = make_layout(W);
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (dev < 0 || dev >= 64) return fail(NS_ERR_UNSUPPORTED, "ns_sample: device ordinal >= 64");
    if (g_dev[dev].smem_set < L.total) {
      err = cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total);
      if (err != cudaSuccess)
        return fail(NS_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(err));
      g_dev[dev].smem_set = L.total;
    }
  }
  const uintptr_t p = reinterpret_cast<uintptr_t>(a.logits);
  const int tma_ok = (a.logits_dtype == NS_DTYPE_F32) && (p % 16 == 0) && (a.logits_row_stride % 4 == 0);
  const int vec16_ok = (a.logits_dtype == NS_DTYPE_BF16) && (p % 8 == 0) && (a.logits_row_stride % 4 == 0);

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(a.num_rows * kCluster), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  err = cudaLaunchKernelEx(&cfg, sample_kernel, a, W, tma_ok, vec16_ok);
  if (err != cudaSuccess) return fail(NS_ERR_CUDA, std::string("sample kernel launch: ") + cudaGetErrorString(err));
  return NS_OK;
}

}  // extern "C"

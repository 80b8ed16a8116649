// ns_sample.cu -- B200 (sm_100a) token sampling: one kernel launch per step.
//
// Replaces nanoserve/scheduler/sampler.py:21-89 (Sampler.sample).  Design:
//
//  * Persistent thread-block clusters of kCluster (8) CTAs, as many as are
//    co-resident (two CTAs per SM); cluster c samples rows c, c+G, c+2G...
//    CTA r of a cluster owns the contiguous vocabulary slice [r*W, r*W+W)
//    of the current row and keeps it in its shared memory while it needs
//    it, so every row crosses HBM exactly once.  Each warp moves its own
//    contiguous piece of the slice with one mbarrier-tracked bulk copy
//    (cp.async.bulk, global -> own shared memory, no multicast) and issues
//    the copy for the NEXT row as soon as it has finished with the current
//    one, so HBM keeps streaming while the cluster exchanges statistics,
//    waits at barriers and decides.  The next row's parameters are fetched
//    with cp.async during the current row.
//  * Row statistics, histograms and candidate lists are exchanged through
//    distributed shared memory (st/ld/red/atom .shared::cluster) between
//    cluster barriers.  Areas that peers write into are double-buffered by
//    row parity; the row's leader CTA rotates.  No global scratch memory.
//  * Three row paths, chosen per row (uniformly across the cluster):
//      GREEDY   temperature == 0 and no debug output: first-index argmax
//               (sampler.py:82-83); one exchange.
//      TOPK     0 < top_k <= kTopkSmall: a histogram of per-thread maxima
//               bounds the k-th largest logit from below; every element
//               above the bound goes to the row's leader CTA, which
//               finishes top-k (sampler.py:53-58), top-p (sampler.py:60-73),
//               softmax and the inverse-CDF draw on that short list.
//      GENERAL  anything else: exp(s - max) is computed once per element and
//               kept in place.  Top-p locates its boundary with a histogram
//               of approximate masses keyed on the bits of exp(s - max)
//               (log-spaced buckets, one 32-bit shared atomic per element),
//               narrows it to a window of buckets that must contain the
//               boundary, then ships the window's elements to the leader,
//               which sorts them and decides exactly with the exact mass
//               above the window.  Large top-k runs an exact 3-level radix
//               select first.  The draw walks per-warp masses in vocabulary
//               order, then one warp's piece of the slice.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <climits>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/nanoserve_sampler.h"
#include "ns_device.cuh"
#include "ns_rows.h"

namespace ns {

constexpr int kCluster = 8;
constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kBins = 4096;          // top-p locator histogram (u32 approximate masses)
constexpr int kCoarse = 64;          // coarse buckets of kFine fine buckets
constexpr int kFine = kBins / kCoarse;
constexpr int kRadixBins = 2048;     // radix-select level histogram (u32 counts), 2 buffers
constexpr int kRadixCoarse = 32;
constexpr int kCap = 512;            // leader candidate list capacity (a power of two)
constexpr int kTopkSmall = 128;      // largest top_k served by the TOPK path
constexpr int kTmBins = 2048;        // per-thread-maximum histogram (u16 counts), quarter binades
constexpr int kTmShift = 21;
constexpr int kMaxSlice = 24576;     // largest slice (elements) one CTA holds
constexpr int kMaxShift = 17;        // locator buckets cover >= 63.9 binades of exp(s - max)
constexpr uint32_t kOne = 0x3F800000u;           // bits of 1.0f
constexpr double kWindowSlack = 1.0 + 0x1p-14;  // > 1 / (1 - 2^-15): locator mass error bound
constexpr double kFixedScale = 17592186044416.0;  // 2^44

// What peers write into this CTA during one row; double-buffered by row parity.
struct __align__(16) Recv {
  uint32_t rec_kmax[kCluster];   // orderable key of the CTA maximum (0xffffffff: NaN seen)
  uint32_t rec_kmin[kCluster];   // orderable key of the CTA minimum
  float rec_amin[kCluster];      // smallest |x|
  int32_t rec_amax[kCluster];    // first index of the CTA maximum
  int32_t rec_nan[kCluster];
  int32_t rec_pinf[kCluster];
  double rec_z[kCluster];
  double rec_above[kCluster];
  uint32_t cand_n;
  uint32_t overflow;
  uint32_t pad[2];
  uint32_t tm_global[kTmBins / 2];
};

// One row's inputs, fetched one row ahead.
struct __align__(16) RowIn {
  NsRowParams P;
  int64_t h[2];
  int64_t src;
  int64_t pad;
};

// Fixed-size control block at the start of dynamic shared memory.
struct __align__(16) Ctl {
  uint64_t mbar[kWarps];
  RowIn rin[2];
  // own coarse sums, double-buffered by level (peers read them)
  double cmass[2][kCoarse];
  uint32_t ccnt[2][kRadixCoarse];
  double cz[2];
  // leader broadcast
  float bc_thr;
  int32_t bc_thr_idx;
  int32_t bc_owner;
  float bc_m;
  double bc_tloc;
  double bc_z;
  // CTA-local results
  int32_t sel_found;
  int32_t sel_lo;
  int32_t sel_hi;
  uint32_t sel_cnt;
  uint32_t sel_before_cnt;
  float sel_est;
  double sel_z;
  // reductions
  uint32_t red_k[kWarps];
  uint32_t red_m[kWarps];
  uint32_t red_a[kWarps];
  int32_t red_i[kWarps];
  int32_t red_j[kWarps];
  uint32_t red_u[kWarps];
  double wmass[kWarps];
  unsigned long long wfix[kWarps];
  int32_t misc_i;
  int32_t misc_j;
  // top-p tie resolution (leader broadcast, peer reports)
  uint32_t bc_tie;
  uint32_t bc_bits;
  int32_t bc_q;
  int32_t bc_cq;
  float tie_smin[kCluster];
  float tie_smax[kCluster];
  int32_t token;
  uint32_t mem_n;
};

struct Layout {
  size_t ctl, recv, hist, bitmap, cand_s, cand_i, keys, mem_s, mem_i, mem_e, vals, total;
};

__host__ __device__ inline size_t align16(size_t x) { return (x + 15) & ~size_t(15); }

__host__ __device__ inline Layout make_layout(int W) {
  Layout L;
  size_t o = 0;
  L.ctl = o;    o = align16(o + sizeof(Ctl));
  L.recv = o;   o = align16(o + 2 * sizeof(Recv));
  L.hist = o;   o = align16(o + sizeof(uint32_t) * kBins);
  L.bitmap = o; o = align16(o + sizeof(uint32_t) * ((W + 31) / 32));
  L.cand_s = o; o = align16(o + sizeof(float) * kCap);
  L.cand_i = o; o = align16(o + sizeof(int32_t) * kCap);
  L.keys = o;   o = align16(o + sizeof(unsigned long long) * kCap);
  L.mem_s = o;  o = align16(o + sizeof(float) * kCap);
  L.mem_i = o;  o = align16(o + sizeof(int32_t) * kCap);
  L.mem_e = o;  o = align16(o + sizeof(float) * kCap);
  L.vals = o;   o = align16(o + sizeof(float) * W);
  L.total = o;
  return L;
}

// Bitonic sort of keys[0, n) ascending in place (n <= kCap), by the whole CTA.
// Entries [n, pow2) are filled with the largest key.
__device__ void bitonic_sort(unsigned long long* keys, int n, int tid) {
  int np = 1;
  while (np < n) np <<= 1;
  for (int i = n + tid; i < np; i += kThreads) keys[i] = ~0ull;
  __syncthreads();
  for (int k = 2; k <= np; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < np; i += kThreads) {
        const int l = i ^ j;
        if (l > i) {
          const unsigned long long a = keys[i], b = keys[l];
          const bool up = (i & k) == 0;
          if ((a > b) == up) { keys[i] = b; keys[l] = a; }
        }
      }
      __syncthreads();
    }
  }
}

// ---------------------------------------------------------------- contexts
// Where logits rows come from (copied out of the kernel parameters).
struct Src {
  const void* logits;
  const int64_t* sidx;
  int64_t nrows;
  int64_t stride;
  bool bf16;
};
__device__ __forceinline__ int64_t source_row(const Src& S, int row, bool& bad) {
  int64_t src = row;
  bad = false;
  if (S.sidx) src = S.sidx[row];
  if (src < 0 || src >= S.nrows) { bad = true; src = 0; }
  return src;
}

// The CTA's slice geometry (the same for every row).
struct Geo {
  int V, W, base, len, nf4, full4, chunk, f_begin, f_end;
  uint32_t rank;
  bool tma, vec16;
};

// One row being sampled.
struct Row {
  int row;
  uint32_t lead;  // the row's leader CTA
  const float* src32;
  const __nv_bfloat16* src16;
  float T, rT;
  bool t_one, greedy, topp, pen;
  int k;
  float p, rp;
};

__device__ __forceinline__ float load_scalar(const Geo& g, const Row& R, int local) {
  if (R.src16) return __bfloat162float(R.src16[g.base + local]);
  return R.src32[g.base + local];
}
// Logit after the repetition penalty for one element of this CTA's slice,
// re-read from global memory.
__device__ __forceinline__ float penalized_from_global(const Geo& g, const Row& R, const uint32_t* bitmap, int local) {
  float x = load_scalar(g, R, local);
  if (R.pen && ((bitmap[local >> 5] >> (local & 31)) & 1u)) x = penalize(x, R.rp);
  return x;
}
__device__ __forceinline__ float scaled(const Row& R, float x) {
  return R.t_one ? x : div_by_const(x, R.T, R.rT);
}
// Markstein's division without the range guard: exact whenever every |x| of
// the row lies in [2^-40, 2^80] and the temperature is at most 2^20 (then
// both |x| and |x/T| stay inside the guard of div_by_const).
__device__ __forceinline__ float scaled_fast(const Row& R, float x) {
  const float q0 = __fmul_rn(x, R.rT);
  return __fmaf_rn(__fmaf_rn(-q0, R.T, x), R.rT, q0);
}

// Load float4 slot f (4 logits) of this CTA's slice with the penalty applied,
// store it to shared memory when it did not arrive there by bulk copy or was
// changed, and emit the penalized debug output.  Elements past the slice end
// read as -inf.
__device__ __forceinline__ float4 load_slot(const Geo& g, const Row& R, float* vals, const uint32_t* bitmap, int f,
                                            float* pen_out) {
  float4 v;
  const int e0 = f * 4;
  bool dirty = false;
  if (g.tma && f < g.full4) {
    v = reinterpret_cast<const float4*>(vals)[f];
  } else if (g.vec16 && e0 + 3 < g.len) {
    uint2 raw = *reinterpret_cast<const uint2*>(R.src16 + g.base + e0);
    __nv_bfloat162 lo = *reinterpret_cast<__nv_bfloat162*>(&raw.x);
    __nv_bfloat162 hi = *reinterpret_cast<__nv_bfloat162*>(&raw.y);
    float2 a = __bfloat1622float2(lo), b = __bfloat1622float2(hi);
    v = make_float4(a.x, a.y, b.x, b.y);
    dirty = true;
  } else {
    float t[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) t[c] = (e0 + c < g.len) ? load_scalar(g, R, e0 + c) : -INFINITY;
    v = make_float4(t[0], t[1], t[2], t[3]);
    dirty = true;
  }
  if (R.pen) {
    const uint32_t nib = (bitmap[f >> 3] >> ((f & 7) << 2)) & 0xFu;
    if (nib) {
      if (nib & 1u) v.x = penalize(v.x, R.rp);
      if (nib & 2u) v.y = penalize(v.y, R.rp);
      if (nib & 4u) v.z = penalize(v.z, R.rp);
      if (nib & 8u) v.w = penalize(v.w, R.rp);
      dirty = true;
    }
  }
  if (dirty) reinterpret_cast<float4*>(vals)[f] = v;
  if (pen_out) {
    const float t[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int c = 0; c < 4; ++c)
      if (e0 + c < g.len) pen_out[e0 + c] = t[c];
  }
  return v;
}

// Issue this warp's bulk copy of row `row` into its piece of the slice.  The
// warp must be done reading and writing that piece for the current row.
// Every lane orders its own earlier shared-memory writes before the copy.
__device__ __forceinline__ void issue_chunk(const Src& S, const Geo& g, Ctl& ctl, float* vals, int row, int warp,
                                            int lane) {
  fence_proxy_async_smem();
  __syncwarp();
  if (!g.tma || lane != 0) return;
  const int fe = min(g.f_end, g.full4);
  if (fe <= g.f_begin) return;
  bool bad;
  const int64_t src = source_row(S, row, bad);
  const float* p = reinterpret_cast<const float*>(S.logits) + src * S.stride + g.base + 4 * g.f_begin;
  const uint32_t bytes = (uint32_t)(fe - g.f_begin) * 16u;
  mbar_arrive_expect_tx(&ctl.mbar[warp], bytes);
  bulk_g2s(vals + 4 * g.f_begin, p, bytes, &ctl.mbar[warp]);
}

// Bounded wait for this warp's bulk copy of the current row.  On give-up the
// status word is set and the kernel carries on, so that no cluster barrier
// is left waiting.
__device__ __forceinline__ void wait_chunk(const Geo& g, Ctl& ctl, int warp, uint32_t parity, uint32_t* status) {
  if (!g.tma || g.f_begin >= min(g.f_end, g.full4)) return;
  uint32_t spins = 0;
  while (!mbar_try_wait(&ctl.mbar[warp], parity)) {
    if (++spins > (1u << 22)) {
      if (status) atomicOr(status, NS_STATUS_WAIT_TIMEOUT);
      break;
    }
    if (spins > 64) __nanosleep(64);
  }
}

// Threads 0..3 start fetching row `row`'s inputs into `dst` (cp.async).
__device__ __forceinline__ void fetch_row_inputs(const NsSampleArgs& a, RowIn& dst, int row, int tid) {
  if (tid == 0) {
    cp_async16(&dst.P, &a.row_params[row]);
  } else if (tid == 1) {
    cp_async16(reinterpret_cast<char*>(&dst.P) + 16, reinterpret_cast<const char*>(&a.row_params[row]) + 16);
  } else if (tid == 2) {
    if (a.history_offsets) {
      cp_async8(&dst.h[0], &a.history_offsets[row]);
      cp_async8(&dst.h[1], &a.history_offsets[row + 1]);
    } else {
      dst.h[0] = 0;
      dst.h[1] = 0;
    }
  } else if (tid == 3) {
    if (a.sample_indices) cp_async8(&dst.src, &a.sample_indices[row]);
    else dst.src = row;
  }
  if (tid < 4) cp_async_commit();
}

// Row taken at position t of the row order (NsSampleArgs.row_order, a
// scheduling hint); an entry outside [0, S) takes row t and, with `flag`,
// sets NS_STATUS_BAD_ROW_ORDER.
__device__ __forceinline__ int ordered_row(const NsSampleArgs& a, int t, bool flag) {
  if (!a.row_order) return t;
  const int r = __ldg(&a.row_order[t]);
  if (r >= 0 && r < a.num_rows) return r;
  if (flag && a.status) atomicOr(a.status, NS_STATUS_BAD_ROW_ORDER);
  return t;
}

// Smallest float c <= b with RN(c/T) == RN(b/T): the lower end of the set of
// logits whose scaled value is at least RN(b/T).
__device__ float lower_preimage(const Row& R, float b) {
  if (R.t_one || !(b > -INFINITY) || !(b < INFINITY)) return b;
  const float target = div_by_const(b, R.T, R.rT);
  float c = b;
  for (int i = 0; i < 64; ++i) {
    const float d = nextafterf(c, -INFINITY);
    if (div_by_const(d, R.T, R.rT) == target) c = d; else return c;
  }
  return -INFINITY;
}


// Block-wide exclusive scan of one u32 per thread (thread 0 first).
__device__ uint32_t block_excl_u32(Ctl& ctl, uint32_t v, uint32_t& total, int tid) {
  const int lane = tid & 31, warp = tid >> 5;
  const uint32_t inc = warp_incl_u32(v, lane);
  if (lane == 31) ctl.red_u[warp] = inc;
  __syncthreads();
  uint32_t wpre = 0, tot = 0;
  for (int w = 0; w < kWarps; ++w) {
    const uint32_t x = ctl.red_u[w];
    if (w < warp) wpre += x;
    tot += x;
  }
  __syncthreads();
  total = tot;
  return wpre + inc - v;
}

// ---------------------------------------------------------------- radix crossing (counts)
// Over the kRadixBins-bucket count histogram `h` (bucket 0 = largest keys):
// first bucket whose inclusive count over the whole cluster reaches `kneed`.
// Contains one cluster barrier; `h` and ctl.ccnt[buf] must stay untouched by
// this CTA until the next cluster barrier.
__device__ void radix_crossing(Ctl& ctl, const uint32_t* h, int buf, uint32_t kneed, int tid) {
  const int lane = tid & 31, warp = tid >> 5;
  {
    const int c = tid >> 4;  // 32 coarse buckets x 64 fine; 16 threads each
    uint32_t cnt = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) cnt += h[tid * 4 + j];
#pragma unroll
    for (int o = 8; o; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    if ((tid & 15) == 0) ctl.ccnt[buf][c] = cnt;
  }
  cluster_sync();
  if (warp == 0) {
    uint32_t cnt = 0;
    const uint32_t ac = smem_addr(&ctl.ccnt[buf][lane]);
#pragma unroll
    for (int r = 0; r < kCluster; ++r) cnt += dsmem_ld_u32(dsmem_map(ac, r));
    const uint32_t ic = warp_incl_u32(cnt, lane);
    const uint32_t bal = __ballot_sync(0xffffffffu, ic >= kneed);
    int found = bal != 0u, bsel = 0;
    uint32_t bcnt = 0, bbefore = 0;
    if (found) {
      const int cb = __ffs(bal) - 1;
      uint32_t run = __shfl_sync(0xffffffffu, ic - cnt, cb);
      found = 0;
      for (int hh = 0; hh < 2 && !found; ++hh) {
        const int b = cb * 64 + hh * 32 + lane;
        const uint32_t ah = smem_addr(&h[b]);
        uint32_t f = 0;
#pragma unroll
        for (int r = 0; r < kCluster; ++r) f += dsmem_ld_u32(dsmem_map(ah, r));
        const uint32_t inc = warp_incl_u32(f, lane) + run;
        const uint32_t b2 = __ballot_sync(0xffffffffu, inc >= kneed);
        if (b2) {
          const int l = __ffs(b2) - 1;
          bsel = cb * 64 + hh * 32 + l;
          bcnt = __shfl_sync(0xffffffffu, f, l);
          bbefore = __shfl_sync(0xffffffffu, inc - f, l);
          found = 1;
        } else {
          run = __shfl_sync(0xffffffffu, inc, 31);
        }
      }
    }
    if (lane == 0) {
      ctl.sel_found = found;
      ctl.sel_lo = bsel;
      ctl.sel_cnt = bcnt;
      ctl.sel_before_cnt = bbefore;
    }
  }
  __syncthreads();
}

// ---------------------------------------------------------------- top-p locator
// Bucket b of a locator level covers keys (bits of exp(s - max)) in
// [top - (b+1)*2^sh + 1, top - b*2^sh]; top + 1 is a multiple of 2^sh, so each
// bucket lies inside one binade and its elements share one exponent.
struct Level {
  uint32_t top;
  int sh;
  bool last_is_overflow;  // level 0: the last bucket collects everything below
  __device__ __forceinline__ uint32_t lo_key(int b) const { return top - (uint32_t)(b + 1) * (1u << sh) + 1u; }
  __device__ __forceinline__ uint32_t hi_key(int b) const { return top - (uint32_t)b * (1u << sh); }
  __device__ __forceinline__ double mass(uint32_t sum16, int b) const {
    if (sum16 == 0u || (last_is_overflow && b == kBins - 1)) return 0.0;
    const int ex = (int)(lo_key(b) >> 23);
    return ldexp((double)sum16, ex - 142);
  }
};

// Cluster-wide window search.  Every CTA has its approximate-mass histogram
// in `h` and its exact mass (the total at level 0, the mass above the level's
// key range otherwise) in ctl.cz[buf].  Finds the bucket window [lo, hi] that
// must contain the top-p boundary, given that each bucket's approximate mass
// is within a factor (1 - 2^-15) of its exact mass, and an estimate of the
// number of elements in it.  One cluster barrier; the caller must leave `h`
// and ctl.cmass/cz[buf] untouched until the next cluster barrier.
__device__ void topp_window(Ctl& ctl, const uint32_t* h, int buf, const Level& lv, bool level0, double zin,
                            float p, int tid) {
  const int lane = tid & 31, warp = tid >> 5;
  {
    // own coarse sums: 8 threads per coarse bucket, 8 fine buckets each
    const int c = tid >> 3;
    double m = 0.0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int b = tid * 8 + j;
      m += lv.mass(h[b], b);
    }
#pragma unroll
    for (int o = 4; o; o >>= 1) m += __shfl_xor_sync(0xffffffffu, m, o);
    if ((tid & 7) == 0) ctl.cmass[buf][c] = m;
  }
  cluster_sync();
  if (warp == 0) {
    double zsum = 0.0;
#pragma unroll
    for (int r = 0; r < kCluster; ++r) zsum += dsmem_ld_f64(dsmem_map(smem_addr(&ctl.cz[buf]), r));
    const double z = level0 ? zsum : zin;
    const double base = level0 ? 0.0 : zsum;
    double cm[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const uint32_t ad = smem_addr(&ctl.cmass[buf][hh * 32 + lane]);
      double s = 0.0;
#pragma unroll
      for (int r = 0; r < kCluster; ++r) s += dsmem_ld_f64(dsmem_map(ad, r));
      cm[hh] = s;
    }
    // first coarse buckets where the upper (slack) and the lower estimate cross
    int c_lo = -1, c_hi = -1;
    double run = base, pre_lo = 0.0;
    for (int hh = 0; hh < 2; ++hh) {
      const double inc = warp_incl_f64(cm[hh], lane) + run;
      const uint32_t bl = __ballot_sync(0xffffffffu, topp_crossed(inc * kWindowSlack, z, p));
      const uint32_t bh = __ballot_sync(0xffffffffu, topp_crossed(inc, z, p));
      if (c_lo < 0 && bl) {
        const int l = __ffs(bl) - 1;
        c_lo = hh * 32 + l;
        pre_lo = __shfl_sync(0xffffffffu, inc - cm[hh], l);
      }
      if (c_hi < 0 && bh) c_hi = hh * 32 + __ffs(bh) - 1;
      run = __shfl_sync(0xffffffffu, inc, 31);
    }
    int found = (c_lo >= 0);
    int b_lo = 0, b_hi = 0;
    float est = 0.f;
    if (found) {
      if (c_hi < 0) c_hi = kCoarse - 1;
      double frun = pre_lo;
      int fl = -1, fh = -1;
      double est_d = 0.0;
      for (int c = c_lo; c <= c_hi && fh < 0; ++c) {
        for (int hh = 0; hh < 2 && fh < 0; ++hh) {
          const int b = c * kFine + hh * 32 + lane;
          const uint32_t ah = smem_addr(&h[b]);
          uint32_t s16 = 0;
#pragma unroll
          for (int r = 0; r < kCluster; ++r) s16 += dsmem_ld_u32(dsmem_map(ah, r));
          const double m = lv.mass(s16, b);
          const double inc = warp_incl_f64(m, lane) + frun;
          const uint32_t bl = __ballot_sync(0xffffffffu, topp_crossed(inc * kWindowSlack, z, p));
          const uint32_t bh = __ballot_sync(0xffffffffu, topp_crossed(inc, z, p));
          const int flo = (fl < 0 && bl) ? c * kFine + hh * 32 + (__ffs(bl) - 1) : fl;
          const int fhi = bh ? c * kFine + hh * 32 + (__ffs(bh) - 1) : -1;
          // elements in the window ~ mass / smallest value of the bucket
          const bool inwin = (flo >= 0) && b >= flo && (fhi < 0 || b <= fhi);
          const double e_bot = (double)__uint_as_float(lv.lo_key(b));
          est_d += warp_dsum((inwin && m > 0.0 && e_bot > 0.0) ? m / e_bot : 0.0);
          fl = flo;
          fh = fhi;
          frun = __shfl_sync(0xffffffffu, inc, 31);
        }
      }
      if (fl < 0) fl = c_lo * kFine;
      if (fh < 0) fh = c_hi * kFine + kFine - 1;
      if (lv.last_is_overflow && fh == kBins - 1) fh = kBins - 2;
      if (fl > fh) fl = fh;
      b_lo = fl;
      b_hi = fh;
      est = (float)(est_d * 1.001 + 1.0);
    }
    if (lane == 0) {
      ctl.sel_found = found;
      ctl.sel_lo = b_lo;
      ctl.sel_hi = b_hi;
      ctl.sel_est = est;
      ctl.sel_z = z;
    }
  }
  __syncthreads();
}

// Per-warp sums of lane values (into ctl.wmass) and their CTA total.
__device__ __forceinline__ double cta_warp_sums(Ctl& ctl, float lane_v, int lane, int warp) {
  const double w = warp_dsum((double)lane_v);
  if (lane == 0) ctl.wmass[warp] = w;
  __syncthreads();
  double s = 0.0;
  for (int i = 0; i < kWarps; ++i) s += ctl.wmass[i];
  return s;
}

// First CTA whose mass prefix passes target, and the target within it.
__device__ __forceinline__ void pick_owner(const double* m, double target, int& owner, double& tloc) {
  double run = 0.0, last_pre = 0.0;
  int last = -1;
  owner = -1;
  for (int r = 0; r < kCluster; ++r) {
    const double mr = m[r];
    if (mr > 0.0) { last = r; last_pre = run; }
    if (owner < 0 && mr > 0.0 && run + mr > target) { owner = r; tloc = target - run; }
    run += mr;
  }
  if (owner < 0) { owner = last; tloc = target - last_pre; }
}
// First warp whose mass prefix passes target, and the target within it.
__device__ __forceinline__ void pick_warp(const double* m, double target, int& w, double& tw) {
  double run = 0.0, lastpre = 0.0;
  int lastw = -1;
  w = -1;
  for (int i = 0; i < kWarps; ++i) {
    const double x = m[i];
    if (x > 0.0) { lastw = i; lastpre = run; }
    if (w < 0 && x > 0.0 && run + x > target) { w = i; tw = target - run; }
    run += x;
  }
  if (w < 0) { w = lastw; tw = target - lastpre; }
}

// What the debug outputs need to recompute kept masses from global memory.
struct Keep {
  float m;             // max scaled logit
  bool have_thr_k;     // large top-k mask: s >= thr_k_s
  float thr_k_s;
  bool window;         // top-p window decision
  uint32_t win_lo, win_hi;
  float thr;           // last kept (s, idx) inside the window
  int thr_idx;
};
__device__ __forceinline__ float kept_mass(const Geo& g, const Row& R, const Keep& K, const uint32_t* bitmap,
                                           int local) {
  if (local >= g.len) return 0.f;
  const float s = scaled(R, penalized_from_global(g, R, bitmap, local));
  if (K.have_thr_k && !(s >= K.thr_k_s)) return 0.f;
  const float e = exp_shifted(s, K.m);
  if (!(e > 0.f)) return 0.f;
  if (K.window) {
    const uint32_t bits = __float_as_uint(e);
    if (bits < K.win_lo) return 0.f;
    if (bits <= K.win_hi && (s < K.thr || (s == K.thr && g.base + local > K.thr_idx))) return 0.f;
  }
  return e;
}

// The selected warp walks its piece of the slice (masses e in shared memory,
// kept <=> bits(e) >= keep_lo and e > 0) in vocabulary order until the mass
// passes tw; returns the token (lane-uniform).
__device__ int walk_warp(const Geo& g, const float4* vals4, int wsel, uint32_t keep_lo, double tw, int lane,
                         int fallback) {
  const int w_begin = min(g.nf4, wsel * g.chunk), w_end = min(g.nf4, w_begin + g.chunk);
  double run = 0.0;
  int tok = -1, last_kept = -1;
  for (int f0 = w_begin; f0 < w_end && tok < 0; f0 += 32) {
    const int f = f0 + lane;
    float q[4] = {0.f, 0.f, 0.f, 0.f};
    if (f < w_end) {
      const float4 v = vals4[f];
      const float t[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int c = 0; c < 4; ++c) q[c] = (__float_as_uint(t[c]) >= keep_lo && t[c] > 0.f) ? t[c] : 0.f;
    }
    const float ls = __fadd_rn(__fadd_rn(__fadd_rn(q[0], q[1]), q[2]), q[3]);
    const double inc = warp_incl_f64((double)ls, lane);
    const double rowtot = __shfl_sync(0xffffffffu, inc, 31);
    int lk = -1;
#pragma unroll
    for (int c = 0; c < 4; ++c)
      if (q[c] > 0.f) lk = g.base + 4 * f + c;
    lk = __reduce_max_sync(0xffffffffu, (uint32_t)(lk + 1)) - 1;
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
          tok = g.base + 4 * f + pick;
        }
        tok = __shfl_sync(0xffffffffu, tok, l);
      }
    }
    run += rowtot;
  }
  if (tok < 0) tok = last_kept;
  if (tok < 0) tok = fallback;
  return tok;
}

// ---------------------------------------------------------------- one row
struct Shared {
  Ctl* ctl;
  Recv* recv;
  uint32_t* hist;
  uint32_t* bitmap;
  float* cand_s;
  int32_t* cand_i;
  unsigned long long* keys;
  float* mem_s;
  int32_t* mem_i;
  float* mem_e;
  float* vals;
};

// ---------------------------------------------------------------- top-p ties
// Exact top-p decision for a window whose members overflow the leader's list
// while the window is at single-value resolution (one bits(e) value per
// bucket, at most kBins of them).  Each value's mass is then count x e
// exactly, so the crossing value e* and the number c of its members kept
// follow from counts alone (sampler.py:66-70: rank j is kept iff j == 0 or
// cum[j-1] <= top_p).  Members of one e* are ranked by scaled logit, then
// index; when they share one scaled logit (a tie group) the kept ones are
// the c of smallest index.  Members of e* with different scaled logits (they
// would have to lie within an ulp of e) set NS_STATUS_CAP_OVERFLOW and are
// taken in index order.  Whole cluster, three cluster barriers.  On return
// K.thr / K.thr_idx name the last kept member, this CTA's dropped members
// are zeroed in `vals`, its kept members' masses are added to ctl.wmass, and
// owner / tloc / zkept describe the draw.
__device__ __noinline__ void tie_resolve(const Geo& g, const Row& R, const Shared& sm, const Recv& rv, Keep& K,
                                         uint32_t win_lo, uint32_t win_hi, double z, double u, uint32_t lead,
                                         bool leader, int tid, uint32_t* status, int& owner, double& tloc,
                                         double& zkept) {
  Ctl& ctl = *sm.ctl;
  uint32_t* hist = sm.hist;
  float4* vals4 = reinterpret_cast<float4*>(sm.vals);
  double* scr = reinterpret_cast<double*>(sm.keys);  // kCap doubles of scratch
  const uint32_t* bitmap = sm.bitmap;
  const int lane = tid & 31, warp = tid >> 5;
  const uint32_t lo = max(win_lo, 1u);
  const uint32_t span_m1 = win_hi - lo;  // < kBins

  // A: this CTA's member counts by value, bucket win_hi - bits(e)
  for (int i = tid; i < kBins / 4; i += kThreads) reinterpret_cast<uint4*>(hist)[i] = make_uint4(0, 0, 0, 0);
  if (tid == 0) {
    ctl.misc_i = INT_MAX;
    ctl.misc_j = -1;
  }
  __syncthreads();
  for (int f = g.f_begin + lane; f < g.f_end; f += 32) {
    const float4 v = vals4[f];
    const float t[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint32_t bits = __float_as_uint(t[c]);
      if (bits - lo <= span_m1) atomicAdd(&hist[win_hi - bits], 1u);
    }
  }
  cluster_sync();  // every CTA's counts are complete

  // B: the leader finds e*, c, the CTA q holding the c-th member of e* and
  // the kept mass of every CTA, and broadcasts them
  if (leader) {
    double before = 0.0;
    for (int r = 0; r < kCluster; ++r) before += rv.rec_above[r];
    uint32_t cnt[8];
    double m[8], tot = 0.0;
    int last = -1;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int b = 8 * tid + j;
      cnt[j] = 0u;
      if ((uint32_t)b <= span_m1) {
        const uint32_t ad = smem_addr(&hist[b]);
#pragma unroll
        for (int r = 0; r < kCluster; ++r) cnt[j] += dsmem_ld_u32(dsmem_map(ad, r));
      }
      m[j] = (double)cnt[j] * (double)__uint_as_float(win_hi - (uint32_t)b);
      tot += m[j];
      if (cnt[j]) last = b;
    }
    const double incl = warp_incl_f64(tot, lane);
    if (lane == 31) scr[warp] = incl;
    if (last >= 0) atomicMax(&ctl.misc_j, last);
    __syncthreads();
    double run = before + incl - tot;
    for (int w = 0; w < warp; ++w) run += scr[w];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (cnt[j] && topp_crossed(run + m[j], z, R.p)) {
        atomicMin(&ctl.misc_i, 8 * tid + j);
        break;
      }
      run += m[j];
    }
    __syncthreads();
    const bool none = ctl.misc_i == INT_MAX;  // no crossing in the window: keep all of it
    const int bstar = none ? ctl.misc_j : ctl.misc_i;
    const uint32_t estar_bits = win_hi - (uint32_t)max(bstar, 0);
    // kept masses per CTA above e*, and the per-CTA counts of e*
    double acc[kCluster];
#pragma unroll
    for (int r = 0; r < kCluster; ++r) acc[r] = 0.0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int b = 8 * tid + j;
      if (b < bstar && cnt[j]) {
        const uint32_t ad = smem_addr(&hist[b]);
        const double e = (double)__uint_as_float(win_hi - (uint32_t)b);
#pragma unroll
        for (int r = 0; r < kCluster; ++r) acc[r] += (double)dsmem_ld_u32(dsmem_map(ad, r)) * e;
      }
    }
#pragma unroll
    for (int r = 0; r < kCluster; ++r) {
      const double s = warp_dsum(acc[r]);
      if (lane == 0) scr[32 + warp * kCluster + r] = s;
    }
    if (bstar >= 0 && tid == (bstar >> 3)) {
      // c: the smallest count of e* members whose inclusive mass crosses
      double pre = before + incl - tot;  // the mass before e*
      for (int w = 0; w < warp; ++w) pre += scr[w];
      for (int j = 0; j < (bstar & 7); ++j) pre += m[j];
      const uint32_t n = cnt[bstar & 7];
      const double e = (double)__uint_as_float(estar_bits);
      uint32_t c = n;
      if (!none) {
        uint32_t lo_c = 1u, hi_c = n;  // crossed(pre + hi_c * e) holds
        while (lo_c < hi_c) {
          const uint32_t mid = lo_c + (hi_c - lo_c) / 2u;
          if (topp_crossed(pre + (double)mid * e, z, R.p)) hi_c = mid;
          else lo_c = mid + 1u;
        }
        c = lo_c;
      }
      const uint32_t ad = smem_addr(&hist[bstar]);
      uint32_t prefix = 0u;
      int q = kCluster - 1;
      uint32_t cq = 0u;
      bool found = false;
      for (int r = 0; r < kCluster; ++r) {
        const uint32_t nr = dsmem_ld_u32(dsmem_map(ad, r));
        const uint32_t cr = c > prefix ? min(nr, c - prefix) : 0u;
        scr[32 + kWarps * kCluster + r] = (double)cr * e;
        if (!found && nr > 0u && prefix + nr >= c) {
          found = true;
          q = r;
          cq = c - prefix;
        }
        prefix += nr;
      }
      ctl.bc_q = q;
      ctl.bc_cq = (int32_t)cq;
    }
    __syncthreads();
    if (tid == 0) {
      double kept[kCluster], zk = 0.0;
      for (int r = 0; r < kCluster; ++r) {
        double s = rv.rec_above[r] + (bstar >= 0 ? scr[32 + kWarps * kCluster + r] : 0.0);
        for (int w = 0; w < kWarps; ++w) s += scr[32 + w * kCluster + r];
        kept[r] = s;
        zk += s;
      }
      int own;
      double t_own = 0.0;
      pick_owner(kept, u * zk, own, t_own);
      const int q = bstar >= 0 ? ctl.bc_q : -1;
      const int cq = bstar >= 0 ? ctl.bc_cq : 0;
      for (uint32_t r = 0; r < (uint32_t)kCluster; ++r) {
        dsmem_st_u32(dsmem_map(smem_addr(&ctl.bc_bits), r), bstar >= 0 ? estar_bits : 0u);
        dsmem_st_u32(dsmem_map(smem_addr(&ctl.bc_q), r), (uint32_t)q);
        dsmem_st_u32(dsmem_map(smem_addr(&ctl.bc_cq), r), (uint32_t)cq);
        dsmem_st_u32(dsmem_map(smem_addr(&ctl.bc_owner), r), (uint32_t)own);
        dsmem_st_f64(dsmem_map(smem_addr(&ctl.bc_tloc), r), t_own);
        dsmem_st_f64(dsmem_map(smem_addr(&ctl.bc_z), r), zk);
      }
    }
  }
  cluster_sync();  // decision delivered

  // C: CTA q finds the cq-th member of e* in index order (the threshold
  // element); every CTA reports the range of scaled logits among its e* members
  const uint32_t estar = ctl.bc_bits;
  const int q = ctl.bc_q;
  {
    float smin = INFINITY, smax = -INFINITY;
    uint32_t ncount = 0u;
    for (int f = g.f_begin + lane; f < g.f_end; f += 32) {
      const float4 v = vals4[f];
      const float t[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (__float_as_uint(t[c]) == estar && estar != 0u) {
          const float s = scaled(R, penalized_from_global(g, R, bitmap, 4 * f + c));
          smin = fminf(smin, s);
          smax = fmaxf(smax, s);
          ++ncount;
        }
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      smin = fminf(smin, __shfl_xor_sync(0xffffffffu, smin, o));
      smax = fmaxf(smax, __shfl_xor_sync(0xffffffffu, smax, o));
      ncount += __shfl_xor_sync(0xffffffffu, ncount, o);
    }
    float* fs = reinterpret_cast<float*>(scr);
    uint32_t* us = reinterpret_cast<uint32_t*>(scr) + 2 * kWarps;
    if (lane == 0) {
      fs[warp] = smin;
      fs[kWarps + warp] = smax;
      us[warp] = ncount;
    }
    __syncthreads();
    if (tid == 0) {
      float a = INFINITY, b = -INFINITY;
      for (int w = 0; w < kWarps; ++w) {
        a = fminf(a, fs[w]);
        b = fmaxf(b, fs[kWarps + w]);
      }
      dsmem_st_f32(dsmem_map(smem_addr(&ctl.tie_smin[g.rank]), lead), a);
      dsmem_st_f32(dsmem_map(smem_addr(&ctl.tie_smax[g.rank]), lead), b);
    }
    if ((int)g.rank == q) {
      // the warp holding the cq-th member walks its piece
      uint32_t target = (uint32_t)ctl.bc_cq;
      int wsel = -1;
      for (int w = 0; w < kWarps; ++w) {
        if (us[w] >= target) { wsel = w; break; }
        target -= us[w];
      }
      if (warp == wsel) {
        uint32_t run = 0u;
        for (int f0 = g.f_begin; f0 < g.f_end; f0 += 32) {
          const int f = f0 + lane;
          uint32_t mask = 0u;
          if (f < g.f_end) {
            const float4 v = vals4[f];
            const float t[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int c = 0; c < 4; ++c) mask |= (__float_as_uint(t[c]) == estar ? 1u : 0u) << c;
          }
          const uint32_t n = (uint32_t)__popc(mask);
          const uint32_t inc = warp_incl_u32(n, lane) + run;
          const uint32_t hit = __ballot_sync(0xffffffffu, inc >= target && inc - n < target);
          if (hit) {
            if (lane == __ffs(hit) - 1) {
              uint32_t k = target - (inc - n);  // 1-based within this lane's members
              int c = 0;
              for (; c < 4; ++c) {
                if ((mask >> c) & 1u) {
                  if (--k == 0u) break;
                }
              }
              const int local = 4 * f + c;
              const float s = scaled(R, penalized_from_global(g, R, bitmap, local));
              for (uint32_t r = 0; r < (uint32_t)kCluster; ++r) {
                dsmem_st_f32(dsmem_map(smem_addr(&ctl.bc_thr), r), s);
                dsmem_st_u32(dsmem_map(smem_addr(&ctl.bc_thr_idx), r), (uint32_t)(g.base + local));
              }
            }
            break;
          }
          run = __shfl_sync(0xffffffffu, inc, 31);
        }
      }
    }
    if (q < 0 && tid == 0) {
      // nothing in the window: keep it all (the threshold is the last member)
      ctl.bc_thr = -INFINITY;
      ctl.bc_thr_idx = INT_MAX;
    }
  }
  cluster_sync();  // threshold element and scaled-logit ranges delivered

  if (leader && tid == 0 && q >= 0) {
    float a = INFINITY, b = -INFINITY;
    for (int r = 0; r < kCluster; ++r) {
      a = fminf(a, ctl.tie_smin[r]);
      b = fmaxf(b, ctl.tie_smax[r]);
    }
    if (a != b && status) atomicOr(status, NS_STATUS_CAP_OVERFLOW);
  }
  K.thr = ctl.bc_thr;
  K.thr_idx = ctl.bc_thr_idx;
  owner = ctl.bc_owner;
  tloc = ctl.bc_tloc;
  zkept = ctl.bc_z;

  // D: drop this CTA's members ranked after the threshold element; add the
  // kept ones to this warp's mass
  double lane_kept = 0.0;
  for (int f = g.f_begin + lane; f < g.f_end; f += 32) {
    float4 v = vals4[f];
    float t[4] = {v.x, v.y, v.z, v.w};
    bool dirty = false;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint32_t bits = __float_as_uint(t[c]);
      if (bits - lo > span_m1) continue;
      bool keep = bits > estar;
      if (bits == estar) {
        const int local = 4 * f + c;
        const float s = scaled(R, penalized_from_global(g, R, bitmap, local));
        keep = s > K.thr || (s == K.thr && g.base + local <= K.thr_idx);
      }
      if (keep) {
        lane_kept += (double)t[c];
      } else {
        t[c] = 0.0f;
        dirty = true;
      }
    }
    if (dirty) vals4[f] = make_float4(t[0], t[1], t[2], t[3]);
  }
  const double wk = warp_dsum(lane_kept);
  if (lane == 0) ctl.wmass[warp] += wk;
  fence_proxy_async_smem();
  __syncthreads();
}

// Samples `row` (its inputs are in ctl.rin[par]).  Every path issues this
// warp's bulk copy of `next_row` as soon as the warp has finished with its
// piece of the slice and records that in `prefetched`; the caller issues it
// at the end of the row otherwise.
__device__ __forceinline__ void process_row(const NsSampleArgs& a, const Src& S, const Geo& g, const Shared& sm,
                                            int row, int next_row, uint32_t par, uint32_t lead, int tid,
                                            bool& prefetched) {
  const int lane = tid & 31, warp = tid >> 5;
  Ctl& ctl = *sm.ctl;
  Recv& rv = sm.recv[par];
  uint32_t* hist = sm.hist;
  uint32_t* bitmap = sm.bitmap;
  float* vals = sm.vals;
  float4* vals4 = reinterpret_cast<float4*>(vals);
  uint32_t* const status = a.status;
  prefetched = false;
  auto prefetch = [&]() {
    if (!prefetched) {
      prefetched = true;
      if (next_row >= 0) issue_chunk(S, g, ctl, vals, next_row, warp, lane);
    }
  };

  const RowIn& in = ctl.rin[par];
  Row R;
  R.row = row;
  R.lead = lead;
  const bool leader = (g.rank == lead);
  int64_t src = in.src;
  const bool bad_row = (src < 0 || src >= S.nrows);
  if (bad_row) src = 0;
  if (S.bf16) {
    R.src16 = reinterpret_cast<const __nv_bfloat16*>(S.logits) + src * S.stride;
    R.src32 = nullptr;
  } else {
    R.src32 = reinterpret_cast<const float*>(S.logits) + src * S.stride;
    R.src16 = nullptr;
  }
  const NsRowParams P = in.P;
  R.greedy = (P.flags & NS_ROW_GREEDY) != 0u;
  R.T = R.greedy ? 1.0f : P.temperature;
  R.rT = __frcp_rn(R.T);
  R.t_one = (R.T == 1.0f);
  R.topp = (P.flags & NS_ROW_TOP_P) != 0u;
  R.p = P.top_p;
  R.k = (P.top_k > 0 && P.top_k < g.V) ? P.top_k : 0;
  R.rp = P.repetition_penalty;
  const int64_t h0 = in.h[0], h1 = in.h[1];
  R.pen = (P.flags & NS_ROW_PENALTY) != 0u && a.history_offsets && h1 > h0;
  const bool debug = (a.out_filtered != nullptr) || (a.out_probs != nullptr);
  const int64_t out_off = (int64_t)row * g.V + g.base;
  float* pen_out = a.out_penalized ? a.out_penalized + out_off : nullptr;
  const bool out_i32 = (a.out_dtype == NS_OUT_I32);

  enum { kGreedy, kTopk, kGeneral };
  const int mode0 = (R.greedy && !debug) ? kGreedy : (R.k > 0 && R.k <= kTopkSmall) ? kTopk : kGeneral;

  // ---------------- per-row setup (the caller synchronised the CTA)
  if (tid == 0) ctl.mem_n = 0u;
  if (mode0 == kTopk)
    for (int i = tid; i < kTmBins / 8; i += kThreads) reinterpret_cast<uint4*>(hist)[i] = make_uint4(0, 0, 0, 0);
  if (R.pen) {
    for (int i = tid; i < (g.W + 31) / 32; i += kThreads) bitmap[i] = 0u;
    __syncthreads();
    uint32_t bad = 0;
    for (int64_t i = h0 + tid; i < h1; i += kThreads) {
      const int id = a.history_ids[i];
      if (id < 0 || id >= g.V) { bad = 1; continue; }
      const int local = id - g.base;
      if (local >= 0 && local < g.len) atomicOr(&bitmap[local >> 5], 1u << (local & 31));
    }
    if (bad && leader && status) atomicOr(status, NS_STATUS_BAD_HISTORY_ID);
  }
  __syncthreads();
  if (bad_row && leader && tid == 0 && status) atomicOr(status, NS_STATUS_BAD_SAMPLE_INDEX);

  // row uniform
  const double u = row_uniform(a, P, row);

  wait_chunk(g, ctl, warp, par, status);

  // ---------------- pass 1 (mode-specific statistics)
  float st_max = -INFINITY, st_min = INFINITY, st_amin = INFINITY;
  int st_amax = INT_MAX;
  if (mode0 == kTopk && !R.greedy) {
    for (int f = g.f_begin + lane; f < g.f_end; f += 32) {
      const float4 v = load_slot(g, R, vals, bitmap, f, pen_out);
      st_max = fmax_nan(st_max, fmax_nan(fmax_nan(v.x, v.y), fmax_nan(v.z, v.w)));
    }
  } else {
    const bool want_min = (mode0 == kGeneral);
    const bool want_amin = want_min && !R.t_one;
    for (int f = g.f_begin + lane; f < g.f_end; f += 32) {
      const float4 v = load_slot(g, R, vals, bitmap, f, pen_out);
      const float m4 = fmax_nan(fmax_nan(v.x, v.y), fmax_nan(v.z, v.w));
      if (m4 > st_max) {
        const int c = (v.x == m4) ? 0 : (v.y == m4) ? 1 : (v.z == m4) ? 2 : 3;
        st_amax = g.base + 4 * f + c;
      }
      st_max = fmax_nan(st_max, m4);
      if (want_min) st_min = fminf(st_min, fminf(fminf(v.x, v.y), fminf(v.z, v.w)));
      if (want_amin)
        st_amin = fminf(st_amin, fminf(fminf(fabsf(v.x), fabsf(v.y)), fminf(fabsf(v.z), fabsf(v.w))));
    }
    if (mode0 == kGreedy) prefetch();  // the slice is no longer needed
  }
  if (mode0 == kTopk) {
    // local histogram of thread maxima (u16 counts packed in u32 words)
    const uint32_t b = f2key(st_max) >> kTmShift;
    atomicAdd(&hist[b >> 1], 1u << ((b & 1u) << 4));
  }
  // CTA reduction: (max with NaN seen, first argmax, min, min |x|) via redux
  {
    const bool lane_nan = (st_max != st_max);
    const uint32_t kmax = lane_nan ? 0u : f2key(st_max);
    const uint32_t wk = __reduce_max_sync(0xffffffffu, kmax);
    const int wi = (int)__reduce_min_sync(0xffffffffu, (kmax == wk) ? (uint32_t)st_amax : 0x7fffffffu);
    const bool wnan = __any_sync(0xffffffffu, lane_nan);
    const uint32_t wmin = __reduce_min_sync(0xffffffffu, f2key(st_min));
    const uint32_t wamin = __reduce_min_sync(0xffffffffu, __float_as_uint(st_amin));
    if (lane == 0) {
      ctl.red_k[warp] = wnan ? 0xffffffffu : wk;
      ctl.red_i[warp] = wi;
      ctl.red_m[warp] = wmin;
      ctl.red_a[warp] = wamin;
    }
    __syncthreads();
    if (warp == 0) {
      const bool live = lane < kWarps;
      const uint32_t k = live ? ctl.red_k[lane] : 0u;
      const uint32_t ck = __reduce_max_sync(0xffffffffu, k);
      const int ci = (int)__reduce_min_sync(0xffffffffu, (live && k == ck) ? (uint32_t)ctl.red_i[lane] : 0x7fffffffu);
      const uint32_t cm = __reduce_min_sync(0xffffffffu, live ? ctl.red_m[lane] : 0xffffffffu);
      const uint32_t ca = __reduce_min_sync(0xffffffffu, live ? ctl.red_a[lane] : 0x7f800000u);
      if (lane < kCluster) {
        const uint32_t r = (uint32_t)lane;
        dsmem_st_u32(dsmem_map(smem_addr(&rv.rec_kmax[g.rank]), r), ck);
        dsmem_st_u32(dsmem_map(smem_addr(&rv.rec_kmin[g.rank]), r), cm);
        dsmem_st_u32(dsmem_map(smem_addr(&rv.rec_amin[g.rank]), r), ca);
        dsmem_st_u32(dsmem_map(smem_addr(&rv.rec_amax[g.rank]), r), (uint32_t)ci);
      }
    }
  }
  if (mode0 == kTopk) {
    for (int w = tid; w < kTmBins / 2; w += kThreads) {
      const uint32_t v = hist[w];
      if (v) {
        const uint32_t ad = smem_addr(&rv.tm_global[w]);
#pragma unroll
        for (int r = 0; r < kCluster; ++r) dsmem_red_add_u32(dsmem_map(ad, r), v);
      }
    }
  }
  cluster_sync();  // barrier 1: records (and maxima histograms) delivered

  uint32_t gk = 0u, gkmin = 0xffffffffu;
  float gamin = INFINITY;
  int gamax = INT_MAX;
  for (int r = 0; r < kCluster; ++r) {
    const uint32_t k = rv.rec_kmax[r];
    if (k > gk) { gk = k; gamax = rv.rec_amax[r]; }
    gkmin = min(gkmin, rv.rec_kmin[r]);
    gamin = fminf(gamin, rv.rec_amin[r]);
  }
  const bool gnan = (gk == 0xffffffffu);
  const float gmax = gnan ? __int_as_float(0x7fc00000) : key2f(gk);
  const float gmin = key2f(gkmin);
  if (gmax == -INFINITY) gamax = 0;

  // ---------------- rows whose softmax is NaN: uniform 1/V (sampler.py:76-80)
  if (gnan || gmax == INFINITY || gmax == -INFINITY) {
    prefetch();
    int tok = 0;
    if (R.greedy) {
      // torch.argmax: the first NaN, else the first +inf, else index 0.  The
      // penalty keeps NaN and +inf, so the raw logits in global memory decide.
      int my_nan = INT_MAX, my_pinf = INT_MAX;
      for (int i = tid; i < g.len; i += kThreads) {
        const float x = load_scalar(g, R, i);
        if (x != x) my_nan = min(my_nan, g.base + i);
        if (x == INFINITY) my_pinf = min(my_pinf, g.base + i);
      }
      my_nan = (int)__reduce_min_sync(0xffffffffu, (uint32_t)my_nan);
      my_pinf = (int)__reduce_min_sync(0xffffffffu, (uint32_t)my_pinf);
      if (lane == 0) { ctl.red_i[warp] = my_nan; ctl.red_j[warp] = my_pinf; }
      __syncthreads();
      if (tid < kCluster) {
        int n = INT_MAX, q = INT_MAX;
        for (int w = 0; w < kWarps; ++w) { n = min(n, ctl.red_i[w]); q = min(q, ctl.red_j[w]); }
        dsmem_st_u32(dsmem_map(smem_addr(&rv.rec_nan[g.rank]), tid), (uint32_t)n);
        dsmem_st_u32(dsmem_map(smem_addr(&rv.rec_pinf[g.rank]), tid), (uint32_t)q);
      }
      cluster_sync();
      int fn = INT_MAX, fp = INT_MAX;
      for (int r = 0; r < kCluster; ++r) { fn = min(fn, rv.rec_nan[r]); fp = min(fp, rv.rec_pinf[r]); }
      tok = (fn != INT_MAX) ? fn : (fp != INT_MAX) ? fp : 0;
    } else {
      tok = min(g.V - 1, (int)(u * (double)g.V));
    }
    if (leader && tid == 0) write_token(a.out_tokens, out_i32, row, tok);
    if (debug) {
      const float pu = 1.0f / (float)g.V;
      for (int i = tid; i < g.len; i += kThreads) {
        if (a.out_probs) a.out_probs[out_off + i] = pu;
        if (a.out_filtered) a.out_filtered[out_off + i] = scaled(R, penalized_from_global(g, R, bitmap, i));
      }
    }
    return;
  }

  // ================================================================ GREEDY
  if (mode0 == kGreedy) {
    if (leader && tid == 0) write_token(a.out_tokens, out_i32, row, gamax);
    return;
  }

  const uint32_t cand_n_lead = dsmem_map(smem_addr(&rv.cand_n), lead);
  bool need_min = false;

  // ================================================================ TOPK
  if (mode0 == kTopk) {
    {
      // thread t owns buckets [kTmBins-4(t+1), kTmBins-4t), scanned from the top
      uint32_t cnt[4];
      uint32_t s = 0;
      const int bhi = kTmBins - 1 - 4 * tid;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int b = bhi - j;
        cnt[j] = (rv.tm_global[b >> 1] >> ((b & 1) << 4)) & 0xFFFFu;
        s += cnt[j];
      }
      uint32_t tot;
      const uint32_t pre = block_excl_u32(ctl, s, tot, tid);
      if (pre < (uint32_t)R.k && pre + s >= (uint32_t)R.k) {
        uint32_t run = pre;
        for (int j = 0; j < 4; ++j) {
          run += cnt[j];
          if (run >= (uint32_t)R.k) { ctl.misc_i = bhi - j; break; }
        }
      }
      if (tid == 0 && tot < (uint32_t)R.k) ctl.misc_i = 0;
      __syncthreads();
    }
    const uint32_t bkey = (uint32_t)ctl.misc_i << kTmShift;
    float bound = (bkey < 0x00800000u) ? -INFINITY : key2f(bkey);
    bound = lower_preimage(R, bound);

    // every element >= bound goes to the leader (warp-aggregated slots)
    for (int f = g.f_begin + lane; f - lane < g.f_end; f += 32) {
      const bool live = f < g.f_end;
      const float4 v = live ? vals4[f] : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      const float m4 = fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w));
      if (!__any_sync(0xffffffffu, m4 >= bound)) continue;
      const float t[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const bool take = live && (4 * f + c < g.len) && (t[c] >= bound);
        const uint32_t bal = __ballot_sync(0xffffffffu, take);
        if (bal) {
          uint32_t slot0 = 0;
          const int first = __ffs(bal) - 1;
          if (lane == first) slot0 = dsmem_atom_add_u32(cand_n_lead, (uint32_t)__popc(bal));
          slot0 = __shfl_sync(0xffffffffu, slot0, first);
          if (take) {
            const uint32_t slot = slot0 + (uint32_t)__popc(bal & ((1u << lane) - 1u));
            if (slot < (uint32_t)kCap) {
              dsmem_st_f32(dsmem_map(smem_addr(&sm.cand_s[slot]), lead), scaled(R, t[c]));
              dsmem_st_u32(dsmem_map(smem_addr(&sm.cand_i[slot]), lead), (uint32_t)(g.base + 4 * f + c));
            } else if (slot == (uint32_t)kCap) {
              for (int r = 0; r < kCluster; ++r) dsmem_st_u32(dsmem_map(smem_addr(&rv.overflow), r), 1u);
            }
          }
        }
      }
    }
    cluster_sync();  // barrier 2: candidates delivered (and any overflow flagged everywhere)
    if (!rv.overflow) {
      prefetch();
      if (leader) {
        const int n = (int)rv.cand_n;
        float* cand_s = sm.cand_s;
        int32_t* cand_i = sm.cand_i;
        unsigned long long* keys = sm.keys;
        if (n == 0) {  // impossible while the bound holds; keep the kernel total anyway
          if (tid == 0) write_token(a.out_tokens, out_i32, row, gamax);
        } else {
          // candidates in rank order (value desc, index asc)
          for (int i = tid; i < n; i += kThreads) keys[i] = rank_key(cand_s[i], cand_i[i]);
          bitonic_sort(keys, n, tid);
          for (int r = tid; r < n; r += kThreads) {
            cand_s[r] = key_value(keys[r]);
            cand_i[r] = key_index(keys[r]);
          }
          __syncthreads();
          const float s0 = cand_s[0];
          const float thr = cand_s[min(R.k, n) - 1];
          if (tid == 0) { ctl.misc_i = n; ctl.token = INT_MAX; }
          __syncthreads();
          for (int r = tid; r < n; r += kThreads) {
            const bool in1 = cand_s[r] >= thr;
            const bool nxt = (r + 1 < n) && (cand_s[r + 1] >= thr);
            if (in1 && !nxt) ctl.misc_i = r + 1;
          }
          __syncthreads();
          const int n1 = ctl.misc_i;  // survivors of top-k (ties at the threshold kept)
          float* cand_e = sm.mem_e;   // masses by rank (the member list is unused on this path)
          for (int r = tid; r < n1; r += kThreads) cand_e[r] = exp_shifted(cand_s[r], s0);
          __syncthreads();
          int n2 = n1;
          if (warp == 0) {
            double z = 0.0;
            for (int c0 = 0; c0 < n1; c0 += 32) {
              const int r = c0 + lane;
              z += warp_dsum(r < n1 ? (double)cand_e[r] : 0.0);
            }
            int m2 = n1;
            if (R.topp) {
              double run = 0.0;
              int j0 = -1;
              for (int c0 = 0; c0 < n1 && j0 < 0; c0 += 32) {
                const int r = c0 + lane;
                const double inc = warp_incl_f64(r < n1 ? (double)cand_e[r] : 0.0, lane) + run;
                const uint32_t bal = __ballot_sync(0xffffffffu, r < n1 && topp_crossed(inc, z, R.p));
                if (bal) j0 = c0 + __ffs(bal) - 1;
                run = __shfl_sync(0xffffffffu, inc, 31);
              }
              // keep exactly ranks 0..j0 in (value desc, index asc) order
              if (j0 >= 0) m2 = j0 + 1;
              z = 0.0;
              for (int c0 = 0; c0 < m2; c0 += 32) {
                const int r = c0 + lane;
                z += warp_dsum(r < m2 ? (double)cand_e[r] : 0.0);
              }
            }
            if (lane == 0) { ctl.misc_i = m2; ctl.sel_z = z; }
          }
          __syncthreads();
          n2 = ctl.misc_i;
          const double z2 = ctl.sel_z;
          const double target = u * z2;
          // inverse CDF in vocabulary order over the kept ranks
          for (int r = tid; r < n2; r += kThreads) {
            const int ir = cand_i[r];
            const double er = (double)cand_e[r];
            double before = 0.0;
            for (int q = 0; q < n2; ++q)
              if (cand_i[q] < ir) before += (double)cand_e[q];
            if (er > 0.0 && before <= target && target < before + er) atomicMin(&ctl.token, ir);
          }
          __syncthreads();
          if (tid == 0) {
            int tok = ctl.token;
            if (tok == INT_MAX) {
              // target at the very top (rounding): the last kept element with mass
              int last = -1;
              for (int r = 0; r < n2; ++r)
                if (cand_e[r] > 0.f && cand_i[r] > last) last = cand_i[r];
              tok = last >= 0 ? last : cand_i[0];
            }
            if (R.greedy) tok = cand_i[0];
            write_token(a.out_tokens, out_i32, row, tok);
            if (debug) {
              for (int r = 0; r < kCluster; ++r) {
                dsmem_st_f32(dsmem_map(smem_addr(&ctl.bc_thr), r), cand_s[n2 - 1]);
                dsmem_st_u32(dsmem_map(smem_addr(&ctl.bc_thr_idx), r), (uint32_t)cand_i[n2 - 1]);
                dsmem_st_f32(dsmem_map(smem_addr(&ctl.bc_m), r), s0);
                dsmem_st_f64(dsmem_map(smem_addr(&ctl.bc_z), r), z2);
              }
            }
          }
        }
      }
      if (debug) {
        cluster_sync();  // barrier 3: leader's broadcast delivered
        const float thr2 = ctl.bc_thr, m = ctl.bc_m;
        const int thr_idx = ctl.bc_thr_idx;
        const double z = ctl.bc_z;
        for (int i = tid; i < g.len; i += kThreads) {
          const float s = scaled(R, penalized_from_global(g, R, bitmap, i));
          const bool kept = s > thr2 || (s == thr2 && g.base + i <= thr_idx);
          if (a.out_filtered) a.out_filtered[out_off + i] = kept ? s : -INFINITY;
          if (a.out_probs) a.out_probs[out_off + i] = kept ? (float)((double)exp_shifted(s, m) / z) : 0.0f;
        }
      }
      return;
    }
    // the candidate list overflowed: this row takes the (exact) general path
    need_min = true;
  }

  // ================================================================ GENERAL
  float gmin2 = gmin, gamin2 = gamin;
  if (need_min) {
    // statistics the TOPK pass did not gather: min and min |x|
    float mn = INFINITY, amn = INFINITY;
    for (int f = g.f_begin + lane; f < g.f_end; f += 32) {
      const float4 v = vals4[f];
      mn = fminf(mn, fminf(fminf(v.x, v.y), fminf(v.z, v.w)));
      amn = fminf(amn, fminf(fminf(fabsf(v.x), fabsf(v.y)), fminf(fabsf(v.z), fabsf(v.w))));
    }
    const uint32_t wm = __reduce_min_sync(0xffffffffu, f2key(mn));
    const uint32_t wa = __reduce_min_sync(0xffffffffu, __float_as_uint(amn));
    if (lane == 0) { ctl.red_m[warp] = wm; ctl.red_a[warp] = wa; }
    __syncthreads();
    if (tid < kCluster) {
      uint32_t m2 = 0xffffffffu, a2 = 0x7f800000u;
      for (int w = 0; w < kWarps; ++w) { m2 = min(m2, ctl.red_m[w]); a2 = min(a2, ctl.red_a[w]); }
      dsmem_st_u32(dsmem_map(smem_addr(&rv.rec_kmin[g.rank]), tid), m2);
      dsmem_st_u32(dsmem_map(smem_addr(&rv.rec_amin[g.rank]), tid), a2);
    }
    if (leader && tid == 0) rv.cand_n = 0u;
    cluster_sync();
    uint32_t km = 0xffffffffu;
    gamin2 = INFINITY;
    for (int r = 0; r < kCluster; ++r) { km = min(km, rv.rec_kmin[r]); gamin2 = fminf(gamin2, rv.rec_amin[r]); }
    gmin2 = key2f(km);
  }
  // The guard-free division needs every |x| of the row in [2^-40, 2^80] and T <= 2^20.
  const float gabsmax = fmaxf(fabsf(gmax), fabsf(gmin2));
  const bool fast_div = !R.t_one && gamin2 >= 0x1p-40f && gabsmax <= 0x1p+80f && R.T <= 0x1p+20f;
  Keep K;
  K.m = R.t_one ? gmax : __fdiv_rn(gmax, R.T);  // max scaled logit (division is monotone)
  K.have_thr_k = false;
  K.thr_k_s = -INFINITY;
  K.window = false;
  K.win_lo = K.win_hi = 0u;
  K.thr = -INFINITY;
  K.thr_idx = INT_MAX;
  const float min_s =
      (gmin2 < INFINITY && gmin2 > -INFINITY) ? (R.t_one ? gmin2 : __fdiv_rn(gmin2, R.T)) : -INFINITY;
  int hbuf = 0;

  // ---- large top-k: exact radix select of the k-th largest penalized logit
  if (R.k > 0) {
    uint32_t prefix = 0, krem = (uint32_t)R.k;
    const int shifts[3] = {21, 10, 0};
    const int widths[3] = {11, 11, 10};
    bool ok = true;
    for (int lvl = 0; lvl < 3; ++lvl) {
      const int sh = shifts[lvl], wd = widths[lvl];
      const uint32_t nbm = (1u << wd) - 1u;
      uint32_t* h = hist + hbuf * kRadixBins;
      for (int i = tid; i < kRadixBins; i += kThreads) h[i] = 0u;
      __syncthreads();
      for (int f = g.f_begin + lane; f < g.f_end; f += 32) {
        const float4 v = vals4[f];
        const float t[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if (4 * f + c >= g.len) continue;
          const uint32_t key = f2key(t[c]);
          if (lvl > 0 && (key >> (sh + wd)) != prefix) continue;
          atomicAdd(&h[nbm - ((key >> sh) & nbm)], 1u);
        }
      }
      __syncthreads();
      radix_crossing(ctl, h, hbuf, krem, tid);
      hbuf ^= 1;
      if (!ctl.sel_found) { ok = false; break; }
      krem -= ctl.sel_before_cnt;
      prefix = (prefix << wd) | (nbm - (uint32_t)ctl.sel_lo);
    }
    if (ok) {
      K.have_thr_k = true;
      K.thr_k_s = scaled(R, key2f(prefix));
    }
    cluster_sync();  // peers done reading the radix histograms
  }

  // ---- pass 2: e = exp(s - m) in place; locator histogram; lane masses
  const float e_lo = exp_shifted(K.have_thr_k ? fmaxf(min_s, K.thr_k_s) : min_s, K.m);
  int SH = 0;
  {
    const uint32_t D = (e_lo > 0.0f) ? (kOne - __float_as_uint(e_lo)) : kOne;
    while (SH < kMaxShift && (int64_t)((D + (1u << SH) - 1u) >> SH) > kBins - 2) ++SH;
  }
  const uint32_t KC = kOne - 1u + (1u << SH);
  const bool topp = R.topp;
  if (topp) {
    for (int i = tid; i < kBins / 4; i += kThreads) reinterpret_cast<uint4*>(hist)[i] = make_uint4(0, 0, 0, 0);
    __syncthreads();
  }
  float lane_z = 0.0f;
  {
    const float m = K.m, thr_k_s = K.thr_k_s;
    const bool have_thr_k = K.have_thr_k;
    for (int f = g.f_begin + lane; f < g.f_end; f += 32) {
      const float4 v = vals4[f];
      float t[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float s = R.t_one ? t[c] : (fast_div ? scaled_fast(R, t[c]) : div_by_const(t[c], R.T, R.rT));
        float e = exp_shifted(s, m);
        if (have_thr_k && !(s >= thr_k_s)) e = 0.0f;
        t[c] = e;
        lane_z = __fadd_rn(lane_z, e);
        if (topp) {
          const uint32_t bits = __float_as_uint(e);
          const int d = max(0, (int)(KC - bits));
          const uint32_t b = min((uint32_t)(kBins - 1), (uint32_t)d >> SH);
          atomicAdd(&hist[b], approx_mass16(bits));
        }
      }
      vals4[f] = make_float4(t[0], t[1], t[2], t[3]);
    }
  }
  {
    const double cz = cta_warp_sums(ctl, lane_z, lane, warp);  // ctl.wmass = per-warp totals
    if (tid == 0) ctl.cz[0] = cz;
    __syncthreads();
  }

  double zkept = 0.0;
  int owner = -1;
  double tloc = 0.0;
  bool crossed = false;
  uint32_t keep_lo = 1u;  // kept <=> bits(e) >= keep_lo and e > 0

  if (topp) {
    // ---- top-p locator: a window of buckets that must contain the boundary
    Level lv{KC, SH, true};
    uint32_t win_lo = 0, win_hi = 0;
    topp_window(ctl, hist, 0, lv, true, 0.0, R.p, tid);
    const double z = ctl.sel_z;
    for (int lvl = 0;; ++lvl) {
      if (!ctl.sel_found) break;
      win_lo = lv.lo_key(ctl.sel_hi);
      win_hi = lv.hi_key(ctl.sel_lo);
      crossed = true;
      if (ctl.sel_est <= 0.9f * (float)kCap || lv.sh == 0 || lvl >= 5) break;
      // refine inside [win_lo, win_hi]: finer buckets, exact mass above the window
      const uint32_t span = win_hi - win_lo + 1u;
      int sh2 = 0;
      while (((span + (1u << sh2) - 1u) >> sh2) > (uint32_t)(kBins - 1)) ++sh2;
      if (sh2 >= lv.sh) sh2 = lv.sh - 1;
      cluster_sync();  // peers done reading this level's histogram and sums
      for (int i = tid; i < kBins / 4; i += kThreads) reinterpret_cast<uint4*>(hist)[i] = make_uint4(0, 0, 0, 0);
      __syncthreads();
      float lane_above = 0.0f;
      for (int f = g.f_begin + lane; f < g.f_end; f += 32) {
        const float4 v = vals4[f];
        const float t[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t bits = __float_as_uint(t[c]);
          if (bits > win_hi) lane_above = __fadd_rn(lane_above, t[c]);
          else if (bits >= win_lo) atomicAdd(&hist[(win_hi - bits) >> sh2], approx_mass16(bits));
        }
      }
      {
        const double s = cta_warp_sums(ctl, lane_above, lane, warp);
        if (tid == 0) ctl.cz[1] = s;
        __syncthreads();
      }
      lv = Level{win_hi, sh2, false};
      topp_window(ctl, hist, 1, lv, false, z, R.p, tid);
    }
    cluster_sync();  // peers done reading the locator histograms
    if (crossed) {
      // ---- collection: exact mass above the window; window members -> leader
      float lane_above = 0.0f;
      for (int f = g.f_begin + lane; f - lane < g.f_end; f += 32) {
        const bool live = f < g.f_end;
        const float4 v = live ? vals4[f] : make_float4(0.f, 0.f, 0.f, 0.f);
        const float t[4] = {v.x, v.y, v.z, v.w};
        bool any_mem = false;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t bits = __float_as_uint(t[c]);
          if (bits > win_hi) lane_above = __fadd_rn(lane_above, t[c]);
          any_mem |= (bits >= win_lo && bits <= win_hi);
        }
        if (!__any_sync(0xffffffffu, any_mem)) continue;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t bits = __float_as_uint(t[c]);
          const bool take = live && bits >= win_lo && bits <= win_hi;
          const uint32_t bal = __ballot_sync(0xffffffffu, take);
          if (bal) {
            uint32_t slot0 = 0;
            const int first = __ffs(bal) - 1;
            if (lane == first) slot0 = dsmem_atom_add_u32(cand_n_lead, (uint32_t)__popc(bal));
            slot0 = __shfl_sync(0xffffffffu, slot0, first);
            if (take) {
              const uint32_t slot = slot0 + (uint32_t)__popc(bal & ((1u << lane) - 1u));
              const int local = 4 * f + c;
              const float s = scaled(R, penalized_from_global(g, R, bitmap, local));
              if (slot < (uint32_t)kCap) {
                dsmem_st_f32(dsmem_map(smem_addr(&sm.cand_s[slot]), lead), s);
                dsmem_st_u32(dsmem_map(smem_addr(&sm.cand_i[slot]), lead), (uint32_t)(g.base + local));
              }
              const uint32_t ms = atomicAdd(&ctl.mem_n, 1u);
              if (ms < (uint32_t)kCap) { sm.mem_s[ms] = s; sm.mem_i[ms] = local; sm.mem_e[ms] = t[c]; }
            }
          }
        }
      }
      {
        const double s = cta_warp_sums(ctl, lane_above, lane, warp);  // ctl.wmass = above masses
        if (tid == 0) dsmem_st_f64(dsmem_map(smem_addr(&rv.rec_above[g.rank]), lead), s);
      }
      cluster_sync();  // barrier: members and above-window masses delivered
      if (leader) {
        float* cand_s = sm.cand_s;
        int32_t* cand_i = sm.cand_i;
        unsigned long long* keys = sm.keys;
        const uint32_t ntot = rv.cand_n;
        const int n = (int)min(ntot, (uint32_t)kCap);
        for (int i = tid; i < n; i += kThreads) keys[i] = rank_key(cand_s[i], cand_i[i]);
        bitonic_sort(keys, n, tid);
        if (warp == 0) {
          double before = 0.0;
          for (int r = 0; r < kCluster; ++r) before += rv.rec_above[r];
          int j0 = -1;
          double run = before;
          if (ntot <= (uint32_t)kCap) {
            for (int c0 = 0; c0 < n && j0 < 0; c0 += 32) {
              const int r = c0 + lane;
              const float er = r < n ? exp_shifted(key_value(keys[r]), K.m) : 0.f;
              const double inc = warp_incl_f64((double)er, lane) + run;
              const uint32_t bal = __ballot_sync(0xffffffffu, r < n && er > 0.f && topp_crossed(inc, z, R.p));
              if (bal) j0 = c0 + __ffs(bal) - 1;
              run = __shfl_sync(0xffffffffu, inc, 31);
            }
          }
          if (j0 < 0) j0 = n - 1;  // no crossing inside (or overflow): keep the window
          const float thr = n > 0 ? key_value(keys[j0]) : -INFINITY;
          const int thr_idx = n > 0 ? key_index(keys[j0]) : INT_MAX;
          // kept mass per CTA: above-window mass + kept members (lane-strided, then combined)
          double kept[kCluster];
#pragma unroll
          for (int r = 0; r < kCluster; ++r) kept[r] = 0.0;
          for (int r = lane; r <= j0 && r < n; r += 32) {
            const unsigned long long kk = keys[r];
            const int owner_r = key_index(kk) / g.W;
            const double add = (double)exp_shifted(key_value(kk), K.m);
#pragma unroll
            for (int q = 0; q < kCluster; ++q)
              if (q == owner_r) kept[q] += add;
          }
          double zk = 0.0;
#pragma unroll
          for (int r = 0; r < kCluster; ++r) {
            kept[r] = warp_dsum(kept[r]) + rv.rec_above[r];
            zk += kept[r];
          }
          int own;
          double t_own = 0.0;
          pick_owner(kept, u * zk, own, t_own);
          // too many members, but one bits(e) value per bucket: exact by counts
          const bool tie = ntot > (uint32_t)kCap && lv.sh == 0 && (win_hi - win_lo) < (uint32_t)kBins;
          if (lane < kCluster) {
            const uint32_t r = (uint32_t)lane;
            dsmem_st_u32(dsmem_map(smem_addr(&ctl.bc_tie), r), tie ? 1u : 0u);
            dsmem_st_f32(dsmem_map(smem_addr(&ctl.bc_thr), r), thr);
            dsmem_st_u32(dsmem_map(smem_addr(&ctl.bc_thr_idx), r), (uint32_t)thr_idx);
            dsmem_st_u32(dsmem_map(smem_addr(&ctl.bc_owner), r), (uint32_t)own);
            dsmem_st_f64(dsmem_map(smem_addr(&ctl.bc_tloc), r), t_own);
            dsmem_st_f64(dsmem_map(smem_addr(&ctl.bc_z), r), zk);
          }
          if (ntot > (uint32_t)kCap && !tie && lane == 0 && status) atomicOr(status, NS_STATUS_CAP_OVERFLOW);
        }
      }
      cluster_sync();  // barrier: decision delivered
      K.window = true;
      K.win_lo = win_lo;
      K.win_hi = win_hi;
      keep_lo = win_lo;
      if (ctl.bc_tie) {
        tie_resolve(g, R, sm, rv, K, win_lo, win_hi, z, u, lead, leader, tid, status, owner, tloc, zkept);
      } else {
        K.thr = ctl.bc_thr;
        K.thr_idx = ctl.bc_thr_idx;
        owner = ctl.bc_owner;
        tloc = ctl.bc_tloc;
        zkept = ctl.bc_z;
        // drop this CTA's members ranked after the threshold element and add
        // the kept ones to the per-warp masses (fixed point: order-independent)
        if (tid < kWarps) ctl.wfix[tid] = 0ull;
        __syncthreads();
        const int nm = (int)min(ctl.mem_n, (uint32_t)kCap);
        for (int i = tid; i < nm; i += kThreads) {
          const float sm_s = sm.mem_s[i];
          const int li = sm.mem_i[i];
          if (sm_s < K.thr || (sm_s == K.thr && g.base + li > K.thr_idx)) {
            vals[li] = 0.0f;
          } else {
            const int w = min(kWarps - 1, (li >> 2) / g.chunk);
            atomicAdd(&ctl.wfix[w], (unsigned long long)llrint((double)sm.mem_e[i] * kFixedScale));
          }
        }
        fence_proxy_async_smem();  // the zeroed elements may sit in another warp's piece
        __syncthreads();
        if (tid < kWarps) ctl.wmass[tid] += (double)ctl.wfix[tid] * kFixedToReal;
        __syncthreads();
      }
    }
  }
  if (!topp || !crossed) {
    // plain sampling, large top-k alone, or a top-p that never crosses: draw over all e
    if (tid < kCluster) dsmem_st_f64(dsmem_map(smem_addr(&rv.rec_z[g.rank]), tid), ctl.cz[0]);
    cluster_sync();
    for (int r = 0; r < kCluster; ++r) zkept += rv.rec_z[r];
    pick_owner(rv.rec_z, u * zkept, owner, tloc);
  }

  // ---- the draw: the owning CTA picks a warp, the warp walks its piece of the slice
  if (R.greedy || owner < 0) {
    prefetch();
    if (leader && tid == 0) write_token(a.out_tokens, out_i32, row, gamax);
  } else if ((int)g.rank != owner) {
    prefetch();
  } else {
    int wsel;
    double tw = 0.0;
    pick_warp(ctl.wmass, tloc, wsel, tw);
    if (warp == wsel) {
      const int tok = walk_warp(g, vals4, wsel, keep_lo, tw, lane, gamax);
      if (lane == 0) write_token(a.out_tokens, out_i32, row, tok);
    }
    prefetch();
  }
  if (debug) {
    for (int i = tid; i < g.len; i += kThreads) {
      const float e = kept_mass(g, R, K, bitmap, i);
      if (a.out_probs) a.out_probs[out_off + i] = e > 0.f ? (float)((double)e / zkept) : 0.0f;
      if (a.out_filtered) {
        // a zero mass is filtered out only behind a crossed top-p boundary
        // (every positive mass ranks ahead of it); top-k alone keeps it
        const float s = scaled(R, penalized_from_global(g, R, bitmap, i));
        const bool keep = e > 0.f || (!K.window && (!K.have_thr_k || s >= K.thr_k_s));
        a.out_filtered[out_off + i] = keep ? s : -INFINITY;
      }
    }
  }
}

// ---------------------------------------------------------------- the kernel
__global__ void __launch_bounds__(kThreads, 2) sample_kernel(const NsSampleArgs a, int W, int tma_ok, int vec16_ok) {
  extern __shared__ __align__(128) unsigned char smem[];
  const Layout L = make_layout(W);
  Shared sm;
  sm.ctl = reinterpret_cast<Ctl*>(smem + L.ctl);
  sm.recv = reinterpret_cast<Recv*>(smem + L.recv);
  sm.hist = reinterpret_cast<uint32_t*>(smem + L.hist);
  sm.bitmap = reinterpret_cast<uint32_t*>(smem + L.bitmap);
  sm.cand_s = reinterpret_cast<float*>(smem + L.cand_s);
  sm.cand_i = reinterpret_cast<int32_t*>(smem + L.cand_i);
  sm.keys = reinterpret_cast<unsigned long long*>(smem + L.keys);
  sm.mem_s = reinterpret_cast<float*>(smem + L.mem_s);
  sm.mem_i = reinterpret_cast<int32_t*>(smem + L.mem_i);
  sm.mem_e = reinterpret_cast<float*>(smem + L.mem_e);
  sm.vals = reinterpret_cast<float*>(smem + L.vals);
  Ctl& ctl = *sm.ctl;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  Src S;
  S.logits = a.logits;
  S.sidx = a.sample_indices;
  S.nrows = a.num_logit_rows;
  S.stride = a.logits_row_stride;
  S.bf16 = (a.logits_dtype == NS_DTYPE_BF16);
  Geo g;
  g.rank = cluster_ctarank();
  g.V = a.vocab_size;
  g.W = W;
  g.base = (int)g.rank * W;
  g.len = max(0, min(W, g.V - g.base));
  g.nf4 = (g.len + 3) >> 2;
  g.full4 = g.len >> 2;
  g.chunk = max(1, (g.nf4 + kWarps - 1) / kWarps);
  g.f_begin = min(g.nf4, warp * g.chunk);
  g.f_end = min(g.nf4, g.f_begin + g.chunk);
  g.tma = tma_ok && !S.bf16;
  g.vec16 = vec16_ok && S.bf16;
  const int cid = blockIdx.x / kCluster;
  const int ncl = gridDim.x / kCluster;
  const int nrows = a.num_rows;

  // one-time setup: barriers, both receive areas, the first row's inputs
  if (tid == 0) {
    for (int w = 0; w < kWarps; ++w) mbar_init(&ctl.mbar[w], 1);
    fence_mbar_init();
  }
  {
    uint4* r4 = reinterpret_cast<uint4*>(sm.recv);
    for (int i = tid; i < (int)(2 * sizeof(Recv) / 16); i += kThreads) r4[i] = make_uint4(0, 0, 0, 0);
  }
  if (cid < nrows) {
    fetch_row_inputs(a, ctl.rin[0], ordered_row(a, cid, false), tid);
    if (tid < 4) cp_async_wait_all();
  }
  __syncthreads();
  cluster_sync();  // every CTA of the cluster runs and is initialised
  if (cid < nrows) issue_chunk(S, g, ctl, sm.vals, ordered_row(a, cid, false), warp, lane);

  uint32_t it = 0;
  for (int t = cid; t < nrows; t += ncl, ++it) {
    const int row = ordered_row(a, t, tid == 0 && g.rank == 0);
    __syncthreads();  // the previous row is finished in this CTA
    // clear what peers will write for the next row (they write it only after
    // this row's first cluster barrier, which waits for this CTA)
    {
      uint4* r4 = reinterpret_cast<uint4*>(&sm.recv[(it & 1u) ^ 1u]);
      for (int i = tid; i < (int)(sizeof(Recv) / 16); i += kThreads) r4[i] = make_uint4(0, 0, 0, 0);
    }
    const int next = (t + ncl < nrows) ? ordered_row(a, t + ncl, false) : -1;
    if (next >= 0) fetch_row_inputs(a, ctl.rin[(it & 1u) ^ 1u], next, tid);
    bool prefetched = false;
    process_row(a, S, g, sm, row, next, it & 1u, it & (kCluster - 1), tid, prefetched);
    if (!prefetched && next >= 0) issue_chunk(S, g, ctl, sm.vals, next, warp, lane);
    if (tid < 4) cp_async_wait_all();  // the next row's inputs have landed
  }
  cluster_sync();  // nobody leaves while a peer may still address its shared memory
}

// ---------------------------------------------------------------- host side
thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

struct DeviceState {
  size_t smem_set = 0;
  int max_clusters = 0;
  size_t clusters_for = 0;
};
std::mutex g_mu;
DeviceState g_dev[64];

// Batches of at least this many rows use the row kernel.
constexpr int kRowsMinBatch = 32;

int slice_width(int V) {
  const int W = (V + kCluster - 1) / kCluster;
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

int64_t ns_workspace_bytes(int32_t num_rows) { return ns::rows_workspace_bytes(num_rows); }

}  // extern "C"

namespace ns {

// One sampling step (ns_sample's body).  `noalloc`: the row kernel runs
// on the library's static workspace (ns_sample_noalloc).
static int sample_call(const NsSampleArgs* args, void* stream, bool noalloc) {
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
  const uintptr_t rp = reinterpret_cast<uintptr_t>(a.row_params);
  if (rp % 16 != 0) return fail(NS_ERR_INVALID_ARG, "ns_sample: row_params must be 16-byte aligned");
  if ((a.history_offsets && reinterpret_cast<uintptr_t>(a.history_offsets) % 8 != 0) ||
      (a.sample_indices && reinterpret_cast<uintptr_t>(a.sample_indices) % 8 != 0))
    return fail(NS_ERR_INVALID_ARG, "ns_sample: history_offsets / sample_indices must be 8-byte aligned");

  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return fail(NS_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(err));
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);

  if (a.kernel != NS_KERNEL_AUTO && a.kernel != NS_KERNEL_CLUSTER && a.kernel != NS_KERNEL_SPLIT)
    return fail(NS_ERR_INVALID_ARG, "ns_sample: kernel must be NS_KERNEL_AUTO, NS_KERNEL_CLUSTER or NS_KERNEL_SPLIT");
  // Kernel choice: the row kernel once the batch is large enough, the
  // cluster kernel otherwise (NsSampleArgs.kernel may force either).
  if (rows_supported(a) && (a.kernel == NS_KERNEL_SPLIT || (a.kernel == NS_KERNEL_AUTO && a.num_rows >= kRowsMinBatch))) {
    std::string msg;
    const int rc = noalloc ? rows_launch_noalloc(a, st, dev, msg) : rows_launch(a, st, dev, msg);
    return rc == NS_OK ? NS_OK : fail(rc, msg);
  }
  const int W = slice_width(a.vocab_size);
  const Layout L = make_layout(W);

  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;

  int max_clusters = 0;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (dev < 0 || dev >= 64) return fail(NS_ERR_UNSUPPORTED, "ns_sample: device ordinal >= 64");
    DeviceState& ds = g_dev[dev];
    if (ds.smem_set < L.total) {
      err = cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total);
      if (err != cudaSuccess)
        return fail(NS_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(err));
      ds.smem_set = L.total;
    }
    if (ds.clusters_for != L.total) {
      cfg.gridDim = dim3(kCluster, 1, 1);
      int n = 0;
      err = cudaOccupancyMaxActiveClusters(&n, sample_kernel, &cfg);
      if (err != cudaSuccess || n <= 0)
        return fail(NS_ERR_CUDA, std::string("cudaOccupancyMaxActiveClusters: ") +
                                     (err != cudaSuccess ? cudaGetErrorString(err) : "no cluster fits"));
      ds.max_clusters = n;
      ds.clusters_for = L.total;
    }
    max_clusters = ds.max_clusters;
  }
  const int clusters = a.num_rows < max_clusters ? a.num_rows : max_clusters;
  cfg.gridDim = dim3((unsigned)(clusters * kCluster), 1, 1);
  const uintptr_t p = reinterpret_cast<uintptr_t>(a.logits);
  const int tma_ok = (a.logits_dtype == NS_DTYPE_F32) && (p % 16 == 0) && (a.logits_row_stride % 4 == 0);
  const int vec16_ok = (a.logits_dtype == NS_DTYPE_BF16) && (p % 8 == 0) && (a.logits_row_stride % 4 == 0);
  err = cudaLaunchKernelEx(&cfg, sample_kernel, a, W, tma_ok, vec16_ok);
  if (err != cudaSuccess) return fail(NS_ERR_CUDA, std::string("sample kernel launch: ") + cudaGetErrorString(err));
  return NS_OK;
}

}  // namespace ns

extern "C" {

int ns_sample(const NsSampleArgs* args, void* stream) { return ns::sample_call(args, stream, false); }

int ns_sample_noalloc(const NsSampleArgs* args, void* stream) {
  using namespace ns;
  if (!args) return fail(NS_ERR_INVALID_ARG, "ns_sample_noalloc: args is NULL");
  return sample_call(args, stream, true);
}

}  // extern "C"

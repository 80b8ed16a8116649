// ns_row_core.cuh -- device building blocks of the row sampling kernel
// (ns_rows.cu): element formats, the row layout used by its whole-row passes,
// block reductions and sorts over the 512 consumer threads, the exact top-k
// radix select, the top-p window search, member decision and tie resolution,
// and the inverse-CDF draws.  Every function here runs on the block's 512
// consumer threads (warps 0-15) and synchronises them with csync(), a named
// barrier that the block's producer warp never joins.
//
// The semantics are those of nanoserve/scheduler/sampler.py:21-89: penalty
// :31-38, temperature :40-51, top-k :53-58, top-p :60-73, softmax and NaN
// guard :75-80, greedy :82-83, multinomial draw :84-89.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <climits>

#include "../../include/nanoserve_sampler.h"
#include "ns_device.cuh"

namespace ns {
namespace rk {

constexpr int kThreads = 512;             // consumer threads of a block
constexpr int kWarps = kThreads / 32;     // the row layout's warp ranges
constexpr int kPieceBytes = 512;          // one warp's share of a chunk in the row layout
constexpr int kBins = 4096;               // top-p locator histogram (u32 approximate masses)
constexpr int kRadixBins = 2048;          // radix-select level histogram (u32 counts)
constexpr int kTopkMax = 128;             // largest top_k served from per-part candidate lists
constexpr int kCandCap = 2048;            // block candidate / window-member list (u64 keys)
constexpr uint32_t kTopFine = 0x4F7FFFFFu;  // first locator level: e = exp(s - m0) in [2^-32, 2^32)
constexpr int kShFine = 17;                  // 1/64 binade per bucket
constexpr uint32_t kTopWide = 0x5F7FFFFFu;  // fallback level: e < 2^64, every normal float
constexpr int kShWide = 19;                  // 1/16 binade per bucket
constexpr double kSlack = 1.0 + 0x1p-11;  // > 1 / (1 - 2^-12): locator mass error bound
constexpr int kMinVocab = 24576;
constexpr int kMaxVocab = 196608;
constexpr int kStages = 6;                 // chunks per draw piece of a warp range
constexpr int kMaxChunks = (kMaxVocab / kWarps + 127) / 128;  // 512-byte pieces per warp range (fp32)
constexpr int kPiecesMax = (kMaxChunks + kStages - 1) / kStages;  // draw pieces per warp range
constexpr int kSub = 256;                  // top-p member sub-buckets

// Barrier of the 512 consumer threads (named barrier 1); the producer warp
// (warp 16) never takes part.
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, 512;" ::: "memory"); }

// ---------------------------------------------------------------- element formats
// 16 bytes of a row as logits.
struct EF32 {
  static constexpr uint32_t kNegInf2 = 0xFF800000u;  // a 32-bit word of -inf logits
  static constexpr int kEPT = 4;            // elements per thread per chunk
  static constexpr int kPiece = 32 * kEPT;  // elements per warp piece
  using Raw = float4;
  static __device__ __forceinline__ Raw zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }
  static __device__ __forceinline__ Raw lds(const unsigned char* p) { return *reinterpret_cast<const float4*>(p); }
  static __device__ __forceinline__ Raw lds_s(uint32_t a) {
    Raw r;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w) : "r"(a));
    return r;
  }
  static __device__ __forceinline__ Raw ldg(const char* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
  static __device__ __forceinline__ void unpack(const Raw& r, float (&x)[kEPT]) {
    x[0] = r.x;
    x[1] = r.y;
    x[2] = r.z;
    x[3] = r.w;
  }
};
struct EBF16 {
  static constexpr uint32_t kNegInf2 = 0xFF80FF80u;
  static constexpr int kEPT = 8;
  static constexpr int kPiece = 32 * kEPT;
  using Raw = uint4;
  static __device__ __forceinline__ Raw zero() { return make_uint4(0u, 0u, 0u, 0u); }
  static __device__ __forceinline__ Raw lds(const unsigned char* p) { return *reinterpret_cast<const uint4*>(p); }
  static __device__ __forceinline__ Raw lds_s(uint32_t a) {
    Raw r;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(a));
    return r;
  }
  static __device__ __forceinline__ Raw ldg(const char* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
  // bf16 -> fp32 is exact: the bf16 bits are the high half of the fp32 bits
  static __device__ __forceinline__ void unpack(const Raw& r, float (&x)[kEPT]) {
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      x[2 * q] = __uint_as_float(w[q] << 16);
      x[2 * q + 1] = __uint_as_float(w[q] & 0xffff0000u);
    }
  }
};

// ---------------------------------------------------------------- locator masses
// Approximate mass of one positive normal float: the top 13 of its 24
// significand bits.  All elements of one locator bucket share their binary
// exponent, so a bucket's sum of these values, scaled by 2^(exponent - 139),
// under-estimates its exact mass by less than a factor (1 - 2^-12); a bucket
// of up to 2^18 elements sums below 2^31.
__device__ __forceinline__ uint32_t approx_mass13(uint32_t bits) { return ((bits >> 11) & 0xfffu) | 0x1000u; }

// Bucket b of a locator level covers bits of e in [top - (b+1)*2^sh + 1,
// top - b*2^sh]; top + 1 is a multiple of 2^sh, so each bucket lies inside
// one binade.  Masses are added without a range test: indices past the last
// bucket are clamped into it, and where that happens (lump_last) its mass is
// left out of the search.
struct Level {
  uint32_t top;
  int sh;
  bool lump_last;  // the last bucket also holds everything below the level: its mass is unknown
  __device__ __forceinline__ uint32_t lo_key(int b) const {
    const uint64_t span = (uint64_t)(b + 1) << sh;
    return span > (uint64_t)top + 1u ? 0u : top - (uint32_t)span + 1u;
  }
  __device__ __forceinline__ uint32_t hi_key(int b) const { return top - ((uint32_t)b << sh); }
  __device__ __forceinline__ double mass(uint32_t sum13, int b) const {
    if (sum13 == 0u || (lump_last && b == kBins - 1)) return 0.0;
    // sum13 * 2^(exponent - 139), the power of two built from its bits
    const int ex = (int)(lo_key(b) >> 23) - 139 + 1023;
    return (double)sum13 * __longlong_as_double((long long)ex << 52);
  }
};

// ---------------------------------------------------------------- shared state
// Per-row working state of the finishing passes.
struct __align__(16) Ctl {
  double seg[kWarps];        // kept mass per warp range
  double piece[kMaxChunks];  // kept mass per piece of the drawn warp range
  double pm[kWarps][kPiecesMax];  // top-p: kept mass per kStages-chunk piece of every warp range
  unsigned long long dec_key;     // top-p: rank key of the last kept member
  uint32_t red_k[kWarps];
  uint32_t red_b[kWarps];
  int32_t red_i[kWarps];
  int32_t red_j[kWarps];
  uint32_t red_u[kWarps];
  uint32_t red_o[kWarps];
  double red_e[kWarps];
  double pick_t;
  double dec_z;
  float sel_est;
  int sel_found;
  int sel_lo;
  int sel_hi;
  uint32_t sel_before;
  int pick;
  uint32_t cand_n;
  uint32_t list_n;
  int misc;
  int misc2;
  int token;
  float dec_thr;
  int dec_thr_idx;
};

struct Sh {
  Ctl* ctl;
  uint32_t* bitmap;          // penalty bitmap, one bit per vocabulary id
  unsigned long long* cand;  // candidates / top-p window members (kCandCap keys)
  uint32_t* hist;            // locator or radix histogram (kBins u32); also a sorted u64 list
  unsigned long long* small; // 32 keys: a crossing sub-bucket
};

// One row being sampled, with the row layout shared by every row.
// Repetition penalty of a row: rp and RN(1/rp).
struct Pen {
  float rp;
  double inv;  // RN64(1 / rp)
  __device__ static Pen of(float rp) { return Pen{rp, __drcp_rn((double)rp)}; }
};

struct RowCtx {
  const char* src;
  int V, W, nch, row;
  float T, rT, rp, p;
  double invT;  // RN64(1 / T): scaled() divides with no out-of-line call
  Pen pp;
  int k;  // top-k (0: none)
  bool t_one, greedy, topp, pen;
};

// This thread's place in the row layout (the same for every row).
struct Lane {
  int tid, lane, warp;
  int base;  // element index of this thread's first element in chunk 0
  int nv;    // chunks in which this thread holds elements
  int nvw;   // chunks in which every lane of this warp holds elements
};

template <class E>
__device__ __forceinline__ Lane make_lane(int V, int W, int tid) {
  Lane ln;
  ln.tid = tid;
  ln.lane = tid & 31;
  ln.warp = tid >> 5;
  ln.base = ln.warp * W + ln.lane * E::kEPT;
  const int ww = max(0, min(W, V - ln.warp * W));  // this warp's range length
  ln.nv = ww > ln.lane * E::kEPT ? (ww - ln.lane * E::kEPT + E::kPiece - 1) / E::kPiece : 0;
  ln.nvw = ww > 31 * E::kEPT ? (ww - 31 * E::kEPT + E::kPiece - 1) / E::kPiece : 0;
  return ln;
}

// This thread's bytes of row `src` in the row layout (16-byte aligned: the
// host admits only such rows).
template <class E>
__device__ __forceinline__ const char* lane_src(const char* src, const Lane& ln) {
  return src + (size_t)ln.base * (sizeof(typename E::Raw) / E::kEPT);
}

enum { kGreedy = 0, kTopk = 1, kGeneral = 2 };

__device__ __forceinline__ int row_mode(const NsRowParams& P, int V, bool debug) {
  const bool greedy = (P.flags & NS_ROW_GREEDY) != 0u;
  if (greedy && !debug) return kGreedy;
  const int k = (P.top_k > 0 && P.top_k < V) ? P.top_k : 0;
  return (k > 0 && k <= kTopkMax) ? kTopk : kGeneral;
}

__device__ __forceinline__ float scaled(const RowCtx& R, float x) {
  return R.t_one ? x : div_by_row_const(x, R.T, R.invT);
}

// Smallest float c <= b with RN(c/T) == RN(b/T): the lower end of the set of
// logits whose scaled value is at least RN(b/T).
__device__ __noinline__ float lower_preimage(float b, bool t_one, float T, float rT) {
  if (t_one || !(b > -INFINITY) || !(b < INFINITY)) return b;
  const float target = div_by_const(b, T, rT);
  float c = b;
  for (int i = 0; i < 64; ++i) {
    const float d = nextafterf(c, -INFINITY);
    if (div_by_const(d, T, rT) == target) c = d; else return c;
  }
  return -INFINITY;
}

// The thread's 16 bytes of a row as penalized logits (sampler.py:31-38).
template <class E, bool PEN>
__device__ __forceinline__ void penalized(const uint32_t* bitmap, Pen pp, const typename E::Raw& raw, int idx0,
                                          float (&x)[E::kEPT], bool live = true) {
  E::unpack(raw, x);
  if (PEN && live) {
    const uint32_t m = (bitmap[idx0 >> 5] >> (idx0 & 31)) & ((1u << E::kEPT) - 1u);
    if (m) {
#pragma unroll
      for (int j = 0; j < E::kEPT; ++j)
        if ((m >> j) & 1u) x[j] = penalize(x[j], pp.rp, pp.inv);
    }
  }
}

// Calls f(c, x, idx0, live) for every chunk c of the row with this thread's
// penalized logits, re-read from global memory (eight chunks in flight).
template <class E, class F>
__device__ __forceinline__ void global_pass(const RowCtx& R, const uint32_t* bitmap, int tid, F&& f) {
  constexpr int EPT = E::kEPT, U = 8;
  const Lane ln = make_lane<E>(R.V, R.W, tid);
  const char* src = lane_src<E>(R.src, ln);
  for (int c0 = 0; c0 < R.nch; c0 += U) {
    typename E::Raw raw[U];
#pragma unroll
    for (int u = 0; u < U; ++u) raw[u] = (c0 + u < ln.nv) ? E::ldg(src + (c0 + u) * kPieceBytes) : E::zero();
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = c0 + u;
      if (c < R.nch) {
        const int idx0 = ln.base + c * E::kPiece;
        const bool live = c < ln.nv;
        float x[EPT];
        if (live) {
          if (R.pen) penalized<E, true>(bitmap, R.pp, raw[u], idx0, x);
          else penalized<E, false>(bitmap, R.pp, raw[u], idx0, x);
        } else {
#pragma unroll
          for (int j = 0; j < EPT; ++j) x[j] = -INFINITY;
        }
        f(c, x, idx0, live);
      }
    }
  }
}

// ---------------------------------------------------------------- block reductions
// Block-wide exclusive scan of one u32 per thread (thread 0 first).
__device__ __forceinline__ uint32_t block_excl_u32(Ctl& ctl, uint32_t v, uint32_t& total, int tid) {
  const int lane = tid & 31, warp = tid >> 5;
  const uint32_t inc = warp_incl_u32(v, lane);
  if (lane == 31) ctl.red_u[warp] = inc;
  csync();
  uint32_t wpre = 0, tot = 0;
  for (int w = 0; w < kWarps; ++w) {
    const uint32_t x = ctl.red_u[w];
    if (w < warp) wpre += x;
    tot += x;
  }
  csync();
  total = tot;
  return wpre + inc - v;
}

__device__ __forceinline__ double block_dsum(Ctl& ctl, double v, int tid) {
  const double w = warp_dsum(v);
  if ((tid & 31) == 0) ctl.red_e[tid >> 5] = w;
  csync();
  double s = 0.0;
  for (int i = 0; i < kWarps; ++i) s += ctl.red_e[i];
  csync();
  return s;
}

// Per-warp-range totals of per-thread masses into ctl.seg, and their sum.
__device__ __forceinline__ double block_segments(Ctl& ctl, double v, int tid) {
  const double w = warp_dsum(v);
  if ((tid & 31) == 0) ctl.seg[tid >> 5] = w;
  csync();
  double s = 0.0;
  for (int i = 0; i < kWarps; ++i) s += ctl.seg[i];
  csync();
  return s;
}

// Row statistics after the first pass: NaN-propagating maximum with its first
// index, the row total of the per-thread masses `z` (also kept per warp range
// in ctl.seg) and whether any e left the locator level above (flag bit 0) or
// below (bit 1).
struct Stats {
  float mx;
  bool nan;
  int arg;
  double z;
  bool over;
  bool lumped;
};
__device__ __forceinline__ Stats block_stats(Ctl& ctl, float v, int arg, double z, uint32_t flags, int tid) {
  const int lane = tid & 31, warp = tid >> 5;
  const bool nan = (v != v);
  const uint32_t k = nan ? 0u : f2key(v);
  const uint32_t wk = __reduce_max_sync(0xffffffffu, k);
  const uint32_t wi = __reduce_min_sync(0xffffffffu, k == wk ? (uint32_t)arg : 0x7fffffffu);
  const bool wn = __any_sync(0xffffffffu, nan);
  const uint32_t wo = __reduce_or_sync(0xffffffffu, flags);
  const double wz = warp_dsum(z);
  if (lane == 0) {
    ctl.red_k[warp] = wn ? 0xffffffffu : wk;
    ctl.red_i[warp] = (int)wi;
    ctl.red_o[warp] = wo;
    ctl.seg[warp] = wz;
  }
  csync();
  uint32_t ck = 0u, co = 0u;
  int ci = INT_MAX;
  double cz = 0.0;
  for (int w = 0; w < kWarps; ++w) {
    const uint32_t kk = ctl.red_k[w];
    if (kk > ck) {
      ck = kk;
      ci = ctl.red_i[w];
    } else if (kk == ck) {
      ci = min(ci, ctl.red_i[w]);
    }
    co |= ctl.red_o[w];
    cz += ctl.seg[w];
  }
  csync();
  Stats S;
  S.nan = (ck == 0xffffffffu);
  S.mx = S.nan ? __int_as_float(0x7fc00000) : key2f(ck);
  S.arg = ci;
  S.z = cz;
  S.over = (co & 1u) != 0u;
  S.lumped = (co & 2u) != 0u;
  return S;
}

// Bitonic sorting of up to kCandCap 64-bit keys.  Every stage with stride
// below 128 runs inside one warp on a 128-key segment held in registers
// (element i = base + 32 r + lane), so only strides >= 128 need the block.
__device__ __forceinline__ void cmpx_regs(unsigned long long& a, unsigned long long& b, bool up) {
  const bool sw = (a > b) == up;
  const unsigned long long t = a;
  a = sw ? b : a;
  b = sw ? t : b;
}
__device__ __forceinline__ void cmpx_lanes(unsigned long long& v, int j, bool up, int lane) {
  const unsigned long long o = __shfl_xor_sync(0xffffffffu, v, j);
  const bool lower = (lane & j) == 0;
  v = (lower == up) ? (v < o ? v : o) : (v < o ? o : v);
}
// Stages j = 64 .. 1 of bitonic level k on one segment.
__device__ __forceinline__ void seg_merge(unsigned long long (&v)[4], int base, int lane, int k) {
  bool up[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) up[r] = ((base + 32 * r + lane) & k) == 0;
  cmpx_regs(v[0], v[2], up[0]);
  cmpx_regs(v[1], v[3], up[1]);
  cmpx_regs(v[0], v[1], up[0]);
  cmpx_regs(v[2], v[3], up[2]);
#pragma unroll
  for (int j = 16; j > 0; j >>= 1) {
#pragma unroll
    for (int r = 0; r < 4; ++r) cmpx_lanes(v[r], j, up[r], lane);
  }
}
// Levels k = 2 .. 128 on one segment (ascending or descending by bit 128 of base).
__device__ __forceinline__ void seg_sort(unsigned long long (&v)[4], int base, int lane) {
#pragma unroll
  for (int k = 2; k <= 128; k <<= 1) {
    bool up[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) up[r] = ((base + 32 * r + lane) & k) == 0;
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j == 64) {
        cmpx_regs(v[0], v[2], up[0]);
        cmpx_regs(v[1], v[3], up[1]);
      } else if (j == 32) {
        cmpx_regs(v[0], v[1], up[0]);
        cmpx_regs(v[2], v[3], up[2]);
      } else {
#pragma unroll
        for (int r = 0; r < 4; ++r) cmpx_lanes(v[r], j, up[r], lane);
      }
    }
  }
}

// Sort keys[0, n) ascending in place (n <= kCandCap; the buffer holds
// kCandCap keys).  Whole block; ends with a barrier.
__device__ __forceinline__ void sort_keys(unsigned long long* keys, int n, int tid) {
  const int lane = tid & 31, warp = tid >> 5;
  int np = 128;
  while (np < n) np <<= 1;
  for (int i = n + tid; i < np; i += kThreads) keys[i] = ~0ull;
  csync();
  const int nseg = np >> 7;
  unsigned long long v[4];
  if (warp < nseg) {
    const int base = warp << 7;
#pragma unroll
    for (int r = 0; r < 4; ++r) v[r] = keys[base + 32 * r + lane];
    seg_sort(v, base, lane);
#pragma unroll
    for (int r = 0; r < 4; ++r) keys[base + 32 * r + lane] = v[r];
  }
  csync();
  for (int k = 256; k <= np; k <<= 1) {
    for (int j = k >> 1; j >= 128; j >>= 1) {
      for (int i = tid; i < np; i += kThreads) {
        const int l = i ^ j;
        if (l > i) {
          const unsigned long long a = keys[i], b = keys[l];
          if ((a > b) == ((i & k) == 0)) {
            keys[i] = b;
            keys[l] = a;
          }
        }
      }
      csync();
    }
    if (warp < nseg) {
      const int base = warp << 7;
#pragma unroll
      for (int r = 0; r < 4; ++r) v[r] = keys[base + 32 * r + lane];
      seg_merge(v, base, lane, k);
#pragma unroll
      for (int r = 0; r < 4; ++r) keys[base + 32 * r + lane] = v[r];
    }
    csync();
  }
}

// Append keys to a block-shared list (warp-aggregated slots); entries past
// `cap` are counted but dropped.
__device__ __forceinline__ void list_append(unsigned long long* list, uint32_t* count, bool take,
                                            unsigned long long key, int cap, int lane) {
  const uint32_t bal = __ballot_sync(0xffffffffu, take);
  if (bal) {
    const int first = __ffs(bal) - 1;
    uint32_t base = 0;
    if (lane == first) base = atomicAdd(count, (uint32_t)__popc(bal));
    base = __shfl_sync(0xffffffffu, base, first);
    if (take) {
      const uint32_t slot = base + (uint32_t)__popc(bal & ((1u << lane) - 1u));
      if (slot < (uint32_t)cap) list[slot] = key;
    }
  }
}

// ---------------------------------------------------------------- radix select
// k-th largest penalized logit by a 3-level radix select over its key
// (11/11/10 bits), re-reading the row three times.  Whole block.
template <class E>
__device__ __forceinline__ float radix_select(const RowCtx R, const Sh sh, int tid) {
  Ctl& ctl = *sh.ctl;
  uint32_t* h = sh.hist;
  uint32_t prefix = 0u, krem = (uint32_t)R.k;
  const int shifts[3] = {21, 10, 0};
  const int widths[3] = {11, 11, 10};
  for (int lvl = 0; lvl < 3; ++lvl) {
    const int shl = shifts[lvl], wd = widths[lvl];
    const uint32_t nbm = (1u << wd) - 1u;
    for (int b = tid; b < kRadixBins; b += kThreads) h[b] = 0u;
    csync();
    if (tid == 0) ctl.misc = -1;
    global_pass<E>(R, sh.bitmap, tid, [&](int, const float(&x)[E::kEPT], int, bool live) {
      if (!live) return;
#pragma unroll
      for (int j = 0; j < E::kEPT; ++j) {
        const uint32_t key = f2key(x[j]);
        if (lvl > 0 && (key >> (shl + wd)) != prefix) continue;
        atomicAdd(&h[nbm - ((key >> shl) & nbm)], 1u);
      }
    });
    csync();
    // bucket 0 holds the largest keys; thread t owns buckets [4t, 4t+4)
    uint32_t cnt[4], s = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      cnt[j] = h[4 * tid + j];
      s += cnt[j];
    }
    uint32_t tot;
    const uint32_t pre = block_excl_u32(ctl, s, tot, tid);
    if (pre < krem && pre + s >= krem) {
      uint32_t run = pre;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (run + cnt[j] >= krem) {
          ctl.misc = 4 * tid + j;
          ctl.sel_before = run;
          break;
        }
        run += cnt[j];
      }
    }
    csync();
    const int b = ctl.misc;
    if (b < 0) return -INFINITY;  // fewer than k elements (k < V makes this impossible)
    krem -= ctl.sel_before;
    prefix = (prefix << wd) | (nbm - (uint32_t)b);
    csync();
  }
  return key2f(prefix);
}

// ---------------------------------------------------------------- top-p window
// Reference rule (sampler.py:66-70): sorted rank j is kept iff j == 0 or
// float32(cum[j-1]) <= top_p; with thr = topp_threshold(z, top_p) the rank
// whose inclusive mass first exceeds thr is the last one kept.  Finds the
// bucket window [lo, hi] of level `lv` that must contain that rank, given
// that each bucket's approximate mass is within a factor (1 - 2^-12) of its
// exact mass: lo is the first bucket whose inclusive mass times kSlack passes
// thr, hi the first whose inclusive mass does (the level's last bucket when
// none does).  `base` is the exact mass above the level's range.  Also sets
// an estimate of the number of elements in the window.  Whole block: thread
// t owns buckets [8t, 8t + 8) and one block scan orders them.
__device__ __forceinline__ void topp_window(Ctl* ctlp, const uint32_t* h, const Level lv, double base, double thr,
                                         int tid) {
  constexpr int kPer = kBins / kThreads;
  static_assert(kPer == 8, "two 16-byte loads per thread");
  Ctl& ctl = *ctlp;
  const int lane = tid & 31, warp = tid >> 5;
  const uint4 q0 = reinterpret_cast<const uint4*>(h)[2 * tid];
  const uint4 q1 = reinterpret_cast<const uint4*>(h)[2 * tid + 1];
  const uint32_t v[kPer] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
  double m[kPer], tot = 0.0;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    m[j] = lv.mass(v[j], kPer * tid + j);
    tot += m[j];
  }
  const double inc = warp_incl_f64(tot, lane);
  if (lane == 31) ctl.red_e[warp] = inc;
  if (tid == 0) {
    ctl.misc = INT_MAX;
    ctl.misc2 = INT_MAX;
  }
  csync();
  double run = base + (inc - tot);
  for (int w = 0; w < warp; ++w) run += ctl.red_e[w];
  int lo = INT_MAX, hi = INT_MAX;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    run += m[j];
    if (lo == INT_MAX && run * kSlack > thr) lo = kPer * tid + j;
    if (hi == INT_MAX && run > thr) hi = kPer * tid + j;
  }
  if (lo != INT_MAX) atomicMin(&ctl.misc, lo);
  if (hi != INT_MAX) atomicMin(&ctl.misc2, hi);
  csync();
  const bool found = ctl.misc != INT_MAX;
  const int fh = ctl.misc2 == INT_MAX ? kBins - 1 : ctl.misc2;
  const int fl = found ? min(ctl.misc, fh) : 0;
  // elements in the window ~ mass / smallest value of the bucket
  double est = 0.0;
  if (found) {
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int b = kPer * tid + j;
      const float e_bot = __uint_as_float(lv.lo_key(b));
      if (b >= fl && b <= fh && m[j] > 0.0 && e_bot > 0.0f) est += (double)__fdividef((float)m[j], e_bot);
    }
  }
  est = warp_dsum(est);
  if (lane == 0) ctl.red_e[warp] = est;
  csync();
  if (tid == 0) {
    double e = 0.0;
    for (int w = 0; w < kWarps; ++w) e += ctl.red_e[w];
    ctl.sel_found = found;
    ctl.sel_lo = found ? fl : 0;
    ctl.sel_hi = found ? fh : 0;
    ctl.sel_est = found ? (float)(e * 1.001 + 1.0) : 0.0f;
  }
  csync();
}

// ---------------------------------------------------------------- the draw
// Which elements survive filtering, and their masses e = exp(s - m0).
struct Keep {
  float m0;
  bool have_k;  // top-k by threshold: s >= thr_k
  float thr_k;
  bool window;  // top-p decided inside [win_lo, win_hi]
  uint32_t win_lo, win_hi;
  float thr;    // last kept (s, idx) inside the window
  int thr_idx;
  __device__ __forceinline__ float mass(float s) const {
    return (have_k && !(s >= thr_k)) ? 0.0f : exp_shifted(s, m0);
  }
  __device__ __forceinline__ bool kept(float s, float e, int idx) const {
    if (have_k && !(s >= thr_k)) return false;
    if (!window) return true;
    const uint32_t bits = __float_as_uint(e);
    if (bits > win_hi) return true;
    if (bits < win_lo || bits == 0u) return false;
    return s > thr || (s == thr && idx <= thr_idx);
  }
};

// Kept masses of 16 bytes of logits (`valid` false: all zero).
template <class E>
__device__ __forceinline__ void kept_masses(const RowCtx& R, const uint32_t* bitmap, const Keep& K,
                                            const typename E::Raw& raw, int idx0, bool valid, float (&q)[E::kEPT]) {
  if (valid) {
    float x[E::kEPT];
    if (R.pen) penalized<E, true>(bitmap, R.pp, raw, idx0, x);
    else penalized<E, false>(bitmap, R.pp, raw, idx0, x);
#pragma unroll
    for (int j = 0; j < E::kEPT; ++j) {
      const float s = scaled(R, x[j]);
      const float e = K.mass(s);
      q[j] = (e > 0.f && K.kept(s, e, idx0 + j)) ? e : 0.f;
    }
  } else {
#pragma unroll
    for (int j = 0; j < E::kEPT; ++j) q[j] = 0.f;
  }
}

// The inverse-CDF draw in vocabulary order over the kept masses, whole block:
// the warp range whose mass prefix (ctl.seg) passes `target`, then the piece
// inside it (masses recomputed from a re-read of the range), then the
// element, walked by warp 0.  Falls back to the last kept element when
// rounding leaves the target past the total, then to `fallback`.
template <class E>
__device__ __forceinline__ int draw_token(const RowCtx R, const Sh sh, const Keep K, double target, int fallback,
                                       int tid) {
  constexpr int kPer = (kMaxChunks + kWarps - 1) / kWarps;  // pieces per warp at most
  Ctl& ctl = *sh.ctl;
  const int lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    double run = 0.0, t = 0.0;
    int pick = -1, last = -1;
    for (int w = 0; w < kWarps; ++w) {
      const double m = ctl.seg[w];
      if (m > 0.0) last = w;
      if (pick < 0 && m > 0.0 && target < run + m) {
        pick = w;
        t = target - run;
      }
      run += m;
    }
    if (pick < 0) {
      pick = last;
      t = 1e300;
    }
    ctl.pick = pick;
    ctl.pick_t = t;
  }
  csync();
  const int wr = ctl.pick;
  const double t1 = ctl.pick_t;
  if (wr < 0) return fallback;
  const int ww = max(0, min(R.W, R.V - wr * R.W));
  const int npieces = (ww + E::kPiece - 1) / E::kPiece;
  const char* base = R.src + (size_t)wr * R.W * (sizeof(typename E::Raw) / E::kEPT);
  {
    // piece masses: warp w takes pieces w, w + 16, ...; all loads first
    typename E::Raw raw[kPer];
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      const int off = (warp + q * kWarps) * E::kPiece + lane * E::kEPT;
      raw[q] = off < ww ? E::ldg(base + (size_t)off * (sizeof(typename E::Raw) / E::kEPT)) : E::zero();
    }
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      const int p = warp + q * kWarps;
      if (p < npieces) {
        const int off = p * E::kPiece + lane * E::kEPT;
        float m[E::kEPT];
        kept_masses<E>(R, sh.bitmap, K, raw[q], wr * R.W + off, off < ww, m);
        float ls = 0.f;
#pragma unroll
        for (int j = 0; j < E::kEPT; ++j) ls = __fadd_rn(ls, m[j]);
        const double ps = warp_dsum((double)ls);
        if (lane == 0) ctl.piece[p] = ps;
      }
    }
  }
  csync();
  if (warp == 0) {
    int pick = -1, last = -1;
    double t2 = 0.0, run = 0.0;
    for (int p0 = 0; p0 < npieces; p0 += 32) {
      const int p = p0 + lane;
      const double m = p < npieces ? ctl.piece[p] : 0.0;
      const double inc = warp_incl_f64(m, lane) + run;
      const uint32_t pos = __ballot_sync(0xffffffffu, m > 0.0);
      const uint32_t hit = __ballot_sync(0xffffffffu, m > 0.0 && t1 < inc);
      if (pos) last = p0 + 31 - __clz(pos);
      if (pick < 0 && hit) {
        const int l = __ffs(hit) - 1;
        pick = p0 + l;
        t2 = t1 - __shfl_sync(0xffffffffu, inc - m, l);
      }
      run = __shfl_sync(0xffffffffu, inc, 31);
    }
    if (pick < 0) {
      pick = last;
      t2 = 1e300;
    }
    int tok = fallback;
    if (pick >= 0) {
      const int off = pick * E::kPiece + lane * E::kEPT;
      const int idx0 = wr * R.W + off;
      const typename E::Raw raw =
          off < ww ? E::ldg(base + (size_t)off * (sizeof(typename E::Raw) / E::kEPT)) : E::zero();
      float q[E::kEPT];
      kept_masses<E>(R, sh.bitmap, K, raw, idx0, off < ww, q);
      float ls = 0.f;
      int lk = -1;
#pragma unroll
      for (int j = 0; j < E::kEPT; ++j) {
        ls = __fadd_rn(ls, q[j]);
        if (q[j] > 0.f) lk = idx0 + j;
      }
      const double inc = warp_incl_f64((double)ls, lane);
      const uint32_t bal = __ballot_sync(0xffffffffu, inc > t2 && ls > 0.f);
      if (bal) {
        const int l = __ffs(bal) - 1;
        int mine = -1;
        if (lane == l) {
          double cum = inc - (double)ls;
          int pk = -1, lastc = -1;
#pragma unroll
          for (int j = 0; j < E::kEPT; ++j) {
            if (q[j] > 0.f) {
              lastc = j;
              cum += (double)q[j];
              if (pk < 0 && cum > t2) pk = j;
            }
          }
          if (pk < 0) pk = lastc;
          mine = idx0 + pk;
        }
        tok = __shfl_sync(0xffffffffu, mine, l);
      } else {
        const int lastk = (int)__reduce_max_sync(0xffffffffu, (uint32_t)(lk + 1)) - 1;
        if (lastk >= 0) tok = lastk;
      }
    }
    if (lane == 0) ctl.token = tok;
  }
  csync();
  return ctl.token;
}

// ---------------------------------------------------------------- top-p ties
// Exact top-p decision for a window whose members overflow the candidate
// list while the window is at single-value resolution (one bits(e) value per
// bucket, at most kBins of them): each value's mass is count x e exactly, so
// the crossing value e* and the number c of its members kept follow from
// counts alone (sampler.py:66-70: rank j is kept iff j == 0 or cum[j-1] <=
// top_p).  Members of e* rank by scaled logit, then index; a tie group's
// kept members are its c of smallest index.  Members of e* with different
// scaled logits (they lie within an ulp of e) set NS_STATUS_CAP_OVERFLOW and
// are taken in index order.  Re-reads the row three times.  `above` is the
// exact mass above the window, which ctl.seg holds per warp range; on return
// ctl.seg includes the kept members, K describes the decision and the kept
// total is returned.  Whole block.
template <class E>
__device__ __forceinline__ double topp_ties(const RowCtx& R, const Sh& sh, Keep& K, uint32_t wlo, uint32_t whi,
                                         double above, double z, uint32_t* status, int tid) {
  constexpr int EPT = E::kEPT;
  Ctl& ctl = *sh.ctl;
  uint32_t* hist = sh.hist;
  const int lane = tid & 31, warp = tid >> 5;
  const uint32_t span_m1 = whi - wlo;  // < kBins
  const Keep K1 = K;
  // counts by value, bucket whi - bits(e)
  for (int b = tid; b < kBins / 4; b += kThreads) reinterpret_cast<uint4*>(hist)[b] = make_uint4(0, 0, 0, 0);
  if (tid == 0) {
    ctl.misc = INT_MAX;
    ctl.misc2 = -1;
  }
  csync();
  global_pass<E>(R, sh.bitmap, tid, [&](int, const float(&x)[EPT], int, bool live) {
    if (!live) return;
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
      const uint32_t bits = __float_as_uint(K1.mass(scaled(R, x[j])));
      if (bits - wlo <= span_m1) atomicAdd(&hist[whi - bits], 1u);
    }
  });
  csync();
  // the crossing value e*: thread t owns buckets [8t, 8t+8)
  uint32_t cnt[8];
  double m[8], tot = 0.0;
  int last = -1;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int b = 8 * tid + j;
    cnt[j] = (uint32_t)b <= span_m1 ? hist[b] : 0u;
    m[j] = (double)cnt[j] * (double)__uint_as_float(whi - (uint32_t)b);
    tot += m[j];
    if (cnt[j]) last = b;
  }
  const double incl = warp_incl_f64(tot, lane);
  if (lane == 31) ctl.red_e[warp] = incl;
  if (last >= 0) atomicMax(&ctl.misc2, last);
  csync();
  double pre = above + incl - tot;
  for (int w = 0; w < warp; ++w) pre += ctl.red_e[w];
  {
    double run = pre;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (cnt[j] && topp_crossed(run + m[j], z, R.p)) {
        atomicMin(&ctl.misc, 8 * tid + j);
        break;
      }
      run += m[j];
    }
  }
  csync();
  const bool none = ctl.misc == INT_MAX;  // no crossing inside: the whole window stays
  const int bstar = none ? ctl.misc2 : ctl.misc;
  const uint32_t estar = whi - (uint32_t)bstar;
  const float ef = __uint_as_float(estar);
  if (tid == (bstar >> 3)) {
    // c: the fewest members of e* whose inclusive mass crosses
    double p0 = pre;
    for (int j = 0; j < (bstar & 7); ++j) p0 += m[j];
    const uint32_t n = cnt[bstar & 7];
    uint32_t lo = 1u, hi = n;
    if (!none) {
      while (lo < hi) {
        const uint32_t mid = lo + (hi - lo) / 2u;
        if (topp_crossed(p0 + (double)mid * (double)ef, z, R.p)) hi = mid;
        else lo = mid + 1u;
      }
    }
    ctl.sel_before = none ? n : lo;
  }
  csync();
  const uint32_t c = ctl.sel_before;
  // per warp range: members of e*, the range of their scaled logits, and the
  // (kept) mass of the window above e*
  uint32_t nme = 0u;
  float smin = INFINITY, smax = -INFINITY;
  double la = 0.0;
  global_pass<E>(R, sh.bitmap, tid, [&](int, const float(&x)[EPT], int, bool live) {
    if (!live) return;
    float part = 0.0f;
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
      const float s = scaled(R, x[j]);
      const float e = K1.mass(s);
      const uint32_t bits = __float_as_uint(e);
      if (bits == estar) {
        ++nme;
        smin = fminf(smin, s);
        smax = fmaxf(smax, s);
      } else if (bits > estar && bits <= whi) {
        part = __fadd_rn(part, e);
      }
    }
    la += (double)part;
  });
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    nme += __shfl_xor_sync(0xffffffffu, nme, o);
    smin = fminf(smin, __shfl_xor_sync(0xffffffffu, smin, o));
    smax = fmaxf(smax, __shfl_xor_sync(0xffffffffu, smax, o));
  }
  const double wa = warp_dsum(la);
  if (lane == 0) {
    ctl.red_u[warp] = nme;
    ctl.red_i[warp] = __float_as_int(smin);
    ctl.red_j[warp] = __float_as_int(smax);
  }
  csync();
  uint32_t pw = 0u;  // members of e* in the warp ranges before this one
  for (int w = 0; w < warp; ++w) pw += ctl.red_u[w];
  const uint32_t kc = c > pw ? min(nme, c - pw) : 0u;
  if (lane == 0) ctl.seg[warp] += wa + (double)kc * (double)ef;
  if (tid == 0) {
    float a = INFINITY, b = -INFINITY;
    for (int w = 0; w < kWarps; ++w) {
      a = fminf(a, __int_as_float(ctl.red_i[w]));
      b = fmaxf(b, __int_as_float(ctl.red_j[w]));
    }
    if (a != b && status) atomicOr(status, NS_STATUS_CAP_OVERFLOW);
    ctl.dec_thr = -INFINITY;
    ctl.dec_thr_idx = INT_MAX;
  }
  const double zk = above + block_dsum(ctl, la, tid) + (double)c * (double)ef;
  // the warp holding the c-th member of e* finds it (index order)
  const bool mine = nme > 0u && pw < c && c <= pw + nme;
  const uint32_t target = c - pw;
  uint32_t run = 0u;
  bool done = !mine;
  global_pass<E>(R, sh.bitmap, tid, [&](int, const float(&x)[EPT], int idx0, bool live) {
    if (done) return;
    uint32_t mask = 0u;
    if (live) {
#pragma unroll
      for (int j = 0; j < EPT; ++j) mask |= (__float_as_uint(K1.mass(scaled(R, x[j]))) == estar ? 1u : 0u) << j;
    }
    const uint32_t n = (uint32_t)__popc(mask);
    const uint32_t inc = warp_incl_u32(n, lane) + run;
    const uint32_t hit = __ballot_sync(0xffffffffu, inc >= target && inc - n < target);
    if (hit) {
      if (lane == __ffs(hit) - 1) {
        uint32_t k = target - (inc - n);
        int j = 0;
        for (; j < EPT; ++j)
          if (((mask >> j) & 1u) && --k == 0u) break;
        ctl.dec_thr = scaled(R, x[j]);
        ctl.dec_thr_idx = idx0 + j;
      }
      done = true;
    } else {
      run = __shfl_sync(0xffffffffu, inc, 31);
    }
  });
  csync();
  K.window = true;
  K.win_lo = wlo;
  K.win_hi = whi;
  K.thr = ctl.dec_thr;
  K.thr_idx = ctl.dec_thr_idx;
  return zk;
}

// ---------------------------------------------------------------- top-p members
// Decision among the window members sh.cand[0, n) (rank keys; every member
// has bits(e) in [wlo, whi], wlo >= 1): the first member in rank order (value
// descending, index ascending) whose inclusive mass -- `above` plus the
// members up to it -- passes thr (topp_threshold of the row total).  Members
// are grouped by bits(e) into at most kSub sub-buckets whose masses are
// summed in fixed point (2^-40 of the window top; order-independent), and
// only the crossing sub-bucket's members are ordered, by one warp.  Returns
// false, with nothing decided, when that sub-bucket holds more than 32
// members (the caller then sorts them all).  Otherwise sets ctl.dec_thr /
// dec_thr_idx to the last kept member, adds the kept members' masses to
// ctl.seg (per warp range) and ctl.pm (per piece), and returns their total
// in `kept`.  Uses sh.hist and sh.small as scratch.  Whole block.
template <class E>
__device__ __forceinline__ bool member_decide(const Sh sh, int n, uint32_t wlo, uint32_t whi, float m0, double above,
                                           double thr, int W, double& kept, int tid) {
  constexpr int kPer = kCandCap / kThreads;
  Ctl& ctl = *sh.ctl;
  const int lane = tid & 31, warp = tid >> 5;
  unsigned long long* sbm = reinterpret_cast<unsigned long long*>(sh.hist);  // [kSub] fixed-point masses
  uint32_t* sbc = sh.hist + 2 * kSub;                                          // [kSub] counts
  unsigned long long* small = sh.small;  // [32] crossing sub-bucket
  int shs = 0;
  while (((whi - wlo) >> shs) >= (uint32_t)kSub) ++shs;
  // F = e * 2^(40 - (E_top - 126)) < 2^41 for every member (E_top: biased exponent of whi)
  const int etop = (int)(whi >> 23);
  const double scale = __longlong_as_double((long long)(1023 + 166 - etop) << 52);
  const double unit = __longlong_as_double((long long)(1023 - 166 + etop) << 52);
  if (tid < kSub) {
    sbm[tid] = 0ull;
    sbc[tid] = 0u;
  }
  if (tid == 0) {
    ctl.misc = INT_MAX;
    ctl.list_n = 0u;
    ctl.dec_key = 0ull;
  }
  csync();
  unsigned long long key[kPer];
  int sb[kPer];
  float e[kPer];
#pragma unroll
  for (int q = 0; q < kPer; ++q) {
    const int r = tid + q * kThreads;
    key[q] = ~0ull;
    sb[q] = -1;
    e[q] = 0.0f;
    if (r < n) {
      key[q] = sh.cand[r];
      e[q] = exp_shifted(key_value(key[q]), m0);
      sb[q] = (int)((whi - __float_as_uint(e[q])) >> shs);
      atomicAdd(&sbc[sb[q]], 1u);
      atomicAdd(&sbm[sb[q]], (unsigned long long)__double2ull_rz((double)e[q] * scale));
      atomicMax(&ctl.dec_key, key[q]);  // with no crossing, the last member stays last
    }
  }
  csync();
  // the crossing sub-bucket: threads 0..kSub-1 scan the sub-bucket masses
  double pre = 0.0, m = 0.0;
  if (tid < kSub) {
    m = (double)sbm[tid] * unit;
    const double inc = warp_incl_f64(m, lane);
    if (lane == 31) ctl.red_e[warp] = inc;
    pre = inc - m;
  }
  csync();
  if (tid < kSub) {
    for (int w = 0; w < warp; ++w) pre += ctl.red_e[w];
    pre += above;
    if (sbc[tid] != 0u && pre + m > thr) atomicMin(&ctl.misc, tid);
  }
  csync();
  const int sbs = ctl.misc;
  if (tid == sbs) ctl.pick_t = pre;  // mass before the crossing sub-bucket
#pragma unroll
  for (int q = 0; q < kPer; ++q) {
    if (sb[q] >= 0 && sb[q] == sbs) {
      const uint32_t slot = atomicAdd(&ctl.list_n, 1u);
      if (slot < 32u) small[slot] = key[q];
    }
  }
  csync();
  if (sbs != INT_MAX && ctl.list_n > 32u) return false;
  if (sbs != INT_MAX && warp == 0) {
    // order the crossing sub-bucket (bitonic across the warp, ascending keys)
    const int ns = (int)ctl.list_n;
    unsigned long long k = lane < ns ? small[lane] : ~0ull;
#pragma unroll
    for (int kk = 2; kk <= 32; kk <<= 1) {
#pragma unroll
      for (int j = kk >> 1; j > 0; j >>= 1) {
        const unsigned long long o = __shfl_xor_sync(0xffffffffu, k, j);
        const bool take_min = ((lane & j) == 0) == ((lane & kk) == 0);
        k = take_min ? (k < o ? k : o) : (k < o ? o : k);
      }
    }
    const float ee = lane < ns ? exp_shifted(key_value(k), m0) : 0.0f;
    const double inc = warp_incl_f64((double)ee, lane) + ctl.pick_t;
    const uint32_t bal = __ballot_sync(0xffffffffu, lane < ns && inc > thr);
    const int l = bal ? __ffs(bal) - 1 : ns - 1;
    const unsigned long long kl = __shfl_sync(0xffffffffu, k, l);
    if (lane == 0) ctl.dec_key = kl;
  }
  csync();
  const unsigned long long last = ctl.dec_key;
  if (tid == 0) {
    ctl.dec_thr = n > 0 ? key_value(last) : -INFINITY;
    ctl.dec_thr_idx = n > 0 ? key_index(last) : INT_MAX;
  }
  // kept members (rank key <= the last kept one's) join their range and piece masses
  double lk = 0.0;
#pragma unroll
  for (int q = 0; q < kPer; ++q) {
    if (sb[q] >= 0 && key[q] <= last && e[q] > 0.0f) {
      const int idx = key_index(key[q]);
      const int w = idx / W;
      const int c = (idx - w * W) / E::kPiece;
      atomicAdd(&ctl.seg[w], (double)e[q]);
      atomicAdd(&ctl.pm[w][c / kStages], (double)e[q]);
      lk += (double)e[q];
    }
  }
  kept = block_dsum(ctl, lk, tid);  // (its barriers order the mass updates and ctl.dec_*)
  return true;
}

// Inverse-CDF draw in vocabulary order from the kept masses per warp range
// (ctl.seg) and per kStages-chunk piece of it (ctl.pm): warp 0 picks both
// from shared memory, reads the chosen piece (one round trip) and walks it
// chunk by chunk.  Falls back to the last kept element when rounding leaves
// the target past the total, then to `fallback`.  The token is returned in
// warp 0 (other warps get `fallback`); no barrier.
template <class E>
__device__ __forceinline__ int draw_piece(const RowCtx R, const Sh sh, const Keep K, double target, int fallback,
                                       int tid) {
  if (tid >= 32) return fallback;
  const Ctl& ctl = *sh.ctl;
  const int lane = tid;
  // the warp range
  const double ms = lane < kWarps ? ctl.seg[lane] : 0.0;
  const double incs = warp_incl_f64(ms, lane);
  const uint32_t poss = __ballot_sync(0xffffffffu, ms > 0.0);
  if (!poss) return fallback;
  uint32_t hit = __ballot_sync(0xffffffffu, ms > 0.0 && target < incs);
  int wr;
  double t1;
  if (hit) {
    wr = __ffs(hit) - 1;
    t1 = target - __shfl_sync(0xffffffffu, incs - ms, wr);
  } else {
    wr = 31 - __clz(poss);
    t1 = 1e300;
  }
  // the piece
  const int np = (R.nch + kStages - 1) / kStages;
  const double mp = lane < np ? ctl.pm[wr][lane] : 0.0;
  const double incp = warp_incl_f64(mp, lane);
  const uint32_t posp = __ballot_sync(0xffffffffu, mp > 0.0);
  if (!posp) return fallback;
  hit = __ballot_sync(0xffffffffu, mp > 0.0 && t1 < incp);
  int pc;
  double t2;
  if (hit) {
    pc = __ffs(hit) - 1;
    t2 = t1 - __shfl_sync(0xffffffffu, incp - mp, pc);
  } else {
    pc = 31 - __clz(posp);
    t2 = 1e300;
  }
  // walk the piece's chunks in vocabulary order
  constexpr int esz = sizeof(typename E::Raw) / E::kEPT;
  const int ww = max(0, min(R.W, R.V - wr * R.W));
  const int c0 = pc * kStages, c1 = min(R.nch, c0 + kStages);
  const char* base = R.src + (size_t)wr * R.W * esz;
  typename E::Raw raw[kStages];
#pragma unroll
  for (int u = 0; u < kStages; ++u) {
    const int off = (c0 + u) * E::kPiece + lane * E::kEPT;
    raw[u] = (c0 + u < c1 && off < ww) ? E::ldg(base + (size_t)off * esz) : E::zero();
  }
  int tok = -1, lastk = -1;
  double run = 0.0;
#pragma unroll
  for (int u = 0; u < kStages; ++u) {
    const int off = (c0 + u) * E::kPiece + lane * E::kEPT;
    const int idx0 = wr * R.W + off;
    float q[E::kEPT];
    kept_masses<E>(R, sh.bitmap, K, raw[u], idx0, c0 + u < c1 && off < ww, q);
    float ls = 0.f;
    int lk = -1;
#pragma unroll
    for (int j = 0; j < E::kEPT; ++j) {
      ls = __fadd_rn(ls, q[j]);
      if (q[j] > 0.f) lk = idx0 + j;
    }
    lastk = max(lastk, (int)__reduce_max_sync(0xffffffffu, (uint32_t)(lk + 1)) - 1);
    const double inc = warp_incl_f64((double)ls, lane) + run;
    const uint32_t bal = __ballot_sync(0xffffffffu, inc > t2 && ls > 0.f);
    if (bal) {
      const int l = __ffs(bal) - 1;
      int mine = -1;
      if (lane == l) {
        double cum = inc - (double)ls;
        int pk = -1, lastc = -1;
#pragma unroll
        for (int j = 0; j < E::kEPT; ++j) {
          if (q[j] > 0.f) {
            lastc = j;
            cum += (double)q[j];
            if (pk < 0 && cum > t2) pk = j;
          }
        }
        if (pk < 0) pk = lastc;
        mine = idx0 + pk;
      }
      tok = __shfl_sync(0xffffffffu, mine, l);
      break;
    }
    run = __shfl_sync(0xffffffffu, inc, 31);
  }
  if (tok < 0) tok = lastk >= 0 ? lastk : fallback;
  return tok;
}

}  // namespace rk
}  // namespace ns

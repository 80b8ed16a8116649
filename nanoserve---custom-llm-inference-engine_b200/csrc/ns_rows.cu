// ns_rows.cu -- B200 (sm_100a) token sampling for large batches: one thread
// block per row, every row streamed from HBM once.
//
// Replaces nanoserve/scheduler/sampler.py:21-89 (Sampler.sample) when the
// batch has enough rows to occupy the SMs; the cluster kernel in
// ns_sample.cu serves small batches, unaligned rows and small vocabularies.
// Design:
//
//  * Persistent blocks of 512 threads, two per SM; block b samples rows
//    b, b+G, b+2G...  Warp w owns the contiguous range [w*W, (w+1)*W) of
//    every row (W = V/16 rounded up), which it reads as 512-byte pieces,
//    16 bytes (4 fp32 or 8 bf16 logits) per lane.  Chunk c of a row is the
//    c-th piece of all 16 ranges, one 8 KB stage of a shared-memory ring.
//  * Thread t only ever reads the t-th 16 bytes of a stage, so it fills that
//    slot itself with cp.async, kStages chunks ahead of its reads (one commit
//    group per chunk).  Nothing ties the warps together while they stream,
//    and the copies run on into the row's second pass or the next row while
//    the block is still deciding the current one.
//  * The first pass gathers everything a row's path needs, so greedy and
//    top-k rows read HBM exactly once:
//      GREEDY  temperature 0 and no debug output: first-index argmax
//              (sampler.py:82-83).
//      TOPK    0 < top_k <= kTopkMax: the k-th largest of the per-thread
//              maxima seen so far bounds the k-th largest logit from below;
//              it is refreshed after chunks 0 and kRefreshAt, and every
//              element above it goes to its warp's own candidate list.  At
//              the end the candidates above the final bound are sorted, and
//              top-k (sampler.py:53-58), top-p (sampler.py:60-73), softmax
//              and the draw finish on that short list.
//      GENERAL the rest.  e = exp(s - m0), m0 the first chunk's maximum, is
//              summed per thread (plain sampling) and, for top-p, also fed to
//              a histogram of approximate masses keyed on the bits of e
//              (log-spaced buckets, one 32-bit shared atomic per element).  A
//              top-p row then takes a second pass through the ring (an L2
//              re-read, fetched while the histogram is searched) that sums the
//              exact mass above a window of buckets that must contain the
//              boundary and collects the window's elements, which are sorted
//              to decide exactly.
//  * The draw is an inverse CDF in vocabulary order driven by the row's
//    uniform: the warp range whose kept-mass prefix passes the target, then
//    the 512-byte piece inside it (masses recomputed from an L2 re-read of
//    that range), then the element, walked by one warp.
//  * Rare cases -- top_k > kTopkMax, candidate-list overflow, a row maximum
//    far above the first chunk's, NaN/inf rows, debug outputs -- re-read the
//    row from global memory as often as they need.
#include <cuda_runtime.h>
#include <stdint.h>

#include <climits>
#include <mutex>
#include <cstdlib>
#include <string>

#include "../../include/nanoserve_sampler.h"
#include "ns_device.cuh"
#include "ns_rows.h"

namespace ns {
namespace rk {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kStages = 6;                // ring depth (chunks in flight per thread)
constexpr int kPieceBytes = 512;          // one warp's share of a chunk
constexpr int kChunkBytes = kWarps * kPieceBytes;
constexpr int kBins = 4096;               // top-p locator histogram (u32 approximate masses)
constexpr int kTmBins = 2048;             // per-thread-maximum histogram, quarter binades
constexpr int kTmShift = 21;
constexpr int kRadixBins = 2048;          // radix-select level histogram (u32 counts)
constexpr int kTopkMax = 128;             // largest top_k served by the TOPK path
constexpr int kRefreshAt = 8;             // TOPK bound refreshes after chunks 0 and 8
constexpr int kCandCap = 2048;            // candidate / window-member capacity (u64 keys)
constexpr int kWarpCands = kCandCap / kWarps;  // TOPK: each warp's own candidate list
constexpr uint32_t kTopFine = 0x4F7FFFFFu;  // first locator level: e = exp(s - m0) in [2^-32, 2^32)
constexpr int kShFine = 17;                  // 1/64 binade per bucket
constexpr uint32_t kTopWide = 0x5F7FFFFFu;  // fallback level: e < 2^64, every normal float
constexpr int kShWide = 19;                  // 1/16 binade per bucket
constexpr double kSlack = 1.0 + 0x1p-11;  // > 1 / (1 - 2^-12): locator mass error bound
constexpr int kMinVocab = 24576;          // a row spans more chunks than the ring has stages
constexpr int kMaxVocab = 196608;
constexpr int kMaxChunks = (kMaxVocab / kWarps + 127) / 128;  // pieces per warp range (fp32)
constexpr int kPiecesMax = (kMaxChunks + kStages - 1) / kStages;  // draw pieces (kStages chunks) per warp range
constexpr int kSub = 256;                  // top-p member sub-buckets

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
// One row's inputs, fetched two rows ahead.
struct __align__(16) RowIn {
  NsRowParams P;
  int64_t h[2];
  int64_t src;
  int64_t row;  // the row this slot samples (row_order applied)
};

// Where a row comes from and how often the ring streams it.
struct RowPlan {
  const char* src;  // the row in global memory
  int passes;       // passes through the ring (1, or 2 for top-p rows)
  int valid;        // the row exists
  int pre;          // the pre-pass has streamed its first pass
};

struct __align__(16) Ctl {
  RowIn rin[4];
  RowPlan plan[2];
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

struct Layout {
  size_t ctl, ring, bitmap, cand, hist, tm, total;
};

__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) & ~(a - 1); }

__host__ __device__ inline Layout make_layout(int V) {
  Layout L;
  size_t o = 0;
  L.ctl = o;    o = align_up(o + sizeof(Ctl), 128);
  L.ring = o;   o = align_up(o + (size_t)kStages * kChunkBytes, 16);
  L.bitmap = o; o = align_up(o + sizeof(uint32_t) * (size_t)((V + 31) / 32), 16);
  L.cand = o;   o = align_up(o + sizeof(unsigned long long) * kCandCap, 16);
  L.hist = o;   o = align_up(o + sizeof(uint32_t) * kBins, 16);
  L.tm = o;     o = align_up(o + sizeof(uint32_t) * kTmBins, 16);
  L.total = o;
  return L;
}

struct Sh {
  Ctl* ctl;
  unsigned char* ring;
  uint32_t* bitmap;
  unsigned long long* cand;  // TOPK candidates / top-p window members
  uint32_t* hist;            // locator or radix histogram; TOPK: the final sorted list (u64)
  uint32_t* tm;              // per-thread-maximum histogram
};

// One row being sampled, with the row layout shared by every row.
// Repetition penalty of a row: rp and RN(1/rp).
struct Pen {
  float rp, rrp;
};

struct RowCtx {
  const char* src;
  int V, W, nch, row;
  float T, rT, rp, p;
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

enum { kGreedy = 0, kTopk = 1, kGeneral = 2 };

__device__ __forceinline__ int row_mode(const NsRowParams& P, int V, bool debug) {
  const bool greedy = (P.flags & NS_ROW_GREEDY) != 0u;
  if (greedy && !debug) return kGreedy;
  const int k = (P.top_k > 0 && P.top_k < V) ? P.top_k : 0;
  return (k > 0 && k <= kTopkMax) ? kTopk : kGeneral;
}

__device__ __forceinline__ float scaled(const RowCtx& R, float x) {
  return R.t_one ? x : div_by_const(x, R.T, R.rT);
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
        if ((m >> j) & 1u) x[j] = penalize(x[j], pp.rp, pp.rrp);
    }
  }
}

// ---------------------------------------------------------------- the ring
// Where this thread's refills come from during one pass over a row, offset
// to its own 16 bytes: chunk c + kStages of the pass if that is still inside
// it (`cur`), else chunk c + kStages - nch of what follows the pass
// (`after`: the row's second pass or the next row).  nullptr: nothing.
struct Feed {
  const char* cur;
  const char* after;
};

// Wait until this thread's copy kStages - 1 groups back has landed.
__device__ __forceinline__ void cp_async_wait_ring() {
  asm volatile("cp.async.wait_group %0;" ::"n"(kStages - 1) : "memory");
}

__device__ __forceinline__ unsigned char* stage_slot(unsigned char* ring, int stage, int tid) {
  return ring + stage * kChunkBytes + tid * 16;
}

// This thread's bytes of row `src` (16-byte aligned: the host admits only
// such rows).
template <class E>
__device__ __forceinline__ const char* lane_src(const char* src, const Lane& ln) {
  return src + (size_t)ln.base * (sizeof(typename E::Raw) / E::kEPT);
}

// Refill sources for the first pass over the block's i-th row, and for its
// second pass (`wanted` false: the second pass is only drained).
template <class E>
__device__ __forceinline__ Feed feed_first(const Ctl& ctl, int i, const Lane& ln) {
  const RowPlan& p = ctl.plan[i & 1];
  const RowPlan& n = ctl.plan[(i + 1) & 1];
  Feed f;
  f.cur = lane_src<E>(p.src, ln);
  f.after = p.passes == 2 ? f.cur : (n.valid ? lane_src<E>(n.src, ln) : nullptr);
  return f;
}
template <class E>
__device__ __forceinline__ Feed feed_second(const Ctl& ctl, int i, const Lane& ln, bool wanted) {
  const RowPlan& p = ctl.plan[i & 1];
  const RowPlan& n = ctl.plan[(i + 1) & 1];
  Feed f;
  f.cur = wanted ? lane_src<E>(p.src, ln) : nullptr;
  f.after = n.valid ? lane_src<E>(n.src, ln) : nullptr;
  return f;
}

// Prologue: the first kStages chunks of the block's first row.
template <class E>
__device__ __forceinline__ void ring_start(const Ctl& ctl, unsigned char* ring, const Lane& ln) {
  const RowPlan& pl = ctl.plan[0];
  const char* src = lane_src<E>(pl.src, ln);
  for (int c = 0; c < kStages; ++c) {
    unsigned char* dst = stage_slot(ring, c, ln.tid);
    if (pl.valid && c < ln.nv) cp_async16(dst, src + c * kPieceBytes);
    else *reinterpret_cast<uint4*>(dst) = make_uint4(E::kNegInf2, E::kNegInf2, E::kNegInf2, E::kNegInf2);
    cp_async_commit();
  }
}

__device__ __forceinline__ void cp_async16_s(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

// This thread's walk through the ring during one pass: the shared address of
// its slot in the stage it reads next, and where its refills (kStages chunks
// ahead) come from -- a running pointer with a count of refills left from
// the current source, switched to `after` when the refills leave the pass.
struct RingWalk {
  uint32_t slot, ring_lo, ring_hi;
  const char* gp;
  int left;
  int plain_end;  // chunks below this refill from `cur` in every lane of the warp
  __device__ __forceinline__ RingWalk(const Sh& sh, const Lane& ln, const Feed& fd, int stage) {
    ring_lo = smem_addr(sh.ring) + ln.tid * 16;
    ring_hi = ring_lo + kStages * kChunkBytes;
    slot = ring_lo + stage * kChunkBytes;
    gp = fd.cur + kStages * kPieceBytes;
    left = fd.cur ? ln.nv - kStages : 0;
    plain_end = fd.cur ? ln.nvw - kStages : 0;
  }
  // refill the slot just read with chunk c + kStages (one commit group); a
  // slot this lane has no data for is filled with -inf logits instead
  __device__ __forceinline__ void refill(const Feed& fd, const Lane& ln, int c, int nch, uint32_t pad) {
    if (c == nch - kStages) {
      gp = fd.after;
      left = fd.after ? ln.nv : 0;
    }
    if (left > 0) cp_async16_s(slot, gp);
    else asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(slot), "r"(pad) : "memory");
    gp += kPieceBytes;
    --left;
    cp_async_commit();
    slot += kChunkBytes;
    if (slot == ring_hi) slot = ring_lo;
  }
};

// One pass of the current row through the ring: body(c, x, idx0, live) for
// every chunk c with this thread's penalized logits (-inf where the lane has
// no element: live false).
template <class E, bool PEN, class F>
__device__ __forceinline__ void ring_range(const Sh& sh, const Lane& ln, const Feed& fd, RingWalk& rw, int c0, int c1,
                                           int nch, Pen pp, F&& body) {
  constexpr int EPT = E::kEPT;
  int c = c0;
  int idx0 = ln.base + c0 * E::kPiece;
  // whole turns of the ring in which every lane of the warp has data and
  // refills from the current source: fixed slot addresses, immediate source
  // offsets, no per-chunk bookkeeping (the bound is warp-uniform, so bodies
  // may use warp collectives)
  const int cm = min(c1, rw.plain_end);
  if (c + kStages <= cm) {
    uint32_t slots[kStages];
#pragma unroll
    for (int u = 0; u < kStages; ++u) {
      const uint32_t a = rw.slot + u * kChunkBytes;
      slots[u] = a >= rw.ring_hi ? a - kStages * kChunkBytes : a;
    }
    const char* gp = rw.gp;
    do {
#pragma unroll
      for (int u = 0; u < kStages; ++u) {
        cp_async_wait_ring();
        const typename E::Raw raw = E::lds_s(slots[u]);
        cp_async16_s(slots[u], gp + u * kPieceBytes);
        cp_async_commit();
        float x[EPT];
        penalized<E, PEN>(sh.bitmap, pp, raw, idx0 + u * E::kPiece, x);
        body(c + u, x, idx0 + u * E::kPiece, true);
      }
      c += kStages;
      idx0 += kStages * E::kPiece;
      gp += kStages * kPieceBytes;
    } while (c + kStages <= cm);
    rw.left -= c - c0;
    rw.gp = gp;
  }
  for (; c < c1; ++c, idx0 += E::kPiece) {
    cp_async_wait_ring();
    const typename E::Raw raw = E::lds_s(rw.slot);
    rw.refill(fd, ln, c, nch, E::kNegInf2);
    const bool live = c < ln.nv;
    float x[EPT];
    penalized<E, PEN>(sh.bitmap, pp, raw, idx0, x, live);
    body(c, x, idx0, live);
  }
}
template <class E, bool PEN, class F>
__device__ __forceinline__ void ring_pass(const Sh& sh, const Lane& ln, const Feed& fd, int nch, int& stage, Pen pp,
                                          F&& body) {
  RingWalk rw(sh, ln, fd, stage);
  ring_range<E, PEN>(sh, ln, fd, rw, 0, nch, nch, pp, body);
  stage = (stage + nch) % kStages;
}

// Maximum of this thread's penalized logits in the pass's first chunk, read
// ahead of the pass (which then finds the chunk already landed).
template <class E>
__device__ __forceinline__ float peek_max(const Sh& sh, const Lane& ln, int stage, bool pen, Pen pp) {
  cp_async_wait_ring();
  const typename E::Raw raw = E::lds_s(smem_addr(sh.ring) + stage * kChunkBytes + ln.tid * 16);
  float x[E::kEPT];
  if (pen) penalized<E, true>(sh.bitmap, pp, raw, ln.base, x, ln.nv > 0);
  else penalized<E, false>(sh.bitmap, pp, raw, ln.base, x);
  float mv = x[0];
#pragma unroll
  for (int j = 1; j < E::kEPT; ++j) mv = fmax_nan(mv, x[j]);
  return mv;
}

// Consume a second pass nobody needs without fetching it; returns the new
// ring stage.  (Out of line, so everything is passed by value.)
__device__ __noinline__ int drain_pass(unsigned char* ring, Feed fd, Lane ln, int nch, int stage, uint32_t pad) {
  Sh sh;
  sh.ring = ring;
  RingWalk rw(sh, ln, fd, stage);
  for (int c = 0; c < nch; ++c) {
    cp_async_wait_ring();
    rw.refill(fd, ln, c, nch, pad);
  }
  return (stage + nch) % kStages;
}

// Calls f(c, x, idx0, live) for every chunk c of the row with this thread's
// penalized logits, re-read from global memory (four chunks in flight).
template <class E, class F>
__device__ __forceinline__ void global_pass(const RowCtx& R, const uint32_t* bitmap, int tid, F&& f) {
  constexpr int EPT = E::kEPT, U = 4;
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

// Threads 0..3 copy row `row`'s inputs (64 bytes) into `dst` with plain
// loads; cp.async is kept for the ring, whose group count must stay exact.
__device__ __forceinline__ void fetch_row_inputs(const NsSampleArgs& a, RowIn& dst, int ticket, int tid) {
  if (tid >= 4) return;
  int row = ticket;
  if (a.row_order) {
    const int r = __ldg(&a.row_order[ticket]);
    if (r >= 0 && r < a.num_rows) row = r;
    else if (tid == 3 && a.status) atomicOr(a.status, NS_STATUS_BAD_ROW_ORDER);
  }
  uint4 v;
  if (tid < 2) {
    v = __ldg(reinterpret_cast<const uint4*>(&a.row_params[row]) + tid);
  } else {
    int64_t x0, x1 = row;
    if (tid == 2) {
      x0 = a.history_offsets ? a.history_offsets[row] : 0;
      x1 = a.history_offsets ? a.history_offsets[row + 1] : 0;
    } else {
      x0 = a.sample_indices ? a.sample_indices[row] : row;
    }
    v = make_uint4((uint32_t)x0, (uint32_t)((uint64_t)x0 >> 32), (uint32_t)x1, (uint32_t)((uint64_t)x1 >> 32));
  }
  reinterpret_cast<uint4*>(&dst)[tid] = v;
}

// ---------------------------------------------------------------- pre-pass
// The first pass of top-p rows without top-k, split over kPreParts blocks per
// row and run as its own kernel ahead of the row kernel (same stream): each
// block streams one contiguous part of the row and leaves the part's
// locator histogram and statistics in g_pre_*; the row kernel adds the parts
// and goes straight to the top-p window, so such a row streams through its
// own block once instead of twice.  Every part uses the row kernel's m0 (the
// maximum of the row's first chunk, which every part reads), so the parts'
// histograms add up exactly to the one the row kernel would have built.
constexpr int kPreRows = 256;  // calls with at most this many rows use the pre-pass
constexpr int kPreParts = 4;   // blocks per row
static_assert(kPreRows == kRowsScratchRows, "the header's limit is the scratch size");

struct PreStats {
  double z;        // sum over the part of e = exp(s - m0)
  uint32_t mxkey;  // orderable key of the part's largest penalized logit (0xffffffff: a NaN)
  float m0;
  uint32_t pad[2];
};

// Scratch of the pre-pass: file-scope device arrays of the library (16 MB
// of histograms and 32 KB of statistics, held by every GPU that loads it);
// slot r belongs to row r of the current call.  Nothing in them needs
// clearing: a call reads only slots it wrote earlier in the same call.
// Calls that overlap on the GPU race on them.
static __device__ __align__(256) uint32_t g_pre_hist[kPreRows][kPreParts][kBins];
static __device__ __align__(256) PreStats g_pre_stats[kPreRows][kPreParts];

// Rows the pre-pass serves: top-p on, top-k off, no debug outputs.
__device__ __forceinline__ bool pre_row(const NsRowParams& P, int V, bool debug) {
  const bool k_on = P.top_k > 0 && P.top_k < V;
  return !debug && (P.flags & NS_ROW_GREEDY) == 0u && (P.flags & NS_ROW_TOP_P) != 0u && !k_on;
}

// Plan of this block's i-th row (taken at position `ticket` of the row
// order), from its fetched inputs.
__device__ __forceinline__ void make_plan(const NsSampleArgs& a, Ctl& ctl, int i, int ticket, bool debug,
                                          bool pre_on) {
  RowPlan& pl = ctl.plan[i & 1];
  if (ticket >= a.num_rows) {
    pl.valid = 0;
    return;
  }
  const RowIn& in = ctl.rin[i & 3];
  int64_t src = in.src;
  if (src < 0 || src >= a.num_logit_rows) src = 0;
  const size_t esize = a.logits_dtype == NS_DTYPE_BF16 ? 2 : 4;
  pl.src = static_cast<const char*>(a.logits) + (size_t)src * (size_t)a.logits_row_stride * esize;
  const int mode = row_mode(in.P, a.vocab_size, debug);
  pl.pre = (pre_on && in.row < kPreRows && pre_row(in.P, a.vocab_size, debug)) ? 1 : 0;
  pl.passes = (!pl.pre && mode == kGeneral && (in.P.flags & NS_ROW_TOP_P)) ? 2 : 1;
  pl.valid = 1;
}

// ---------------------------------------------------------------- block reductions
// Block-wide exclusive scan of one u32 per thread (thread 0 first).
__device__ __forceinline__ uint32_t block_excl_u32(Ctl& ctl, uint32_t v, uint32_t& total, int tid) {
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

__device__ __forceinline__ double block_dsum(Ctl& ctl, double v, int tid) {
  const double w = warp_dsum(v);
  if ((tid & 31) == 0) ctl.red_e[tid >> 5] = w;
  __syncthreads();
  double s = 0.0;
  for (int i = 0; i < kWarps; ++i) s += ctl.red_e[i];
  __syncthreads();
  return s;
}

// Per-warp-range totals of per-thread masses into ctl.seg, and their sum.
__device__ __forceinline__ double block_segments(Ctl& ctl, double v, int tid) {
  const double w = warp_dsum(v);
  if ((tid & 31) == 0) ctl.seg[tid >> 5] = w;
  __syncthreads();
  double s = 0.0;
  for (int i = 0; i < kWarps; ++i) s += ctl.seg[i];
  __syncthreads();
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
  __syncthreads();
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
  __syncthreads();
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
__device__ __noinline__ void sort_keys(unsigned long long* keys, int n, int tid) {
  const int lane = tid & 31, warp = tid >> 5;
  int np = 128;
  while (np < n) np <<= 1;
  for (int i = n + tid; i < np; i += kThreads) keys[i] = ~0ull;
  __syncthreads();
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
  __syncthreads();
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
      __syncthreads();
    }
    if (warp < nseg) {
      const int base = warp << 7;
#pragma unroll
      for (int r = 0; r < 4; ++r) v[r] = keys[base + 32 * r + lane];
      seg_merge(v, base, lane, k);
#pragma unroll
      for (int r = 0; r < 4; ++r) keys[base + 32 * r + lane] = v[r];
    }
    __syncthreads();
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

// ---------------------------------------------------------------- top-k bound
// Over the kTmBins-bucket count histogram `tm` (bucket kTmBins - 1 holds the
// largest keys): the bucket where the count from the top reaches `need`, and
// the count above it.  Whole block; thread t scans buckets from the top.
__device__ __forceinline__ int tm_crossing(Ctl& ctl, const uint32_t* tm, uint32_t need, uint32_t& above, int tid) {
  uint32_t cnt[4];
  uint32_t s = 0;
  const int bhi = kTmBins - 1 - 4 * tid;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    cnt[j] = tm[bhi - j];
    s += cnt[j];
  }
  uint32_t tot;
  const uint32_t pre = block_excl_u32(ctl, s, tot, tid);
  if (pre < need && pre + s >= need) {
    uint32_t run = pre;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (run + cnt[j] >= need) {
        ctl.misc = bhi - j;
        ctl.sel_before = run;
        break;
      }
      run += cnt[j];
    }
  }
  __syncthreads();
  above = ctl.sel_before;
  return ctl.misc;
}

// The k-th largest per-thread maximum (a logit before temperature), rounded
// down to 2^10 units of its order key (two histogram levels) and extended to
// every logit whose scaled value ties with it: a lower bound for the k-th
// largest scaled logit of the row.  Whole block.
__device__ __noinline__ float topk_bound(int topk, bool t_one, float T, float rT, Ctl* ctlp, uint32_t* tm, float tmax,
                                         int tid) {
  Ctl& ctl = *ctlp;
  const uint32_t key = (tmax == tmax) ? f2key(tmax) : 0u;  // NaN maxima take no part
  for (int b = tid; b < kTmBins; b += kThreads) tm[b] = 0u;
  __syncthreads();
  if (tid == 0) ctl.misc = -1;
  if (key) atomicAdd(&tm[key >> kTmShift], 1u);
  __syncthreads();
  uint32_t above;
  const int b1 = tm_crossing(ctl, tm, (uint32_t)topk, above, tid);
  if (b1 < 0) return -INFINITY;  // fewer maxima than k
  // second level inside bucket b1: bits 20..10 of the key
  for (int b = tid; b < kTmBins; b += kThreads) tm[b] = 0u;
  __syncthreads();
  if (tid == 0) ctl.misc = -1;
  if (key && (int)(key >> kTmShift) == b1) atomicAdd(&tm[(key >> 10) & (kTmBins - 1)], 1u);
  __syncthreads();
  uint32_t above2;
  const int b2 = tm_crossing(ctl, tm, (uint32_t)topk - above, above2, tid);
  const uint32_t bkey = ((uint32_t)b1 << kTmShift) | ((uint32_t)max(b2, 0) << 10);
  const float bound = bkey < 0x00800000u ? -INFINITY : key2f(bkey);
  return lower_preimage(bound, t_one, T, rT);
}

// ---------------------------------------------------------------- radix select
// k-th largest penalized logit by a 3-level radix select over its key
// (11/11/10 bits), re-reading the row three times.  Whole block.
template <class E>
__device__ __noinline__ float radix_select(const RowCtx R, const Sh sh, int tid) {
  Ctl& ctl = *sh.ctl;
  uint32_t* h = sh.hist;
  uint32_t prefix = 0u, krem = (uint32_t)R.k;
  const int shifts[3] = {21, 10, 0};
  const int widths[3] = {11, 11, 10};
  for (int lvl = 0; lvl < 3; ++lvl) {
    const int shl = shifts[lvl], wd = widths[lvl];
    const uint32_t nbm = (1u << wd) - 1u;
    for (int b = tid; b < kRadixBins; b += kThreads) h[b] = 0u;
    __syncthreads();
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
    __syncthreads();
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
    __syncthreads();
    const int b = ctl.misc;
    if (b < 0) return -INFINITY;  // fewer than k elements (k < V makes this impossible)
    krem -= ctl.sel_before;
    prefix = (prefix << wd) | (nbm - (uint32_t)b);
    __syncthreads();
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
__device__ __noinline__ void topp_window(Ctl* ctlp, const uint32_t* h, const Level lv, double base, double thr,
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
  __syncthreads();
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
  __syncthreads();
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
  __syncthreads();
  if (tid == 0) {
    double e = 0.0;
    for (int w = 0; w < kWarps; ++w) e += ctl.red_e[w];
    ctl.sel_found = found;
    ctl.sel_lo = found ? fl : 0;
    ctl.sel_hi = found ? fh : 0;
    ctl.sel_est = found ? (float)(e * 1.001 + 1.0) : 0.0f;
  }
  __syncthreads();
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
__device__ __noinline__ int draw_token(const RowCtx R, const Sh sh, const Keep K, double target, int fallback,
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
  __syncthreads();
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
  __syncthreads();
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
  __syncthreads();
  return ctl.token;
}

// The first index at which this thread holds `best`, which it first saw in
// chunk `bc` (re-read from global memory); INT_MAX when it saw none.
template <class E>
__device__ __forceinline__ int arg_of(const RowCtx& R, const uint32_t* bitmap, const Lane& ln, float best, int bc) {
  if (bc < 0) return INT_MAX;
  const int idx0 = ln.base + bc * E::kPiece;
  const typename E::Raw raw = E::ldg(lane_src<E>(R.src, ln) + bc * kPieceBytes);
  float x[E::kEPT];
  if (R.pen) penalized<E, true>(bitmap, R.pp, raw, idx0, x);
  else penalized<E, false>(bitmap, R.pp, raw, idx0, x);
  int jj = E::kEPT - 1;
#pragma unroll
  for (int j = E::kEPT - 1; j >= 0; --j)
    if (x[j] == best) jj = j;
  return idx0 + jj;
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
__device__ __noinline__ double topp_ties(const RowCtx& R, const Sh& sh, Keep& K, uint32_t wlo, uint32_t whi,
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
  __syncthreads();
  global_pass<E>(R, sh.bitmap, tid, [&](int, const float(&x)[EPT], int, bool live) {
    if (!live) return;
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
      const uint32_t bits = __float_as_uint(K1.mass(scaled(R, x[j])));
      if (bits - wlo <= span_m1) atomicAdd(&hist[whi - bits], 1u);
    }
  });
  __syncthreads();
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
  __syncthreads();
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
  __syncthreads();
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
  __syncthreads();
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
  __syncthreads();
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
  __syncthreads();
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
// in `kept`.  Uses sh.hist and sh.tm as scratch.  Whole block.
template <class E>
__device__ __noinline__ bool member_decide(const Sh sh, int n, uint32_t wlo, uint32_t whi, float m0, double above,
                                           double thr, int W, double& kept, int tid) {
  constexpr int kPer = kCandCap / kThreads;
  Ctl& ctl = *sh.ctl;
  const int lane = tid & 31, warp = tid >> 5;
  unsigned long long* sbm = reinterpret_cast<unsigned long long*>(sh.hist);  // [kSub] fixed-point masses
  uint32_t* sbc = sh.hist + 2 * kSub;                                          // [kSub] counts
  unsigned long long* small = reinterpret_cast<unsigned long long*>(sh.tm);  // [32] crossing sub-bucket
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
  __syncthreads();
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
  __syncthreads();
  // the crossing sub-bucket: threads 0..kSub-1 scan the sub-bucket masses
  double pre = 0.0, m = 0.0;
  if (tid < kSub) {
    m = (double)sbm[tid] * unit;
    const double inc = warp_incl_f64(m, lane);
    if (lane == 31) ctl.red_e[warp] = inc;
    pre = inc - m;
  }
  __syncthreads();
  if (tid < kSub) {
    for (int w = 0; w < warp; ++w) pre += ctl.red_e[w];
    pre += above;
    if (sbc[tid] != 0u && pre + m > thr) atomicMin(&ctl.misc, tid);
  }
  __syncthreads();
  const int sbs = ctl.misc;
  if (tid == sbs) ctl.pick_t = pre;  // mass before the crossing sub-bucket
#pragma unroll
  for (int q = 0; q < kPer; ++q) {
    if (sb[q] >= 0 && sb[q] == sbs) {
      const uint32_t slot = atomicAdd(&ctl.list_n, 1u);
      if (slot < 32u) small[slot] = key[q];
    }
  }
  __syncthreads();
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
  __syncthreads();
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
__device__ __noinline__ int draw_piece(const RowCtx R, const Sh sh, const Keep K, double target, int fallback,
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

// ---------------------------------------------------------------- top-k lists
// One chunk's logits of a thread, passed by value to out-of-line helpers.
template <class E>
struct Chunk {
  float v[E::kEPT];
};

// Appends this warp's elements >= tau of one chunk to the warp's candidate
// list (slots counted in the warp-uniform wcnt; entries past kWarpCands are
// counted but not stored) and returns the new count.  Rare once the bound is
// tight, so it stays out of the streaming loop.  Whole warp.
template <class E>
__device__ __noinline__ int topk_insert(unsigned long long* wl, int wcnt, const Chunk<E> ch, int idx0, float tau,
                                        bool live, bool t_one, float T, float rT, int lane) {
  const uint32_t lt = (1u << lane) - 1u;
#pragma unroll
  for (int j = 0; j < E::kEPT; ++j) {
    const bool tk = live && (ch.v[j] >= tau);
    const uint32_t bal = __ballot_sync(0xffffffffu, tk);
    if (tk) {
      const int slot = wcnt + __popc(bal & lt);
      if (slot < kWarpCands) wl[slot] = rank_key(t_one ? ch.v[j] : div_by_const(ch.v[j], T, rT), idx0 + j);
    }
    wcnt += __popc(bal);
  }
  return wcnt;
}

// ---------------------------------------------------------------- pre-pass kernel
template <class E>
__device__ __forceinline__ void pre_pass(const NsSampleArgs& a, int W, uint32_t* scratch_hist,
                                         PreStats* scratch_stats) {
  constexpr int EPT = E::kEPT;
  constexpr int esz = sizeof(typename E::Raw) / EPT;
  __shared__ __align__(16) uint32_t hist[kBins];
  __shared__ uint32_t bitmap[(kMaxVocab + 31) / 32];
  __shared__ uint32_t red_k[kWarps];
  __shared__ double red_z[kWarps];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row = blockIdx.x / kPreParts, part = blockIdx.x % kPreParts;
  if (row >= a.num_rows) return;
  const NsRowParams P = a.row_params[row];
  const int V = a.vocab_size;
  const bool debug = (a.out_filtered != nullptr) || (a.out_probs != nullptr);
  if (!pre_row(P, V, debug)) return;
  int64_t src = a.sample_indices ? a.sample_indices[row] : row;
  if (src < 0 || src >= a.num_logit_rows) src = 0;  // the row kernel reports it
  const char* rs = static_cast<const char*>(a.logits) + (size_t)src * (size_t)a.logits_row_stride * esz;
  const float T = P.temperature;
  const float rT = __frcp_rn(T);
  const bool t_one = (T == 1.0f);
  const int64_t h0 = a.history_offsets ? a.history_offsets[row] : 0;
  const int64_t h1 = a.history_offsets ? a.history_offsets[row + 1] : 0;
  const bool pen = (P.flags & NS_ROW_PENALTY) != 0u && a.history_offsets && h1 > h0;
  const Pen pp{P.repetition_penalty, __frcp_rn(P.repetition_penalty)};

  for (int b = tid; b < kBins / 4; b += kThreads) reinterpret_cast<uint4*>(hist)[b] = make_uint4(0, 0, 0, 0);
  if (pen)
    for (int w = tid; w < (V + 31) / 32; w += kThreads) bitmap[w] = 0u;
  __syncthreads();
  if (pen) {
    for (int64_t h = h0 + tid; h < h1; h += kThreads) {
      const int id = a.history_ids[h];
      if (id >= 0 && id < V) atomicOr(&bitmap[id >> 5], 1u << (id & 31));
    }
  }
  __syncthreads();
  // m0: the row kernel's first chunk (thread t: warp range t / 32, its lane's 16 bytes)
  float pm = -INFINITY;
  {
    const int ww = max(0, min(W, V - warp * W));
    const int idx0 = warp * W + lane * EPT;
    if (lane * EPT < ww) {
      float x[EPT];
      const typename E::Raw raw = E::ldg(rs + (size_t)idx0 * esz);
      if (pen) penalized<E, true>(bitmap, pp, raw, idx0, x);
      else penalized<E, false>(bitmap, pp, raw, idx0, x);
      pm = x[0];
#pragma unroll
      for (int j = 1; j < EPT; ++j) pm = fmax_nan(pm, x[j]);
    }
  }
  {
    const uint32_t wk = __reduce_max_sync(0xffffffffu, pm != pm ? 0u : f2key(pm));
    if (lane == 0) red_k[warp] = wk;
  }
  __syncthreads();
  uint32_t ck = 0u;
  for (int w = 0; w < kWarps; ++w) ck = max(ck, red_k[w]);
  const float mx0 = key2f(ck);
  const float m0 = (mx0 > -INFINITY && mx0 < INFINITY) ? (t_one ? mx0 : div_by_const(mx0, T, rT)) : 0.0f;
  __syncthreads();  // red_k is reused below
  // this part's 16-byte slots, block-strided
  const int nslots = V / EPT;
  const int s_lo = (int)((int64_t)part * nslots / kPreParts), s_hi = (int)((int64_t)(part + 1) * nslots / kPreParts);
  float lmax = -INFINITY;
  double lz = 0.0;
  constexpr int U = 4;
  for (int s0 = s_lo + tid; s0 < s_hi; s0 += U * kThreads) {
    typename E::Raw raw[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int sl = s0 + u * kThreads;
      raw[u] = sl < s_hi ? E::ldg(rs + (size_t)sl * sizeof(typename E::Raw)) : E::zero();
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int sl = s0 + u * kThreads;
      if (sl >= s_hi) continue;
      float x[EPT];
      if (pen) penalized<E, true>(bitmap, pp, raw[u], sl * EPT, x);
      else penalized<E, false>(bitmap, pp, raw[u], sl * EPT, x);
      float part_z = 0.0f;
#pragma unroll
      for (int j = 0; j < EPT; ++j) {
        lmax = fmax_nan(lmax, x[j]);
        const float s = t_one ? x[j] : div_by_const(x[j], T, rT);
        const float e = exp_shifted(s, m0);
        part_z = __fadd_rn(part_z, e);
        const uint32_t bits = __float_as_uint(e);
        atomicAdd(&hist[min((kTopFine - bits) >> kShFine, (uint32_t)(kBins - 1))], approx_mass13(bits));
      }
      lz += (double)part_z;
    }
  }
  {
    const bool nan = (lmax != lmax);
    const uint32_t wk = __reduce_max_sync(0xffffffffu, nan ? 0u : f2key(lmax));
    const bool wn = __any_sync(0xffffffffu, nan);
    const double wz = warp_dsum(lz);
    if (lane == 0) {
      red_k[warp] = wn ? 0xffffffffu : wk;
      red_z[warp] = wz;
    }
  }
  __syncthreads();
  uint32_t* gh = scratch_hist + ((size_t)row * kPreParts + part) * kBins;
  for (int b = tid; b < kBins / 4; b += kThreads)
    reinterpret_cast<uint4*>(gh)[b] = reinterpret_cast<const uint4*>(hist)[b];
  if (tid == 0) {
    uint32_t k = 0u;
    double z = 0.0;
    for (int w = 0; w < kWarps; ++w) {
      k = max(k, red_k[w]);
      z += red_z[w];
    }
    PreStats st;
    st.z = z;
    st.mxkey = k;
    st.m0 = m0;
    st.pad[0] = st.pad[1] = 0u;
    scratch_stats[(size_t)row * kPreParts + part] = st;
  }
}

// The pre-pass as ns_sample launches it: the scratch named directly.
template <class E>
__global__ void __launch_bounds__(kThreads) pre_kernel(const NsSampleArgs a, int W) {
  pre_pass<E>(a, W, &g_pre_hist[0][0][0], &g_pre_stats[0][0]);
}

// The same pre-pass given the scratch's device address, which the host
// looked up with cudaGetSymbolAddress (ns_sample_noalloc).
template <class E>
__global__ void __launch_bounds__(kThreads) pre_kernel_at(const NsSampleArgs a, int W, uint32_t* scratch_hist,
                                                          PreStats* scratch_stats) {
  pre_pass<E>(a, W, scratch_hist, scratch_stats);
}

// ---------------------------------------------------------------- one row
template <class E>
__device__ __forceinline__ void sample_row(const NsSampleArgs& a, const Sh& sh, const Lane& ln, int& stage, int i,
                                           int row, int nch, int W) {
  constexpr int EPT = E::kEPT;
  const int tid = ln.tid, lane = ln.lane, warp = ln.warp;
  Ctl& ctl = *sh.ctl;
  uint32_t* const status = a.status;
  const int V = a.vocab_size;
  const bool debug = (a.out_filtered != nullptr) || (a.out_probs != nullptr);
  const bool out_i32 = (a.out_dtype == NS_OUT_I32);
  const RowIn& in = ctl.rin[i & 3];
  const NsRowParams P = in.P;
  RowCtx R;
  R.src = ctl.plan[i & 1].src;
  R.V = V;
  R.W = W;
  R.nch = nch;
  R.row = row;
  R.greedy = (P.flags & NS_ROW_GREEDY) != 0u;
  R.T = R.greedy ? 1.0f : P.temperature;
  R.rT = __frcp_rn(R.T);
  R.t_one = (R.T == 1.0f);
  R.topp = (P.flags & NS_ROW_TOP_P) != 0u;
  R.p = P.top_p;
  R.k = (P.top_k > 0 && P.top_k < V) ? P.top_k : 0;
  R.rp = P.repetition_penalty;
  R.pp = Pen{R.rp, __frcp_rn(R.rp)};
  const int64_t h0 = in.h[0], h1 = in.h[1];
  R.pen = (P.flags & NS_ROW_PENALTY) != 0u && a.history_offsets && h1 > h0;
  const bool ring2 = ctl.plan[i & 1].passes == 2;
  const bool pre = ctl.plan[i & 1].pre != 0;  // first pass done by the pre-pass; the ring has the second
  int mode = row_mode(P, V, debug);
  const int64_t out_off = (int64_t)row * V;

  // ---------------- setup: penalty bitmap, histograms, counters
  const bool want_hist = (mode == kGeneral) && R.topp && R.k == 0;
  if (R.pen)
    for (int w = tid; w < (V + 31) / 32; w += kThreads) sh.bitmap[w] = 0u;
  if (want_hist)
    for (int b = tid; b < kBins / 4; b += kThreads) reinterpret_cast<uint4*>(sh.hist)[b] = make_uint4(0, 0, 0, 0);
  if (tid == 0) ctl.cand_n = 0u;
  __syncthreads();
  if (R.pen) {
    uint32_t bad = 0;
    for (int64_t h = h0 + tid; h < h1; h += kThreads) {
      const int id = a.history_ids[h];
      if (id < 0 || id >= V) {
        bad = 1;
        continue;
      }
      atomicOr(&sh.bitmap[id >> 5], 1u << (id & 31));
    }
    if (bad && status) atomicOr(status, NS_STATUS_BAD_HISTORY_ID);
  }
  if (tid == 0 && status && (in.src < 0 || in.src >= a.num_logit_rows)) atomicOr(status, NS_STATUS_BAD_SAMPLE_INDEX);
  __syncthreads();

  // row uniform
  double u;
  if (a.uniforms) {
    u = (double)a.uniforms[row];
  } else {
    const uint64_t key = (P.flags & NS_ROW_SEED) ? P.seed : a.philox_seed;
    u = philox_uniform(key, a.philox_offset, (uint64_t)(a.row_offset + row));
  }
  if (!(u >= 0.0)) u = 0.0;
  if (u >= 1.0) u = 0x1.fffffffffffffp-1;

  const Feed fd1 = feed_first<E>(ctl, i, ln);
  RingWalk rw(sh, ln, fd1, stage);
  // chunks [c0, c1) of this row's first pass, specialised on whether the penalty is on
  auto first_range = [&](int c0, int c1, auto&& body) {
    if (R.pen) ring_range<E, true>(sh, ln, fd1, rw, c0, c1, nch, R.pp, body);
    else ring_range<E, false>(sh, ln, fd1, rw, c0, c1, nch, R.pp, body);
  };

  // ================================================================ first pass
  Stats S;
  float m0 = 0.0f;
  bool over = false;      // GENERAL: some e >= 2^32 (the row maximum is far above m0)
  uint32_t lumped = 0u;   // top-p: some e fell into the level's lumped last bucket
  float tau = -INFINITY;  // TOPK: bound on the k-th largest penalized logit
  // argmax bookkeeping for greedy rows: the largest value and the chunk it
  // was first seen in; the element index is recovered after the pass
  float best = -INFINITY;
  int best_c = -1;
  if (pre) {
    // the pre-pass streamed this row: add its parts' histograms and statistics
    const uint4* gh = reinterpret_cast<const uint4*>(&g_pre_hist[row][0][0]);
    for (int b = tid; b < kBins / 4; b += kThreads) {
      uint4 acc = gh[b];
#pragma unroll
      for (int q = 1; q < kPreParts; ++q) {
        const uint4 v = gh[q * (kBins / 4) + b];
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      reinterpret_cast<uint4*>(sh.hist)[b] = acc;
    }
    uint32_t key = 0u;
    double zz = 0.0;
#pragma unroll
    for (int q = 0; q < kPreParts; ++q) {
      key = max(key, g_pre_stats[row][q].mxkey);
      zz += g_pre_stats[row][q].z;
    }
    m0 = g_pre_stats[row][0].m0;
    S.nan = (key == 0xffffffffu);
    S.mx = S.nan ? __int_as_float(0x7fc00000) : key2f(key);
    S.arg = INT_MAX;
    S.z = zz;
    S.over = false;
    S.lumped = false;
    __syncthreads();
    if (!(S.nan || S.mx == INFINITY || S.mx == -INFINITY)) {
      over = __float_as_uint(exp_shifted(scaled(R, S.mx), m0)) > kTopFine;
      lumped = (sh.hist[kBins - 1] != 0u) ? 1u : 0u;
    }
  } else {
  if (mode == kGreedy) {
    float st = -INFINITY;
    first_range(0, nch, [&](int c, const float(&x)[EPT], int, bool) {
      float mv = x[0];
#pragma unroll
      for (int j = 1; j < EPT; ++j) mv = fmax_nan(mv, x[j]);
      if (mv > best) {
        best = mv;
        best_c = c;
      }
      st = fmax_nan(st, mv);
    });
    S = block_stats(ctl, st, arg_of<E>(R, sh.bitmap, ln, best, best_c), 0.0, 0u, tid);
  } else if (mode == kTopk) {
    // the bound from chunk 0's thread maxima, refreshed after chunk kRefreshAt
    float tmax = peek_max<E>(sh, ln, stage, R.pen, R.pp);
    tau = topk_bound(R.k, R.t_one, R.T, R.rT, &ctl, sh.tm, tmax, tid);
    // each warp appends to its own list (slots counted in a warp-uniform register)
    unsigned long long* wl = sh.cand + warp * kWarpCands;
    int wcnt = 0;
    auto body = [&](int c, const float(&x)[EPT], int idx0, bool live) {
      float mv = x[0];
#pragma unroll
      for (int j = 1; j < EPT; ++j) mv = fmax_nan(mv, x[j]);
      if (R.greedy && mv > best) {
        best = mv;
        best_c = c;
      }
      tmax = fmax_nan(tmax, mv);
      if (__any_sync(0xffffffffu, live && mv >= tau)) {
        Chunk<E> ch;
#pragma unroll
        for (int j = 0; j < EPT; ++j) ch.v[j] = x[j];
        wcnt = topk_insert<E>(wl, wcnt, ch, idx0, tau, live, R.t_one, R.T, R.rT, lane);
      }
    };
    const int cr = min(kRefreshAt + 1, nch);
    first_range(0, cr, body);
    tau = topk_bound(R.k, R.t_one, R.T, R.rT, &ctl, sh.tm, tmax, tid);
    first_range(cr, nch, body);
    if (lane == 0) ctl.red_j[warp] = wcnt;
    S = block_stats(ctl, tmax, R.greedy ? arg_of<E>(R, sh.bitmap, ln, best, best_c) : INT_MAX, 0.0, 0u, tid);
    if (!(S.nan || S.mx == INFINITY || S.mx == -INFINITY))
      tau = topk_bound(R.k, R.t_one, R.T, R.rT, &ctl, sh.tm, tmax, tid);
  } else {
    // GENERAL: e = exp(s - m0) with m0 the first chunk's maximum
    float lmax = -INFINITY;
    double lz = 0.0;
    const bool with_e = R.k == 0;  // large top-k computes its masses after the select
    if (with_e) {
      const float pm = peek_max<E>(sh, ln, stage, R.pen, R.pp);
      const uint32_t wk = __reduce_max_sync(0xffffffffu, pm != pm ? 0u : f2key(pm));
      if (lane == 0) ctl.red_b[warp] = wk;
      __syncthreads();
      uint32_t ck = 0u;
      for (int w = 0; w < kWarps; ++w) ck = max(ck, ctl.red_b[w]);
      const float mx = key2f(ck);
      m0 = (mx > -INFINITY && mx < INFINITY) ? scaled(R, mx) : 0.0f;
    }
    first_range(0, nch, [&](int c, const float(&x)[EPT], int, bool) {
      float mv = x[0];
#pragma unroll
      for (int j = 1; j < EPT; ++j) mv = fmax_nan(mv, x[j]);
      if (R.greedy && mv > best) {
        best = mv;
        best_c = c;
      }
      lmax = fmax_nan(lmax, mv);
      if (!with_e) return;
      float s[EPT];
      if (R.t_one) {
#pragma unroll
        for (int j = 0; j < EPT; ++j) s[j] = x[j];
      } else {
#pragma unroll
        for (int j = 0; j < EPT; ++j) s[j] = div_by_const(x[j], R.T, R.rT);
      }
      float part = 0.0f;
#pragma unroll
      for (int j = 0; j < EPT; ++j) {
        const float e = exp_shifted(s[j], m0);
        part = __fadd_rn(part, e);
        if (want_hist) {
          // no range test: e >= 2^32 and e < 2^-32 both clamp into the last bucket
          const uint32_t bits = __float_as_uint(e);
          atomicAdd(&sh.hist[min((kTopFine - bits) >> kShFine, (uint32_t)(kBins - 1))], approx_mass13(bits));
        }
      }
      lz += (double)part;
    });
    S = block_stats(ctl, lmax, R.greedy ? arg_of<E>(R, sh.bitmap, ln, best, best_c) : INT_MAX, lz, 0u, tid);
    if (with_e && !(S.nan || S.mx == INFINITY || S.mx == -INFINITY)) {
      over = __float_as_uint(exp_shifted(scaled(R, S.mx), m0)) > kTopFine;
      lumped = (want_hist && sh.hist[kBins - 1] != 0u) ? 1u : 0u;
    }
  }
  stage = (stage + nch) % kStages;
  }

  if (a.out_penalized) {
    // debug output: the logits after the repetition penalty (sampler.py:31-38)
    float* const pen_out = a.out_penalized + out_off;
    global_pass<E>(R, sh.bitmap, tid, [&](int, const float(&x)[EPT], int idx0, bool live) {
      if (!live) return;
#pragma unroll
      for (int j = 0; j < EPT; ++j) pen_out[idx0 + j] = x[j];
    });
  }

  // ================================================================ rows whose softmax is NaN
  // NaN or +inf logits, or all -inf: uniform probabilities 1/V (sampler.py:76-80)
  if (S.nan || S.mx == INFINITY || S.mx == -INFINITY) {
    if (ring2 || pre) stage = drain_pass(sh.ring, feed_second<E>(ctl, i, ln, false), ln, nch, stage, E::kNegInf2);
    int tok;
    if (R.greedy) {
      // torch.argmax: the first NaN, else the first +inf, else index 0.  The
      // penalty keeps NaN and +inf, so the raw logits decide.
      int my_nan = INT_MAX, my_pinf = INT_MAX;
      global_pass<E>(R, sh.bitmap, tid, [&](int, const float(&x)[EPT], int idx0, bool live) {
        if (!live) return;
#pragma unroll
        for (int j = 0; j < EPT; ++j) {
          if (x[j] != x[j]) my_nan = min(my_nan, idx0 + j);
          if (x[j] == INFINITY) my_pinf = min(my_pinf, idx0 + j);
        }
      });
      my_nan = (int)__reduce_min_sync(0xffffffffu, (uint32_t)my_nan);
      my_pinf = (int)__reduce_min_sync(0xffffffffu, (uint32_t)my_pinf);
      if (lane == 0) {
        ctl.red_i[warp] = my_nan;
        ctl.red_j[warp] = my_pinf;
      }
      __syncthreads();
      int fn = INT_MAX, fp = INT_MAX;
      for (int w = 0; w < kWarps; ++w) {
        fn = min(fn, ctl.red_i[w]);
        fp = min(fp, ctl.red_j[w]);
      }
      tok = (fn != INT_MAX) ? fn : (fp != INT_MAX) ? fp : 0;
    } else {
      tok = min(V - 1, (int)(u * (double)V));
    }
    if (tid == 0) write_token(a.out_tokens, out_i32, row, tok);
    if (debug) {
      const float pu = 1.0f / (float)V;
      global_pass<E>(R, sh.bitmap, tid, [&](int, const float(&x)[EPT], int idx0, bool live) {
        if (!live) return;
#pragma unroll
        for (int j = 0; j < EPT; ++j) {
          if (a.out_probs) a.out_probs[out_off + idx0 + j] = pu;
          if (a.out_filtered) a.out_filtered[out_off + idx0 + j] = scaled(R, x[j]);
        }
      });
    }
    return;
  }

  // ================================================================ GREEDY
  if (mode == kGreedy) {
    if (tid == 0) write_token(a.out_tokens, out_i32, row, S.arg);
    return;
  }

  // ================================================================ TOPK
  if (mode == kTopk) {
    bool fits = true;
    for (int w = 0; w < kWarps; ++w) fits &= ctl.red_j[w] <= kWarpCands;
    if (fits) {
      // the candidates at or above the final bound, from every warp's list
      const float sig = scaled(R, tau);
      unsigned long long* list = reinterpret_cast<unsigned long long*>(sh.hist);
      if (tid == 0) ctl.list_n = 0u;
      __syncthreads();
      for (int r = tid; r < kCandCap; r += kThreads) {
        const bool valid = (r % kWarpCands) < ctl.red_j[r / kWarpCands];
        const unsigned long long key = valid ? sh.cand[r] : 0ull;
        list_append(list, &ctl.list_n, valid && key_value(key) >= sig, key, kCandCap, lane);
      }
      __syncthreads();
      const int nl = (int)ctl.list_n;
      if (nl > 0) {
        sort_keys(list, nl, tid);
        if (warp == 0) {
          // top-k keeps every rank whose value ties the k-th (sampler.py:53-58)
          const float s0 = key_value(list[0]);
          const float thr = key_value(list[min(R.k, nl) - 1]);
          int n1 = nl;
          for (int c0 = 0; c0 < nl; c0 += 32) {
            const int r = c0 + lane;
            const uint32_t below = __ballot_sync(0xffffffffu, r < nl && key_value(list[r]) < thr);
            if (below) {
              n1 = c0 + __ffs(below) - 1;
              break;
            }
          }
          float* ce = reinterpret_cast<float*>(sh.cand);  // masses by rank (the candidates are consumed)
          double z = 0.0;
          for (int r = lane; r < n1; r += 32) {
            const float e = exp_shifted(key_value(list[r]), s0);
            ce[r] = e;
            z += (double)e;
          }
          z = warp_dsum(z);
          __syncwarp();
          int m2 = n1;
          if (R.topp) {
            // keep exactly ranks 0..j0 in (value desc, index asc) order (sampler.py:60-73)
            double run = 0.0;
            int j0 = -1;
            for (int c0 = 0; c0 < n1 && j0 < 0; c0 += 32) {
              const int r = c0 + lane;
              const double inc = warp_incl_f64(r < n1 ? (double)ce[r] : 0.0, lane) + run;
              const uint32_t bal = __ballot_sync(0xffffffffu, r < n1 && topp_crossed(inc, z, R.p));
              if (bal) j0 = c0 + __ffs(bal) - 1;
              run = __shfl_sync(0xffffffffu, inc, 31);
            }
            if (j0 >= 0) m2 = j0 + 1;
            z = 0.0;
            for (int r = lane; r < m2; r += 32) z += (double)ce[r];
            z = warp_dsum(z);
          }
          // inverse CDF in vocabulary order over the kept ranks
          const double target = u * z;
          int tok = INT_MAX, last = -1;
          for (int r = lane; r < m2; r += 32) {
            const int ir = key_index(list[r]);
            const double er = (double)ce[r];
            if (er > 0.0) last = max(last, ir);
            double before = 0.0;
            for (int q2 = 0; q2 < m2; ++q2)
              if (key_index(list[q2]) < ir) before += (double)ce[q2];
            if (er > 0.0 && before <= target && target < before + er) tok = min(tok, ir);
          }
          tok = (int)__reduce_min_sync(0xffffffffu, (uint32_t)tok);
          last = (int)__reduce_max_sync(0xffffffffu, (uint32_t)(last + 1)) - 1;
          if (tok == INT_MAX) tok = last >= 0 ? last : key_index(list[0]);  // rounding at the very top
          if (R.greedy) tok = key_index(list[0]);
          if (lane == 0) {
            write_token(a.out_tokens, out_i32, row, tok);
            ctl.dec_thr = key_value(list[m2 - 1]);
            ctl.dec_thr_idx = key_index(list[m2 - 1]);
            ctl.dec_z = z;
          }
        }
        if (debug) {
          __syncthreads();
          const float s0 = key_value(list[0]);
          const float thr2 = ctl.dec_thr;
          const int thr_idx2 = ctl.dec_thr_idx;
          const double z2 = ctl.dec_z;
          global_pass<E>(R, sh.bitmap, tid, [&](int, const float(&x)[EPT], int idx0, bool live) {
            if (!live) return;
#pragma unroll
            for (int j = 0; j < EPT; ++j) {
              const float s = scaled(R, x[j]);
              const bool kept = s > thr2 || (s == thr2 && idx0 + j <= thr_idx2);
              if (a.out_filtered) a.out_filtered[out_off + idx0 + j] = kept ? s : -INFINITY;
              if (a.out_probs)
                a.out_probs[out_off + idx0 + j] = kept ? (float)((double)exp_shifted(s, s0) / z2) : 0.0f;
            }
          });
        }
        return;
      }
    }
    // a warp's candidate list overflowed: the row takes the (exact) general path
    mode = kGeneral;
  }

  // ================================================================ GENERAL
  const float m = scaled(R, S.mx);
  Keep K;
  K.m0 = m0;
  K.have_k = false;
  K.thr_k = -INFINITY;
  K.window = false;
  K.win_lo = K.win_hi = 0u;
  K.thr = -INFINITY;
  K.thr_idx = INT_MAX;
  double z = S.z;
  // the first pass's masses hold unless top-k comes first or e passed 2^32
  const bool first_ok = R.k == 0 && !over;
  if (R.k > 0) {
    K.have_k = true;
    K.thr_k = scaled(R, radix_select<E>(R, sh, tid));
  }
  // (Re)compute the masses against m0 with a re-read of the row, plus the
  // locator histogram of level `lv` for top-p rows.
  auto stats_pass = [&](const Level& lv, bool hist_only) {
    const Keep K0 = K;
    if (R.topp)
      for (int b = tid; b < kBins / 4; b += kThreads) reinterpret_cast<uint4*>(sh.hist)[b] = make_uint4(0, 0, 0, 0);
    __syncthreads();
    double lz = 0.0;
    const bool hist = R.topp;
    global_pass<E>(R, sh.bitmap, tid, [&](int, const float(&x)[EPT], int, bool live) {
      if (!live) return;
      float part = 0.0f;
#pragma unroll
      for (int j = 0; j < EPT; ++j) {
        const float e = K0.mass(scaled(R, x[j]));
        part = __fadd_rn(part, e);
        if (hist) {
          const uint32_t bits = __float_as_uint(e);
          atomicAdd(&sh.hist[min((lv.top - bits) >> lv.sh, (uint32_t)(kBins - 1))], approx_mass13(bits));
        }
      }
      lz += (double)part;
    });
    __syncthreads();
    lumped = (hist && sh.hist[kBins - 1] != 0u) ? 1u : 0u;
    if (!hist_only) z = block_segments(ctl, lz, tid);
  };
  Level lv{kTopFine, kShFine, true};
  if (!first_ok) {
    m0 = m;
    K.m0 = m0;
    stats_pass(lv, false);
  }

  double zk = z;
  bool ring_used = false;
  bool pm_ok = false;  // ctl.pm holds the kept masses per draw piece
  if (R.topp) {
    topp_window(&ctl, sh.hist, lv, 0.0, topp_threshold(z, R.p), tid);
    if (!ctl.sel_found && lumped) {
      // the boundary may lie among masses below the level: locate it on the wide one
      lv = Level{kTopWide, kShWide, true};
      stats_pass(lv, true);
      topp_window(&ctl, sh.hist, lv, 0.0, topp_threshold(z, R.p), tid);
    }
    const bool crossed = ctl.sel_found != 0;
    uint32_t win_lo = 0u, win_hi = 0u;
    float est = 0.0f;
    if (crossed) {
      win_lo = lv.lo_key(ctl.sel_hi);
      win_hi = lv.hi_key(ctl.sel_lo);
      est = ctl.sel_est;
    }
    int refines = 0;
    bool force_refine = false;
    while (crossed) {
      if ((est > 0.9f * (float)kCandCap || force_refine) && lv.sh > 0 && refines < 5) {
        // ---- refine inside [win_lo, win_hi]: finer buckets, exact mass above the window
        const uint32_t span = win_hi - win_lo + 1u;
        int sh2 = 0;
        while (((span + (1u << sh2) - 1u) >> sh2) > (uint32_t)(kBins - 1)) ++sh2;
        if (sh2 >= lv.sh) {
          refines = 5;  // the window is too wide to split further: collect it as it is
          continue;
        }
        force_refine = false;
        ++refines;
        for (int b = tid; b < kBins / 4; b += kThreads) reinterpret_cast<uint4*>(sh.hist)[b] = make_uint4(0, 0, 0, 0);
        __syncthreads();
        double la = 0.0;
        const Keep K1 = K;
        const uint32_t wlo = max(win_lo, 1u), whi = win_hi;
        global_pass<E>(R, sh.bitmap, tid, [&](int, const float(&x)[EPT], int, bool live) {
          if (!live) return;
          float part = 0.0f;
#pragma unroll
          for (int j = 0; j < EPT; ++j) {
            const float e = K1.mass(scaled(R, x[j]));
            const uint32_t bits = __float_as_uint(e);
            if (bits > whi) part = __fadd_rn(part, e);
            else if (bits >= wlo) atomicAdd(&sh.hist[(whi - bits) >> sh2], approx_mass13(bits));
          }
          la += (double)part;
        });
        const double above_lv = block_dsum(ctl, la, tid);
        const Level lv2{win_hi, sh2, false};
        topp_window(&ctl, sh.hist, lv2, above_lv, topp_threshold(z, R.p), tid);
        if (ctl.sel_found) {
          lv = lv2;
          win_lo = lv.lo_key(ctl.sel_hi);
          win_hi = lv.hi_key(ctl.sel_lo);
          est = ctl.sel_est;
        } else {
          refines = 5;  // keep the previous window: it still contains the boundary
        }
        continue;
      }
      // ---- collection: exact mass above the window per warp range; window members
      if (tid == 0) ctl.cand_n = 0u;
      __syncthreads();
      double la = 0.0;
      const Keep K1 = K;
      const uint32_t wlo = max(win_lo, 1u), whi = win_hi;
      // per-thread mass above the window in the current draw piece (kStages
      // chunks; chunks are visited in order from 0, the same in every lane)
      float pacc = 0.0f;
      int pleft = kStages, pidx = 0;
      auto piece_end = [&](int c, float part) {
        pacc = __fadd_rn(pacc, part);
        if (--pleft == 0 || c == nch - 1) {
          const double ps = warp_dsum((double)pacc);
          if (lane == 0) ctl.pm[warp][pidx] = ps;
          pacc = 0.0f;
          pleft = kStages;
          ++pidx;
        }
      };
      auto collect = [&](int c, const float(&x)[EPT], int idx0, bool live) {
        float part = 0.0f;
        if (live) {
          float s[EPT];
          if (R.t_one) {
#pragma unroll
            for (int j = 0; j < EPT; ++j) s[j] = x[j];
          } else {
#pragma unroll
            for (int j = 0; j < EPT; ++j) s[j] = div_by_const(x[j], R.T, R.rT);
          }
          bool anym = false;
          uint32_t bits[EPT];
#pragma unroll
          for (int j = 0; j < EPT; ++j) {
            const float e = K1.mass(s[j]);
            bits[j] = __float_as_uint(e);
            if (bits[j] > whi) part = __fadd_rn(part, e);
            anym |= (bits[j] >= wlo && bits[j] <= whi);
          }
          if (anym) {
            // rare: append this thread's window members one by one
#pragma unroll
            for (int j = 0; j < EPT; ++j) {
              if (bits[j] >= wlo && bits[j] <= whi) {
                const uint32_t slot = atomicAdd(&ctl.cand_n, 1u);
                if (slot < (uint32_t)kCandCap) sh.cand[slot] = rank_key(s[j], idx0 + j);
              }
            }
          }
        }
        la += (double)part;
        piece_end(c, part);
      };
      if ((ring2 || pre) && !ring_used && !K.have_k) {
        ring_used = true;
        const Feed fd2 = pre ? fd1 : feed_second<E>(ctl, i, ln, true);
        const float mm = m0;
        auto collect_ring = [&](int c, const float(&x)[EPT], int idx0, bool) {
          float s[EPT];
          if (R.t_one) {
#pragma unroll
            for (int j = 0; j < EPT; ++j) s[j] = x[j];
          } else {
#pragma unroll
            for (int j = 0; j < EPT; ++j) s[j] = div_by_const(x[j], R.T, R.rT);
          }
          float part = 0.0f;
          bool anym = false;
          uint32_t bits[EPT];
#pragma unroll
          for (int j = 0; j < EPT; ++j) {
            const float e = exp_shifted(s[j], mm);
            bits[j] = __float_as_uint(e);
            part = bits[j] > whi ? __fadd_rn(part, e) : part;
            anym |= (bits[j] - wlo) <= (whi - wlo);
          }
          la += (double)part;
          if (anym) {
#pragma unroll
            for (int j = 0; j < EPT; ++j) {
              if ((bits[j] - wlo) <= (whi - wlo)) {
                const uint32_t slot = atomicAdd(&ctl.cand_n, 1u);
                if (slot < (uint32_t)kCandCap) sh.cand[slot] = rank_key(s[j], idx0 + j);
              }
            }
          }
          piece_end(c, part);
        };
        if (R.pen) ring_pass<E, true>(sh, ln, fd2, nch, stage, R.pp, collect_ring);
        else ring_pass<E, false>(sh, ln, fd2, nch, stage, R.pp, collect_ring);
      } else {
        global_pass<E>(R, sh.bitmap, tid, collect);
      }
      const double above = block_segments(ctl, la, tid);
      const uint32_t ntot = ctl.cand_n;
      if (ntot > (uint32_t)kCandCap && lv.sh > 0 && refines < 5) {
        force_refine = true;  // the window held more elements than estimated
        continue;
      }
      if (ntot > (uint32_t)kCandCap && lv.sh == 0 && win_hi - max(win_lo, 1u) < (uint32_t)kBins) {
        // a tie group (or many members of few values) at single-value resolution
        zk = topp_ties<E>(R, sh, K, max(win_lo, 1u), win_hi, above, z, status, tid);
        break;
      }
      const int n = (int)min(ntot, (uint32_t)kCandCap);
      if (ntot <= (uint32_t)kCandCap) {
        // ---- decision by sub-buckets of the members (the usual case)
        double kept_m = 0.0;
        if (member_decide<E>(sh, n, max(win_lo, 1u), win_hi, m0, above, topp_threshold(z, R.p), W, kept_m, tid)) {
          zk = above + kept_m;
          pm_ok = true;
          K.window = true;
          K.win_lo = win_lo;
          K.win_hi = win_hi;
          K.thr = ctl.dec_thr;
          K.thr_idx = ctl.dec_thr_idx;
          break;
        }
      }
      // ---- decision on the sorted window members: the first rank whose
      // inclusive mass crosses (block-wide scan, 4 ranks per thread)
      if (ntot > (uint32_t)kCandCap && tid == 0 && status) atomicOr(status, NS_STATUS_CAP_OVERFLOW);
      sort_keys(sh.cand, n, tid);
      if (tid == 0) ctl.misc = INT_MAX;
      float er[4];
      double tsum = 0.0;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int r = 4 * tid + q;
        er[q] = r < n ? exp_shifted(key_value(sh.cand[r]), m0) : 0.0f;
        tsum += (double)er[q];
      }
      {
        const double inc = warp_incl_f64(tsum, lane);
        if (lane == 31) ctl.red_e[warp] = inc;
        __syncthreads();
        double run = above + inc - tsum;
        for (int w = 0; w < warp; ++w) run += ctl.red_e[w];
        if (ntot <= (uint32_t)kCandCap) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            run += (double)er[q];
            if (er[q] > 0.0f && topp_crossed(run, z, R.p)) {
              atomicMin(&ctl.misc, 4 * tid + q);
              break;
            }
          }
        }
        __syncthreads();
      }
      // no crossing inside (or overflow): keep the whole window
      const int j0 = ctl.misc == INT_MAX ? n - 1 : ctl.misc;
      if (tid == 0) {
        ctl.dec_thr = n > 0 ? key_value(sh.cand[j0]) : -INFINITY;
        ctl.dec_thr_idx = n > 0 ? key_index(sh.cand[j0]) : INT_MAX;
      }
      // kept members join their warp ranges' masses
      double lk = 0.0;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int r = 4 * tid + q;
        if (r <= j0 && er[q] > 0.0f) {
          const int idx = key_index(sh.cand[r]);
          atomicAdd(&ctl.seg[idx / W], (double)er[q]);
          atomicAdd(&ctl.pm[idx / W][(idx % W) / E::kPiece / kStages], (double)er[q]);
          lk += (double)er[q];
        }
      }
      zk = above + block_dsum(ctl, lk, tid);  // (its barriers order the range updates)
      pm_ok = ntot <= (uint32_t)kCandCap;
      K.window = true;
      K.win_lo = win_lo;
      K.win_hi = win_hi;
      K.thr = ctl.dec_thr;
      K.thr_idx = ctl.dec_thr_idx;
      break;
    }
    if (!crossed) {
      // top-p never crosses: every element stays; draw over all masses
      double lz = 0.0;
      const Keep K1 = K;
      auto plain = [&](int, const float(&x)[EPT], int, bool live) {
        if (!live) return;
        float part = 0.0f;
#pragma unroll
        for (int j = 0; j < EPT; ++j) part = __fadd_rn(part, K1.mass(scaled(R, x[j])));
        lz += (double)part;
      };
      if ((ring2 || pre) && !ring_used) {
        ring_used = true;
        const Feed fd2 = pre ? fd1 : feed_second<E>(ctl, i, ln, true);
        if (R.pen) ring_pass<E, true>(sh, ln, fd2, nch, stage, R.pp, plain);
        else ring_pass<E, false>(sh, ln, fd2, nch, stage, R.pp, plain);
      } else {
        global_pass<E>(R, sh.bitmap, tid, plain);
      }
      zk = block_segments(ctl, lz, tid);
    }
  }
  if ((ring2 || pre) && !ring_used)
    stage = drain_pass(sh.ring, feed_second<E>(ctl, i, ln, false), ln, nch, stage, E::kNegInf2);

  // ---- the draw
  const int tok = R.greedy ? S.arg
                 : pm_ok   ? draw_piece<E>(R, sh, K, u * zk, S.arg, tid)
                           : draw_token<E>(R, sh, K, u * zk, S.arg, tid);
  if (tid == 0) write_token(a.out_tokens, out_i32, row, tok == INT_MAX ? 0 : tok);
  if (debug) {
    global_pass<E>(R, sh.bitmap, tid, [&](int, const float(&x)[EPT], int idx0, bool live) {
      if (!live) return;
#pragma unroll
      for (int j = 0; j < EPT; ++j) {
        const float s = scaled(R, x[j]);
        const float e = K.mass(s);
        const bool kept = K.kept(s, e, idx0 + j);
        if (a.out_filtered) a.out_filtered[out_off + idx0 + j] = kept ? s : -INFINITY;
        if (a.out_probs) a.out_probs[out_off + idx0 + j] = (kept && e > 0.f) ? (float)((double)e / zk) : 0.0f;
      }
    });
  }
}

// ---------------------------------------------------------------- the kernel
template <class E>
__global__ void __launch_bounds__(kThreads, 2) row_kernel(const NsSampleArgs a, int W, int nch, int pre_on) {
  extern __shared__ __align__(128) unsigned char smem[];
  const Layout L = make_layout(a.vocab_size);
  Sh sh;
  sh.ctl = reinterpret_cast<Ctl*>(smem + L.ctl);
  sh.ring = smem + L.ring;
  sh.bitmap = reinterpret_cast<uint32_t*>(smem + L.bitmap);
  sh.cand = reinterpret_cast<unsigned long long*>(smem + L.cand);
  sh.hist = reinterpret_cast<uint32_t*>(smem + L.hist);
  sh.tm = reinterpret_cast<uint32_t*>(smem + L.tm);
  Ctl& ctl = *sh.ctl;
  const int tid = threadIdx.x;
  const int G = gridDim.x;
  const int t0 = blockIdx.x;  // this block takes positions t0, t0 + G, ... of the row order
  const bool debug = (a.out_filtered != nullptr) || (a.out_probs != nullptr);
  const Lane ln = make_lane<E>(a.vocab_size, W, tid);

  if (t0 < a.num_rows) fetch_row_inputs(a, ctl.rin[0], t0, tid);
  if (t0 + G < a.num_rows) fetch_row_inputs(a, ctl.rin[1], t0 + G, tid);
  __syncthreads();
  if (tid == 0) make_plan(a, ctl, 0, t0, debug, pre_on != 0);
  __syncthreads();
  ring_start<E>(ctl, sh.ring, ln);
  int stage = 0;
  for (int i = 0, t = t0; t < a.num_rows; ++i, t += G) {
    __syncthreads();  // the previous row is finished; row i+1's inputs are in place
    if (tid == 0) make_plan(a, ctl, i + 1, t + G, debug, pre_on != 0);
    if (t + 2 * G < a.num_rows) fetch_row_inputs(a, ctl.rin[(i + 2) & 3], t + 2 * G, tid);
    sample_row<E>(a, sh, ln, stage, i, (int)ctl.rin[i & 3].row, nch, W);
  }
  cp_async_wait_all();  // nothing may land in shared memory after the block exits
}

// ---------------------------------------------------------------- host side
struct DevState {
  size_t smem_set[2] = {0, 0};
  int blocks_per_sm[2] = {0, 0};
  size_t occ_for[2] = {0, 0};
  int sms = 0;
  uint32_t* scratch_hist = nullptr;  // device addresses of the pre-pass scratch (ns_sample_noalloc)
  PreStats* scratch_stats = nullptr;
};

// Where a launch's pre-pass writes: nullptr in both = the scratch named in
// device code (ns_sample); else its device address (ns_sample_noalloc).
struct ScratchAt {
  uint32_t* hist = nullptr;
  PreStats* stats = nullptr;
};
std::mutex g_mu;
DevState g_dev[64];

}  // namespace rk

bool rows_supported(const NsSampleArgs& a) {
  const int esize = a.logits_dtype == NS_DTYPE_BF16 ? 2 : 4;
  const uintptr_t p = reinterpret_cast<uintptr_t>(a.logits);
  return a.vocab_size >= rk::kMinVocab && a.vocab_size <= rk::kMaxVocab && p % 16 == 0 &&
         ((int64_t)a.logits_row_stride * esize) % 16 == 0 && ((int64_t)a.vocab_size * esize) % 16 == 0;
}

static int rows_launch_at(const NsSampleArgs& a, cudaStream_t stream, int device, std::string& err,
                          const rk::ScratchAt& at);

int rows_launch(const NsSampleArgs& a, cudaStream_t stream, int device, std::string& err) {
  return rows_launch_at(a, stream, device, err, rk::ScratchAt{});
}

int rows_noalloc_setup(int device, std::string& err) {
  using namespace rk;
  std::lock_guard<std::mutex> lk(g_mu);
  if (device < 0 || device >= 64) {
    err = "device ordinal >= 64";
    return NS_ERR_UNSUPPORTED;
  }
  DevState& ds = g_dev[device];
  if (ds.scratch_hist && ds.scratch_stats) return NS_OK;
  // the arrays' names are host-side stand-ins; the kernels need their device
  // addresses on this (the current) device
  void* h = nullptr;
  void* st = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&h, g_pre_hist);
  if (e == cudaSuccess) e = cudaGetSymbolAddress(&st, g_pre_stats);
  if (e != cudaSuccess || !h || !st) {
    err = std::string("cudaGetSymbolAddress of the pre-pass scratch: ") + cudaGetErrorString(e);
    return NS_ERR_CUDA;
  }
  ds.scratch_hist = static_cast<uint32_t*>(h);
  ds.scratch_stats = static_cast<PreStats*>(st);
  return NS_OK;
}

int rows_launch_noalloc(const NsSampleArgs& a, cudaStream_t stream, int device, std::string& err) {
  using namespace rk;
  ScratchAt at;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (device < 0 || device >= 64 || !g_dev[device].scratch_hist) {
      err = "ns_sample_noalloc: the device's scratch address was not set up";
      return NS_ERR_CUDA;
    }
    at.hist = g_dev[device].scratch_hist;
    at.stats = g_dev[device].scratch_stats;
  }
  return rows_launch_at(a, stream, device, err, at);
}

static int rows_launch_at(const NsSampleArgs& a, cudaStream_t stream, int device, std::string& err,
                          const rk::ScratchAt& at) {
  using namespace rk;
  const bool bf16 = a.logits_dtype == NS_DTYPE_BF16;
  const int ept = bf16 ? EBF16::kEPT : EF32::kEPT;
  // warp range: V / 16 rounded up to whole 16-byte slots
  const int W = ((a.vocab_size + kWarps - 1) / kWarps + ept - 1) / ept * ept;
  const int nch = (W + 32 * ept - 1) / (32 * ept);
  const Layout L = make_layout(a.vocab_size);
  const void* fn = bf16 ? reinterpret_cast<const void*>(&row_kernel<EBF16>)
                        : reinterpret_cast<const void*>(&row_kernel<EF32>);
  const int fi = bf16 ? 1 : 0;
  int per_sm = 0, sms = 0;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (device < 0 || device >= 64) {
      err = "ns_sample: device ordinal >= 64";
      return NS_ERR_UNSUPPORTED;
    }
    DevState& ds = g_dev[device];
    cudaError_t e;
    if (ds.sms == 0) {
      e = cudaDeviceGetAttribute(&ds.sms, cudaDevAttrMultiProcessorCount, device);
      if (e != cudaSuccess) {
        err = std::string("cudaDeviceGetAttribute: ") + cudaGetErrorString(e);
        return NS_ERR_CUDA;
      }
    }
    if (ds.smem_set[fi] < L.total) {
      e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total);
      if (e != cudaSuccess) {
        err = std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e);
        return NS_ERR_CUDA;
      }
      ds.smem_set[fi] = L.total;
    }
    if (ds.occ_for[fi] != L.total) {
      int n = 0;
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, kThreads, L.total);
      if (e != cudaSuccess || n <= 0) {
        err = std::string("cudaOccupancyMaxActiveBlocksPerMultiprocessor: ") +
              (e != cudaSuccess ? cudaGetErrorString(e) : "no block fits");
        return NS_ERR_CUDA;
      }
      ds.blocks_per_sm[fi] = n;
      ds.occ_for[fi] = L.total;
    }
    per_sm = ds.blocks_per_sm[fi];
    sms = ds.sms;
  }
  const int cap = per_sm * sms;
  const int grid = a.num_rows < cap ? a.num_rows : cap;
  // top-p rows of small batches: their first pass runs split over several
  // blocks per row first (same stream), the row kernel picks it up
  const bool debug = a.out_filtered != nullptr || a.out_probs != nullptr;
  const char* pe_env = std::getenv("NS_PREPASS");  // "0": every row streams in its own block
  int pre_on = (!debug && a.num_rows <= kPreRows && !(pe_env && pe_env[0] == '0')) ? 1 : 0;
  if (pre_on) {
    cudaError_t pe;
    if (at.hist) {
      const void* pfn = bf16 ? reinterpret_cast<const void*>(&pre_kernel_at<EBF16>)
                             : reinterpret_cast<const void*>(&pre_kernel_at<EF32>);
      uint32_t* h = at.hist;
      PreStats* st = at.stats;
      void* pargs[] = {const_cast<NsSampleArgs*>(&a), const_cast<int*>(&W), &h, &st};
      pe = cudaLaunchKernel(pfn, dim3((unsigned)(a.num_rows * kPreParts)), dim3(kThreads), pargs, 0, stream);
    } else {
      const void* pfn = bf16 ? reinterpret_cast<const void*>(&pre_kernel<EBF16>)
                             : reinterpret_cast<const void*>(&pre_kernel<EF32>);
      void* pargs[] = {const_cast<NsSampleArgs*>(&a), const_cast<int*>(&W)};
      pe = cudaLaunchKernel(pfn, dim3((unsigned)(a.num_rows * kPreParts)), dim3(kThreads), pargs, 0, stream);
    }
    if (pe != cudaSuccess) {
      err = std::string("pre-pass launch: ") + cudaGetErrorString(pe);
      return NS_ERR_CUDA;
    }
  }
  void* args[] = {const_cast<NsSampleArgs*>(&a), const_cast<int*>(&W), const_cast<int*>(&nch), &pre_on};
  const cudaError_t e = cudaLaunchKernel(fn, dim3((unsigned)grid), dim3(kThreads), args, L.total, stream);
  if (e != cudaSuccess) {
    err = std::string("row kernel launch: ") + cudaGetErrorString(e);
    return NS_ERR_CUDA;
  }
  return NS_OK;
}

}  // namespace ns

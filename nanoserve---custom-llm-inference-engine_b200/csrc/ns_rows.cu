// ns_rows.cu -- B200 (sm_100a) token sampling for batches of aligned rows:
// persistent blocks stream whole rows through a bulk-copy ring, and finish
// each row while the next one is already streaming.
//
// Replaces nanoserve/scheduler/sampler.py:21-89 (Sampler.sample); the
// cluster kernel in ns_sample.cu serves unaligned rows and small
// vocabularies.  Design:
//
//  * One block per SM, 17 warps.  Warp 16 is the producer: it takes rows
//    from a global ticket counter (the caller's row order), fetches a row's
//    inputs and moves the row in chunks of about 32 KB into a shared-memory
//    ring, one cp.async.bulk copy per chunk (global -> own shared memory,
//    mbarrier completion, no multicast).  It takes the next row's ticket
//    while the current row's last chunks are in flight and keeps the ring
//    full across row boundaries, so HBM keeps streaming while the consumers
//    finish a row.
//  * Warps 0-15 consume the ring chunk by chunk, with no block barrier per
//    chunk (each warp releases a slot on its own).  What a row's path needs
//    accumulates in registers and shared memory as the chunks pass:
//      GREEDY   the maximum and its first index (sampler.py:82-83);
//      TOPK     (0 < top_k <= 128) a lower bound on the k-th largest logit
//               (the k-th largest of the warps' top-8 per-thread maxima,
//               taken after the first chunk and refreshed after chunk 2 and
//               at the end) and every element at or above it, kept in a
//               shared candidate list (sampler.py:53-58);
//      GENERAL  masses e = exp(s - m0), m0 the scaled maximum of the first
//               chunk, summed, and for top-p rows added to a locator
//               histogram of approximate masses (sampler.py:60-76).
//    The penalty (sampler.py:31-38) and temperature (sampler.py:40-51) are
//    applied on the fly from the row's penalty bitmap.
//  * After a row's last chunk the consumers finish it: greedy and top-k
//    rows from what accumulated (top-k, top-p over the sorted candidates and
//    the draw); top-p rows locate the boundary window in the histogram and
//    re-read their row (from L2: it streamed moments before) to collect and
//    rank the window's members exactly.  The draw is an inverse CDF in
//    vocabulary order.  Rare cases (top_k > 128, candidate overflow, a row
//    maximum far above m0, NaN/inf rows, debug outputs) take exact
//    whole-row passes.
#include <cuda_runtime.h>
#include <stdint.h>

#include <climits>
#include <mutex>
#include <string>

#include "../../include/nanoserve_sampler.h"
#include "ns_device.cuh"
#include "ns_row_core.cuh"
#include "ns_rows.h"

namespace ns {
namespace rk {

constexpr int kBlockThreads = kThreads + 32;  // 16 consumer warps + the producer warp
constexpr int kChunkTarget = 32768;           // bytes per chunk (rounded to whole units)
constexpr int kMaxChunksRow = 32;             // chunks per row at most
constexpr int kUnit = 32;                     // chunk boundaries fall on multiples of 32 elements
constexpr int kRingMax = 8;                   // ring slots at most
constexpr int kRefreshChunk = 2;              // TOPK: the bound is refreshed after this chunk ...
constexpr int kRefreshMinK = 64;              // ... when k exceeds this: the bound from chunk 0 leaves
                                              // about k * chunks candidates, which fits kCandCap below it
constexpr long long kSpinLimit = 1ll << 22;   // bounded waits (a few seconds at most)

// ---------------------------------------------------------------- global workspace
// The only global state: the next row ticket and the count of blocks done
// with the call (the last one returns both to zero).
struct WsHeader {
  uint32_t ticket;
  uint32_t exited;
  uint32_t pad[30];
};
static_assert(sizeof(WsHeader) == NS_NOALLOC_WORKSPACE_BYTES, "the workspace is the header's size");

// The workspace of ns_sample_noalloc: zero when the library loads, left zero
// by every call (128 bytes, held by every GPU that loads the library).
static __device__ __align__(256) unsigned char g_static_ws[sizeof(WsHeader)];

// ---------------------------------------------------------------- the ring
// One chunk's origin, written by the producer next to its ring slot.
struct __align__(16) ChunkDesc {
  NsRowParams P;
  int64_t h0, h1;  // history range
  int64_t src;     // logits row (validated)
  int32_t row;     // the row sampled (row order applied, validated); < 0: no more work
  int32_t chunk;   // index of the chunk in the row
  int32_t e_lo;    // its first element
  int32_t nsl;     // its 16-byte slots
  uint32_t bad;    // NS_STATUS bits found by the producer (reported with chunk 0)
  int32_t pass;    // 0: the row's streaming pass; 1: its second pass (top-p rows)
  uint32_t pad[2];
};

// Launch geometry, computed on the host.
struct Geo {
  int W, nch;          // the row layout of the whole-row passes
  int nchunk, units;   // chunks per row, 32-element units per row
  int nslot;           // ring slots
  int slot_bytes;      // bytes per ring slot (the largest chunk)
  int ppc;             // second-pass pieces (kPieceSlots slots) per chunk, at most kWarps
  int o_ctl, o_bitmap, o_hist, o_cand, o_small, o_ring, smem;
};

// The second pass keeps its piece masses in the locator histogram's space,
// past the 4 KB that the member decision uses as scratch.
constexpr int kPm2Offset = 1024;               // u32 words into sh.hist
constexpr int kPm2Cap = kBins - kPm2Offset;    // floats

struct __align__(16) Ring {
  uint64_t full[kRingMax];   // the slot's bytes have landed (one arrival + the transaction count)
  uint64_t empty[kRingMax];  // every consumer warp is done with the slot (16 arrivals)
  ChunkDesc desc[kRingMax];
  // what the finishing work reads, kept here once per block (not copied per
  // thread into each call's frame)
  NsSampleArgs args;
  Geo geo;
  Sh sh;
  ChunkDesc cur;  // the row being finished
  Stats S;        // its statistics
  int n;          // ring position of the next chunk (the finisher consumes a top-p row's second pass)
  uint32_t wkey[kWarps];
  int32_t warg[kWarps];
  uint32_t wspec[kWarps];
  double wz[kWarps];
  uint32_t top8[kWarps * 8];
  float bound;   // TOPK: current lower bound (penalized logit space)
  float m0;      // GENERAL: the row's mass anchor
  uint32_t nlist;  // TOPK: candidates appended to sh.cand
  uint32_t bad;
};

__host__ __device__ inline int chunk_lo(const Geo& g, int c) {
  return (c * g.units / g.nchunk) * kUnit;  // c * units < 2^31: at most 32 * 6144
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Bounded wait on phase `parity`; false (and NS_STATUS_WAIT_TIMEOUT) if it
// never completed.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t* status) {
  for (long long i = 0; i < kSpinLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  if (status) atomicOr(status, NS_STATUS_WAIT_TIMEOUT);
  return false;
}

// ---------------------------------------------------------------- producer
// One row's inputs, as the producer fetched them.
struct RowFetch {
  bool ok;
  int row;
  uint32_t bad;
  uint4 p0, p1;
  int64_t h0, h1, src;
};

__device__ __forceinline__ RowFetch claim_row(const NsSampleArgs& a, WsHeader* hdr) {
  RowFetch f;
  f.ok = false;
  const uint32_t t = atomicAdd(&hdr->ticket, 1u);
  if (t >= (uint32_t)a.num_rows) return f;
  f.ok = true;
  f.bad = 0u;
  int row = (int)t;
  if (a.row_order) {
    const int r = __ldg(&a.row_order[t]);
    if (r >= 0 && r < a.num_rows) row = r;
    else f.bad |= NS_STATUS_BAD_ROW_ORDER;
  }
  f.row = row;
  f.p0 = __ldg(reinterpret_cast<const uint4*>(&a.row_params[row]));
  f.p1 = __ldg(reinterpret_cast<const uint4*>(&a.row_params[row]) + 1);
  f.h0 = a.history_offsets ? __ldg(&a.history_offsets[row]) : 0;
  f.h1 = a.history_offsets ? __ldg(&a.history_offsets[row + 1]) : 0;
  int64_t src = a.sample_indices ? __ldg(&a.sample_indices[row]) : (int64_t)row;
  if (src < 0 || src >= a.num_logit_rows) {
    f.bad |= NS_STATUS_BAD_SAMPLE_INDEX;
    src = 0;
  }
  f.src = src;
  return f;
}

// Rows whose finishing work reads a second pass of the row from the ring:
// top-p without top-k (the GENERAL path's locator histogram).
__host__ __device__ inline bool two_pass_row(const NsRowParams& P, int V, bool debug) {
  const bool greedy = (P.flags & NS_ROW_GREEDY) != 0u;
  const int k = (P.top_k > 0 && P.top_k < V) ? P.top_k : 0;
  return (!greedy || debug) && k == 0 && (P.flags & NS_ROW_TOP_P) != 0u;
}

// Lane 0 of warp 16: rows in ticket order, every chunk of a row in turn; the
// next row is claimed (and its inputs fetched) while the current row's last
// chunks go out, so the ring stays full across rows.
template <class E>
__device__ void producer(const NsSampleArgs& a, const Geo& g, Ring& rg, unsigned char* ring, WsHeader* hdr) {
  constexpr int esz = sizeof(typename E::Raw) / E::kEPT;
  const char* logits = static_cast<const char*>(a.logits);
  const bool debug = (a.out_filtered != nullptr) || (a.out_probs != nullptr);
  RowFetch cur = claim_row(a, hdr);
  int n = 0;
  while (cur.ok) {
    RowFetch next;
    next.ok = false;
    const char* rowp = logits + (size_t)cur.src * (size_t)a.logits_row_stride * esz;
    // top-p rows stream twice: their finishing work collects the boundary
    // window from a second pass through the ring (an L2 re-read)
    NsRowParams P;
    reinterpret_cast<uint4*>(&P)[0] = cur.p0;
    reinterpret_cast<uint4*>(&P)[1] = cur.p1;
    const int total = two_pass_row(P, a.vocab_size, debug) ? 2 * g.nchunk : g.nchunk;
    const int claim_at = max(0, total - g.nslot);
    for (int t = 0; t < total; ++t) {
      const int c = t < g.nchunk ? t : t - g.nchunk;
      if (t == claim_at) next = claim_row(a, hdr);
      const int s = n % g.nslot;
      const int use = n / g.nslot;
      if (use > 0) mbar_wait_bounded(&rg.empty[s], (uint32_t)(use - 1) & 1u, a.status);
      ChunkDesc& d = rg.desc[s];
      reinterpret_cast<uint4*>(&d.P)[0] = cur.p0;
      reinterpret_cast<uint4*>(&d.P)[1] = cur.p1;
      d.h0 = cur.h0;
      d.h1 = cur.h1;
      d.src = cur.src;
      const int lo = chunk_lo(g, c), hi = min(a.vocab_size, chunk_lo(g, c + 1));
      const uint32_t bytes = (uint32_t)(hi - lo) * esz;
      d.row = cur.row;
      d.chunk = c;
      d.e_lo = lo;
      d.nsl = (int)(bytes / 16u);
      d.bad = cur.bad;
      d.pass = t < g.nchunk ? 0 : 1;
      mbar_arrive_expect_tx(&rg.full[s], bytes);
      bulk_g2s(ring + (size_t)s * g.slot_bytes, rowp + (size_t)lo * esz, bytes, &rg.full[s]);
      ++n;
    }
    cur = next;
  }
  // no more work: a descriptor with row -1 ends the consumers' loop
  const int s = n % g.nslot;
  const int use = n / g.nslot;
  if (use > 0) mbar_wait_bounded(&rg.empty[s], (uint32_t)(use - 1) & 1u, a.status);
  rg.desc[s].row = -1;
  mbar_arrive(&rg.full[s]);
}

// ---------------------------------------------------------------- chunk passes
// Per-thread state of the row being streamed.
struct RowAcc {
  float st;    // NaN-propagating maximum of the penalized logits seen
  float best;  // largest (non-NaN) value seen, first occurrence
  int bidx;    // its index
  double lz;   // GENERAL, k == 0: sum of e = exp(s - m0)
};

// Maximum bookkeeping for one 16-byte slot.
template <class E>
__device__ __forceinline__ void track_max(RowAcc& acc, const float (&x)[E::kEPT], int idx0) {
  float mv = x[0];
#pragma unroll
  for (int q = 1; q < E::kEPT; ++q) mv = fmax_nan(mv, x[q]);
  acc.st = fmax_nan(acc.st, mv);
  if (mv > acc.best) {
    int jj = E::kEPT - 1;
#pragma unroll
    for (int q = E::kEPT - 1; q >= 0; --q)
      if (x[q] == mv) jj = q;
    acc.best = mv;
    acc.bidx = idx0 + jj;
  }
}

// The passes below take a thread's slots of a chunk (16-byte slots tid,
// tid + 512, ...) in batches of kRounds: every load of a batch first, then
// kRounds independent chains of work, so the few warps of a block keep
// enough instructions in flight.
constexpr int kRounds = 4;
constexpr int kPieceSlots = 32 * kRounds;  // slots of a second-pass piece (one warp's share of a chunk)

template <class E>
struct Batch {
  typename E::Raw raw[kRounds];
};

__device__ __forceinline__ void red_add_shared(uint32_t addr, uint32_t v) {
  asm volatile("red.shared.add.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

// Element q of a thread's slot (an unrolled select: a register array indexed
// at run time would live in local memory).
template <int N>
__device__ __forceinline__ float pick(const float (&x)[N], int q) {
  float v = x[0];
#pragma unroll
  for (int i = 1; i < N; ++i) v = (q == i) ? x[i] : v;
  return v;
}

// (shared-space loads: the ring's address reaches these loops as a generic
// pointer, and generic loads of shared memory cost more latency)
template <class E>
__device__ __forceinline__ void load_batch(const unsigned char* tile, int j0, int nsl, Batch<E>& b) {
  const uint32_t t = smem_addr(tile);
#pragma unroll
  for (int r = 0; r < kRounds; ++r) {
    const int j = j0 + r * kThreads;
    b.raw[r] = j < nsl ? E::lds_s(t + (uint32_t)j * 16u) : E::zero();
  }
}

template <class E, bool PEN>
__device__ __forceinline__ void max_pass(const unsigned char* tile, const uint32_t* bitmap, Pen pp, int e_lo, int nsl,
                                         int tid, RowAcc& acc) {
  for (int j0 = tid; j0 < nsl; j0 += kRounds * kThreads) {
    Batch<E> b;
    load_batch<E>(tile, j0, nsl, b);
#pragma unroll
    for (int r = 0; r < kRounds; ++r) {
      const int j = j0 + r * kThreads;
      if (j < nsl) {
        float x[E::kEPT];
        penalized<E, PEN>(bitmap, pp, b.raw[r], e_lo + j * E::kEPT, x);
        track_max<E>(acc, x, e_lo + j * E::kEPT);
      }
    }
  }
}

// GENERAL masses: e = exp(s - m0) summed per slot in fp32, then per thread in
// fp64, and for top-p rows added to the locator histogram; with TRACK the
// maximum bookkeeping rides along.
template <class E, bool PEN, bool TONE, bool HIST, bool TRACK>
__device__ __forceinline__ void mass_pass(const unsigned char* tile, const uint32_t* bitmap, uint32_t* hist, Pen pp,
                                          float T, double invT, float m0, int e_lo, int nsl, int tid, RowAcc& acc) {
  const uint32_t hs = smem_addr(hist);
  for (int j0 = tid; j0 < nsl; j0 += kRounds * kThreads) {
    Batch<E> b;
    load_batch<E>(tile, j0, nsl, b);
#pragma unroll
    for (int r = 0; r < kRounds; ++r) {
      const int j = j0 + r * kThreads;
      if (j < nsl) {
        float x[E::kEPT];
        penalized<E, PEN>(bitmap, pp, b.raw[r], e_lo + j * E::kEPT, x);
        if (TRACK) track_max<E>(acc, x, e_lo + j * E::kEPT);
        float part = 0.0f;
#pragma unroll
        for (int q = 0; q < E::kEPT; ++q) {
          const float sv = TONE ? x[q] : div_by_row_const(x[q], T, invT);
          const float e = exp_shifted(sv, m0);
          part = __fadd_rn(part, e);
          if (HIST) {
            // no range test: e >= 2^32 and e < 2^-32 both clamp into the last bucket
            const uint32_t bits = __float_as_uint(e);
            red_add_shared(hs + 4u * min((kTopFine - bits) >> kShFine, (uint32_t)(kBins - 1)), approx_mass13(bits));
          }
        }
        acc.lz += (double)part;
      }
    }
  }
}

// TOPK candidates: every element >= tau, as rank keys, appended to the
// row's list (sh.cand; one shared atomic per candidate: candidates are few,
// and warp-wide appends cost more in collectives than they save; entries past
// kCandCap are counted but dropped); with TRACK the maximum bookkeeping rides
// along.  A bit mask marks a batch's candidates, which a short loop re-reads
// from the ring.
template <class E, bool PEN, bool TRACK>
__device__ __forceinline__ void cand_pass(const unsigned char* tile, const Sh& sh, Ring& rg, Pen pp, float tau,
                                          bool t_one, float T, double invT, int e_lo, int nsl, int tid, RowAcc& acc) {
  constexpr int EPT = E::kEPT;
  static_assert(kRounds * EPT <= 32, "one candidate bit per element of a batch");
  const uint32_t ts = smem_addr(tile);
  for (int j0 = tid; j0 < nsl; j0 += kRounds * kThreads) {
    Batch<E> b;
    load_batch<E>(tile, j0, nsl, b);
    uint32_t memb = 0u;
#pragma unroll
    for (int r = 0; r < kRounds; ++r) {
      const int j = j0 + r * kThreads;
      const bool live = j < nsl;
      float x[EPT];
      penalized<E, PEN>(sh.bitmap, pp, b.raw[r], e_lo + j * EPT, x, live);
      if (TRACK && live) track_max<E>(acc, x, e_lo + j * EPT);
#pragma unroll
      for (int q = 0; q < EPT; ++q) memb |= (live && x[q] >= tau) ? (1u << (r * EPT + q)) : 0u;
    }
    while (memb) {
      const int bit = __ffs(memb) - 1;
      memb &= memb - 1u;
      const int r = bit / EPT, q = bit % EPT;
      const int j = j0 + r * kThreads;
      float x[EPT];
      penalized<E, PEN>(sh.bitmap, pp, E::lds_s(ts + (uint32_t)j * 16u), e_lo + j * EPT, x);
      const float xq = pick(x, q);
      const float sv = t_one ? xq : div_by_row_const(xq, T, invT);
      const uint32_t slot = atomicAdd(&rg.nlist, 1u);
      if (slot < (uint32_t)kCandCap) sh.cand[slot] = rank_key(sv, e_lo + j * EPT + q);
    }
  }
}

// The k-th largest per-thread maximum among the top 8 of every warp (128
// values), extended to every logit whose scaled value ties with it: at least
// k elements of the row are at or above it, so it bounds the row's k-th
// largest penalized logit from below.  -inf when fewer than k maxima are
// finite.  Consumer threads; the result is in rg.bound.
__device__ __noinline__ void topk_bound8(Ring* rgp, float tmax, int k, bool t_one, float T, float rT, int tid) {
  Ring& rg = *rgp;
  const int lane = tid & 31, warp = tid >> 5;
  uint32_t key = (tmax == tmax && tmax > -INFINITY) ? f2key(tmax) : 0u;
  // bitonic sort of the warp's 32 keys, descending
#pragma unroll
  for (int kk = 2; kk <= 32; kk <<= 1) {
#pragma unroll
    for (int j = kk >> 1; j > 0; j >>= 1) {
      const uint32_t o = __shfl_xor_sync(0xffffffffu, key, j);
      const bool desc = ((lane & kk) == 0);
      const bool lower = ((lane & j) == 0);
      key = (lower == desc) ? max(key, o) : min(key, o);
    }
  }
  if (lane < 8) rg.top8[warp * 8 + lane] = key;
  csync();
  if (warp == 0) {
    unsigned long long v[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) v[r] = ~(unsigned long long)rg.top8[32 * r + lane];  // ascending ~key = descending key
    seg_sort(v, 0, lane);
    // element k-1 of the 128 sorted values sits in register (k-1)/32 of lane (k-1)%32
    const int r = (k - 1) >> 5, l = (k - 1) & 31;
    const unsigned long long sel = (r == 0) ? v[0] : (r == 1) ? v[1] : (r == 2) ? v[2] : v[3];
    const uint32_t bk = ~(uint32_t)__shfl_sync(0xffffffffu, (uint32_t)sel, l);
    if (lane == 0) rg.bound = bk == 0u ? -INFINITY : lower_preimage(key2f(bk), t_one, T, rT);
  }
  csync();
}

// Row statistics after the last chunk: NaN-propagating maximum key, its first
// index, whether any thread saw a NaN or +inf, and the ordered sum of z.
// Consumer threads; every thread returns them.
__device__ __forceinline__ Stats row_stats(Ring& rg, const RowAcc& acc, int tid, bool& special) {
  const int lane = tid & 31, warp = tid >> 5;
  const bool nan = (acc.st != acc.st);
  const uint32_t k = nan ? 0xffffffffu : f2key(acc.st);
  const uint32_t wk = __reduce_max_sync(0xffffffffu, k);
  const uint32_t wi = __reduce_min_sync(0xffffffffu, k == wk ? (uint32_t)acc.bidx : 0x7fffffffu);
  const uint32_t ws = __reduce_or_sync(0xffffffffu, (nan || acc.st == INFINITY) ? 1u : 0u);
  const double wz = warp_dsum(acc.lz);
  if (lane == 0) {
    rg.wkey[warp] = wk;
    rg.warg[warp] = (int)wi;
    rg.wspec[warp] = ws;
    rg.wz[warp] = wz;
  }
  csync();
  uint32_t ck = 0u, cs = 0u;
  int ci = INT_MAX;
  double cz = 0.0;
  for (int w = 0; w < kWarps; ++w) {
    const uint32_t kk = rg.wkey[w];
    if (kk > ck) {
      ck = kk;
      ci = rg.warg[w];
    } else if (kk == ck) {
      ci = min(ci, rg.warg[w]);
    }
    cs |= rg.wspec[w];
    cz += rg.wz[w];
  }
  csync();  // rg.w* are reused
  Stats S;
  S.nan = (ck == 0xffffffffu);
  S.mx = S.nan ? __int_as_float(0x7fc00000) : key2f(ck);
  S.arg = ci;
  S.z = cz;
  S.over = false;
  S.lumped = false;
  special = cs != 0u;
  return S;
}

// ---------------------------------------------------------------- one row's chunks
// The ring position of the row's first chunk is n; its full barrier has been
// waited on.  These loops take every chunk of the row in turn (waiting for
// each, releasing each slot warp by warp), keep the row's descriptor in
// rg.cur before the last slot is released, and return with n past the row.
// One loop per row path, specialised on what its elements need, so that
// nothing but the path's own state is live while chunks stream.
struct ChunkPos {
  int s;             // ring slot
  const unsigned char* tile;
  int e_lo, nsl;
};

__device__ __forceinline__ ChunkPos chunk_at(Ring& rg, unsigned char* ring, const Geo& g, int n, bool wait,
                                             uint32_t* status) {
  ChunkPos c;
  c.s = n % g.nslot;
  if (wait) mbar_wait_bounded(&rg.full[c.s], (uint32_t)(n / g.nslot) & 1u, status);
  c.tile = ring + (size_t)c.s * g.slot_bytes;
  c.e_lo = rg.desc[c.s].e_lo;
  c.nsl = rg.desc[c.s].nsl;
  return c;
}

// Releases a slot; with `last`, keeps its descriptor in rg.cur first (warp 0
// copies it before its own arrival, which the producer waits for).
__device__ __forceinline__ void chunk_done(Ring& rg, int s, bool last, int tid) {
  if (last && tid == 0) rg.cur = rg.desc[s];
  __syncwarp();
  if ((tid & 31) == 0) mbar_arrive(&rg.empty[s]);
}

template <class E, bool PEN>
__device__ __noinline__ int stream_max(Ring* rgp, unsigned char* ring, Pen pp, int n, RowAcc* out, uint32_t* status,
                                       int tid) {
  Ring& rg = *rgp;
  const Geo g = rg.geo;
  uint32_t* const bitmap = rg.sh.bitmap;
  RowAcc acc{-INFINITY, -INFINITY, INT_MAX, 0.0};
  for (int c = 0; c < g.nchunk; ++c, ++n) {
    const ChunkPos p = chunk_at(rg, ring, g, n, c > 0, status);
    max_pass<E, PEN>(p.tile, bitmap, pp, p.e_lo, p.nsl, tid, acc);
    chunk_done(rg, p.s, c == g.nchunk - 1, tid);
  }
  *out = acc;
  return n;
}

template <class E, bool PEN>
__device__ __noinline__ int stream_topk(Ring* rgp, unsigned char* ring, Pen pp, int k, bool t_one, float T, float rT,
                                        int n, RowAcc* out, uint32_t* status, int tid) {
  Ring& rg = *rgp;
  const Geo g = rg.geo;
  const Sh sh = rg.sh;
  const double invT = t_one ? 1.0 : __drcp_rn((double)T);  // (the quotients stay IEEE; no call in the loops)
  RowAcc acc{-INFINITY, -INFINITY, INT_MAX, 0.0};
  for (int c = 0; c < g.nchunk; ++c, ++n) {
    const ChunkPos p = chunk_at(rg, ring, g, n, c > 0, status);
    if (c == 0 || (c == kRefreshChunk && k > kRefreshMinK)) {
      // the maxima first, then the (new) bound, then the candidates
      max_pass<E, PEN>(p.tile, sh.bitmap, pp, p.e_lo, p.nsl, tid, acc);
      topk_bound8(&rg, acc.st, k, t_one, T, rT, tid);
      cand_pass<E, PEN, false>(p.tile, sh, rg, pp, rg.bound, t_one, T, invT, p.e_lo, p.nsl, tid, acc);
    } else {
      cand_pass<E, PEN, true>(p.tile, sh, rg, pp, rg.bound, t_one, T, invT, p.e_lo, p.nsl, tid, acc);
    }
    chunk_done(rg, p.s, c == g.nchunk - 1, tid);
  }
  *out = acc;
  return n;
}

template <class E, bool PEN, bool TONE, bool HIST>
__device__ __noinline__ int stream_mass(Ring* rgp, unsigned char* ring, Pen pp, float T, float rT, int n, RowAcc* out,
                                        uint32_t* status, int tid) {
  Ring& rg = *rgp;
  const Geo g = rg.geo;
  const Sh sh = rg.sh;
  const int lane = tid & 31;
  const double invT = TONE ? 1.0 : __drcp_rn((double)T);  // (the quotients stay IEEE; no call in the loops)
  RowAcc acc{-INFINITY, -INFINITY, INT_MAX, 0.0};
  // chunk 0: its maximum gives m0, then its masses
  {
    const ChunkPos p = chunk_at(rg, ring, g, n, false, status);
    max_pass<E, PEN>(p.tile, sh.bitmap, pp, p.e_lo, p.nsl, tid, acc);
    const uint32_t wk = __reduce_max_sync(0xffffffffu, acc.st != acc.st ? 0xffffffffu : f2key(acc.st));
    if (lane == 0) rg.wkey[tid >> 5] = wk;
    csync();
    uint32_t ck = 0u;
    for (int w = 0; w < kWarps; ++w) ck = max(ck, rg.wkey[w]);
    const float mx = ck == 0xffffffffu ? __int_as_float(0x7fc00000) : key2f(ck);
    const float m0 = (mx > -INFINITY && mx < INFINITY) ? (TONE ? mx : div_by_const(mx, T, rT)) : 0.0f;
    if (tid == 0) rg.m0 = m0;
    csync();  // rg.wkey is reused
    mass_pass<E, PEN, TONE, HIST, false>(p.tile, sh.bitmap, sh.hist, pp, T, invT, m0, p.e_lo, p.nsl, tid, acc);
    chunk_done(rg, p.s, g.nchunk == 1, tid);
    ++n;
  }
  const float m0 = rg.m0;
  for (int c = 1; c < g.nchunk; ++c, ++n) {
    const ChunkPos p = chunk_at(rg, ring, g, n, true, status);
    mass_pass<E, PEN, TONE, HIST, true>(p.tile, sh.bitmap, sh.hist, pp, T, invT, m0, p.e_lo, p.nsl, tid, acc);
    chunk_done(rg, p.s, c == g.nchunk - 1, tid);
  }
  *out = acc;
  return n;
}

template <class E, bool PEN>
__device__ __forceinline__ int stream_mass_sel(bool t_one, bool hist, Ring* rgp, unsigned char* ring, Pen pp, float T,
                                               float rT, int n, RowAcc* out, uint32_t* status, int tid) {
  if (t_one) {
    return hist ? stream_mass<E, PEN, true, true>(rgp, ring, pp, T, rT, n, out, status, tid)
                : stream_mass<E, PEN, true, false>(rgp, ring, pp, T, rT, n, out, status, tid);
  }
  return hist ? stream_mass<E, PEN, false, true>(rgp, ring, pp, T, rT, n, out, status, tid)
              : stream_mass<E, PEN, false, false>(rgp, ring, pp, T, rT, n, out, status, tid);
}

// ---------------------------------------------------------------- the second pass
// A top-p row's second pass through the ring.  Its pieces are kPieceSlots
// consecutive 16-byte slots of a chunk: warp w reads piece w of every chunk,
// slots kPieceSlots * w + 32 r + lane for its kRounds rounds.  With
// `collect`: the exact mass above the window [wlo, whi] in a fixed summation
// order (returned), the kept mass of every piece (pm2[chunk * ppc + piece],
// fp32, in vocabulary order) and, with `take_members`, the window's members
// appended to sh.cand (ctl.cand_n); otherwise the chunks are only released.
// The work on a piece is straight-line: a bit mask flags the rare window
// members, which a short loop then re-reads from the ring and appends, and
// one warp reduction per chunk gives the piece's mass.  The row's constants
// come by value and stay in registers.  Consumer threads.
template <class E, bool PEN, bool TONE>
__device__ __noinline__ double ring_pass2(Ring* rgp, Pen pp, float T, float rT, float m0, uint32_t wlo, uint32_t whi,
                                          bool take_members, float* pm2, int ppc, bool collect, int tid) {
  constexpr int EPT = E::kEPT;
  static_assert(kRounds * EPT <= 32, "one member bit per element of a piece");
  Ring& rg = *rgp;
  const Geo g = rg.geo;
  const Sh sh = rg.sh;
  Ctl& ctl = *sh.ctl;
  uint32_t* const status = rg.args.status;
  unsigned char* ring = reinterpret_cast<unsigned char*>(rgp) + g.o_ring;
  const int lane = tid & 31, warp = tid >> 5;
  const uint32_t span = whi - wlo;
  const double invT = TONE ? 1.0 : __drcp_rn((double)T);  // (T / rT: the IEEE quotient, no call in the loop)
  (void)rT;
  int n = rg.n;
  double la = 0.0;
  if (collect) {
    for (int i = tid; i < g.nchunk * ppc; i += kThreads) pm2[i] = 0.0f;
    if (tid == 0) ctl.cand_n = 0u;
    csync();
  }
  const int jw = kPieceSlots * warp + lane;  // this thread's first slot of its piece
  for (int c = 0; c < g.nchunk; ++c, ++n) {
    const ChunkPos p = chunk_at(rg, ring, g, n, true, status);
    if (collect && kPieceSlots * warp < p.nsl) {  // (warp-uniform)
      const uint32_t tile = smem_addr(p.tile);
      typename E::Raw raw[kRounds];
#pragma unroll
      for (int r = 0; r < kRounds; ++r) {
        const int j = jw + 32 * r;
        if (j < p.nsl) {
          raw[r] = E::lds_s(tile + (uint32_t)j * 16u);
        } else {
          // past the chunk: -inf logits (no mass, never a member)
          const uint4 ninf = make_uint4(E::kNegInf2, E::kNegInf2, E::kNegInf2, E::kNegInf2);
          raw[r] = *reinterpret_cast<const typename E::Raw*>(&ninf);
        }
      }
      float piece = 0.0f;
      uint32_t memb = 0u;
#pragma unroll
      for (int r = 0; r < kRounds; ++r) {
        const int j = jw + 32 * r;
        const bool live = j < p.nsl;
        float x[EPT];
        penalized<E, PEN>(sh.bitmap, pp, raw[r], p.e_lo + j * EPT, x, live);
        float part = 0.0f;
#pragma unroll
        for (int q = 0; q < EPT; ++q) {
          const float sv = TONE ? x[q] : div_by_row_const(x[q], T, invT);
          const float e = exp_shifted(sv, m0);
          const uint32_t bits = __float_as_uint(e);
          part = __fadd_rn(part, bits > whi ? e : 0.0f);  // (+0 leaves the sum as it is)
          // a window that reaches e = 0 would take -inf logits too, never a slot past the chunk
          memb |= (take_members && live && bits - wlo <= span) ? (1u << (r * EPT + q)) : 0u;
        }
        la += (double)part;
        piece = __fadd_rn(piece, part);
      }
      while (memb) {
        // a window member: re-read its slot, append its rank key
        const int bit = __ffs(memb) - 1;
        memb &= memb - 1u;
        const int r = bit / EPT, q = bit % EPT;
        const int j = jw + 32 * r;
        float x[EPT];
        penalized<E, PEN>(sh.bitmap, pp, E::lds_s(tile + (uint32_t)j * 16u), p.e_lo + j * EPT, x);
        const float xq = pick(x, q);
        const float sv = TONE ? xq : div_by_row_const(xq, T, invT);
        const uint32_t slot = atomicAdd(&ctl.cand_n, 1u);
        if (slot < (uint32_t)kCandCap) sh.cand[slot] = rank_key(sv, p.e_lo + j * EPT + q);
      }
      // the piece's mass, summed in a fixed order
#pragma unroll
      for (int o = 16; o; o >>= 1) piece += __shfl_xor_sync(0xffffffffu, piece, o);
      if (lane == 0) pm2[c * ppc + warp] = piece;
    }
    chunk_done(rg, p.s, false, tid);
  }
  rg.n = n;  // (every thread writes the same value)
  if (!collect) return 0.0;
  return block_dsum(ctl, la, tid);
}

template <class E>
__device__ __forceinline__ double ring_pass2_sel(Ring& rg, const RowCtx& R, float m0, uint32_t wlo, uint32_t whi,
                                                 bool take_members, float* pm2, int ppc, bool collect, int tid) {
  if (R.pen) {
    return R.t_one ? ring_pass2<E, true, true>(&rg, R.pp, R.T, R.rT, m0, wlo, whi, take_members, pm2, ppc, collect, tid)
                   : ring_pass2<E, true, false>(&rg, R.pp, R.T, R.rT, m0, wlo, whi, take_members, pm2, ppc, collect, tid);
  }
  return R.t_one ? ring_pass2<E, false, true>(&rg, R.pp, R.T, R.rT, m0, wlo, whi, take_members, pm2, ppc, collect, tid)
                 : ring_pass2<E, false, false>(&rg, R.pp, R.T, R.rT, m0, wlo, whi, take_members, pm2, ppc, collect, tid);
}

// The chunk of element idx, and its piece in pm2.
__device__ __forceinline__ int piece_of(const Geo& g, int ppc, int ept, int idx) {
  int c = (int)(((idx >> 5) * (int64_t)g.nchunk) / g.units);
  while (c + 1 < g.nchunk && chunk_lo(g, c + 1) <= idx) ++c;
  while (c > 0 && chunk_lo(g, c) > idx) --c;
  return c * ppc + ((idx - chunk_lo(g, c)) / ept) / kPieceSlots;
}

// Adds the kept window members (rank key <= last) to their pieces' masses.
template <class E>
__device__ void members_to_pieces(const Geo& g, const Sh& sh, int nmem, unsigned long long last, float m0, float* pm2,
                                  int ppc, int tid) {
  for (int r = tid; r < nmem; r += kThreads) {
    const unsigned long long key = sh.cand[r];
    if (key > last) continue;
    const float e = exp_shifted(key_value(key), m0);
    if (e > 0.0f) atomicAdd(&pm2[piece_of(g, ppc, E::kEPT, key_index(key))], e);
  }
  csync();
}

// Inverse-CDF draw in vocabulary order over the piece masses of the second
// pass: a block scan finds the piece whose mass prefix passes `target`, then
// warp 0 reads that piece (one round trip for its kRounds rounds) and walks it.  Falls back to the
// last kept element when rounding leaves the target past the total, then to
// `fallback`.  Consumer threads; every thread returns the token.
template <class E>
__device__ int draw_ring(Ring& rg, const Sh& sh, const RowCtx& R, const Keep& K, const float* pm2, int ppc,
                         double target, int fallback, int tid) {
  constexpr int EPT = E::kEPT;
  constexpr int esz = sizeof(typename E::Raw) / EPT;
  const Geo& g = rg.geo;
  Ctl& ctl = *sh.ctl;
  const int lane = tid & 31, warp = tid >> 5;
  const int np = g.nchunk * ppc;
  const int per = (np + kThreads - 1) / kThreads;
  const int q0 = tid * per;
  double tot = 0.0;
  int lastp = -1;
  for (int i = 0; i < per; ++i) {
    const int q = q0 + i;
    const float m = q < np ? pm2[q] : 0.0f;
    tot += (double)m;
    if (m > 0.0f) lastp = q;
  }
  const double inc = warp_incl_f64(tot, lane);
  if (lane == 31) ctl.red_e[warp] = inc;
  if (tid == 0) {
    ctl.misc = INT_MAX;
    ctl.misc2 = -1;
  }
  csync();
  double run = inc - tot;
  for (int w = 0; w < warp; ++w) run += ctl.red_e[w];
  if (lastp >= 0) atomicMax(&ctl.misc2, lastp);
  int hit = -1;
  double before = 0.0;
  for (int i = 0; i < per && hit < 0; ++i) {
    const int q = q0 + i;
    const float m = q < np ? pm2[q] : 0.0f;
    if (m > 0.0f && target < run + (double)m) {
      hit = q;
      before = run;
    }
    run += (double)m;
  }
  if (hit >= 0) atomicMin(&ctl.misc, hit);
  csync();
  if (hit >= 0 && hit == ctl.misc) ctl.pick_t = target - before;
  csync();
  int pc = ctl.misc;
  double t2 = ctl.pick_t;
  if (pc == INT_MAX) {
    pc = ctl.misc2;  // rounding: the last piece with mass, its last kept element
    t2 = 1e300;
  }
  if (pc < 0) return fallback;
  if (warp == 0) {
    // the piece's rounds in vocabulary order: slots kPieceSlots * w + 32 r + lane
    const int c = pc / ppc, w = pc % ppc;
    const int e_lo = chunk_lo(g, c), e_hi = min(R.V, chunk_lo(g, c + 1));
    typename E::Raw raw[kRounds];
#pragma unroll
    for (int r = 0; r < kRounds; ++r) {
      const int idx0 = e_lo + (kPieceSlots * w + 32 * r + lane) * EPT;
      raw[r] = idx0 < e_hi ? E::ldg(R.src + (size_t)idx0 * esz) : E::zero();
    }
    int tok = -1, lastk = -1;
    double run2 = 0.0;  // kept mass of the piece's earlier rounds
#pragma unroll
    for (int r = 0; r < kRounds; ++r) {
      if (tok >= 0) break;  // (warp-uniform)
      const int idx0 = e_lo + (kPieceSlots * w + 32 * r + lane) * EPT;
      float q[EPT];
      kept_masses<E>(R, sh.bitmap, K, raw[r], idx0, idx0 < e_hi, q);
      float ls = 0.f;
      int lk = -1;
#pragma unroll
      for (int j = 0; j < EPT; ++j) {
        ls = __fadd_rn(ls, q[j]);
        if (q[j] > 0.f) lk = idx0 + j;
      }
      lastk = max(lastk, (int)__reduce_max_sync(0xffffffffu, (uint32_t)(lk + 1)) - 1);
      const double inc2 = warp_incl_f64((double)ls, lane) + run2;
      const uint32_t bal = __ballot_sync(0xffffffffu, inc2 > t2 && ls > 0.f);
      if (bal) {
        const int l = __ffs(bal) - 1;
        int mine = -1;
        if (lane == l) {
          double cum = inc2 - (double)ls;
          int pk = -1, lastc = -1;
#pragma unroll
          for (int j = 0; j < EPT; ++j) {
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
      }
      run2 = __shfl_sync(0xffffffffu, inc2, 31);
    }
    if (tok < 0) tok = lastk >= 0 ? lastk : fallback;
    if (lane == 0) ctl.token = tok;
  }
  csync();
  return ctl.token;
}

// ---------------------------------------------------------------- finisher
// Finishes row rg.cur.row once its last chunk has streamed: the decision and
// the draw from what accumulated (rg.S, sh.hist, sh.cand, rg), re-reading the
// row where the path needs it.  Its inputs are read from shared memory (rg),
// so the call copies nothing into a per-thread frame.  Consumer threads.
template <class E>
__device__ __noinline__ void finish_row(Ring* rgp, int tid) {
  constexpr int EPT = E::kEPT;
  constexpr int esz = sizeof(typename E::Raw) / EPT;
  const int lane = tid & 31, warp = tid >> 5;
  Ring& rg = *rgp;
  const NsSampleArgs& a = rg.args;
  const Geo& g = rg.geo;
  const ChunkDesc& d = rg.cur;
  const Stats S = rg.S;
  const Sh sh = rg.sh;
  Ctl& ctl = *sh.ctl;
  uint32_t* const status = a.status;
  const int V = a.vocab_size;
  const bool debug = (a.out_filtered != nullptr) || (a.out_probs != nullptr);
  const bool out_i32 = (a.out_dtype == NS_OUT_I32);
  const NsRowParams P = d.P;
  const int row = d.row;
  RowCtx R;
  R.src = static_cast<const char*>(a.logits) + (size_t)d.src * (size_t)a.logits_row_stride * esz;
  R.V = V;
  R.W = g.W;
  R.nch = g.nch;
  R.row = row;
  R.greedy = (P.flags & NS_ROW_GREEDY) != 0u;
  R.T = R.greedy ? 1.0f : P.temperature;
  R.rT = __frcp_rn(R.T);
  R.invT = __drcp_rn((double)R.T);
  R.t_one = (R.T == 1.0f);
  R.topp = (P.flags & NS_ROW_TOP_P) != 0u;
  R.p = P.top_p;
  R.k = (P.top_k > 0 && P.top_k < V) ? P.top_k : 0;
  R.rp = P.repetition_penalty;
  R.pp = Pen::of(R.rp);
  R.pen = (P.flags & NS_ROW_PENALTY) != 0u && a.history_offsets && d.h1 > d.h0;
  int mode = row_mode(P, V, debug);
  const bool hist_used = (mode == kGeneral) && R.k == 0 && R.topp;  // the chunks built sh.hist
  const bool ring2 = hist_used;  // its second pass waits in the ring (two_pass_row)
  bool ring_used = false;
  bool pm2_ok = false;  // pm2 holds the kept masses per second-pass piece
  float* const pm2 = reinterpret_cast<float*>(sh.hist) + kPm2Offset;
  const int64_t out_off = (int64_t)row * V;
  const double u = row_uniform(a, P, row);
  const float row_bound = rg.bound;
  const uint32_t cand_total = rg.nlist;
  float m0 = rg.m0;

  if (a.out_penalized) {
    // debug output: the logits after the repetition penalty (sampler.py:31-38)
    float* const pen_out = a.out_penalized + out_off;
    global_pass<E>(R, sh.bitmap, tid, [&](int, const float(&x)[EPT], int idx0, bool live) {
      if (!live) return;
#pragma unroll
      for (int j = 0; j < EPT; ++j) pen_out[idx0 + j] = x[j];
    });
  }

  int tok = 0;
  bool done = false;
  // ================================================================ rows whose softmax is NaN
  // NaN or +inf logits, or all -inf: uniform probabilities 1/V (sampler.py:76-80)
  if (S.nan || S.mx == INFINITY || S.mx == -INFINITY) {
    if (R.greedy) {
      // torch.argmax: the first NaN, else the first +inf, else index 0 (the
      // penalty keeps NaN and +inf, so the raw logits decide)
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
      csync();
      int fn = INT_MAX, fp = INT_MAX;
      for (int w = 0; w < kWarps; ++w) {
        fn = min(fn, ctl.red_i[w]);
        fp = min(fp, ctl.red_j[w]);
      }
      csync();
      tok = (fn != INT_MAX) ? fn : (fp != INT_MAX) ? fp : 0;
    } else {
      tok = min(V - 1, (int)(u * (double)V));
    }
    if (ring2) {
      ring_used = true;
      ring_pass2_sel<E>(rg, R, m0, 1u, 0u, false, pm2, g.ppc, false, tid);
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
    done = true;
  }

  // ================================================================ GREEDY
  if (!done && mode == kGreedy) {
    if (tid == 0) write_token(a.out_tokens, out_i32, row, S.arg);
    done = true;
  }

  // ================================================================ TOPK
  if (!done && mode == kTopk) {
    // the streamed candidates at or above the row's final bound
    unsigned long long* list = reinterpret_cast<unsigned long long*>(sh.hist);
    if (tid == 0) ctl.list_n = 0u;
    csync();
    const bool fits = cand_total <= (uint32_t)kCandCap;
    if (fits) {
      const float sig = scaled(R, row_bound);
      const int ncand = (int)cand_total;
      const int nround = (ncand + kThreads - 1) / kThreads * kThreads;
      for (int r = tid; r < nround; r += kThreads) {
        const bool valid = r < ncand;
        const unsigned long long key = valid ? sh.cand[r] : 0ull;
        list_append(list, &ctl.list_n, valid && key_value(key) >= sig, key, kCandCap, lane);
      }
    }
    csync();
    const int nl = (int)ctl.list_n;
    if (fits && nl > 0 && nl <= kCandCap) {
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
        float* ce = reinterpret_cast<float*>(sh.cand);  // masses by rank
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
        int t = INT_MAX, last = -1;
        for (int r = lane; r < m2; r += 32) {
          const int ir = key_index(list[r]);
          const double er = (double)ce[r];
          if (er > 0.0) last = max(last, ir);
          double before = 0.0;
          for (int q2 = 0; q2 < m2; ++q2)
            if (key_index(list[q2]) < ir) before += (double)ce[q2];
          if (er > 0.0 && before <= target && target < before + er) t = min(t, ir);
        }
        t = (int)__reduce_min_sync(0xffffffffu, (uint32_t)t);
        last = (int)__reduce_max_sync(0xffffffffu, (uint32_t)(last + 1)) - 1;
        if (t == INT_MAX) t = last >= 0 ? last : key_index(list[0]);  // rounding at the very top
        if (R.greedy) t = S.arg;
        if (lane == 0) {
          write_token(a.out_tokens, out_i32, row, t);
          ctl.dec_thr = key_value(list[m2 - 1]);
          ctl.dec_thr_idx = key_index(list[m2 - 1]);
          ctl.dec_z = z;
          ctl.misc2 = __float_as_int(s0);
        }
      }
      if (debug) {
        csync();
        const float s0 = __int_as_float(ctl.misc2);
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
      done = true;
    } else {
      // the candidate list overflowed: the row takes the (exact) general path
      mode = kGeneral;
    }
  }

  // ================================================================ GENERAL
  if (!done) {
    const float m = scaled(R, S.mx);
    Keep K;
    K.have_k = false;
    K.thr_k = -INFINITY;
    K.window = false;
    K.win_lo = K.win_hi = 0u;
    K.thr = -INFINITY;
    K.thr_idx = INT_MAX;
    double z = S.z;
    bool over = false;
    uint32_t lumped = 0u;
    if (hist_used) {
      // the streamed locator histogram is in sh.hist
      over = __float_as_uint(exp_shifted(m, m0)) > kTopFine;
      lumped = (sh.hist[kBins - 1] != 0u) ? 1u : 0u;
    }
    K.m0 = m0;
    // the parts' masses hold for top-p rows unless top-k comes first or e passed 2^32
    const bool first_ok = hist_used && !over;
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
      csync();
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
      csync();
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
          csync();
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
        // ---- collection: exact mass above the window per warp range and per
        // draw piece; the window's members.  The first collection of a top-p
        // row reads its second pass from the ring.
        const bool use_ring = ring2 && !ring_used;
        const uint32_t wlo = max(win_lo, 1u), whi = win_hi;
        double above = 0.0;
        if (use_ring) {
          ring_used = true;
          above = ring_pass2_sel<E>(rg, R, K.m0, wlo, whi, true, pm2, g.ppc, true, tid);
        } else {
        if (tid == 0) ctl.cand_n = 0u;
        csync();
        double la = 0.0;
        const Keep K1 = K;
        // per-thread mass above the window in the current draw piece (kStages
        // chunks; chunks are visited in order from 0, the same in every lane)
        float pacc = 0.0f;
        int pleft = kStages, pidx = 0;
        auto piece_end = [&](int c, float part) {
          pacc = __fadd_rn(pacc, part);
          if (--pleft == 0 || c == R.nch - 1) {
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
              for (int j = 0; j < EPT; ++j) s[j] = div_by_row_const(x[j], R.T, R.invT);
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
                  const uint32_t slotn = atomicAdd(&ctl.cand_n, 1u);
                  if (slotn < (uint32_t)kCandCap) sh.cand[slotn] = rank_key(s[j], idx0 + j);
                }
              }
            }
          }
          la += (double)part;
          piece_end(c, part);
        };
        global_pass<E>(R, sh.bitmap, tid, collect);
        above = block_segments(ctl, la, tid);
        }
        const uint32_t ntot = ctl.cand_n;
        if (use_ring && ntot > (uint32_t)kCandCap) {
          // more members than the list holds: refine, or collect again from
          // global memory (which also fills the per-range masses the tie
          // resolution needs)
          if (lv.sh > 0 && refines < 5) force_refine = true;
          continue;
        }
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
          if (member_decide<E>(sh, n, max(win_lo, 1u), win_hi, m0, above, topp_threshold(z, R.p), R.W, kept_m, tid)) {
            zk = above + kept_m;
            if (use_ring) {
              members_to_pieces<E>(g, sh, n, ctl.dec_key, m0, pm2, g.ppc, tid);
              pm2_ok = true;
            } else {
              pm_ok = true;
            }
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
          csync();
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
          csync();
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
            atomicAdd(&ctl.seg[idx / R.W], (double)er[q]);
            atomicAdd(&ctl.pm[idx / R.W][(idx % R.W) / E::kPiece / kStages], (double)er[q]);
            lk += (double)er[q];
          }
        }
        zk = above + block_dsum(ctl, lk, tid);  // (its barriers order the range updates)
        if (use_ring) {
          members_to_pieces<E>(g, sh, n, n > 0 ? sh.cand[j0] : 0ull, m0, pm2, g.ppc, tid);
          pm2_ok = true;
        } else {
          pm_ok = ntot <= (uint32_t)kCandCap;
        }
        K.window = true;
        K.win_lo = win_lo;
        K.win_hi = win_hi;
        K.thr = ctl.dec_thr;
        K.thr_idx = ctl.dec_thr_idx;
        break;
      }
      if (!crossed && ring2 && !ring_used) {
        // top-p never crosses: every element stays; the second pass gives
        // every piece's mass
        ring_used = true;
        zk = ring_pass2_sel<E>(rg, R, K.m0, 1u, 0u, false, pm2, g.ppc, true, tid);
        pm2_ok = true;
      } else if (!crossed) {
        // top-p never crosses: every element stays; draw over all masses
        double lz = 0.0;
        const Keep K1 = K;
        global_pass<E>(R, sh.bitmap, tid, [&](int, const float(&x)[EPT], int, bool live) {
          if (!live) return;
          float part = 0.0f;
#pragma unroll
          for (int j = 0; j < EPT; ++j) part = __fadd_rn(part, K1.mass(scaled(R, x[j])));
          lz += (double)part;
        });
        zk = block_segments(ctl, lz, tid);
      }
    }

    // ---- the draw
    if (ring2 && !ring_used) {
      ring_used = true;
      ring_pass2_sel<E>(rg, R, K.m0, 1u, 0u, false, pm2, g.ppc, false, tid);  // (not needed: released)
    }
    tok = R.greedy ? S.arg
          : pm2_ok ? draw_ring<E>(rg, sh, R, K, pm2, g.ppc, u * zk, S.arg, tid)
          : pm_ok  ? draw_piece<E>(R, sh, K, u * zk, S.arg, tid)
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

}

// ---------------------------------------------------------------- the kernel
template <class E>
__global__ void __launch_bounds__(kBlockThreads, 1) rows_kernel(const NsSampleArgs a, const Geo g, void* ws) {
  extern __shared__ __align__(128) unsigned char smem[];
  Ring& rg = *reinterpret_cast<Ring*>(smem);
  Sh sh;
  sh.ctl = reinterpret_cast<Ctl*>(smem + g.o_ctl);
  sh.bitmap = reinterpret_cast<uint32_t*>(smem + g.o_bitmap);
  sh.hist = reinterpret_cast<uint32_t*>(smem + g.o_hist);
  sh.cand = reinterpret_cast<unsigned long long*>(smem + g.o_cand);
  sh.small = reinterpret_cast<unsigned long long*>(smem + g.o_small);
  unsigned char* ring = smem + g.o_ring;
  WsHeader* hdr = static_cast<WsHeader*>(ws);
  const int tid = threadIdx.x;
  const int V = a.vocab_size;
  const bool debug = (a.out_filtered != nullptr) || (a.out_probs != nullptr);

  if (tid == 0) {
    for (int s = 0; s < g.nslot; ++s) {
      mbar_init(&rg.full[s], 1);
      mbar_init(&rg.empty[s], kWarps);
    }
    fence_mbar_init();
    rg.args = a;
    rg.geo = g;
    rg.sh = sh;
  }
  __syncthreads();

  if (tid >= kThreads) {
    if (tid == kThreads) producer<E>(a, g, rg, ring, hdr);
  } else {
    const int lane = tid & 31;
    int n = 0;  // ring position of the next chunk
    for (;;) {
      // ---- a new row: its first chunk's descriptor
      const int s0 = n % g.nslot;
      mbar_wait_bounded(&rg.full[s0], (uint32_t)(n / g.nslot) & 1u, a.status);
      const ChunkDesc& ds = rg.desc[s0];
      if (ds.row < 0) break;
      const NsRowParams P = ds.P;
      const int64_t h0 = ds.h0, h1 = ds.h1;
      const uint32_t bad0 = ds.bad;
      const int mode = row_mode(P, V, debug);
      const int k = (P.top_k > 0 && P.top_k < V) ? P.top_k : 0;
      const bool greedy = (P.flags & NS_ROW_GREEDY) != 0u;
      const float T = greedy ? 1.0f : P.temperature;
      const float rT = __frcp_rn(T);
      const bool t_one = (T == 1.0f);
      const bool pen = (P.flags & NS_ROW_PENALTY) != 0u && a.history_offsets && h1 > h0;
      const Pen pp = Pen::of(P.repetition_penalty);
      const bool with_e = (mode == kGeneral) && k == 0;
      const bool want_hist = with_e && (P.flags & NS_ROW_TOP_P) != 0u;

      // ---- its penalty bitmap, histogram and counters
      if (pen)
        for (int w = tid; w < (V + 31) / 32; w += kThreads) sh.bitmap[w] = 0u;
      if (want_hist)
        for (int b = tid; b < kBins / 4; b += kThreads) reinterpret_cast<uint4*>(sh.hist)[b] = make_uint4(0, 0, 0, 0);
      if (tid == 0) {
        rg.nlist = 0u;
        rg.bound = -INFINITY;
        rg.m0 = 0.0f;
        if (bad0 && a.status) atomicOr(a.status, bad0);
      }
      csync();
      if (pen) {
        // every id loaded first (independent loads in flight), then set
        constexpr int kIdBatch = 4;
        uint32_t bad = 0u;
        for (int64_t h = h0 + tid; h < h1; h += (int64_t)kIdBatch * kThreads) {
          int id[kIdBatch];
#pragma unroll
          for (int q = 0; q < kIdBatch; ++q) {
            const int64_t hq = h + (int64_t)q * kThreads;
            id[q] = hq < h1 ? __ldg(&a.history_ids[hq]) : -2;
          }
#pragma unroll
          for (int q = 0; q < kIdBatch; ++q) {
            if (id[q] == -2) continue;
            if (id[q] < 0 || id[q] >= V) {
              bad = 1u;
              continue;
            }
            atomicOr(&sh.bitmap[id[q] >> 5], 1u << (id[q] & 31));
          }
        }
        if (__any_sync(0xffffffffu, bad) && lane == 0 && a.status) atomicOr(a.status, NS_STATUS_BAD_HISTORY_ID);
        csync();
      }

      // ---- every chunk of the row
      RowAcc acc;
      if (mode == kGreedy || (mode == kGeneral && !with_e)) {
        n = pen ? stream_max<E, true>(&rg, ring, pp, n, &acc, a.status, tid)
                : stream_max<E, false>(&rg, ring, pp, n, &acc, a.status, tid);
      } else if (mode == kTopk) {
        n = pen ? stream_topk<E, true>(&rg, ring, pp, k, t_one, T, rT, n, &acc, a.status, tid)
                : stream_topk<E, false>(&rg, ring, pp, k, t_one, T, rT, n, &acc, a.status, tid);
      } else {
        n = pen ? stream_mass_sel<E, true>(t_one, want_hist, &rg, ring, pp, T, rT, n, &acc, a.status, tid)
                : stream_mass_sel<E, false>(t_one, want_hist, &rg, ring, pp, T, rT, n, &acc, a.status, tid);
      }

      // ---- the row's statistics, then the finishing work
      bool special = false;
      const Stats S = row_stats(rg, acc, tid, special);
      if (mode == kTopk && !(S.nan || S.mx == INFINITY || S.mx == -INFINITY))
        topk_bound8(&rg, acc.st, k, t_one, T, rT, tid);  // the final, tightest bound
      (void)special;
      if (tid == 0) {
        rg.S = S;
        rg.n = n;
      }
      csync();
      finish_row<E>(&rg, tid);
      csync();  // the next row may reuse the bitmap, histogram and lists
      n = rg.n;  // past a top-p row's second pass
    }
  }
  __syncthreads();
  // the last block out returns the ticket counter to zero
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(&hdr->exited, 1u) == gridDim.x - 1u) {
      hdr->ticket = 0u;
      hdr->exited = 0u;
      __threadfence();
    }
  }
}

// ---------------------------------------------------------------- host side
struct DevState {
  size_t smem_set[2] = {0, 0};
  int sms = 0;
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

int64_t rows_workspace_bytes(int32_t num_rows) {
  (void)num_rows;
  return (int64_t)sizeof(rk::WsHeader);
}

static int rows_launch_ws(const NsSampleArgs& a, cudaStream_t stream, int device, std::string& err, void* ws,
                          int64_t ws_bytes_avail) {
  using namespace rk;
  const bool bf16 = a.logits_dtype == NS_DTYPE_BF16;
  const int ept = bf16 ? EBF16::kEPT : EF32::kEPT;
  const int esz = bf16 ? 2 : 4;
  if (ws_bytes_avail < (int64_t)sizeof(WsHeader)) {
    err = "ns_sample: workspace of " + std::to_string(ws_bytes_avail) + " bytes is smaller than the " +
          std::to_string(sizeof(WsHeader)) + " it needs (ns_workspace_bytes)";
    return NS_ERR_INVALID_ARG;
  }
  if (reinterpret_cast<uintptr_t>(ws) % 16 != 0) {
    err = "ns_sample: workspace must be 16-byte aligned";
    return NS_ERR_INVALID_ARG;
  }
  Geo g;
  // the whole-row passes' layout: warp range = V / 16 rounded up to whole 16-byte slots
  g.W = ((a.vocab_size + kWarps - 1) / kWarps + ept - 1) / ept * ept;
  g.nch = (g.W + 32 * ept - 1) / (32 * ept);
  g.units = (a.vocab_size + kUnit - 1) / kUnit;
  int nchunk = (int)(((int64_t)a.vocab_size * esz + kChunkTarget - 1) / kChunkTarget);
  nchunk = nchunk < 1 ? 1 : (nchunk > kMaxChunksRow ? kMaxChunksRow : nchunk);
  g.nchunk = nchunk;
  g.slot_bytes = ((g.units + nchunk - 1) / nchunk) * kUnit * esz;
  g.ppc = (g.slot_bytes + 16 * kPieceSlots - 1) / (16 * kPieceSlots);  // at most kWarps: slots <= 32 KB
  if (g.ppc > kWarps || g.nchunk * g.ppc > kPm2Cap) {
    err = "ns_sample: too many second-pass pieces per row";
    return NS_ERR_UNSUPPORTED;
  }
  size_t o = 0;
  auto take = [&](size_t bytes, size_t align) {
    o = (o + align - 1) & ~(align - 1);
    const size_t at = o;
    o += bytes;
    return (int)at;
  };
  take(sizeof(Ring), 128);
  g.o_ctl = take(sizeof(Ctl), 128);
  g.o_bitmap = take(sizeof(uint32_t) * (size_t)((a.vocab_size + 31) / 32), 128);
  g.o_hist = take(sizeof(uint32_t) * kBins, 128);
  g.o_cand = take(sizeof(unsigned long long) * kCandCap, 128);
  g.o_small = take(sizeof(unsigned long long) * 32, 128);
  const size_t fixed = (o + 127) & ~(size_t)127;
  constexpr size_t kSmemMax = 227 * 1024;
  int nslot = (int)((kSmemMax - fixed) / (size_t)g.slot_bytes);
  nslot = nslot > kRingMax ? kRingMax : nslot;
  if (nslot < 2) {
    err = "ns_sample: row chunks do not fit the shared-memory ring";
    return NS_ERR_UNSUPPORTED;
  }
  g.nslot = nslot;
  g.o_ring = take((size_t)nslot * g.slot_bytes, 128);
  g.smem = (int)((o + 127) & ~(size_t)127);

  const void* fn = bf16 ? reinterpret_cast<const void*>(&rows_kernel<EBF16>)
                        : reinterpret_cast<const void*>(&rows_kernel<EF32>);
  const int fi = bf16 ? 1 : 0;
  int sms = 0;
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
    if (ds.smem_set[fi] < (size_t)g.smem) {
      e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, g.smem);
      if (e != cudaSuccess) {
        err = std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e);
        return NS_ERR_CUDA;
      }
      ds.smem_set[fi] = (size_t)g.smem;
    }
    sms = ds.sms;
  }
  const int grid = a.num_rows < sms ? a.num_rows : sms;
  void* args[] = {const_cast<NsSampleArgs*>(&a), &g, &ws};
  const cudaError_t e = cudaLaunchKernel(fn, dim3((unsigned)grid), dim3(kBlockThreads), args, (size_t)g.smem, stream);
  if (e != cudaSuccess) {
    err = std::string("row kernel launch: ") + cudaGetErrorString(e);
    return NS_ERR_CUDA;
  }
  return NS_OK;
}

int rows_launch(const NsSampleArgs& a, cudaStream_t stream, int device, std::string& err) {
  if (!a.workspace) {
    err = "ns_sample: this call takes the row kernel, which needs NsSampleArgs.workspace "
          "(ns_workspace_bytes bytes, zeroed once before first use)";
    return NS_ERR_INVALID_ARG;
  }
  return rows_launch_ws(a, stream, device, err, a.workspace, a.workspace_bytes);
}

int rows_launch_noalloc(const NsSampleArgs& a, cudaStream_t stream, int device, std::string& err) {
  // The array's name is a host-side stand-in; the kernel needs its device
  // address on this (the current) device, looked up on every call (a host-side
  // query; the first one on a device may load the module, so make that first
  // call outside any stream capture).
  void* ws = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&ws, rk::g_static_ws);
  if (e != cudaSuccess || !ws) {
    err = std::string("cudaGetSymbolAddress of the static workspace: ") + cudaGetErrorString(e);
    return NS_ERR_CUDA;
  }
  return rows_launch_ws(a, stream, device, err, ws, (int64_t)sizeof(rk::g_static_ws));
}

}  // namespace ns

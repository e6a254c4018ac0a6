// ascan_tma.cuh -- persistent, TMA-fed scan kernels for sm_100a.
//
// One CTA per SM runs a loop over 4096-element tiles taken, in scan order,
// from an atomic ticket counter.  Warp 8 is the producer: it takes the ticket,
// waits for a free stage of a shared-memory ring, issues 2-D TMA loads of the
// tile's inputs (tensor maps view the flat array as rows of 128 bytes, 128B
// swizzle) and, while they fly, writes the tile's sequence-boundary bitmaps,
// the neighbour scalars at the tile edges and the ragged tail of the array
// into the stage's metadata.  Warps 0-7 consume: thread i owns elements
// [16i, 16i+16) of the tile (the swizzle makes those blocked reads
// bank-conflict free), folds them serially, scans the per-thread aggregates
// across the warp with shuffles and across warps through shared memory,
// obtains the tile's carry-in by decoupled look-back, writes the outputs into
// a double-buffered staging area and hands them to a TMA store.  HBM keeps
// streaming the next stages while a tile is computed or waits on a
// predecessor.
//
// Every wait is bounded: mbarrier waits and look-back polls give up after
// kLookbackTimeoutNs, report ASCAN_DEV_ERR_LOOKBACK and set the launch's abort
// word, after which no wait of the launch blocks again.  Consumers leave their
// loop only together (a bar.red vote), never one warp alone.
#pragma once

#include <cuda.h>

#include "ascan_device.cuh"

namespace ascan {
namespace tma {

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;  // 256
constexpr int kThreads = kConsumers + 32;        // + producer warp
constexpr int kPerThread = 16;                   // elements per consumer thread
constexpr int kTileElems = kConsumers * kPerThread;
static_assert(kTileElems == kTile, "TMA and plain kernels share the tile size");
constexpr int kBitWords = kTileElems / 32;       // 128
constexpr int kCuCache = 1024;                   // cu_seqlens entries cached in smem
constexpr uint32_t kDone = 0xffffffffu;
constexpr int kNamedBarrier = 1;   // consumer-only bar.sync
constexpr int kAgreeBarrier = 2;   // consumer-only bar.red

template <typename T>
struct Fmt {
  static constexpr int kElemsPerRow = 128 / sizeof(T);  // one 128-byte TMA row
  static constexpr int kRows = kTileElems / kElemsPerRow;
  static constexpr int kBytes = kTileElems * sizeof(T);
  static constexpr int kTailMax = kElemsPerRow;         // ragged tail < one row
};

// Byte offset of tile element e inside a 1024-aligned buffer written by TMA
// with CU_TENSOR_MAP_SWIZZLE_128B: the 16-byte chunk index inside each
// 128-byte row is XORed with the row index modulo 8.
template <typename T>
__device__ __forceinline__ uint32_t swz(uint32_t e) {
  const uint32_t byte = e * sizeof(T);
  const uint32_t row = byte >> 7;
  return byte ^ ((row & 7u) << 4);
}

// ---------------------------------------------------------------------------
// PTX wrappers: mbarrier, TMA, bulk groups, named barrier
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase of `parity` to complete; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > kLookbackTimeoutNs) return false;
  }
  return true;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int x, int y,
                                             const void* src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];"
               ::"l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(src))
               : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync %0, %1;" ::"n"(kNamedBarrier), "n"(kConsumers) : "memory");
}

// OR of `pred` over the 256 consumer threads (all of them must call it).
__device__ __forceinline__ bool consumers_any(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.or.pred p, %2, %3, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "n"(kAgreeBarrier), "n"(kConsumers)
      : "memory");
  return r != 0u;
}

__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------
// shared-memory layout
// ---------------------------------------------------------------------------

template <int NIN, typename T>
struct StageMeta {
  uint32_t ticket;     // kDone: no more tiles
  uint32_t n_valid;    // tile elements below N
  uint32_t n_tma;      // tile elements covered by the TMA rows
  uint32_t has_outside;
  int64_t p0;          // flat index of the tile's first element
  float halo[2];       // bwd: [0] gate neighbour, [1] state neighbour at the tile edge
  alignas(16) uint32_t sbits[kBitWords];  // sequence starts (and positions outside any sequence)
  alignas(16) uint32_t ebits[kBitWords];  // sequence ends   (and positions outside any sequence)
  alignas(16) uint32_t obits[kBitWords];  // positions outside any sequence (valid if has_outside)
  float tail[NIN][Fmt<T>::kTailMax];
};

template <int NIN, int NOUT, int NS, typename T>
struct Smem {
  alignas(1024) uint8_t in[NS][NIN][Fmt<T>::kBytes];
  alignas(1024) uint8_t out[2][NOUT][Fmt<T>::kBytes];
  StageMeta<NIN, T> meta[NS];
  uint64_t full[NS];
  uint64_t empty[NS];
  int64_t cu[kCuCache];
  Pfx warp_total[kConsumerWarps];
  Pfx te;
  int abort;
};

template <int NIN, int NOUT, int NS, typename T>
constexpr size_t smem_bytes() {
  return sizeof(Smem<NIN, NOUT, NS, T>) + 1024;  // + alignment slack
}

template <typename Sm>
__device__ __forceinline__ Sm& smem_view() {
  extern __shared__ uint8_t smem_raw[];
  const uintptr_t base = reinterpret_cast<uintptr_t>(smem_raw);
  return *reinterpret_cast<Sm*>((base + 1023) & ~static_cast<uintptr_t>(1023));
}

// ---------------------------------------------------------------------------
// producer helpers
// ---------------------------------------------------------------------------

template <typename IdxT>
struct CuView {
  const IdxT* g;        // global array
  const int64_t* s;     // smem cache or nullptr
  int64_t S, BL;
  __device__ __forceinline__ int64_t at(int64_t i) const {
    if (s) return s[i];
    return cu_at(g, i, BL);
  }
  // first i in [lo, hi) with at(i) >= v (hi if none); entries assumed sorted
  __device__ __forceinline__ int64_t lower_bound(int64_t lo, int64_t hi, int64_t v) const {
    while (lo < hi) {
      const int64_t m = (lo + hi) >> 1;
      if (at(m) < v)
        lo = m + 1;
      else
        hi = m;
    }
    return lo;
  }
};

// Bits [lo, hi) (lo, hi relative to a 128-bit span) into words w[0..3].
__device__ __forceinline__ void set_range(uint32_t (&w)[4], uint32_t lo, uint32_t hi) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t a = lo > 32u * k ? lo - 32u * k : 0u;
    const uint32_t b = hi > 32u * k ? (hi - 32u * k < 32u ? hi - 32u * k : 32u) : 0u;
    if (b > a) w[k] |= (b - a == 32u ? 0xffffffffu : ((1u << (b - a)) - 1u)) << a;
  }
}

__device__ __forceinline__ void set_one(uint32_t (&w)[4], uint32_t bit) {
#pragma unroll
  for (int k = 0; k < 4; ++k) w[k] |= (bit >> 5) == static_cast<uint32_t>(k) ? 1u << (bit & 31) : 0u;
}

// Boundaries of row positions [t, t+len), which sit at bit offset `pos` of
// this lane's 128-element span: starts (cu[i], i < S), ends (cu[j]-1, j >= 1)
// and positions before cu[0] (which belong to no sequence).
template <typename IdxT>
__device__ __forceinline__ void mark_span(uint32_t (&sw)[4], uint32_t (&ew)[4], uint32_t (&ow)[4],
                                          const CuView<IdxT>& cu, int64_t t, int64_t len,
                                          uint32_t pos) {
  const int64_t end = t + len;
  const int64_t cu0 = cu.at(0);
  if (cu0 > t) {
    const uint32_t hi = pos + static_cast<uint32_t>((cu0 < end ? cu0 : end) - t);
    set_range(sw, pos, hi);
    set_range(ew, pos, hi);
    set_range(ow, pos, hi);
  }
  for (int64_t i = cu.lower_bound(0, cu.S, t); i < cu.S; ++i) {
    const int64_t v = cu.at(i);
    if (v >= end) break;
    if (v >= t) set_one(sw, pos + static_cast<uint32_t>(v - t));
  }
  for (int64_t j = cu.lower_bound(1, cu.S + 1, t + 1); j <= cu.S; ++j) {
    const int64_t v = cu.at(j) - 1;
    if (v >= end) break;
    if (v >= t) set_one(ew, pos + static_cast<uint32_t>(v - t));
  }
}

// Builds the boundary bitmaps of the tile that starts at flat index p0.  Lane
// l owns tile elements [128 l, 128 l + 128) and writes its 4 words of each
// bitmap once, without shared-memory atomics.  Called by all 32 lanes.
template <typename IdxT, int NIN, typename T>
__device__ void build_meta(StageMeta<NIN, T>& m, const CuView<IdxT>& cu, int64_t p0, int64_t N,
                           int64_t n_tma_total, int lane) {
  const int64_t rem = N - p0;
  const uint32_t n_valid = static_cast<uint32_t>(rem < kTileElems ? rem : kTileElems);
  int64_t nt = n_tma_total - p0;
  nt = nt < 0 ? 0 : (nt > n_valid ? n_valid : nt);
  uint32_t sw[4] = {0u, 0u, 0u, 0u}, ew[4] = {0u, 0u, 0u, 0u}, ow[4] = {0u, 0u, 0u, 0u};
  const uint32_t e0 = static_cast<uint32_t>(lane) * 128u;
  const int64_t BL = cu.BL;
  if (e0 < n_valid) {
    const int64_t p = p0 + e0;
    int64_t t = (p < 0xffffffffll && BL < 0xffffffffll)
                    ? static_cast<int64_t>(static_cast<uint32_t>(p) % static_cast<uint32_t>(BL))
                    : p % BL;
    const uint32_t stop = (e0 + 128u < n_valid ? e0 + 128u : n_valid) - e0;
    uint32_t pos = 0u;
    while (pos < stop) {
      int64_t len = static_cast<int64_t>(stop - pos);
      if (len > BL - t) len = BL - t;
      mark_span(sw, ew, ow, cu, t, len, pos);
      pos += static_cast<uint32_t>(len);
      t = 0;
    }
  }
  // positions past the end of the array are isolated and never stored
  if (n_valid < e0 + 128u) {
    const uint32_t lo = n_valid > e0 ? n_valid - e0 : 0u;
    set_range(sw, lo, 128u);
    set_range(ew, lo, 128u);
  }
  *reinterpret_cast<uint4*>(&m.sbits[lane * 4]) = make_uint4(sw[0], sw[1], sw[2], sw[3]);
  *reinterpret_cast<uint4*>(&m.ebits[lane * 4]) = make_uint4(ew[0], ew[1], ew[2], ew[3]);
  *reinterpret_cast<uint4*>(&m.obits[lane * 4]) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
  const bool outside = __any_sync(kFull, (ow[0] | ow[1] | ow[2] | ow[3]) != 0u);
  if (lane == 0) {
    m.has_outside = outside ? 1u : 0u;
    m.n_valid = n_valid;
    m.n_tma = static_cast<uint32_t>(nt);
    m.p0 = p0;
  }
}

// ---------------------------------------------------------------------------
// consumer helpers
// ---------------------------------------------------------------------------

// Element e of input k of the current tile, as float.
template <typename T, int NIN>
__device__ __forceinline__ float tile_elem(const uint8_t* buf, const StageMeta<NIN, T>& m, int k,
                                           uint32_t e, uint32_t n_tma, uint32_t n_valid,
                                           float fill) {
  if (e < n_tma) return Cvt<T>::to(*reinterpret_cast<const T*>(buf + swz<T>(e)));
  if (e < n_valid) return m.tail[k][e - n_tma];
  return fill;
}

// This thread's 16 elements [o, o+16) of input k.
template <typename T, int NIN>
__device__ __forceinline__ void read_block(const uint8_t* buf, const StageMeta<NIN, T>& m, int k,
                                           uint32_t o, uint32_t n_tma, uint32_t n_valid,
                                           float fill, float (&v)[kPerThread]) {
  if (o + kPerThread <= n_tma) {
    constexpr int kVec = 16 / sizeof(T);
#pragma unroll
    for (int c = 0; c < kPerThread / kVec; ++c) {
      const uint4 raw = *reinterpret_cast<const uint4*>(buf + swz<T>(o + c * kVec));
      unpack16<T>(raw, &v[c * kVec]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < kPerThread; ++j) v[j] = tile_elem<T, NIN>(buf, m, k, o + j, n_tma, n_valid, fill);
  }
}

template <typename T>
__device__ __forceinline__ void write_block(uint8_t* buf, uint32_t o, const float (&v)[kPerThread]) {
  constexpr int kVec = 16 / sizeof(T);
#pragma unroll
  for (int c = 0; c < kPerThread / kVec; ++c)
    *reinterpret_cast<uint4*>(buf + swz<T>(o + c * kVec)) = pack16<T>(&v[c * kVec]);
}

// Direct global stores of the elements whose bit is set in `mask`.
template <typename T>
__device__ __forceinline__ void store_direct(T* base, int64_t p, uint32_t mask,
                                             const float (&v)[kPerThread]) {
#pragma unroll
  for (int j = 0; j < kPerThread; ++j)
    if ((mask >> j) & 1u) base[p + j] = Cvt<T>::from(v[j]);
}

// Serial fold of 16 elements in scan order with sequence heads.
template <bool REV>
__device__ __forceinline__ Pfx fold16(const float (&a)[kPerThread], const float (&b)[kPerThread],
                                      uint32_t head) {
  constexpr int j0 = REV ? kPerThread - 1 : 0;
  Pfx p{a[j0], b[j0], kValid | static_cast<int>((head >> j0) & 1u)};
  if (head == 0u) {
#pragma unroll
    for (int jj = 1; jj < kPerThread; ++jj) {
      const int j = REV ? kPerThread - 1 - jj : jj;
      p.b = fmaf(a[j], p.b, b[j]);
      p.a *= a[j];
    }
  } else {
#pragma unroll
    for (int jj = 1; jj < kPerThread; ++jj) {
      const int j = REV ? kPerThread - 1 - jj : jj;
      if ((head >> j) & 1u) {
        p.a = a[j];
        p.b = b[j];
        p.f |= kHead;
      } else {
        p.b = fmaf(a[j], p.b, b[j]);
        p.a *= a[j];
      }
    }
  }
  return p;
}

// Tile-level part shared by the forward and backward consumers: combines
// the per-warp totals, publishes this tile's status and looks back.  Returns
// the prefix preceding this thread's first element in scan order.
template <bool REV, typename Sm>
__device__ __forceinline__ Pfx consumer_tile_prefix(Sm& sm, Pfx thread_excl, Pfx warp_total,
                                                    bool first_is_head, uint32_t ticket,
                                                    const TileStatus& st, int warp, int lane) {
  if (lane == 0) sm.warp_total[warp] = warp_total;
  consumer_sync();
  Pfx wex = pfx_empty(), tot = pfx_empty();
#pragma unroll
  for (int ww = 0; ww < kConsumerWarps; ++ww) {
    const int w = REV ? kConsumerWarps - 1 - ww : ww;
    if (w == warp) wex = tot;
    tot = compose(tot, sm.warp_total[w]);
  }
  const bool need_lookback = !first_is_head && ticket > 0;
  if (warp == 0) {
    if (lane == 0) {
      const bool inclusive = (tot.f & kHead) || !need_lookback;
      publish(st, ticket, inclusive ? kStatusInclusive : kStatusAggregate, tot.a, tot.b);
    }
    if (need_lookback) {
      Pfx te = pfx_empty();
      int64_t base = static_cast<int64_t>(ticket) - 1;
      bool timed_out = false;
      while (true) {
        const int64_t q = base - lane;
        Pfx x = pfx_empty();
        bool inc = true;
        if (q >= 0) {
          const uint32_t s = wait_status(st, static_cast<uint32_t>(q));
          if (s == kStatusInclusive || s == kStatusAggregate) {
            const float2 v = ld_relaxed_f2(reinterpret_cast<const float*>(st.vals + q) +
                                           (s == kStatusInclusive ? 2 : 0));
            x = Pfx{v.x, v.y, kValid};
            inc = (s == kStatusInclusive);
          } else {
            timed_out = true;
          }
        }
        const unsigned incmask = __ballot_sync(kFull, inc);
        const int stop = incmask ? (__ffs(incmask) - 1) : 31;
        if (lane > stop) x = pfx_empty();
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          Pfx o{__shfl_down_sync(kFull, x.a, off), __shfl_down_sync(kFull, x.b, off),
                __shfl_down_sync(kFull, x.f, off)};
          if (lane + off < 32) x = compose(o, x);
        }
        const Pfx part{__shfl_sync(kFull, x.a, 0), __shfl_sync(kFull, x.b, 0),
                       __shfl_sync(kFull, x.f, 0)};
        te = compose(part, te);
        if (incmask) break;
        base -= 32;
      }
      // A timed-out wait has set the launch's abort word: the producers stop
      // taking tiles and every consumer leaves through the normal path.
      if (__any_sync(kFull, timed_out) && lane == 0) report(ASCAN_DEV_ERR_LOOKBACK, ticket);
      if (lane == 0) {
        if (!(tot.f & kHead)) {
          const Pfx inc = compose(te, tot);
          publish(st, ticket, kStatusInclusive, inc.a, inc.b);
        }
        sm.te = te;
      }
    }
  }
  Pfx te = pfx_empty();
  if (need_lookback) {
    consumer_sync();
    te = sm.te;
  }
  return compose(te, compose(wex, thread_excl));
}

}  // namespace tma
}  // namespace ascan

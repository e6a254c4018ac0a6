// ascan_tma.cuh -- persistent, TMA-fed scan kernels for sm_100a.
//
// Persistent CTAs (one per SM) run a loop over tiles of kTileElems elements
// dealt to them in scan order.  The last warp is the producer: it takes the ticket,
// waits for a free stage of a shared-memory ring, issues 2-D TMA loads of the
// tile's inputs (tensor maps view the flat array as rows of 128 bytes, 128B
// swizzle) and, while they fly, writes the tile's sequence-boundary bitmaps,
// the neighbour scalars at the tile edges and the ragged tail of the array
// into the stage's metadata.  The other warps consume: thread i owns elements
// [16i, 16i+16) of the tile (the swizzle makes those blocked reads
// bank-conflict free), folds them serially, scans the per-thread aggregates
// across the warp with shuffles and across warps through shared memory,
// obtains the tile's carry-in by decoupled look-back, writes the outputs into
// a double-buffered staging area and hands them to a TMA store.  HBM keeps
// streaming the next stages while a tile is computed or waits on a
// predecessor.
//
// There is no CTA-wide barrier after the prologue: consumer warps hand their
// per-tile totals to each other through tagged shared-memory slots and store
// their own slice of each tile.  Every wait is bounded: mbarrier waits, slot
// waits and look-back polls give up after kLookbackTimeoutNs, report
// ASCAN_DEV_ERR_LOOKBACK and set the CTA's and the launch's abort words, after
// which no wait blocks again.
#pragma once

#include <cuda.h>

#include "ascan_device.cuh"

namespace ascan {
namespace tma {

// CTA geometry: one CTA of 8 consumer warps per SM (4096-element tiles).
// ASCAN_TMA_WARPS=4 at compile time builds two CTAs of 4 consumer warps per
// SM (2048-element tiles) instead; measured on B200 it is within a few
// percent at B=8, C=1536 (the SM still runs 8 consumer warps doing the same
// work per element) and slower when rows are fewer than the CTAs.
#ifndef ASCAN_TMA_WARPS
#define ASCAN_TMA_WARPS 8
#endif
constexpr int kConsumerWarps = ASCAN_TMA_WARPS;
constexpr int kCtasPerSm = 32 / kConsumerWarps / 4;       // 2 for 4 warps, 1 for 8
static_assert(kCtasPerSm >= 1, "4 or 8 consumer warps");
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;        // + producer warp
// Tile geometry per kernel: P elements per consumer thread (16 or 32), so a
// tile holds 256 P elements (8 consumer warps).  P = 32 halves the per-tile
// fixed costs per byte (the consumer warps run one dependent chain per tile)
// at the price of shared memory and registers; the launcher picks P per
// kernel and dtype.
template <int P>
struct Geo {
  static_assert(P == 16 || P == 32, "16 or 32 elements per thread");
  static constexpr int kPerThread = P;
  static constexpr uint32_t kMask = P == 32 ? 0xffffffffu : (1u << (P % 32)) - 1u;
  static constexpr int kTileElems = kConsumers * P;
  static constexpr int kBitWords = kTileElems / 32;
};
// The smallest TMA tile: status slots are counted in it.
constexpr int kMinTileElems = Geo<16>::kTileElems;
static_assert(kTile % kMinTileElems == 0 || kMinTileElems % kTile == 0,
              "TMA tiles and the plain kernels' tiles nest (status slots count the smaller)");
constexpr int kCuCache = 1024;                   // cu_seqlens entries cached in smem
constexpr uint32_t kDone = 0xffffffffu;

template <typename T, int P = 16>
struct Fmt {
  static constexpr int kElemsPerRow = 128 / sizeof(T);  // one 128-byte TMA row
  static constexpr int kRows = Geo<P>::kTileElems / kElemsPerRow;
  static constexpr int kBytes = Geo<P>::kTileElems * sizeof(T);
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

// Bounded wait of a whole warp for the phase of `parity` to complete: every
// lane polls (so every lane acquires), and both the completion and the
// timeout are decided by warp votes, so all 32 lanes leave together with the
// same result.  All lanes must call it.  false on timeout.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity,
                                               unsigned long long limit_ns = kLookbackTimeoutNs) {
  bool done = mbar_try_wait(bar, parity);
  if (__all_sync(kFull, done)) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
    if (!done) done = mbar_try_wait(bar, parity);
    if (__all_sync(kFull, done)) return true;
    if (__any_sync(kFull, wait_expired(t0, limit_ns))) return false;
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

// Untiled bulk copy global -> shared (16-byte aligned addresses, size a
// multiple of 16), completing on the same mbarrier as the tile loads.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes),
      "r"(smem_addr(bar))
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

__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------
// shared-memory layout
// ---------------------------------------------------------------------------

template <int NIN, typename T, int P>
struct StageMeta {
  uint32_t ticket;     // kDone: no more tiles
  uint32_t n_valid;    // tile elements below N
  uint32_t n_tma;      // tile elements covered by the TMA rows
  uint32_t has_outside;
  int64_t p0;          // flat index of the tile's first element
  int64_t row0;        // its row
  int64_t t0;          // its position in that row
  float halo[2];       // bwd: [0] gate neighbour, [1] state neighbour at the tile edge
  uint32_t halo_bulk;  // bit k: halo k is in halo_raw[k] instead of halo[k]
  uint32_t halo_idx[2];  // ragged rows: element of halo_raw[k] that is the neighbour
  uint32_t shift;      // ragged rows: elements between the buffer start and the tile start
  // bwd: the 16-byte block holding halo k, fetched by a bulk copy with the tile
  // (the block starting at the element after the tile, or ending at the
  // element before it)
  alignas(16) T halo_raw[2][16 / sizeof(T)];
  // row mode: copy of the predecessor's 16-byte status slot, fetched by a bulk
  // copy together with the tile (all zero = unknown); an inclusive record in
  // it is the tile's carry-in
  alignas(16) uint32_t te_raw[4];
  // time slabs in the plain kernels: 16-byte blocks of the row carry and row
  // halo arrays, fetched by bulk copies with the tile; io_te / io_halo = 1 +
  // the index of the row's value in its block (0: not fetched this way)
  alignas(16) float io_raw[2][4];
  uint32_t io_te, io_halo;
  alignas(16) uint32_t sbits[Geo<P>::kBitWords];  // sequence starts (and positions outside any sequence)
  alignas(16) uint32_t ebits[Geo<P>::kBitWords];  // sequence ends   (and positions outside any sequence)
  alignas(16) uint32_t obits[Geo<P>::kBitWords];  // positions outside any sequence (valid if has_outside)
  float tail[NIN][Fmt<T>::kTailMax];
};

// Order in which tiles are dealt (as tickets, i.e. in scan order).
//  flat mode: tile k of the flat [C*BL] array is ticket k (reverse scans count
//             from the end); a tile's scan predecessor is ticket - 1.
//  row mode:  every row is cut into row-aligned tiles and the tiles are dealt
//             tile-major across rows (tile j of every row, then tile j+1), so
//             a tile's predecessor in its row is ticket - rows: many waves
//             old when rows >> CTAs, and its status can be read ahead.
//  segment mode (row mode with segs > 1): every row is also cut at its
//             sequence starts into `segs` segments of equal length, a whole
//             number of tiles each, and the (row, segment) pairs are the rows
//             of the tile-major order: a segment's first tile starts a
//             sequence, and a tile's predecessor is rows * segs tickets
//             older.  Valid only when cu_seqlens[i] == i * BL / segs for
//             every i, which the kernels check at start-up (seg_sched).
struct TileSched {
  uint32_t num_tiles;
  uint32_t row_mode;
  uint32_t rows;            // row mode: C
  uint32_t tiles_per_row;   // row mode: ceil(BL / tile elements)
  uint32_t stride;          // ticket distance to the scan predecessor
  uint32_t ragged;          // row mode with BL not a multiple of the tile (last tile of a row partial)
  uint32_t cta0;            // first CTA of this scan's group (0 unless bidirectional)
  uint32_t ctas;            // CTAs of the group (0: the whole grid)
  uint32_t segs;            // segment mode if > 1 (and the start-up check passes)
};

// The schedule a launch runs: segment mode when the host offered it and
// every thread's share of the cu_seqlens check held (`seg_ok`, voted by the
// start-up barrier), else the plain row (or flat) order.
__device__ __forceinline__ TileSched seg_sched(const TileSched& in, bool seg_ok) {
  TileSched s = in;
  if (s.segs > 1u && seg_ok)
    s.stride = s.rows * s.segs;
  else
    s.segs = 1u;
  return s;
}

// Hand-off slots between the consumer warps of one tile (no CTA barrier): the
// per-warp totals and the tile's carry-in, each tagged with the tile's
// ticket.  Warps can drift apart by at most the ring depth (a stage is only
// refilled once every warp has read it), so kXsRing > depth keeps slots apart.
constexpr int kXsRing = 8;
constexpr uint32_t kNoTag = 0xffffffffu;

struct XSlot {
  float4 warp[kConsumerWarps];  // {a, b, flags bits, ticket bits}
  float4 te;                    // tile carry-in {a, b, flags bits, ticket bits}
};

// RG (ragged rows): a tile may start anywhere inside a 128-byte TMA row, so
// each input buffer holds one more TMA row (padded to the 1024-byte swizzle
// atom) and the tile's elements sit `shift` elements into it.
template <typename T, int P, bool RG>
constexpr int in_bytes() {
  return Fmt<T, P>::kBytes + (RG ? 1024 : 0);
}

template <int NIN, int NOUT, int NS, typename T, int P, bool RG>
struct Smem {
  alignas(1024) uint8_t in[NS][NIN][in_bytes<T, P, RG>()];
  // output staging: double-buffered tiles for the TMA stores, or (RG) one
  // tile per output cut into per-warp buffers for the coalesced register
  // stores of store_window
  alignas(1024) uint8_t out[2][NOUT][RG ? Fmt<T, P>::kBytes / 2 : Fmt<T, P>::kBytes];
  StageMeta<NIN, T, P> meta[NS];
  uint64_t full[NS];
  uint64_t empty[NS];
  int64_t cu[kCuCache];
  XSlot xs[kXsRing];
  int abort;  // a consumer warp gave up: the others stop waiting on it
};

// RG kernels: warp w's staging buffer for output k (32 P elements).
template <int NIN, int NOUT, int NS, typename T, int P, bool RG>
__device__ __forceinline__ uint8_t* warp_stage(Smem<NIN, NOUT, NS, T, P, RG>& sm, int k, int warp) {
  constexpr int kWarpBytes = Fmt<T, P>::kBytes / kConsumerWarps;
  return &sm.out[0][0][0] + k * Fmt<T, P>::kBytes + warp * kWarpBytes;
}

template <int NIN, int NOUT, int NS, typename T, int P, bool RG>
constexpr size_t smem_bytes() {
  return sizeof(Smem<NIN, NOUT, NS, T, P, RG>) + 1024;  // + alignment slack
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
  // First i in [lo, hi) with at(i) >= v (hi if none), for sorted entries;
  // any input gives an index in [lo, hi].  Warp-wide: all lanes call and get
  // the same result.  Each round probes 32 evenly spaced entries at once, so
  // up to 32 entries take one round of loads and a ballot.
  __device__ __forceinline__ int64_t lower_bound_warp(int64_t lo, int64_t hi, int64_t v,
                                                      int lane) const {
    while (hi - lo > 32) {
      const int64_t step = (hi - lo + 31) / 32;
      const int64_t idx = lo + lane * step;
      const unsigned ge = __ballot_sync(kFull, idx < hi && at(idx) >= v);
      if (ge & 1u) return lo;
      const int f = ge ? __ffs(ge) - 1 : 32;          // first probe at or above v
      const int64_t below = lo + static_cast<int64_t>(f - 1) * step;  // last probe below v
      const int64_t next_hi = f < 32 ? lo + static_cast<int64_t>(f) * step : hi;
      lo = below + 1;
      hi = next_hi < hi ? next_hi : hi;
    }
    const int64_t idx = lo + lane;
    const unsigned ge = __ballot_sync(kFull, idx < hi && at(idx) >= v);
    return ge ? lo + (__ffs(ge) - 1) : hi;
  }
};

__device__ __forceinline__ void or_bit(uint32_t* words, uint32_t e) {
  atomicOr(&words[e >> 5], 1u << (e & 31));
}

// Marks, for row positions [t, t+len) sitting at tile offset `pos`, the
// sequence starts (cu[i], i < S), the sequence ends (cu[j]-1, j >= 1) and the
// positions before cu[0] (which belong to no sequence).  One warp-wide search
// for the first boundary at or after t, then one pass over the boundaries in
// [t, t+len]: boundary v = cu[i] starts a sequence at v and ends one at v-1.
// Called by all lanes.
template <typename IdxT, int NIN, typename T, int P>
__device__ __forceinline__ void mark_segment(StageMeta<NIN, T, P>& m, const CuView<IdxT>& cu,
                                             int64_t t, int64_t len, uint32_t pos, int lane,
                                             bool& outside) {
  const int64_t end = t + len;
  const int64_t cu0 = cu.at(0);
  if (cu0 > t) {
    const int64_t oend = cu0 < end ? cu0 : end;
    for (int64_t q = t + lane; q < oend; q += 32) {
      const uint32_t e = pos + static_cast<uint32_t>(q - t);
      or_bit(m.sbits, e);
      or_bit(m.ebits, e);
      or_bit(m.obits, e);
    }
    outside = true;
  }
  const int64_t i0 = cu.lower_bound_warp(0, cu.S + 1, t, lane);
  for (int64_t i = i0 + lane;; i += 32) {
    bool in = false;  // this lane's boundary lies in [t, end]
    if (i <= cu.S) {
      const int64_t v = cu.at(i);
      if (v <= end) {
        in = true;
        if (i < cu.S && v >= t && v < end) or_bit(m.sbits, pos + static_cast<uint32_t>(v - t));
        if (i >= 1 && v > t) or_bit(m.ebits, pos + static_cast<uint32_t>(v - 1 - t));
      }
    }
    // sorted boundaries: another round only if the last lane's was still inside
    if (!__shfl_sync(kFull, in, 31)) break;
  }
}

// Builds the boundary bitmaps of the tile that starts at flat index p0, whose
// first element sits at row position t0 of row row0 and whose elements end at flat index
// `limit` (the array end, or the row end in row mode).  Called by all lanes.
template <typename IdxT, int NIN, typename T, int P>
__device__ void build_meta(StageMeta<NIN, T, P>& m, const CuView<IdxT>& cu, int64_t p0, int64_t t0,
                           int64_t row0, int64_t limit, int64_t n_tma_total, int lane) {
  constexpr int kTileElems = Geo<P>::kTileElems, kBitWords = Geo<P>::kBitWords;
  const int64_t rem = limit - p0;  // elements of the tile that belong to it (row or array end)
  const uint32_t n_valid = static_cast<uint32_t>(rem < kTileElems ? rem : kTileElems);
  int64_t nt = n_tma_total - p0;
  nt = nt < 0 ? 0 : (nt > n_valid ? n_valid : nt);
  // positions past the end of the array are isolated and never stored
  for (int w = lane; w < kBitWords; w += 32) {
    const uint32_t e0 = static_cast<uint32_t>(w) * 32u;
    const uint32_t past =
        n_valid >= e0 + 32u ? 0u : (n_valid <= e0 ? 0xffffffffu : 0xffffffffu << (n_valid - e0));
    m.sbits[w] = past;
    m.ebits[w] = past;
    m.obits[w] = 0u;
  }
  __syncwarp();
  const int64_t BL = cu.BL;
  int64_t t = t0;
  uint32_t pos = 0;
  bool outside = false;
  while (pos < n_valid) {
    int64_t len = static_cast<int64_t>(n_valid - pos);
    if (len > BL - t) len = BL - t;
    mark_segment<IdxT, NIN, T, P>(m, cu, t, len, pos, lane, outside);
    pos += static_cast<uint32_t>(len);
    t = 0;
  }
  if (lane == 0) {
    m.has_outside = outside ? 1u : 0u;
    m.n_valid = n_valid;
    m.n_tma = static_cast<uint32_t>(nt);
    m.p0 = p0;
    m.row0 = row0;
    m.t0 = t0;
    m.io_te = m.io_halo = 0u;
  }
}

// ---------------------------------------------------------------------------
// consumer helpers
// ---------------------------------------------------------------------------

// Element e of input k of the current tile, as float (`shift`: elements
// between the buffer start and the tile start, ragged rows only).
template <typename T, int NIN, int P>
__device__ __forceinline__ float tile_elem(const uint8_t* buf, const StageMeta<NIN, T, P>& m, int k,
                                           uint32_t e, uint32_t n_tma, uint32_t n_valid,
                                           float fill, uint32_t shift = 0u) {
  if (e < n_tma) return Cvt<T>::to(*reinterpret_cast<const T*>(buf + swz<T>(e + shift)));
  if (e < n_valid) return m.tail[k][e - n_tma];
  return fill;
}

// Per-thread constants: the swizzled byte offsets of the 16-byte chunks that
// hold this thread's 16 elements (identical for every 1024-aligned buffer).
template <typename T, int P>
struct ThreadChunks {
  static constexpr int kVec = 16 / sizeof(T);
  static constexpr int kChunks = P / kVec;
  uint32_t off[kChunks];
  __device__ __forceinline__ explicit ThreadChunks(uint32_t o) {
#pragma unroll
    for (int c = 0; c < kChunks; ++c) off[c] = swz<T>(o + c * kVec);
  }
};

// This thread's 16 elements [o, o+16) of input k.
template <typename T, int NIN, int P>
__device__ __forceinline__ void read_block(const uint8_t* buf, const ThreadChunks<T, P>& tc,
                                           const StageMeta<NIN, T, P>& m, int k, uint32_t o,
                                           uint32_t n_tma, uint32_t n_valid, float fill,
                                           float (&v)[P]) {
  if (o + P <= n_tma) {
#pragma unroll
    for (int c = 0; c < ThreadChunks<T, P>::kChunks; ++c)
      unpack16<T>(*reinterpret_cast<const uint4*>(buf + tc.off[c]),
                  &v[c * ThreadChunks<T, P>::kVec]);
  } else {
#pragma unroll
    for (int j = 0; j < P; ++j)
      v[j] = tile_elem<T, NIN>(buf, m, k, o + j, n_tma, n_valid, fill);
  }
}

// This thread's P elements [o, o+P) of 16-bit input k, packed two per word
// (element 2i in the low half of w[i]); partial tiles pack the converted
// elements back (exact: they came from T).
template <typename T, int NIN, int P>
__device__ __forceinline__ void read_block_packed(const uint8_t* buf, const ThreadChunks<T, P>& tc,
                                                  const StageMeta<NIN, T, P>& m, int k, uint32_t o,
                                                  uint32_t n_tma, uint32_t n_valid,
                                                  uint32_t (&w)[P / 2]) {
  static_assert(sizeof(T) == 2, "packed reads are for 16-bit types");
  if (o + P <= n_tma) {
#pragma unroll
    for (int c = 0; c < ThreadChunks<T, P>::kChunks; ++c) {
      const uint4 q = *reinterpret_cast<const uint4*>(buf + tc.off[c]);
      w[4 * c] = q.x, w[4 * c + 1] = q.y, w[4 * c + 2] = q.z, w[4 * c + 3] = q.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < P / 2; ++i) {
      const T lo = Cvt<T>::from(tile_elem<T, NIN>(buf, m, k, o + 2 * i, n_tma, n_valid, 0.f));
      const T hi = Cvt<T>::from(tile_elem<T, NIN>(buf, m, k, o + 2 * i + 1, n_tma, n_valid, 0.f));
      w[i] = static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&lo)) |
             (static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&hi)) << 16);
    }
  }
}

// Element j of a packed block, as float (j is a compile-time index in the
// unrolled loops that call this).
template <typename T, int N>
__device__ __forceinline__ float packed_elem(const uint32_t (&w)[N], int j) {
  const uint16_t bits = static_cast<uint16_t>((j & 1) ? (w[j >> 1] >> 16) : (w[j >> 1] & 0xffffu));
  return Cvt<T>::to(*reinterpret_cast<const T*>(&bits));
}

// This thread's 16 elements of a tile that starts `shift` elements into the
// buffer (ragged rows): kChunks+1 aligned 16-byte chunks are read and the 16
// elements taken from offset r = shift % kVec, which is the same for every
// thread of the tile (a warp-uniform switch, so no register is indexed at run
// time).
template <typename T, int R, int P>
__device__ __forceinline__ void take_shifted(const float (&raw)[P + 16 / sizeof(T)],
                                             float (&v)[P]) {
#pragma unroll
  for (int j = 0; j < P; ++j) v[j] = raw[R + j];
}

template <typename T, int NIN, int P>
__device__ __forceinline__ void read_block_shifted(const uint8_t* buf,
                                                   const StageMeta<NIN, T, P>& m, int k,
                                                   uint32_t o, uint32_t shift, uint32_t n_tma,
                                                   uint32_t n_valid, float fill, float (&v)[P]) {
  constexpr int kVec = ThreadChunks<T, P>::kVec;
  constexpr int kChunks = ThreadChunks<T, P>::kChunks;
  if (o + P <= n_tma) {
    const uint32_t r = shift % kVec;
    const uint32_t base = o + shift - r;
    float raw[P + kVec];
#pragma unroll
    for (int c = 0; c <= kChunks; ++c)
      unpack16<T>(*reinterpret_cast<const uint4*>(buf + swz<T>(base + c * kVec)), &raw[c * kVec]);
    switch (r) {
      case 0: take_shifted<T, 0>(raw, v); break;
      case 1: take_shifted<T, 1>(raw, v); break;
      case 2: take_shifted<T, 2>(raw, v); break;
      case 3: take_shifted<T, 3>(raw, v); break;
      default:
        if constexpr (kVec > 4) {
          switch (r) {
            case 4: take_shifted<T, (kVec > 4 ? 4 : 0)>(raw, v); break;
            case 5: take_shifted<T, (kVec > 4 ? 5 : 0)>(raw, v); break;
            case 6: take_shifted<T, (kVec > 4 ? 6 : 0)>(raw, v); break;
            default: take_shifted<T, (kVec > 4 ? 7 : 0)>(raw, v); break;
          }
        }
        break;
    }
  } else {
#pragma unroll
    for (int j = 0; j < P; ++j)
      v[j] = tile_elem<T, NIN>(buf, m, k, o + j, n_tma, n_valid, fill, shift);
  }
}

template <typename T, int P>
__device__ __forceinline__ void write_block(uint8_t* buf, const ThreadChunks<T, P>& tc,
                                            const float (&v)[P]) {
#pragma unroll
  for (int c = 0; c < ThreadChunks<T, P>::kChunks; ++c)
    *reinterpret_cast<uint4*>(buf + tc.off[c]) = pack16<T>(&v[c * ThreadChunks<T, P>::kVec]);
}

// Direct global stores of the elements whose bit is set in `mask`.
template <typename T, int P>
__device__ __forceinline__ void store_direct(T* base, int64_t p, uint32_t mask,
                                             const float (&v)[P]) {
#pragma unroll
  for (int j = 0; j < P; ++j)
    if ((mask >> j) & 1u) base[p + j] = Cvt<T>::from(v[j]);
}

// Lane t holds the P elements [q + P t, q + P t + P) of a warp-contiguous
// run whose start q (lane 0's) lies R elements past a 16-byte boundary.
// Every lane takes the last R elements of its left neighbour, so that it
// holds the aligned window [q + P t - R, q + P t - R + P); the windows go
// through the warp's staging buffer `stage` (32 P elements, 128B-swizzled)
// and leave as 16-byte stores in which consecutive lanes write consecutive
// chunks (a fully coalesced 512-byte run per instruction).  The R elements
// before q are not the warp's: the first chunk is written element by
// element from R on; lane 31's last R elements go out one by one.
// Warp-collective.
template <typename T, int R, int P>
__device__ __forceinline__ void store_window(T* base, int64_t q_lane, const float (&v)[P],
                                             int lane, uint8_t* stage) {
  constexpr int kVec = ThreadChunks<T, P>::kVec, kChunks = ThreadChunks<T, P>::kChunks;
  float w[P];
#pragma unroll
  for (int j = 0; j < R; ++j) w[j] = __shfl_up_sync(kFull, v[P - R + j], 1);
#pragma unroll
  for (int j = R; j < P; ++j) w[j] = v[j - R];
  const uint32_t e0 = static_cast<uint32_t>(lane) * P;
#pragma unroll
  for (int c = 0; c < kChunks; ++c)
    *reinterpret_cast<uint4*>(stage + swz<T>(e0 + c * kVec)) = pack16<T>(&w[c * kVec]);
  __syncwarp();
  const int64_t w0 = q_lane - static_cast<int64_t>(e0) - R;  // the warp's aligned window start
#pragma unroll
  for (int k = 0; k < kChunks; ++k) {
    const uint32_t ci = static_cast<uint32_t>(lane) + 32u * k;  // chunk of the warp's window
    const uint4 val = *reinterpret_cast<const uint4*>(stage + swz<T>(ci * kVec));
    T* dst = base + w0 + static_cast<int64_t>(ci) * kVec;
    if (R != 0 && ci == 0u) {
      const T* e = reinterpret_cast<const T*>(&val);
#pragma unroll
      for (int j = R; j < kVec; ++j) dst[j] = e[j];
    } else {
      st_v4(dst, val);
    }
  }
  if (R != 0 && lane == 31) {
#pragma unroll
    for (int j = P - R; j < P; ++j) base[q_lane + j] = Cvt<T>::from(v[j]);
  }
  __syncwarp();  // the buffer is free again for the next output
}

// store_window for the run's actual misalignment r = q mod (16 bytes).
template <typename T, int P>
__device__ __forceinline__ void store_realigned(T* base, int64_t q, uint32_t r,
                                                const float (&v)[P], int lane, uint8_t* stage) {
  constexpr int kVec = ThreadChunks<T, P>::kVec;
  switch (r) {
    case 0: store_window<T, 0>(base, q, v, lane, stage); break;
    case 1: store_window<T, 1>(base, q, v, lane, stage); break;
    case 2: store_window<T, 2>(base, q, v, lane, stage); break;
    case 3: store_window<T, 3>(base, q, v, lane, stage); break;
    default:
      if constexpr (kVec > 4) {
        switch (r) {
          case 4: store_window<T, (kVec > 4 ? 4 : 0)>(base, q, v, lane, stage); break;
          case 5: store_window<T, (kVec > 4 ? 5 : 0)>(base, q, v, lane, stage); break;
          case 6: store_window<T, (kVec > 4 ? 6 : 0)>(base, q, v, lane, stage); break;
          default: store_window<T, (kVec > 4 ? 7 : 0)>(base, q, v, lane, stage); break;
        }
      }
      break;
  }
}

// Bits j of [0, P) with o + j < limit.
template <int P>
__device__ __forceinline__ uint32_t below_mask(uint32_t o, uint32_t limit) {
  if (limit >= o + P) return Geo<P>::kMask;
  return limit > o ? (1u << (limit - o)) - 1u : 0u;
}

// Serial fold of 16 elements in scan order with sequence heads.  Leaves the
// local inclusive prefix of every element in place (a[j] = product of the
// gates since the last head, b[j] = the state from a zero carry) and returns
// the thread's aggregate.  Two independent chains (a and b).
template <bool REV, int P>
__device__ __forceinline__ Pfx fold16_inplace(float (&a)[P], float (&b)[P], uint32_t head) {
  constexpr int kPerThread = P;
  constexpr int j0 = REV ? kPerThread - 1 : 0;
  float A = a[j0], B = b[j0];
  const int f = kValid | (head != 0u ? kHead : 0);
  // One path per warp (a warp vote, not a per-thread branch): a single lane
  // holding a head must not make its whole warp run both loops.
  if (__all_sync(kFull, head == 0u)) {
#pragma unroll
    for (int jj = 1; jj < kPerThread; ++jj) {
      const int j = REV ? kPerThread - 1 - jj : jj;
      B = fmaf(a[j], B, b[j]);
      A *= a[j];
      a[j] = A;
      b[j] = B;
    }
  } else {
#pragma unroll
    for (int jj = 1; jj < kPerThread; ++jj) {
      const int j = REV ? kPerThread - 1 - jj : jj;
      const bool h = (head >> j) & 1u;  // a head restarts the recurrence (selects, no branch)
      const float Bn = fmaf(a[j], B, b[j]);
      const float An = A * a[j];
      B = h ? b[j] : Bn;
      A = h ? a[j] : An;
      a[j] = A;
      b[j] = B;
    }
  }
  return Pfx{A, B, f};
}

// Elements (bits) that come before the first head in scan order: only these
// take the carry-in.
template <bool REV, int P>
__device__ __forceinline__ uint32_t carry_mask(uint32_t head) {
  if (head == 0u) return Geo<P>::kMask;
  if (!REV) return (1u << (__ffs(head) - 1)) - 1u;
  return Geo<P>::kMask & ~((2u << (31 - __clz(head))) - 1u);
}

// ---- time slabs: per-row carry-in, halo and aggregate --------------------

// Row and row position of a thread's first element, from its tile's row and
// row position (t may run past the row end: the tile spans rows in flat
// order).  The helpers below walk the thread's K elements from there by
// increments -- no division on the consumers' path.
struct RowPos {
  int64_t r, t;
  __device__ __forceinline__ RowPos(int64_t row0, int64_t t, int64_t BL) : r(row0), t(t) {
    while (this->t >= BL) {
      this->t -= BL;
      ++r;
    }
  }
  // From a flat position (one division: for rare paths only).
  __device__ __forceinline__ RowPos(int64_t p, int64_t BL) : r(p / BL), t(p - (p / BL) * BL) {}
  __device__ __forceinline__ void next(int64_t BL) {
    if (++t == BL) {
      t = 0;
      ++r;
    }
  }
};

// Fetches, with the stage's barrier, the 16-byte block of `arr` (`count`
// floats) that holds arr[i .. i + n) into dst and returns 1 + the index of
// arr[i] there, or 0 when no such block lies inside the array (the caller
// then reads the values itself).  Producer lane only.
__device__ __forceinline__ uint32_t fetch_block(float (&dst)[4], const float* arr, int64_t count,
                                                int64_t i, int n, uint64_t* bar) {
  const uintptr_t base = reinterpret_cast<uintptr_t>(arr);
  const uintptr_t at = base + static_cast<uintptr_t>(4 * i);
  const uintptr_t blk = at & ~static_cast<uintptr_t>(15);
  if (blk < base || blk + 16 > base + static_cast<uintptr_t>(4 * count) ||
      at + static_cast<uintptr_t>(4 * n) > blk + 16)
    return 0u;
  mbar_expect_tx(bar, 16u);
  bulk_load(dst, reinterpret_cast<const void*>(blk), 16u, bar);
  return 1u + static_cast<uint32_t>((at - blk) / 4);
}

// Forward: the carried (gate product, state) of each row enters at the row's
// first element in scan order, which is a sequence head: x' = x + g * state
// and g' = g * product reproduce the continued recurrence and its gate
// products exactly.  `bits` holds the thread's heads.
template <bool REV, int K>
__device__ __forceinline__ void apply_row_carry(float (&a)[K], float (&b)[K], uint32_t bits,
                                                RowPos rp, int64_t BL, const float* carry) {
  const int64_t want = REV ? BL - 1 : 0;
#pragma unroll
  for (int j = 0; j < K; ++j) {
    if (((bits >> j) & 1u) && rp.t == want) {
      b[j] = fmaf(a[j], carry[2 * rp.r + 1], b[j]);
      a[j] *= carry[2 * rp.r];
    }
    rp.next(BL);
  }
}

// Backward: the carried adjoint term enters at the row's first element in
// scan order (a head: the end of the slab's last sequence piece); its
// successor gate lives outside the slab and is already part of the term, so
// the element's own coefficient becomes the identity.
template <bool CAUSAL, int K>
__device__ __forceinline__ void apply_row_carry_adjoint(float (&a)[K], float (&b)[K],
                                                        uint32_t bits, RowPos rp, int64_t BL,
                                                        const float* carry) {
  const int64_t want = CAUSAL ? BL - 1 : 0;
#pragma unroll
  for (int j = 0; j < K; ++j) {
    if (((bits >> j) & 1u) && rp.t == want) {
      b[j] += carry[rp.r];
      a[j] = 1.f;
    }
    rp.next(BL);
  }
}

// Backward: the state neighbour of the row element whose neighbour lies
// outside the slab.  Returns the bits that took a halo (their gate gradient
// is not forced to zero).
template <bool CAUSAL, int K>
__device__ __forceinline__ uint32_t apply_row_halo(float (&hv)[K], uint32_t bits, RowPos rp,
                                                   int64_t BL, const float* halo) {
  const int64_t want = CAUSAL ? 0 : BL - 1;
  uint32_t used = 0u;
#pragma unroll
  for (int j = 0; j < K; ++j) {
    if (((bits >> j) & 1u) && rp.t == want) {
      hv[j] = halo[rp.r];
      used |= 1u << j;
    }
    rp.next(BL);
  }
  return used;
}

// Inclusive (gate product, value) at each row's last element in scan order.
// a, b are the thread's local prefixes and P its exclusive prefix; elements in
// `cm` (before the thread's first head) take P.
template <bool REV, int K>
__device__ __forceinline__ void record_row_agg(const float (&a)[K], const float (&b)[K],
                                               uint32_t bits, uint32_t cm, const Pfx& P,
                                               RowPos rp, int64_t BL, float* agg) {
  const int64_t want = REV ? 0 : BL - 1;
#pragma unroll
  for (int j = 0; j < K; ++j) {
    if (((bits >> j) & 1u) && rp.t == want) {
      const bool c = (cm >> j) & 1u;
      agg[2 * rp.r] = c ? a[j] * P.a : a[j];
      agg[2 * rp.r + 1] = c ? fmaf(a[j], P.b, b[j]) : b[j];
    }
    rp.next(BL);
  }
}

// The scan-first warp's early read of its tile's predecessor status: issued
// by lane 0 when the tile starts, so that its round trip overlaps the tile's
// local fold and warp scan; take_early() turns an inclusive record into the
// known carry-in (otherwise the warp looks back as usual).
__device__ __forceinline__ uint4 load_status_raw(const TileStatus& st, uint32_t q) {
  uint4 r;
  asm volatile("ld.relaxed.gpu.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(st.slots + q)
               : "memory");
  return r;
}

// Warp-wide (all lanes call): adopt lane 0's early record if it is inclusive.
__device__ __forceinline__ void take_early(const uint4& raw, bool& te_known, Pfx& te) {
  const uint32_t k1 = __shfl_sync(kFull, raw.y, 0), k3 = __shfl_sync(kFull, raw.w, 0);
  const uint32_t a = __shfl_sync(kFull, raw.x, 0), b = __shfl_sync(kFull, raw.z, 0);
  if (k1 == kStatusInclusive && k3 == kStatusInclusive) {
    te_known = true;
    te = Pfx{__uint_as_float(a), __uint_as_float(b), kValid};
  }
}

// Slot hand-off in shared memory: one 16-byte store of {a, b, flags, tag}.
__device__ __forceinline__ void xs_put(float4* slot, const Pfx& p, uint32_t tag) {
  asm volatile("st.volatile.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(smem_addr(slot)),
               "r"(__float_as_uint(p.a)), "r"(__float_as_uint(p.b)), "r"(static_cast<uint32_t>(p.f)),
               "r"(tag)
               : "memory");
}

__device__ __forceinline__ uint4 xs_load(const float4* slot) {
  uint4 w;
  asm volatile("ld.volatile.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(w.x), "=r"(w.y), "=r"(w.z), "=r"(w.w)
               : "r"(smem_addr(slot))
               : "memory");
  return w;
}

// Bounded wait of a whole warp for slot hand-offs: each lane with `need`
// waits for its `slot` to carry `tag` and then takes its value into `out`
// (other lanes leave `out` alone).  The slot is written and read as one
// 16-byte access, so a matching tag comes with its own value and no fence is
// needed.  Completion, timeout and the CTA's abort word are decided by warp
// votes, so the result is the same in all lanes and the warp never splits.
// All lanes must call it.  false on timeout or abort.
__device__ __forceinline__ bool xs_get_warp(const float4* slot, bool need, uint32_t tag,
                                            Pfx& out, const volatile int* abort_flag,
                                            unsigned long long limit_ns = kLookbackTimeoutNs) {
  uint4 w = make_uint4(0u, 0u, 0u, 0u);
  bool have = !need;
  if (need) {
    w = xs_load(slot);
    have = w.w == tag;
  }
  if (!__all_sync(kFull, have)) {
    const unsigned long long t0 = globaltimer();
    while (true) {
      if (!have) {
        w = xs_load(slot);
        have = w.w == tag;
      }
      if (__all_sync(kFull, have)) break;
      if (__any_sync(kFull, *abort_flag != 0 || wait_expired(t0, limit_ns))) return false;
    }
  }
  if (need) out = Pfx{__uint_as_float(w.x), __uint_as_float(w.y), static_cast<int>(w.z)};
  return true;
}

// Prefix of this thread's first element within the whole scan, for one warp
// of a tile, without any CTA-wide barrier.  Every warp posts its total; the
// scan-first warp looks back over the preceding tiles and posts the tile's
// carry-in; each warp composes the totals of the warps before it; the
// scan-last warp publishes the tile's status.  `ok` turns false when a wait
// gave up (the caller then leaves its loop after this tile).
template <bool REV, typename Sm>
__device__ __forceinline__ Pfx warp_tile_prefix(Sm& sm, uint32_t xi, Pfx thread_excl,
                                                Pfx warp_total, bool first_is_head,
                                                uint32_t ticket, const TileStatus& st,
                                                uint32_t stride, bool te_known, Pfx te_known_val,
                                                int warp, int lane, bool& ok, uint32_t* err_host) {
  constexpr int kLast = kConsumerWarps - 1;
  const int lw = REV ? kLast - warp : warp;  // position of this warp in scan order
  // a row's first tile has no predecessor, unless its carry-in was given with
  // the tile (a time slab's row carry, te_known)
  const bool need_lookback = !first_is_head && (ticket >= stride || te_known);
  XSlot& slot = sm.xs[xi];
  if (lane == 0) xs_put(&slot.warp[warp], warp_total, ticket);
  if (lw == 0 && need_lookback) {
    Pfx te = te_known_val;
    if (!te_known) {
      bool timed_out = false;
      te = lookback_warp<kLookbackPerLane>(st, ticket, lane, &timed_out, stride);
      if (timed_out && lane == 0) report(ASCAN_DEV_ERR_LOOKBACK, ticket, err_host);
    }
    if (lane == 0) xs_put(&slot.te, te, ticket);
  }
  // totals of the warps before this one, lane j holding the j-th in scan order
  Pfx x = pfx_empty();
  const bool before = lane < lw;
  bool got = xs_get_warp(&slot.warp[before ? (REV ? kLast - lane : lane) : 0], before, ticket, x,
                         &sm.abort);
#pragma unroll
  for (int off = 1; off < kConsumerWarps; off <<= 1) {
    const Pfx o{__shfl_down_sync(kFull, x.a, off), __shfl_down_sync(kFull, x.b, off),
                __shfl_down_sync(kFull, x.f, off)};
    if (lane + off < 32) x = compose(x, o);
  }
  const Pfx wex{__shfl_sync(kFull, x.a, 0), __shfl_sync(kFull, x.b, 0), __shfl_sync(kFull, x.f, 0)};
  const Pfx p_in = compose(wex, thread_excl);
  Pfx te = pfx_empty();
  if (lw == kLast) {
    const Pfx tot = compose(wex, warp_total);
    if (need_lookback && te_known && !(tot.f & kHead)) {
      // The carry-in came with the tile (a row carry, or the predecessor's
      // inclusive record): publish the inclusive record at once.  An
      // aggregate would be wrong here, not just early: a row carry is in no
      // earlier status slot, so a successor that composed this aggregate
      // with the tiles before it (or with the empty prefix before ticket 0)
      // would lose the carry.
      const Pfx inc = compose(te_known_val, tot);
      if (lane == 0) publish(st, ticket, kStatusInclusive, inc.a, inc.b);
      ok = got && ok;  // got is warp-uniform
      return compose(te_known_val, p_in);
    }
    if (lane == 0) {
      const bool inclusive = (tot.f & kHead) || !need_lookback;
      publish(st, ticket, inclusive ? kStatusInclusive : kStatusAggregate, tot.a, tot.b);
    }
    if (need_lookback && !(tot.f & kHead)) {
      got = xs_get_warp(&slot.te, true, ticket, te, &sm.abort) && got;
      if (lane == 0) {
        const Pfx inc = compose(te, tot);
        publish(st, ticket, kStatusInclusive, inc.a, inc.b);
      }
      ok = got && ok;  // got is warp-uniform
      return compose(te, p_in);
    }
  }
  if (need_lookback && __any_sync(kFull, !(p_in.f & kHead))) {
    if (te_known)  // warp-uniform; the scan-first warp posts this same value
      te = te_known_val;
    else
      got = xs_get_warp(&slot.te, true, ticket, te, &sm.abort) && got;
  }
  ok = got && ok;  // got is warp-uniform
  return compose(te, p_in);
}

}  // namespace tma
}  // namespace ascan

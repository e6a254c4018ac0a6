// ascan_impl.cuh -- sm_100a kernels and launchers of the packed-varlen linear
// scan, shared by the library's compilation units.
//
// Every unit (ascan_fwd_*.cu, ascan_bwd_*.cu, ascan_bidi.cu, ascan_misc.cu)
// includes this file and explicitly instantiates only its own launchers
// (fwd_typed, bwd_typed, ... for its dtypes), so the kernels are compiled once
// each and the units build in parallel; ascan.cu holds the C ABI and calls the
// launchers through the explicit-instantiation declarations at the end of this
// file.  Each unit's module has its own sticky error word (g_err_code);
// ascan_get_device_error reads all of them through the accessors that
// ASCAN_UNIT_ERROR_ACCESSORS defines in every unit.
//
// Plain family (one CTA per tile; misaligned views and tiny arrays):
//   * The [C, BL] tensors are treated as ONE flat array of N = C*BL elements
//     cut into tiles of kTile = 4096 consecutive elements.  A sequence head
//     sits at every flat index c*BL + cu[i], so a tile may hold several rows
//     or several sequences, and a long sequence spans many tiles.
//   * 256 threads per tile, 8 warps; a warp owns 4096/8 = 512 consecutive
//     elements as R rows of 32 lanes x VEC elements, VEC = one 128-bit vector
//     (4 fp32 / 8 fp16|bf16).  Lane l of row r loads the vector at
//     warp_base + r*32*VEC + l*VEC, so every load and store instruction of a
//     warp touches 512 contiguous bytes.
//   * In-register scan: each lane folds its VEC elements, a shuffle scan runs
//     across the 32 lanes of each row, rows and warps are chained, and the
//     tile's carry-in comes from a decoupled look-back over the tiles that
//     precede it in scan order (tile order = dynamic ticket, so every tile a
//     CTA waits on belongs to a CTA that is already running).  A tile whose
//     first element starts a sequence needs no look-back at all, which is the
//     common case for packed batches whose lengths are multiples of 4096.
//   * All arithmetic is fp32; fp16/bf16 are converted on load and rounded to
//     nearest on store.
//   * The backward is the same scan run in the opposite direction over
//     (a, b) = (gate of the neighbouring element, dy); the one-element shifts
//     of the gates and of the states come from warp shuffles plus one scalar
//     load at each warp edge, so no shifted copy is ever materialised.
// The persistent TMA family (the default) is described in ascan_tma.cuh.
#pragma once

#include <cudaTypedefs.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <type_traits>

#include "../../include/ascan.h"
#include "ascan_device.cuh"

namespace ascan {

// Sticky per-device error word (ASCAN_DEV_ERR_* bits) and a detail value, one
// pair per compilation unit (each unit is its own module on the device).
static __device__ unsigned int g_err_code = 0;
static __device__ unsigned long long g_err_detail = 0;

// Records an error in this unit's sticky word and, when the process enabled
// one (ascan_error_flag), in the pinned host word the host polls without
// synchronising (a plain store: concurrent reports may overwrite each other's
// bits there; the sticky word keeps all of them).
__device__ __forceinline__ void report(unsigned int bits, unsigned long long detail,
                                       uint32_t* host) {
  if (atomicOr(&g_err_code, bits) == 0u) atomicExch(&g_err_detail, detail);
  if (host) asm volatile("st.volatile.global.u32 [%0], %1;" ::"l"(host), "r"(bits) : "memory");
}

// The first tile checks cu_seqlens once per launch.  Every other tile only
// clamps what it reads (cu_at), so a bad array can never move an access.
template <typename IdxT>
__device__ void validate_cu(const IdxT* __restrict__ cu, int64_t S, int64_t BL,
                            uint32_t* err_host) {
  unsigned bits = 0u;
  for (int64_t i = threadIdx.x; i <= S; i += kThreads) {
    const int64_t v = static_cast<int64_t>(__ldg(cu + i));
    if (v < 0 || v > BL) bits |= ASCAN_DEV_ERR_CU_ORDER;
    if (i < S && static_cast<int64_t>(__ldg(cu + i + 1)) < v) bits |= ASCAN_DEV_ERR_CU_ORDER;
    if (i == S && v != BL) bits |= ASCAN_DEV_ERR_CU_END;
  }
  if (bits) report(bits, 0ull, err_host);
}

// Tile-level tail shared by the forward and backward kernels: chains the warp
// totals, publishes this tile's status, looks back when the tile's first
// element does not start a sequence, and returns the prefix that precedes
// this warp's first element in scan order.
template <bool REV>
__device__ __forceinline__ Pfx tile_prefix(Pfx warp_total, bool first_is_head, uint32_t ticket,
                                           const TileStatus& st, int warp, int lane,
                                           uint32_t* err_host) {
  __shared__ Pfx s_warp[kWarps];
  __shared__ int s_first_head;
  __shared__ Pfx s_te;

  if (lane == 0) s_warp[warp] = warp_total;
  if (threadIdx.x == (REV ? kThreads - 1 : 0)) s_first_head = first_is_head ? 1 : 0;
  __syncthreads();

  Pfx wex = pfx_empty(), tot = pfx_empty();
#pragma unroll
  for (int ww = 0; ww < kWarps; ++ww) {
    const int w = REV ? kWarps - 1 - ww : ww;
    if (w == warp) wex = tot;
    tot = compose(tot, s_warp[w]);
  }

  const bool need_lookback = (s_first_head == 0) && (ticket > 0);
  Pfx te = pfx_empty();
  if (warp == 0) {
    if (lane == 0) {
      const bool inclusive = (tot.f & kHead) || !need_lookback;
      publish(st, ticket, inclusive ? kStatusInclusive : kStatusAggregate, tot.a, tot.b);
    }
    if (need_lookback) {
      bool timed_out = false;
      te = lookback_warp<kLookbackPerLane>(st, ticket, lane, &timed_out);
      if (timed_out && lane == 0) report(ASCAN_DEV_ERR_LOOKBACK, ticket, err_host);
      if (lane == 0) {
        if (!(tot.f & kHead)) {
          const Pfx inc = compose(te, tot);
          publish(st, ticket, kStatusInclusive, inc.a, inc.b);
        }
        s_te = te;
      }
    }
  }
  if (need_lookback) {
    __syncthreads();
    te = s_te;
  }
  return compose(te, wex);
}

// Per-row inputs and outputs of a time slab: the launch covers columns
// [t0, t1) of every row of a longer sequence axis, and the rest of each row
// lives elsewhere (another GPU).  All pointers are nullable; only the
// persistent TMA kernels take them.
//   carry: forward: [C][2] = (gate product, state) carried into each row's
//          first element in scan order; backward: [C] = additive term for the
//          adjoint at that element (its successor gate times successor adjoint)
//   halo:  backward: [C] = state neighbour of the row element whose neighbour
//          lies outside the slab (h[t0-1] causal, h[t1] anti-causal)
//   agg:   [C][2] = inclusive (gate product, value) at each row's last element
//          in scan order
struct RowIO {
  const float* carry;
  const float* halo;
  float* agg;
};

template <typename T, typename IdxT>
struct FwdArgs {
  const T* g;
  const T* x;
  T* y;     // nullable with RowIO.agg: aggregate-only pass
  T* gout;
  const IdxT* cu;
  int64_t S, BL, N;
  uint32_t num_tiles;
  uint32_t* ticket;
  TileStatus st;
  RowIO io;
};

// Row position of flat index p.
__device__ __forceinline__ int64_t row_pos(int64_t p, int64_t BL, bool small) {
  return small ? static_cast<int64_t>(static_cast<uint32_t>(p) % static_cast<uint32_t>(BL))
               : p % BL;
}

template <typename T, typename IdxT, int VEC, bool REV, bool GATES_OUT>
__global__ void __launch_bounds__(kThreads) scan_fwd_kernel(const FwdArgs<T, IdxT> args,
                                                            uint32_t* err_host) {
  constexpr int R = kElemsPerThread / VEC;
  constexpr int kRowElems = 32 * VEC;
  constexpr int kWarpElems = R * kRowElems;
  __shared__ uint32_t s_ticket;

  if (threadIdx.x == 0) s_ticket = atomicAdd(args.ticket, 1u);
  __syncthreads();
  const uint32_t ticket = s_ticket;
  const uint32_t tile = REV ? args.num_tiles - 1u - ticket : ticket;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t N = args.N, BL = args.BL, S = args.S;
  const int64_t wbase = static_cast<int64_t>(tile) * kTile + static_cast<int64_t>(warp) * kWarpElems;

  float ga[R][VEC], xb[R][VEC];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int64_t p = wbase + r * kRowElems + lane * VEC;
    load_vec<T, VEC>(args.g, p, N, 1.f, ga[r]);
    load_vec<T, VEC>(args.x, p, N, 0.f, xb[r]);
  }
  if (ticket == 0) validate_cu(args.cu, S, BL, err_host);

  // Sequence boundaries of every element this lane owns.
  unsigned head[R], wmask[R];
  {
    const bool small = (N + kTile) <= 0xffffffffll;
    int64_t t = row_pos(wbase + lane * VEC, BL, small);
    Cursor cur;
    cursor_seek(cur, args.cu, S, BL, t);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      unsigned sm, em;
      vec_bounds<IdxT, VEC>(cur, t, wbase + r * kRowElems + lane * VEC, N, args.cu, S, BL, sm, em,
                            wmask[r]);
      head[r] = REV ? em : sm;
      if (r + 1 < R) cursor_step(cur, t, kRowElems, args.cu, S, BL);
    }
  }

  // Lane, row and warp prefixes within the tile.
  Pfx vpre[R];
  Pfx carry = pfx_empty();
#pragma unroll
  for (int rr = 0; rr < R; ++rr) {
    const int r = REV ? R - 1 - rr : rr;
    Pfx ex, tot;
    warp_scan<REV>(vec_aggregate<VEC, REV>(ga[r], xb[r], head[r]), lane, ex, tot);
    vpre[r] = compose(carry, ex);
    carry = compose(carry, tot);
  }
  const bool first_is_head = (head[REV ? R - 1 : 0] >> (REV ? VEC - 1 : 0)) & 1u;
  const Pfx wpre = tile_prefix<REV>(carry, first_is_head, ticket, args.st, warp, lane, err_host);

  // Final recurrence from the exact carry-in of each vector.
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const Pfx P = compose(wpre, vpre[r]);
    float h = P.b, a = P.a;
    float yo[VEC], go[VEC];
#pragma unroll
    for (int jj = 0; jj < VEC; ++jj) {
      const int j = REV ? VEC - 1 - jj : jj;
      if ((head[r] >> j) & 1u) {
        h = xb[r][j];
        a = ga[r][j];
      } else {
        h = fmaf(ga[r][j], h, xb[r][j]);
        a = a * ga[r][j];
      }
      yo[j] = h;
      go[j] = a;
    }
    const int64_t p = wbase + r * kRowElems + lane * VEC;
    store_vec<T, VEC>(args.y, p, wmask[r], yo);
    if constexpr (GATES_OUT) store_vec<T, VEC>(args.gout, p, wmask[r], go);
  }
}

template <typename T, typename IdxT>
struct BwdArgs {
  const T* dy;
  const T* g;
  const T* h;
  T* dx;    // nullable together with dg: aggregate-only pass
  T* dg;
  const IdxT* cu;
  int64_t S, BL, N;
  uint32_t num_tiles;
  uint32_t* ticket;
  TileStatus st;
  RowIO io;
};

// Element physically after this lane's vector in row r (lane+1, or lane 0 of
// the next row, or the element after the warp's span for the last lane).
template <int R>
__device__ __forceinline__ void next_first(const float (&first)[R], float edge, int lane,
                                           float (&out)[R]) {
  float s[R];
#pragma unroll
  for (int r = 0; r < R; ++r) s[r] = __shfl_sync(kFull, first[r], (lane + 1) & 31);
#pragma unroll
  for (int r = 0; r < R; ++r) out[r] = (lane < 31) ? s[r] : (r + 1 < R ? s[r + 1] : edge);
}

// Element physically before this lane's vector in row r.
template <int R>
__device__ __forceinline__ void prev_last(const float (&last)[R], float edge, int lane,
                                          float (&out)[R]) {
  float s[R];
#pragma unroll
  for (int r = 0; r < R; ++r) s[r] = __shfl_sync(kFull, last[r], (lane + 31) & 31);
#pragma unroll
  for (int r = 0; r < R; ++r) out[r] = (lane > 0) ? s[r] : (r > 0 ? s[r - 1] : edge);
}

// CAUSAL: adjoint of the causal scan, dh[t] = dy[t] + g[t+1] dh[t+1] (scan
// runs right to left), dg[t] = dh[t] h[t-1].  !CAUSAL mirrors both shifts.
template <typename T, typename IdxT, int VEC, bool CAUSAL>
__global__ void __launch_bounds__(kThreads) scan_bwd_kernel(const BwdArgs<T, IdxT> args,
                                                            uint32_t* err_host) {
  constexpr bool REV = CAUSAL;
  constexpr int R = kElemsPerThread / VEC;
  constexpr int kRowElems = 32 * VEC;
  constexpr int kWarpElems = R * kRowElems;
  __shared__ uint32_t s_ticket;

  if (threadIdx.x == 0) s_ticket = atomicAdd(args.ticket, 1u);
  __syncthreads();
  const uint32_t ticket = s_ticket;
  const uint32_t tile = REV ? args.num_tiles - 1u - ticket : ticket;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t N = args.N, BL = args.BL, S = args.S;
  const int64_t wbase = static_cast<int64_t>(tile) * kTile + static_cast<int64_t>(warp) * kWarpElems;

  float dyv[R][VEC], gv[R][VEC], hv[R][VEC];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int64_t p = wbase + r * kRowElems + lane * VEC;
    load_vec<T, VEC>(args.dy, p, N, 0.f, dyv[r]);
    load_vec<T, VEC>(args.g, p, N, 1.f, gv[r]);
    load_vec<T, VEC>(args.h, p, N, 0.f, hv[r]);
  }
  // One scalar at each edge of the warp's span.
  float g_edge = 1.f, h_edge = 0.f;
  if (CAUSAL) {
    const int64_t pn = wbase + kWarpElems, pp = wbase - 1;
    if (lane == 31 && pn < N) g_edge = Cvt<T>::to(args.g[pn]);
    if (lane == 0 && pp >= 0) h_edge = Cvt<T>::to(args.h[pp]);
  } else {
    const int64_t pn = wbase + kWarpElems, pp = wbase - 1;
    if (lane == 0 && pp >= 0) g_edge = Cvt<T>::to(args.g[pp]);
    if (lane == 31 && pn < N) h_edge = Cvt<T>::to(args.h[pn]);
  }
  if (ticket == 0) validate_cu(args.cu, S, BL, err_host);

  unsigned smask[R], emask[R], wmask[R];
  {
    const bool small = (N + kTile) <= 0xffffffffll;
    int64_t t = row_pos(wbase + lane * VEC, BL, small);
    Cursor cur;
    cursor_seek(cur, args.cu, S, BL, t);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      vec_bounds<IdxT, VEC>(cur, t, wbase + r * kRowElems + lane * VEC, N, args.cu, S, BL,
                            smask[r], emask[r], wmask[r]);
      if (r + 1 < R) cursor_step(cur, t, kRowElems, args.cu, S, BL);
    }
  }

  // Shift gates towards the scan's source and states towards its sink, in
  // place: a[t] = g[t+1], hn[t] = h[t-1] (causal) or the mirror image.
  {
    float gfirst[R], glast[R], hfirst[R], hlast[R], nb_g[R], nb_h[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      gfirst[r] = gv[r][0];
      glast[r] = gv[r][VEC - 1];
      hfirst[r] = hv[r][0];
      hlast[r] = hv[r][VEC - 1];
    }
    if (CAUSAL) {
      next_first<R>(gfirst, g_edge, lane, nb_g);
      prev_last<R>(hlast, h_edge, lane, nb_h);
#pragma unroll
      for (int r = 0; r < R; ++r) {
#pragma unroll
        for (int j = 0; j < VEC - 1; ++j) gv[r][j] = gv[r][j + 1];
        gv[r][VEC - 1] = nb_g[r];
#pragma unroll
        for (int j = VEC - 1; j > 0; --j) hv[r][j] = hv[r][j - 1];
        hv[r][0] = nb_h[r];
      }
    } else {
      prev_last<R>(glast, g_edge, lane, nb_g);
      next_first<R>(hfirst, h_edge, lane, nb_h);
#pragma unroll
      for (int r = 0; r < R; ++r) {
#pragma unroll
        for (int j = VEC - 1; j > 0; --j) gv[r][j] = gv[r][j - 1];
        gv[r][0] = nb_g[r];
#pragma unroll
        for (int j = 0; j < VEC - 1; ++j) hv[r][j] = hv[r][j + 1];
        hv[r][VEC - 1] = nb_h[r];
      }
    }
  }

  unsigned head[R], tail[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    head[r] = CAUSAL ? emask[r] : smask[r];
    tail[r] = CAUSAL ? smask[r] : emask[r];
  }

  Pfx vpre[R];
  Pfx carry = pfx_empty();
#pragma unroll
  for (int rr = 0; rr < R; ++rr) {
    const int r = REV ? R - 1 - rr : rr;
    Pfx ex, tot;
    warp_scan<REV>(vec_aggregate<VEC, REV>(gv[r], dyv[r], head[r]), lane, ex, tot);
    vpre[r] = compose(carry, ex);
    carry = compose(carry, tot);
  }
  const bool first_is_head = (head[REV ? R - 1 : 0] >> (REV ? VEC - 1 : 0)) & 1u;
  const Pfx wpre = tile_prefix<REV>(carry, first_is_head, ticket, args.st, warp, lane, err_host);

#pragma unroll
  for (int r = 0; r < R; ++r) {
    const Pfx P = compose(wpre, vpre[r]);
    float d = P.b;
    float dxo[VEC], dgo[VEC];
#pragma unroll
    for (int jj = 0; jj < VEC; ++jj) {
      const int j = REV ? VEC - 1 - jj : jj;
      d = ((head[r] >> j) & 1u) ? dyv[r][j] : fmaf(gv[r][j], d, dyv[r][j]);
      dxo[j] = d;
      dgo[j] = ((tail[r] >> j) & 1u) ? 0.f : d * hv[r][j];
    }
    const int64_t p = wbase + r * kRowElems + lane * VEC;
    store_vec<T, VEC>(args.dx, p, wmask[r], dxo);
    store_vec<T, VEC>(args.dg, p, wmask[r], dgo);
  }
}

}  // namespace ascan

#include "ascan_slab.cuh"
#include "ascan_tma.cuh"

namespace ascan {

// ---------------------------------------------------------------------------
// Persistent TMA kernels (see ascan_tma.cuh for the pipeline)
// ---------------------------------------------------------------------------

// Stages of the input ring: the deepest ring (at most 6) that fits next to the
// output staging buffers in the 227 KB of shared memory a CTA may use.
// Shared memory of one persistent CTA: the SM's 228 KB shared by kCtasPerSm
// CTAs, 1 KB of each reserved by the hardware.
constexpr size_t kSmemBudget = (228 * 1024) / tma::kCtasPerSm - 1024;

template <typename T, int NIN, int NOUT, int P, bool RG, int NS = 6>
constexpr int ring_depth() {
  if constexpr (NS <= 2)
    return 2;
  else if constexpr (tma::smem_bytes<NIN, NOUT, NS, T, P, RG>() <= kSmemBudget)
    return NS;
  else
    return ring_depth<T, NIN, NOUT, P, RG, NS - 1>();
}

// Whether the kernels that stage their outputs for TMA stores fit with a
// two-stage ring; when they do not (large tiles), the register-store (RG)
// kernels serve every schedule.
template <typename T, int NIN, int NOUT, int P>
constexpr bool staged_fits() {
  return tma::smem_bytes<NIN, NOUT, 2, T, P, false>() <= kSmemBudget;
}

// Producer warp of both kernels: TMA loads and per-tile metadata.  Tickets
// are dealt round-robin in scan order (CTA b takes tickets b, b+G, b+2G, ...,
// G = the launch's CTAs for this scan) and the launch is cooperative, so every CTA is resident and
// the CTAs move through the tickets in waves: a tile's predecessor is in the
// same or an earlier wave.  In row mode the producer also copies the status
// slot of the tile's predecessor (many waves older when rows >> CTAs) into the
// stage metadata with an asynchronous bulk copy, so the consumers usually find
// the carry-in there instead of polling global memory, and the producer never
// waits for that read.
// `Extra` fills the halo scalars and the ragged tail of one stage.
// RG (ragged rows): tiles start anywhere inside a 128-byte TMA row; the box is
// one TMA row taller and the tile's offset into it travels in the metadata.
template <typename T, typename IdxT, bool REV, int NIN, int NOUT, int NS, int P, bool RG,
          typename Extra>
__device__ __forceinline__ void run_producer(tma::Smem<NIN, NOUT, NS, T, P, RG>& sm,
                                             const CUtensorMap* const* maps,
                                             const tma::CuView<IdxT>& cu, int64_t N,
                                             int64_t n_tma_total, const tma::TileSched& sch,
                                             const TileStatus& st, int lane, uint32_t* err_host,
                                             Extra extra, int n_load = NIN) {
  using namespace tma;
  constexpr int kTileElems = Geo<P>::kTileElems;
  using F = Fmt<T, P>;
  if (lane == 0)
    for (int k = 0; k < NIN; ++k) prefetch_map(maps[k]);
  uint32_t stage = 0, phase = 0;
  // pending[s]: the last use of stage s was a TMA load that the consumers have
  // not been seen to release yet; last_parity[s]: the full-barrier phase of it.
  bool pending[NS];
  uint32_t last_parity[NS];
#pragma unroll
  for (int s = 0; s < NS; ++s) pending[s] = false, last_parity[s] = 0;
  const int64_t BL = cu.BL;
  // this launch's CTAs for this scan: all of them, or one group of a
  // bidirectional launch (CTAs [cta0, cta0 + ctas))
  const uint32_t G = sch.ctas ? sch.ctas : gridDim.x;
  const uint32_t num_tiles = sch.num_tiles;
  // flat mode: row position of the current tile's first element, advanced by
  // the (constant) distance between this CTA's consecutive tiles
  // (and its row, advanced the same way: no division per tile)
  const int64_t step = (static_cast<int64_t>(G) * kTileElems) % BL;
  const int64_t row_step = (static_cast<int64_t>(G) * kTileElems) / BL;
  uint32_t ticket = blockIdx.x - sch.cta0;
  int64_t t_flat = 0, r_flat = 0;
  if (!sch.row_mode && ticket < num_tiles) {
    const uint32_t tile0 = REV ? num_tiles - 1u - ticket : ticket;
    t_flat = (static_cast<int64_t>(tile0) * kTileElems) % BL;
    r_flat = (static_cast<int64_t>(tile0) * kTileElems) / BL;
  }
  uint32_t abort_seen = 0u;
  uint32_t iter = 0u;
  while (true) {
    if (ticket >= num_tiles || abort_seen) ticket = kDone;
    // Stop early when the launch was aborted: the CTA's own word every tile
    // (shared memory), the launch-wide word every 16th tile -- a global load
    // on every tile would put an L2 round trip on the producer's path.
    uint32_t abort_next = 0u;
    if (lane == 0 && ticket != kDone) {
      abort_next = static_cast<uint32_t>(*reinterpret_cast<volatile int*>(&sm.abort));
      if ((iter & 15u) == 15u) abort_next |= ld_volatile_u32(st.abort);
    }
    ++iter;
    if (!mbar_wait_warp(&sm.empty[stage], phase ^ 1u)) {
      if (lane == 0) {
        report(ASCAN_DEV_ERR_LOOKBACK, 0xfffffffeull, err_host);
        set_aborted(st);
      }
      break;
    }
    pending[stage] = false;  // its previous load was consumed and released
    StageMeta<NIN, T, P>& m = sm.meta[stage];
    if (ticket == kDone) {
      if (lane == 0) {
        m.ticket = kDone;
        mbar_arrive(&sm.full[stage]);
      }
      break;
    }
    int64_t p0, t0, limit, row0;
    if (sch.row_mode) {
      // stride = rows * segs: the (row, segment) pairs of one tile column
      const uint32_t j = ticket / sch.stride;
      const uint32_t v = ticket - j * sch.stride;
      const uint32_t c = v / sch.segs;
      const uint32_t seg = v - c * sch.segs;
      const uint32_t per_seg = sch.tiles_per_row / sch.segs;
      const uint32_t jj = seg * per_seg + (REV ? per_seg - 1u - j : j);
      t0 = static_cast<int64_t>(jj) * kTileElems;
      p0 = static_cast<int64_t>(c) * BL + t0;
      limit = static_cast<int64_t>(c) * BL + BL;
      row0 = c;
    } else {
      const uint32_t tile = REV ? num_tiles - 1u - ticket : ticket;
      p0 = static_cast<int64_t>(tile) * kTileElems;
      t0 = t_flat;
      limit = N;
      row0 = r_flat;
    }
    const int row = static_cast<int>(p0 / F::kElemsPerRow);
    constexpr uint32_t kBoxBytes = (F::kRows + (RG ? 1 : 0)) * 128u;
    const bool read_pred = sch.row_mode && ticket >= sch.stride;
    if (lane == 0) {
      m.ticket = ticket;
      if constexpr (RG)
        m.shift = static_cast<uint32_t>(p0 - static_cast<int64_t>(row) * F::kElemsPerRow);
      if (!read_pred) m.te_raw[1] = m.te_raw[3] = kStatusNone;
      // the first n_load inputs (an aggregate-only backward skips the states)
      mbar_expect_tx(&sm.full[stage], n_load * kBoxBytes + (read_pred ? 16u : 0u));
      for (int k = 0; k < n_load; ++k) tma_load_2d(sm.in[stage][k], maps[k], 0, row, &sm.full[stage]);
      if (read_pred) bulk_load(m.te_raw, st.slots + (ticket - sch.stride), 16u, &sm.full[stage]);
    }
    pending[stage] = true;
    last_parity[stage] = phase;
    build_meta<IdxT, NIN, T, P>(m, cu, p0, t0, row0, limit, n_tma_total, lane);
    const int64_t rem = limit - p0;
    const uint32_t n_valid = static_cast<uint32_t>(rem < kTileElems ? rem : kTileElems);
    int64_t nt = n_tma_total - p0;
    nt = nt < 0 ? 0 : (nt > n_valid ? n_valid : nt);
    extra(m, p0, static_cast<uint32_t>(nt), n_valid, lane, &sm.full[stage]);
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.full[stage]);
    if (++stage == NS) {
      stage = 0;
      phase ^= 1u;
    }
    ticket += G;
    if (REV) {
      t_flat -= step;
      r_flat -= row_step;
      if (t_flat < 0) t_flat += BL, --r_flat;
    } else {
      t_flat += step;
      r_flat += row_step;
      if (t_flat >= BL) t_flat -= BL, ++r_flat;
    }
    abort_seen = __shfl_sync(kFull, abort_next, 0);
  }
  // Never leave the CTA while a TMA load may still be writing shared memory:
  // wait for every load whose stage was not released afterwards (its full
  // barrier is still in the phase that load armed).
#pragma unroll
  for (int s = 0; s < NS; ++s)
    if (pending[s]) mbar_wait_warp(&sm.full[s], last_parity[s]);  // pending is warp-uniform
}

// IO: the launch serves a time slab (RowIO in use or no outputs); compiled
// separately so the ordinary kernels carry none of that code.
// The CTA's part of one forward launch; the tensor maps are kernel
// parameters (__grid_constant__), passed by address.
template <typename T, typename IdxT, bool REV, bool GATES_OUT, int NS, bool IO, int P, bool RG>
__device__ __forceinline__ void fwd_tma_body(const CUtensorMap* map_g, const CUtensorMap* map_x,
                                             const CUtensorMap* map_y,
                                             const CUtensorMap* map_gout,
                                             const FwdArgs<T, IdxT>& args, int64_t n_tma_total,
                                             const tma::TileSched& sch_in, uint32_t* err_host) {
  using namespace tma;
  constexpr int kPerThread = P, kTileElems = Geo<P>::kTileElems, kBitWords = Geo<P>::kBitWords;
  constexpr uint32_t kThreadMask = Geo<P>::kMask;
  using F = Fmt<T, P>;
  constexpr int NIN = 2, NOUT = GATES_OUT ? 2 : 1;
  using Sm = Smem<NIN, NOUT, NS, T, P, RG>;
  Sm& sm = smem_view<Sm>();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t S = args.S, BL = args.BL, N = args.N;

  const bool cache_cu = (S + 1) <= kCuCache;
  // segment mode needs cu_seqlens[i] == i * BL / segs: each thread checks the
  // entries it caches, the start-up barrier takes the vote (time-slab
  // launches never take it)
  bool seg_ok = !IO && sch_in.segs > 1u && cache_cu;
  const int64_t seg_len = seg_ok ? BL / sch_in.segs : 0;
  if (cache_cu)
    for (int64_t i = tid; i <= S; i += tma::kThreads) {
      const int64_t v = cu_at(args.cu, i, BL);
      sm.cu[i] = v;
      seg_ok = seg_ok && v == i * seg_len;
    }
  if (tid < kXsRing * (kConsumerWarps + 1)) {
    float4* f = &sm.xs[0].warp[0] + tid;
    f->w = __uint_as_float(kNoTag);
  }
  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kConsumerWarps);
    }
    sm.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  const tma::TileSched sch = tma::seg_sched(sch_in, __syncthreads_and(seg_ok) != 0);
  const CuView<IdxT> cu{args.cu, cache_cu ? sm.cu : nullptr, S, BL};

  if (warp == kConsumerWarps) {
    const CUtensorMap* maps[NIN] = {map_g, map_x};
    run_producer<T, IdxT, REV, NIN, NOUT, NS, P, RG>(
        sm, maps, cu, N, n_tma_total, sch, args.st, lane, err_host,
        [&](StageMeta<NIN, T, P>& m, int64_t p0, uint32_t n_tma, uint32_t n_valid, int ln,
            uint64_t* bar) {
          for (uint32_t e = n_tma + ln; e < n_valid; e += 32) {
            m.tail[0][e - n_tma] = Cvt<T>::to(args.g[p0 + e]);
            m.tail[1][e - n_tma] = Cvt<T>::to(args.x[p0 + e]);
          }
          // time slabs: a row carry (gate product, state) that enters at the
          // tile's first element in scan order becomes the tile's known
          // carry-in -- the element stops being a head and the carry composes
          // onto it exactly as the slab kernels' row carry does -- so the
          // plain kernels serve seeded passes over rows of whole tiles
          if (args.io.carry != nullptr) {
            __syncwarp();  // every lane's boundary bits are in place
            if (ln == 0) {
              // (reverse order: only a full tile's last element is its first
              // in scan order; a partial tile stays with the consumers)
              const uint32_t e = REV ? n_valid - 1u : 0u;
              int64_t pos = m.t0 + e, q = 0;
              if (pos >= BL) q = pos / BL, pos -= q * BL;  // a tile that crosses a row end
              uint32_t& w = REV ? m.ebits[e >> 5] : m.sbits[e >> 5];
              if (pos == (REV ? BL - 1 : 0) && ((w >> (e & 31u)) & 1u) &&
                  (!REV || n_valid == static_cast<uint32_t>(kTileElems))) {
                const int64_t r = m.row0 + q;
                // the (product, state) pair comes with the tile when one
                // 16-byte block holds it (the producer never waits on a load)
                m.io_te = fetch_block(m.io_raw[0], args.io.carry, 2 * (N / BL), 2 * r, 2, bar);
                if (m.io_te == 0u) {
                  m.te_raw[0] = __float_as_uint(args.io.carry[2 * r]);
                  m.te_raw[2] = __float_as_uint(args.io.carry[2 * r + 1]);
                }
                m.te_raw[1] = m.te_raw[3] = kStatusInclusive;
                w &= ~(1u << (e & 31u));
              }
            }
          }
        });
    return;
  }

  if (blockIdx.x == sch.cta0) validate_cu(args.cu, S, BL, err_host);
  const uint32_t o = static_cast<uint32_t>(tid) * kPerThread;
  const ThreadChunks<T, P> tc(o);
  const uint32_t bit_word = o >> 5, bit_shift = o & 31u;
  constexpr int kPartRows = F::kRows / kConsumerWarps;    // this warp's slice of a tile
  constexpr int kPartBytes = F::kBytes / kConsumerWarps;
  uint32_t stage = 0, phase = 0, obuf = 0, xi = 0;
  bool ok = true;
  while (true) {
    // Every exit is decided by one warp-wide vote: this warp's own status,
    // the stage's arrival and the CTA's abort word.
    bool go = ok && mbar_wait_warp(&sm.full[stage], phase);  // ok is warp-uniform
    go = __all_sync(kFull, go && *reinterpret_cast<volatile int*>(&sm.abort) == 0);
    if (!go) {
      ok = false;
      break;
    }
    const StageMeta<NIN, T, P>& m = sm.meta[stage];
    const uint32_t ticket = m.ticket;
    if (ticket == kDone) break;
    const int64_t p0 = m.p0;
    const uint32_t n_valid = m.n_valid, n_tma = m.n_tma;
    const bool has_outside = m.has_outside != 0u;
    float a[kPerThread], b[kPerThread];
    if constexpr (RG) {
      const uint32_t shift = m.shift;
      read_block_shifted<T, NIN>(sm.in[stage][0], m, 0, o, shift, n_tma, n_valid, 1.f, a);
      read_block_shifted<T, NIN>(sm.in[stage][1], m, 1, o, shift, n_tma, n_valid, 0.f, b);
    } else {
      read_block<T, NIN>(sm.in[stage][0], tc, m, 0, o, n_tma, n_valid, 1.f, a);
      read_block<T, NIN>(sm.in[stage][1], tc, m, 1, o, n_tma, n_valid, 0.f, b);
    }
    const uint32_t head =
        ((REV ? m.ebits[bit_word] : m.sbits[bit_word]) >> bit_shift) & kThreadMask;
    const uint32_t omask = has_outside ? (m.obits[bit_word] >> bit_shift) & kThreadMask : 0u;
    const bool first_is_head =
        REV ? ((m.ebits[kBitWords - 1] >> 31) & 1u) != 0u : (m.sbits[0] & 1u) != 0u;
    bool te_known = m.te_raw[1] == kStatusInclusive && m.te_raw[3] == kStatusInclusive;
    Pfx te_meta{__uint_as_float(m.te_raw[0]), __uint_as_float(m.te_raw[2]), kValid};
    if (m.io_te != 0u)  // a time slab's row carry, fetched with the tile
      te_meta = Pfx{m.io_raw[0][m.io_te - 1u], m.io_raw[0][m.io_te], kValid};
    // the scan-first warp re-reads its predecessor now, while it folds the tile
    const bool early = (REV ? kConsumerWarps - 1 - warp : warp) == 0 && !te_known &&
                       !first_is_head && ticket >= sch.stride;
    uint4 early_raw = make_uint4(0u, 0u, 0u, 0u);
    if (early && lane == 0) early_raw = load_status_raw(args.st, ticket - sch.stride);
    // time slabs: row ends in scan order, where the row aggregate is taken
    const uint32_t lastmask =
        IO && args.io.agg ? ((REV ? m.sbits[bit_word] : m.ebits[bit_word]) >> bit_shift) & kThreadMask
                          : 0u;
    // time slabs: the row carry enters at the row's first element in scan
    // order (read while the stage's metadata is still held: no register
    // carries the tile's row through the scan)
    if (IO && args.io.carry != nullptr && head != 0u)
      apply_row_carry<REV>(a, b, head, RowPos(m.row0, m.t0 + o, BL), BL, args.io.carry);
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[stage]);
    if (++stage == NS) {
      stage = 0;
      phase ^= 1u;
    }

    Pfx ex, wtot;
    warp_scan<REV>(fold16_inplace<REV>(a, b, head), lane, ex, wtot);
    if (early) take_early(early_raw, te_known, te_meta);
    const Pfx Pc = warp_tile_prefix<REV>(sm, xi, ex, wtot, first_is_head, ticket, args.st,
                                        sch.stride, te_known, te_meta, warp, lane, ok,
                                        err_host);
    // a, b hold the local prefixes: h = A_loc * carry + B_loc before the first head
    const uint32_t cm = carry_mask<REV, P>(head);
    if (IO && lastmask != 0u)
      record_row_agg<REV>(a, b, lastmask, cm, Pc, RowPos(p0 + o, BL), BL, args.io.agg);
    if (__all_sync(kFull, cm == kThreadMask)) {  // warp-uniform: no lane holds a head
#pragma unroll
      for (int j = 0; j < kPerThread; ++j) {
        b[j] = fmaf(a[j], Pc.b, b[j]);
        if constexpr (GATES_OUT) a[j] *= Pc.a;
      }
    } else {
#pragma unroll
      for (int j = 0; j < kPerThread; ++j) {
        const bool c = (cm >> j) & 1u;
        b[j] = c ? fmaf(a[j], Pc.b, b[j]) : b[j];
        if constexpr (GATES_OUT) a[j] = c ? a[j] * Pc.a : a[j];
      }
    }
    const bool store = !IO || args.y != nullptr;  // false: aggregate-only pass
    const uint32_t valid = below_mask<P>(o, n_valid) & ~omask;
    uint32_t direct = store ? valid : 0u;
    if (lane == 0) bulk_wait_read<1>();  // this warp's slice of staging buffer obuf is free
    __syncwarp();
    // this warp's slice goes out by TMA when it lies wholly inside the tile's
    // TMA-covered part (never past a row end or the array end)
    const bool slice_tma =
        !RG && store && !has_outside && (warp + 1) * (kTileElems / kConsumerWarps) <= n_tma;
    if constexpr (RG) {
      if (__all_sync(kFull, direct == kThreadMask)) {
        // ragged rows: a wholly valid warp slice leaves by realigned 16-byte stores
        const uint32_t r = static_cast<uint32_t>(p0 % ThreadChunks<T, P>::kVec);
        store_realigned<T>(args.y, p0 + o, r, b, lane, warp_stage(sm, 0, warp));
        if constexpr (GATES_OUT)
          store_realigned<T>(args.gout, p0 + o, r, a, lane, warp_stage(sm, 1, warp));
        direct = 0u;
      }
    }
    if (slice_tma) {
      write_block<T>(sm.out[obuf][0], tc, b);
      if constexpr (GATES_OUT) write_block<T>(sm.out[obuf][1], tc, a);
      direct = 0u;
    }
    if (direct) {
      store_direct<T>(args.y, p0 + o, direct, b);
      if constexpr (GATES_OUT) store_direct<T>(args.gout, p0 + o, direct, a);
    }
    fence_async_smem();
    __syncwarp();
    if (lane == 0) {
      if (slice_tma) {
        const int row = static_cast<int>(p0 / F::kElemsPerRow) + warp * kPartRows;
        tma_store_2d(map_y, 0, row, sm.out[obuf][0] + warp * kPartBytes);
        if constexpr (GATES_OUT) tma_store_2d(map_gout, 0, row, sm.out[obuf][1] + warp * kPartBytes);
      }
      bulk_commit();
    }
    obuf ^= 1u;
    if (++xi == kXsRing) xi = 0;
  }
  if (!ok && lane == 0) {
    *reinterpret_cast<volatile int*>(&sm.abort) = 1;
    report(ASCAN_DEV_ERR_LOOKBACK, 0xfffffffdull, err_host);
    set_aborted(args.st);
  }
  if (lane == 0) bulk_wait_all();
}

// The CTA's part of one backward launch (tensor maps passed by address, as
// in fwd_tma_body).
template <typename T, typename IdxT, bool CAUSAL, int NS, bool IO, int P, bool RG>
__device__ __forceinline__ void bwd_tma_body(const CUtensorMap* map_dy, const CUtensorMap* map_g,
                                             const CUtensorMap* map_h, const CUtensorMap* map_dx,
                                             const CUtensorMap* map_dg,
                                             const BwdArgs<T, IdxT>& args, int64_t n_tma_total,
                                             const tma::TileSched& sch_in, uint32_t* err_host) {
  using namespace tma;
  constexpr int kPerThread = P, kTileElems = Geo<P>::kTileElems, kBitWords = Geo<P>::kBitWords;
  constexpr uint32_t kThreadMask = Geo<P>::kMask;
  using F = Fmt<T, P>;
  constexpr bool REV = CAUSAL;
  constexpr int NIN = 3, NOUT = 2;
  constexpr bool kPackH = sizeof(T) == 2 && !RG && !IO;
  using Sm = Smem<NIN, NOUT, NS, T, P, RG>;
  Sm& sm = smem_view<Sm>();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t S = args.S, BL = args.BL, N = args.N;

  const bool cache_cu = (S + 1) <= kCuCache;
  // segment mode needs cu_seqlens[i] == i * BL / segs: each thread checks the
  // entries it caches, the start-up barrier takes the vote (time-slab
  // launches never take it)
  bool seg_ok = !IO && sch_in.segs > 1u && cache_cu;
  const int64_t seg_len = seg_ok ? BL / sch_in.segs : 0;
  if (cache_cu)
    for (int64_t i = tid; i <= S; i += tma::kThreads) {
      const int64_t v = cu_at(args.cu, i, BL);
      sm.cu[i] = v;
      seg_ok = seg_ok && v == i * seg_len;
    }
  if (tid < kXsRing * (kConsumerWarps + 1)) {
    float4* f = &sm.xs[0].warp[0] + tid;
    f->w = __uint_as_float(kNoTag);
  }
  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kConsumerWarps);
    }
    sm.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  const tma::TileSched sch = tma::seg_sched(sch_in, __syncthreads_and(seg_ok) != 0);
  const CuView<IdxT> cu{args.cu, cache_cu ? sm.cu : nullptr, S, BL};

  if (warp == kConsumerWarps) {
    const CUtensorMap* maps[NIN] = {map_dy, map_g, map_h};
    run_producer<T, IdxT, REV, NIN, NOUT, NS, P, RG>(
        sm, maps, cu, N, n_tma_total, sch, args.st, lane, err_host,
        [&](StageMeta<NIN, T, P>& m, int64_t p0, uint32_t n_tma, uint32_t n_valid, int ln,
            uint64_t* bar) {
          for (uint32_t e = n_tma + ln; e < n_valid; e += 32) {
            m.tail[0][e - n_tma] = Cvt<T>::to(args.dy[p0 + e]);
            m.tail[1][e - n_tma] = Cvt<T>::to(args.g[p0 + e]);
            m.tail[2][e - n_tma] = Cvt<T>::to(args.h[p0 + e]);
          }
          if (ln == 0) {
            // The element after the tile (gate for the causal adjoint, state
            // otherwise) and the one before it (the other array) come by
            // 16-byte bulk copies, so the producer never waits for them: tile
            // starts are 16-byte aligned, and so are the blocks [pn, pn+V) and
            // [p0-V, p0).  A next block that would reach past the array end
            // is read directly (the array's last tile only).
            // Ragged rows (RG): tiles start anywhere, so the copies fetch the
            // aligned 16-byte blocks holding the neighbours, and the index of
            // the neighbour inside its block travels in the metadata.
            constexpr int V = 16 / static_cast<int>(sizeof(T));
            const int64_t pn = p0 + kTileElems;
            const int kn = CAUSAL ? 0 : 1, kp = CAUSAL ? 1 : 0;  // halo slots
            const T* const arr[2] = {args.g, args.h};
            const float ident[2] = {1.f, 0.f};
            uint32_t bulk = 0u;
            int64_t bn = pn, bp = p0 - V;  // the two blocks' first elements
            if constexpr (RG) {
              bn = pn - pn % V;
              bp = p0 > 0 ? (p0 - 1) - (p0 - 1) % V : 0;
            }
            if (bn + V <= N) {
              bulk |= 1u << kn;
              if constexpr (RG) m.halo_idx[kn] = static_cast<uint32_t>(pn - bn);
            } else {
              m.halo[kn] = pn < N ? Cvt<T>::to(arr[kn][pn]) : ident[kn];
            }
            // never a block that reaches past the array end
            if (RG ? (p0 > 0 && bp + V <= N) : p0 >= V) {
              bulk |= 1u << kp;
              if constexpr (RG) m.halo_idx[kp] = static_cast<uint32_t>(p0 - 1 - bp);
            } else {
              m.halo[kp] = p0 > 0 ? Cvt<T>::to(arr[kp][p0 - 1]) : ident[kp];
            }
            m.halo_bulk = bulk;
            if (bulk) mbar_expect_tx(bar, 16u * static_cast<uint32_t>(__popc(bulk)));
            if (bulk & (1u << kn)) bulk_load(m.halo_raw[kn], arr[kn] + bn, 16u, bar);
            if (bulk & (1u << kp)) bulk_load(m.halo_raw[kp], arr[kp] + bp, 16u, bar);
          }
          // time slabs: the row's carried adjoint term at the tile's first
          // element in scan order becomes the tile's known carry-in (1, c)
          // with that element's outside coefficient the identity; the row's
          // state halo becomes the tile-edge state neighbour, and its element
          // stops counting as a sequence start for the gate gradient.  (Only
          // where that element sits on the tile's edge: always for rows of
          // whole tiles, whose launches run the plain kernels; in the slab
          // kernels the consumers handle the other tiles.)
          if (args.io.carry != nullptr || args.io.halo != nullptr) {
            __syncwarp();  // every lane's boundary bits are in place
            if (ln == 0) {
              if (args.io.carry != nullptr) {
                // (causal: only a full tile's last element is its first in
                // scan order; a partial tile stays with the consumers)
                const uint32_t e = CAUSAL ? n_valid - 1u : 0u;
                int64_t pos = m.t0 + e, q = 0;
                if (pos >= BL) q = pos / BL, pos -= q * BL;  // a tile that crosses a row end
                uint32_t& w = CAUSAL ? m.ebits[e >> 5] : m.sbits[e >> 5];
                if (pos == (CAUSAL ? BL - 1 : 0) && ((w >> (e & 31u)) & 1u) &&
                    (!CAUSAL || n_valid == static_cast<uint32_t>(kTileElems))) {
                  m.io_te = fetch_block(m.io_raw[0], args.io.carry, N / BL, m.row0 + q, 1, bar);
                  m.te_raw[0] = __float_as_uint(1.f);
                  if (m.io_te == 0u) m.te_raw[2] = __float_as_uint(args.io.carry[m.row0 + q]);
                  m.te_raw[1] = m.te_raw[3] = kStatusInclusive;
                  m.halo[0] = 1.f;  // the outside successor gate (already in c)
                  m.halo_bulk &= ~1u;
                  w &= ~(1u << (e & 31u));
                }
              }
              // (not when the row aggregate is written: the slab kernels find
              // the row's last element in scan order by this same boundary
              // bit, so their consumers apply the halo themselves)
              if (args.io.halo != nullptr && args.io.agg == nullptr) {
                const uint32_t e = CAUSAL ? 0u : n_valid - 1u;
                int64_t pos = m.t0 + e, q = 0;
                if (pos >= BL) q = pos / BL, pos -= q * BL;  // a tile that crosses a row end
                uint32_t& w = CAUSAL ? m.sbits[e >> 5] : m.ebits[e >> 5];
                // (anti-causal: the neighbour of a partial tile's last element
                // is not the tile-edge one, so that case stays with the consumers)
                if (pos == (CAUSAL ? 0 : BL - 1) && ((w >> (e & 31u)) & 1u) &&
                    (CAUSAL || n_valid == static_cast<uint32_t>(kTileElems))) {
                  m.io_halo = fetch_block(m.io_raw[1], args.io.halo, N / BL, m.row0 + q, 1, bar);
                  if (m.io_halo == 0u) m.halo[1] = args.io.halo[m.row0 + q];
                  m.halo_bulk &= ~2u;
                  w &= ~(1u << (e & 31u));
                }
              }
            }
          }
        },
        IO && args.dx == nullptr ? 2 : NIN);  // aggregate-only: the states are never read
    return;
  }

  if (blockIdx.x == sch.cta0) validate_cu(args.cu, S, BL, err_host);
  const uint32_t o = static_cast<uint32_t>(tid) * kPerThread;
  const ThreadChunks<T, P> tc(o);
  const uint32_t bit_word = o >> 5, bit_shift = o & 31u;
  constexpr int kPartRows = F::kRows / kConsumerWarps;    // this warp's slice of a tile
  constexpr int kPartBytes = F::kBytes / kConsumerWarps;
  uint32_t stage = 0, phase = 0, obuf = 0, xi = 0;
  bool ok = true;
  while (true) {
    // Every exit is decided by one warp-wide vote: this warp's own status,
    // the stage's arrival and the CTA's abort word.
    bool go = ok && mbar_wait_warp(&sm.full[stage], phase);  // ok is warp-uniform
    go = __all_sync(kFull, go && *reinterpret_cast<volatile int*>(&sm.abort) == 0);
    if (!go) {
      ok = false;
      break;
    }
    const StageMeta<NIN, T, P>& m = sm.meta[stage];
    const uint32_t ticket = m.ticket;
    if (ticket == kDone) break;
    const int64_t p0 = m.p0;
    const uint32_t n_valid = m.n_valid, n_tma = m.n_tma;
    const bool has_outside = m.has_outside != 0u;
    float dyv[kPerThread], gv[kPerThread];
    // 16-bit states stay packed (two per word) until the dg epilogue: half the
    // registers of floats through the scan and the carry
    float hv[kPackH ? 1 : kPerThread];
    uint32_t hw[kPackH ? kPerThread / 2 : 1];
    // ragged rows: the tile sits `shift` elements into its buffers
    const uint32_t shift = RG ? m.shift : 0u;
    if constexpr (RG) {
      read_block_shifted<T, NIN>(sm.in[stage][0], m, 0, o, shift, n_tma, n_valid, 0.f, dyv);
      read_block_shifted<T, NIN>(sm.in[stage][1], m, 1, o, shift, n_tma, n_valid, 1.f, gv);
      read_block_shifted<T, NIN>(sm.in[stage][2], m, 2, o, shift, n_tma, n_valid, 0.f, hv);
    } else {
      read_block<T, NIN>(sm.in[stage][0], tc, m, 0, o, n_tma, n_valid, 0.f, dyv);
      read_block<T, NIN>(sm.in[stage][1], tc, m, 1, o, n_tma, n_valid, 1.f, gv);
      if constexpr (kPackH)
        read_block_packed<T, NIN>(sm.in[stage][2], tc, m, 2, o, n_tma, n_valid, hw);
      else
        read_block<T, NIN>(sm.in[stage][2], tc, m, 2, o, n_tma, n_valid, 0.f, hv);
    }
    // neighbours across the thread boundary: from the tile, or the tile-edge halo
    constexpr int V = 16 / static_cast<int>(sizeof(T));
    float halo_g, halo_h;
    if constexpr (RG) {
      halo_g = (m.halo_bulk & 1u) ? Cvt<T>::to(m.halo_raw[0][m.halo_idx[0]]) : m.halo[0];
      halo_h = (m.halo_bulk & 2u) ? Cvt<T>::to(m.halo_raw[1][m.halo_idx[1]]) : m.halo[1];
    } else {  // aligned tiles: the neighbours sit at fixed places of their blocks
      halo_g = (m.halo_bulk & 1u) ? Cvt<T>::to(m.halo_raw[0][CAUSAL ? 0 : V - 1]) : m.halo[0];
      halo_h = m.io_halo != 0u      ? m.io_raw[1][m.io_halo - 1u]  // a time slab's row halo
               : (m.halo_bulk & 2u) ? Cvt<T>::to(m.halo_raw[1][CAUSAL ? V - 1 : 0])
                                    : m.halo[1];
    }
    float g_nb, h_nb;
    if (CAUSAL) {
      g_nb = (o + kPerThread < static_cast<uint32_t>(kTileElems))
                 ? tile_elem<T, NIN>(sm.in[stage][1], m, 1, o + kPerThread, n_tma, n_valid, 1.f,
                                     shift)
                 : halo_g;
      h_nb = (o > 0) ? tile_elem<T, NIN>(sm.in[stage][2], m, 2, o - 1, n_tma, n_valid, 0.f, shift)
                     : halo_h;
    } else {
      g_nb = (o > 0) ? tile_elem<T, NIN>(sm.in[stage][1], m, 1, o - 1, n_tma, n_valid, 1.f, shift)
                     : halo_g;
      h_nb = (o + kPerThread < static_cast<uint32_t>(kTileElems))
                 ? tile_elem<T, NIN>(sm.in[stage][2], m, 2, o + kPerThread, n_tma, n_valid, 0.f,
                                     shift)
                 : halo_h;
    }
    const uint32_t smask = (m.sbits[bit_word] >> bit_shift) & kThreadMask;
    const uint32_t emask = (m.ebits[bit_word] >> bit_shift) & kThreadMask;
    const uint32_t omask = has_outside ? (m.obits[bit_word] >> bit_shift) & kThreadMask : 0u;
    const bool first_is_head =
        REV ? ((m.ebits[kBitWords - 1] >> 31) & 1u) != 0u : (m.sbits[0] & 1u) != 0u;
    bool te_known = m.te_raw[1] == kStatusInclusive && m.te_raw[3] == kStatusInclusive;
    Pfx te_meta{__uint_as_float(m.te_raw[0]), __uint_as_float(m.te_raw[2]), kValid};
    if (m.io_te != 0u) te_meta.b = m.io_raw[0][m.io_te - 1u];  // a time slab's carried adjoint
    // the scan-first warp re-reads its predecessor now, while it folds the tile
    const bool early = (REV ? kConsumerWarps - 1 - warp : warp) == 0 && !te_known &&
                       !first_is_head && ticket >= sch.stride;
    uint4 early_raw = make_uint4(0u, 0u, 0u, 0u);
    if (early && lane == 0) early_raw = load_status_raw(args.st, ticket - sch.stride);

    // a[t] = g[t+1], hn[t] = h[t-1] (causal) or the mirror image (packed
    // states are shifted when they are unpacked)
    if (CAUSAL) {
#pragma unroll
      for (int j = 0; j < kPerThread - 1; ++j) gv[j] = gv[j + 1];
      gv[kPerThread - 1] = g_nb;
      if constexpr (!kPackH) {
#pragma unroll
        for (int j = kPerThread - 1; j > 0; --j) hv[j] = hv[j - 1];
        hv[0] = h_nb;
      }
    } else {
#pragma unroll
      for (int j = kPerThread - 1; j > 0; --j) gv[j] = gv[j - 1];
      gv[0] = g_nb;
      if constexpr (!kPackH) {
#pragma unroll
        for (int j = 0; j < kPerThread - 1; ++j) hv[j] = hv[j + 1];
        hv[kPerThread - 1] = h_nb;
      }
    }
    const uint32_t head = CAUSAL ? emask : smask;
    uint32_t tail = CAUSAL ? smask : emask;
    // time slabs: carried adjoint at the row's first element in scan order,
    // state neighbour from outside the slab, aggregate at the row's last element
    const uint32_t lastmask = IO && args.io.agg ? tail : 0u;
    // (read while the stage's metadata is still held: no register carries the
    // tile's row through the scan)
    if (IO && args.io.carry != nullptr && head != 0u)
      apply_row_carry_adjoint<CAUSAL>(gv, dyv, head, RowPos(m.row0, m.t0 + o, BL), BL,
                                      args.io.carry);
    if constexpr (IO) {
      if (args.io.halo != nullptr && tail != 0u)
        tail &= ~apply_row_halo<CAUSAL>(hv, tail, RowPos(m.row0, m.t0 + o, BL), BL, args.io.halo);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[stage]);
    if (++stage == NS) {
      stage = 0;
      phase ^= 1u;
    }
    Pfx ex, wtot;
    warp_scan<REV>(fold16_inplace<REV>(gv, dyv, head), lane, ex, wtot);
    if (early) take_early(early_raw, te_known, te_meta);
    const Pfx Pc = warp_tile_prefix<REV>(sm, xi, ex, wtot, first_is_head, ticket, args.st,
                                        sch.stride, te_known, te_meta, warp, lane, ok,
                                        err_host);
    // gv, dyv hold the local prefixes: dh = A_loc * carry + B_loc before the first head
    const uint32_t cm = carry_mask<REV, P>(head);
    if (IO && lastmask != 0u)
      record_row_agg<REV>(gv, dyv, lastmask, cm, Pc, RowPos(p0 + o, BL), BL, args.io.agg);
#pragma unroll
    for (int j = 0; j < kPerThread; ++j) {
      const float d = ((cm >> j) & 1u) ? fmaf(gv[j], Pc.b, dyv[j]) : dyv[j];
      float hn;
      if constexpr (kPackH) {
        if (CAUSAL)
          hn = j == 0 ? h_nb : packed_elem<T>(hw, j - 1);
        else
          hn = j == kPerThread - 1 ? h_nb : packed_elem<T>(hw, j + 1);
      } else {
        hn = hv[j];
      }
      dyv[j] = d;                                    // dx
      gv[j] = ((tail >> j) & 1u) ? 0.f : d * hn;     // dg
    }
    const bool store = !IO || args.dx != nullptr;  // false: aggregate-only pass
    const uint32_t valid = below_mask<P>(o, n_valid) & ~omask;
    uint32_t direct = store ? valid : 0u;
    if (lane == 0) bulk_wait_read<1>();  // this warp's slice of staging buffer obuf is free
    __syncwarp();
    // this warp's slice goes out by TMA when it lies wholly inside the tile's
    // TMA-covered part (never past a row end or the array end)
    const bool slice_tma =
        !RG && store && !has_outside && (warp + 1) * (kTileElems / kConsumerWarps) <= n_tma;
    if constexpr (RG) {
      if (__all_sync(kFull, direct == kThreadMask)) {
        // ragged rows: a wholly valid warp slice leaves by realigned 16-byte stores
        const uint32_t r = static_cast<uint32_t>(p0 % ThreadChunks<T, P>::kVec);
        store_realigned<T>(args.dx, p0 + o, r, dyv, lane, warp_stage(sm, 0, warp));
        store_realigned<T>(args.dg, p0 + o, r, gv, lane, warp_stage(sm, 1, warp));
        direct = 0u;
      }
    }
    if (slice_tma) {
      write_block<T>(sm.out[obuf][0], tc, dyv);
      write_block<T>(sm.out[obuf][1], tc, gv);
      direct = 0u;
    }
    if (direct) {
      store_direct<T>(args.dx, p0 + o, direct, dyv);
      store_direct<T>(args.dg, p0 + o, direct, gv);
    }
    fence_async_smem();
    __syncwarp();
    if (lane == 0) {
      if (slice_tma) {
        const int row = static_cast<int>(p0 / F::kElemsPerRow) + warp * kPartRows;
        tma_store_2d(map_dx, 0, row, sm.out[obuf][0] + warp * kPartBytes);
        tma_store_2d(map_dg, 0, row, sm.out[obuf][1] + warp * kPartBytes);
      }
      bulk_commit();
    }
    obuf ^= 1u;
    if (++xi == kXsRing) xi = 0;
  }
  if (!ok && lane == 0) {
    *reinterpret_cast<volatile int*>(&sm.abort) = 1;
    report(ASCAN_DEV_ERR_LOOKBACK, 0xfffffffdull, err_host);
    set_aborted(args.st);
  }
  if (lane == 0) bulk_wait_all();
}

template <typename T, typename IdxT, bool REV, bool GATES_OUT, int NS, bool IO, int P, bool RG>
__global__ void __launch_bounds__(tma::kThreads, tma::kCtasPerSm)
    scan_fwd_tma_kernel(const __grid_constant__ CUtensorMap map_g,
                        const __grid_constant__ CUtensorMap map_x,
                        const __grid_constant__ CUtensorMap map_y,
                        const __grid_constant__ CUtensorMap map_gout, const FwdArgs<T, IdxT> args,
                        int64_t n_tma_total, const tma::TileSched sch, uint32_t* err_host) {
  fwd_tma_body<T, IdxT, REV, GATES_OUT, NS, IO, P, RG>(&map_g, &map_x, &map_y, &map_gout, args,
                                                    n_tma_total, sch, err_host);
}

template <typename T, typename IdxT, bool CAUSAL, int NS, bool IO, int P, bool RG>
__global__ void __launch_bounds__(tma::kThreads, tma::kCtasPerSm)
    scan_bwd_tma_kernel(const __grid_constant__ CUtensorMap map_dy,
                        const __grid_constant__ CUtensorMap map_g,
                        const __grid_constant__ CUtensorMap map_h,
                        const __grid_constant__ CUtensorMap map_dx,
                        const __grid_constant__ CUtensorMap map_dg, const BwdArgs<T, IdxT> args,
                        int64_t n_tma_total, const tma::TileSched sch, uint32_t* err_host) {
  bwd_tma_body<T, IdxT, CAUSAL, NS, IO, P, RG>(&map_dy, &map_g, &map_h, &map_dx, &map_dg, args,
                                            n_tma_total, sch, err_host);
}

// Both directions of a bidirectional scan in one launch: CTAs [0, bs.cta0)
// run the causal branch over (gates_fwd, tokens_fwd), the others the reverse
// branch over (gates_bwd, tokens_bwd).  The two groups share nothing (own
// tickets, status slots and abort words); the launch is cooperative, so both
// groups are resident and each moves through its own tickets as a separate
// launch would.
template <typename T, typename IdxT, int NS, int P, bool RG>
__global__ void __launch_bounds__(tma::kThreads, tma::kCtasPerSm)
    scan_fwd_bidi_tma_kernel(const __grid_constant__ CUtensorMap f_g,
                             const __grid_constant__ CUtensorMap f_x,
                             const __grid_constant__ CUtensorMap f_y,
                             const __grid_constant__ CUtensorMap b_g,
                             const __grid_constant__ CUtensorMap b_x,
                             const __grid_constant__ CUtensorMap b_y, const FwdArgs<T, IdxT> fa,
                             const FwdArgs<T, IdxT> ba, int64_t n_tma_total,
                             const tma::TileSched fs, const tma::TileSched bs,
                             uint32_t* err_host) {
  if (blockIdx.x < bs.cta0)
    fwd_tma_body<T, IdxT, false, false, NS, false, P, RG>(&f_g, &f_x, &f_y, &f_y, fa, n_tma_total, fs,
                                                          err_host);
  else
    fwd_tma_body<T, IdxT, true, false, NS, false, P, RG>(&b_g, &b_x, &b_y, &b_y, ba, n_tma_total, bs,
                                                         err_host);
}

// Adjoint of scan_fwd_bidi_tma_kernel: the causal adjoint on CTAs [0, bs.cta0),
// the reverse adjoint on the others.
template <typename T, typename IdxT, int NS, int P, bool RG>
__global__ void __launch_bounds__(tma::kThreads, tma::kCtasPerSm)
    scan_bwd_bidi_tma_kernel(const __grid_constant__ CUtensorMap f_dy,
                             const __grid_constant__ CUtensorMap f_g,
                             const __grid_constant__ CUtensorMap f_h,
                             const __grid_constant__ CUtensorMap f_dx,
                             const __grid_constant__ CUtensorMap f_dg,
                             const __grid_constant__ CUtensorMap b_dy,
                             const __grid_constant__ CUtensorMap b_g,
                             const __grid_constant__ CUtensorMap b_h,
                             const __grid_constant__ CUtensorMap b_dx,
                             const __grid_constant__ CUtensorMap b_dg, const BwdArgs<T, IdxT> fa,
                             const BwdArgs<T, IdxT> ba, int64_t n_tma_total,
                             const tma::TileSched fs, const tma::TileSched bs,
                             uint32_t* err_host) {
  if (blockIdx.x < bs.cta0)
    bwd_tma_body<T, IdxT, true, NS, false, P, RG>(&f_dy, &f_g, &f_h, &f_dx, &f_dg, fa, n_tma_total, fs,
                                                  err_host);
  else
    bwd_tma_body<T, IdxT, false, NS, false, P, RG>(&b_dy, &b_g, &b_h, &b_dx, &b_dg, ba, n_tma_total,
                                                bs, err_host);
}

#if defined(ASCAN_UNIT_MISC)  // compiled in one unit only
// ---------------------------------------------------------------------------
// Self-test of the bounded waits: three waits on conditions that nothing will
// ever satisfy -- a stage barrier nobody arrives on, a hand-off slot nobody
// tags, a look-back whose predecessor never publishes -- each of which must
// give up after `limit_ns` and say so, leaving the context usable.
// out[0]: barrier wait succeeded, out[1]: slot wait succeeded, out[2]:
// look-back gave up, out[3]: elapsed nanoseconds of the three waits.
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(32) selftest_waits_kernel(uint4* slots, uint32_t* abort_word,
                                                           unsigned long long limit_ns,
                                                           unsigned long long* out) {
  __shared__ alignas(8) uint64_t bar;
  __shared__ float4 slot;
  __shared__ int cta_abort;
  const int lane = threadIdx.x;
  if (lane == 0) {
    tma::mbar_init(&bar, 1);
    slot = make_float4(0.f, 0.f, 0.f, __uint_as_float(tma::kNoTag));
    cta_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  const unsigned long long t0 = globaltimer();
  const bool got_bar = tma::mbar_wait_warp(&bar, 0u, limit_ns);  // phase 0 never completes
  Pfx v = pfx_empty();
  const bool got_slot = tma::xs_get_warp(&slot, true, 7u, v, &cta_abort, limit_ns);
  bool timed_out = false;
  (void)lookback_warp<kLookbackPerLane>(TileStatus{slots, abort_word}, 1u, lane, &timed_out, 1u,
                                        limit_ns);
  if (lane == 0) {
    out[0] = got_bar ? 1ull : 0ull;
    out[1] = got_slot ? 1ull : 0ull;
    out[2] = timed_out ? 1ull : 0ull;
    out[3] = globaltimer() - t0;
  }
}
#endif  // ASCAN_UNIT_MISC

// ---------------------------------------------------------------------------
// shift_pad: out[t] = pad at boundaries, else data[t -/+ 1]
// ---------------------------------------------------------------------------

template <typename IdxT>
__device__ __forceinline__ bool cu_contains(const IdxT* __restrict__ cu, int64_t lo_i, int64_t hi_i,
                                            int64_t v, int64_t BL) {
  // any cu[i] == v for i in [lo_i, hi_i), cu sorted
  int64_t a = lo_i, b = hi_i;
  while (a < b) {
    int64_t m = (a + b) >> 1;
    if (cu_at(cu, m, BL) < v)
      a = m + 1;
    else
      b = m;
  }
  return a < hi_i && cu_at(cu, a, BL) == v;
}

template <typename T, typename IdxT>
__global__ void __launch_bounds__(kThreads)
    shift_pad_kernel(const T* __restrict__ data, T* __restrict__ out, const IdxT* __restrict__ cu,
                     int64_t S, int64_t BL, int64_t N, float pad, int backward, int wrap) {
  const T padv = Cvt<T>::from(pad);
  for (int64_t p = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; p < N;
       p += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int64_t c = p / BL;
    const int64_t t = p - c * BL;
    const bool boundary = backward ? cu_contains(cu, 0, S, t, BL) : cu_contains(cu, 1, S + 1, t + 1, BL);
    if (boundary) {
      out[p] = padv;
      continue;
    }
    int64_t src = backward ? t - 1 : t + 1;
    if (wrap)
      src = (src < 0) ? src + BL : (src >= BL ? src - BL : src);
    else
      src = src < 0 ? 0 : (src >= BL ? BL - 1 : src);
    out[p] = data[c * BL + src];
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

// Device address of the pinned host error flag (ascan_error_flag), or NULL;
// defined in ascan.cu and passed to every kernel as its last parameter (not
// inside the argument structs, whose layout the hot kernels are tuned to).
extern uint32_t* g_err_host;

struct Workspace {
  uint32_t* ticket;
  TileStatus st;
  size_t clear_bytes;
  bool allow_ragged;  // room for the status slots of ragged row order
};

// Tiles of the plain kernels (kTile elements) and of the persistent TMA
// kernels (4096 or 8192 elements; one divides the other); status slots are
// counted in the smallest tiles so that every kernel fits the same workspace.
static size_t tiles_of(int64_t n) { return static_cast<size_t>((n + kTile - 1) / kTile); }
static size_t tma_tiles_of(int64_t n) {
  return static_cast<size_t>((n + tma::kMinTileElems - 1) / tma::kMinTileElems);
}
// Row order with ragged rows (BL not a multiple of the tile) cuts every row
// into ceil(BL / tile) tiles, a few more than the flat count.
static size_t status_slots(int64_t C, int64_t BL, bool ragged) {
  const size_t plain = tiles_of(C * BL), tma_flat = tma_tiles_of(C * BL);
  const size_t flat = plain > tma_flat ? plain : tma_flat;  // either kernel family
  if (!ragged || BL < tma::kMinTileElems) return flat;  // ragged rows are at least a tile
  const size_t rows = static_cast<size_t>(C) *
                      static_cast<size_t>((BL + tma::kMinTileElems - 1) / tma::kMinTileElems);
  return rows > flat ? rows : flat;
}

// 256-byte header (ticket counter, abort word) + one 16-byte status slot per tile.
static size_t workspace_bytes_for(int64_t C, int64_t BL, bool ragged) {
  return 256 + status_slots(C, BL, ragged) * sizeof(uint4);
}

// A workspace of the flat size is accepted; ragged row order is then simply
// not used (the flat order needs fewer status slots).
static int carve(void* ws, size_t ws_bytes, int64_t C, int64_t BL, Workspace& out) {
  if (!ws || (reinterpret_cast<uintptr_t>(ws) & 255u) != 0) return ASCAN_EWORKSPACE;
  if (ws_bytes < workspace_bytes_for(C, BL, false)) return ASCAN_EWORKSPACE;
  char* base = static_cast<char*>(ws);
  out.allow_ragged = ws_bytes >= workspace_bytes_for(C, BL, true);
  const size_t tiles = status_slots(C, BL, out.allow_ragged);
  out.ticket = reinterpret_cast<uint32_t*>(base);
  out.st.abort = reinterpret_cast<uint32_t*>(base + 4);
  out.st.slots = reinterpret_cast<uint4*>(base + 256);
  out.clear_bytes = 256 + tiles * sizeof(uint4);
  return ASCAN_OK;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static int launch_status() {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    fprintf(stderr, "ascan: CUDA error: %s\n", cudaGetErrorString(e));
    return ASCAN_ECUDA;
  }
  return ASCAN_OK;
}

static int sm_count();

// Aggregate-only slab pass by the row reduction of ascan_slab.cuh.  The warps
// that share a row combine their parts through the cleared part of the
// workspace (one counter per row, then one partial per warp and row), so the
// grid is only as wide as that room allows.  `r2l`: the fold runs right to
// left (causal backward, reverse forward).
template <typename T, typename IdxT, bool BWD>
static int launch_slab_aggregate(const T* a, const T* b, const IdxT* cu, int64_t S, int64_t C,
                                 int64_t L, bool r2l, const float* carry, float* agg,
                                 const Workspace& w, cudaStream_t s) {
  if (!agg || C <= 0 || L <= 0) return ASCAN_EINVAL;
  // one resident wave of CTAs (fewer when the rows are short: every warp
  // gets at least one round of loads); each warp leaves one partial per row
  // it touches, and a row spans at most ceil(warps / C) + 1 warps
  constexpr int64_t kVec = 16 / static_cast<int64_t>(sizeof(T));
  const int64_t sms = sm_count() > 0 ? sm_count() : 1;
  const int64_t vectors = C * ((L + 2 * kVec - 2) / kVec);
  int64_t ctas = sms * slab::kAggCtasPerSm;
  const int64_t by_work = (vectors + slab::kAggMinShare * slab::kAggWarps - 1) /
                          (slab::kAggMinShare * slab::kAggWarps);
  if (ctas > by_work) ctas = by_work;
  if (ctas < 1) ctas = 1;
  char* base = reinterpret_cast<char*>(w.ticket);
  const size_t counters_bytes = (static_cast<size_t>(C) * 4u + 15u) & ~static_cast<size_t>(15);
  const size_t room = w.clear_bytes > 256 + counters_bytes ? w.clear_bytes - 256 - counters_bytes : 0;
  const int64_t room_per_row = static_cast<int64_t>(room / (8u * static_cast<size_t>(C)));
  int64_t per_row = (ctas * slab::kAggWarps + C - 1) / C + 1;
  if (per_row > room_per_row) {
    // fewer warps, as many as the partials' room allows, or whole rows per
    // warp (per_row 0: no partials) when it holds fewer than two per row
    const int64_t max_warps = room_per_row >= 2 ? (room_per_row - 1) * C : 0;
    if (max_warps >= slab::kAggWarps) {
      ctas = max_warps / slab::kAggWarps;
      per_row = (ctas * slab::kAggWarps + C - 1) / C + 1;
    } else {
      per_row = 0;
    }
  }
  slab::AggArgs<T, IdxT> args{a, b, cu, S, L, C, carry, agg,
                              reinterpret_cast<uint32_t*>(base + 256),
                              reinterpret_cast<float2*>(base + 256 + counters_bytes),
                              static_cast<uint32_t>(per_row), g_err_host};
  const dim3 grid(static_cast<unsigned>(ctas)), block(slab::kAggThreads);
  if (r2l)
    slab::slab_aggregate_kernel<T, IdxT, true, BWD><<<grid, block, 0, s>>>(args);
  else
    slab::slab_aggregate_kernel<T, IdxT, false, BWD><<<grid, block, 0, s>>>(args);
  return launch_status();
}

// ---- implementation choice ------------------------------------------------

// 0: automatic (the TMA kernels whenever possible, automatic tile order),
// 1: always the plain kernels, 2: TMA kernels whenever possible with the
// automatic tile order (same as 0), 3: TMA kernels with tiles in flat
// order, 4: TMA kernels with row order whenever rows are tile-aligned.
// ASCAN_IMPL=simple|tma|tma-flat|tma-row selects 1..4 at first use.
extern int g_impl;  // defined in ascan.cu (process-wide)

static int impl_mode() {
  if (g_impl < 0) {
    const char* e = getenv("ASCAN_IMPL");
    g_impl = 0;
    if (e && strcmp(e, "simple") == 0) g_impl = 1;
    if (e && strcmp(e, "tma") == 0) g_impl = 2;
    if (e && strcmp(e, "tma-flat") == 0) g_impl = 3;
    if (e && strcmp(e, "tma-row") == 0) g_impl = 4;
  }
  return g_impl;
}

static bool use_tma() { return impl_mode() != 1; }

// ---- TMA descriptors -------------------------------------------------------

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// The flat array seen as `rows` rows of 128 bytes; one box = one 4096-element
// tile, stored in shared memory with the 128-byte swizzle.
template <typename T>
static bool make_map(CUtensorMap* m, const void* base, int64_t rows,
                     int box_rows = tma::Fmt<T>::kRows) {
  const auto fn = encode_fn();
  if (!fn || rows <= 0 || rows > 0x7fffffffll) return false;
  const CUtensorMapDataType dt =
      std::is_same<T, float>::value    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
      : std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                       : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(tma::Fmt<T>::kElemsPerRow),
                              static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {128};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(tma::Fmt<T>::kElemsPerRow),
                             static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  return n;
}

// CTAs of `kern` that fit on the device at once (0: none, <0: error); the
// shared-memory opt-in and the occupancy query run once per kernel and device.
static int coop_capacity(const void* kern, size_t smem) {
  // Per kernel and device: the shared-memory opt-in and the occupancy query
  // run once (they are host-side driver calls, not free at small sizes).
  struct Entry {
    const void* kern;
    int device;
    int per_sm;
  };
  static std::mutex mu;
  static Entry cache[256];
  static int n_cache = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  int per_sm = -1;
  {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < n_cache; ++i)
      if (cache[i].kern == kern && cache[i].device == dev) per_sm = cache[i].per_sm;
  }
  if (per_sm < 0) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return ASCAN_ECUDA;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, tma::kThreads, smem) !=
        cudaSuccess)
      return 0;
    std::lock_guard<std::mutex> lock(mu);
    if (n_cache < 256) cache[n_cache++] = Entry{kern, dev, per_sm};
  }
  if (per_sm <= 0) return 0;
  const int sms = sm_count();
  if (sms <= 0) return 0;
  return sms * per_sm;
}

// Cooperative launch of `grid` CTAs (at most the capacity).  1: launched,
// <0: error.
static int launch_coop_grid(const void* kern, size_t smem, uint32_t grid, void** params,
                            cudaStream_t s) {
  // cooperative through the launch attribute: also valid under stream capture
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(tma::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelExC(&cfg, kern, params);
  if (e != cudaSuccess) {
    fprintf(stderr, "ascan: cooperative launch failed: %s\n", cudaGetErrorString(e));
    cudaGetLastError();
    return ASCAN_ECUDA;
  }
  return 1;
}

// Cooperative launch of a persistent TMA kernel: one CTA per SM that can hold
// it (never more CTAs than tiles).  Co-residency of every CTA is what makes the
// round-robin tile schedule safe.  1: launched, 0: not possible here (the
// caller falls back to the plain kernel), <0: error.
static int launch_cooperative(const void* kern, size_t smem, uint32_t num_tiles, void** params,
                              cudaStream_t s) {
  const int cap = coop_capacity(kern, smem);
  if (cap <= 0) return cap;
  const uint32_t resident = static_cast<uint32_t>(cap);
  const uint32_t grid = num_tiles < resident ? num_tiles : resident;
  return launch_coop_grid(kern, smem, grid, params, s);
}

// Splits a cooperative grid between the two scans of a bidirectional launch
// (each gets at most its tiles and half the resident CTAs).  false: fewer
// than two CTAs fit, so the two scans run as separate launches.
static bool split_bidi(int cap, tma::TileSched& fs, tma::TileSched& bs, uint32_t& grid) {
  if (cap < 2) return false;
  const uint32_t half = static_cast<uint32_t>(cap) / 2u;
  const uint32_t gf = fs.num_tiles < half ? fs.num_tiles : half;
  const uint32_t rest = static_cast<uint32_t>(cap) - gf;
  const uint32_t gb = bs.num_tiles < rest ? bs.num_tiles : rest;
  if (gf == 0 || gb == 0) return false;
  fs.cta0 = 0u;
  fs.ctas = gf;
  bs.cta0 = gf;
  bs.ctas = gb;
  grid = gf + gb;
  return true;
}

// Tile order of the TMA kernels: row mode needs row-aligned tiles (BL a
// multiple of the tile) and pays off when sequences span several tiles: in
// flat order their tiles are consecutive tickets of one wave, so every tile
// waits on a look-back behind the one before it, while in row order a tile's
// predecessor is `rows` tickets older (many waves when rows >> CTAs, and
// never closer than in flat order).  When sequences fit in a tile on average,
// the flat order is slightly faster (a wave reads one contiguous range).
// Implementations 3 and 4 force the flat and the row order; both orders give
// the same results up to floating-point reassociation.
// allow_ragged: rows that are not whole tiles may be cut into whole tiles and
// a partial last one (the workspace has their status slots and the launch
// has no slab I/O).
// row_hint: take the row order whenever it fits, as if sequences were long
// (wide tiles keep the order the narrow ones would have chosen).
static tma::TileSched make_sched(int64_t kT, int64_t N, int64_t BL, int64_t S,
                                 bool allow_ragged, bool row_hint = false) {
  tma::TileSched sch{static_cast<uint32_t>((N + kT - 1) / kT), 0u, 0u, 0u, 1u, 0u, 0u, 0u, 1u};
  const int64_t C = BL > 0 ? N / BL : 0;
  const int mode = impl_mode();
  const int64_t per_row = BL > 0 ? (BL + kT - 1) / kT : 0;
  const bool aligned = BL % kT == 0;
  const bool fits = BL >= kT && C >= 1 && C <= 0x7fffffffll && C * per_row <= 0xffffffffll &&
                    (aligned || allow_ragged);
  const bool long_seqs = BL > S * kT;  // mean length above a tile
  const bool row = mode == 4 ? fits : mode == 3 ? false : fits && (long_seqs || row_hint);
  if (row) {
    sch.row_mode = 1u;
    sch.rows = static_cast<uint32_t>(C);
    sch.tiles_per_row = static_cast<uint32_t>(per_row);
    sch.stride = static_cast<uint32_t>(C);
    sch.ragged = aligned ? 0u : 1u;
    sch.num_tiles = static_cast<uint32_t>(C * per_row);
    // Segment mode is offered when S sequences of equal length would each
    // cover whole tiles; the kernels take it only if cu_seqlens really is
    // that even split.  It moves a tile's predecessor from C to C * S
    // tickets back: with C = 192 rows of 8 sequences of 65536 (one rank's
    // share of B=8, T=65536, C=1536 on 8 GPUs) the row order puts it 1.3
    // waves back and its carry arrives late (fwd 225 / bwd 422 us against
    // 195 / 391 us for the same array with a sequence start at every tile).
    if (aligned && S >= 2 && S + 1 <= tma::kCuCache && BL % S == 0 && (BL / S) % kT == 0 &&
        C * S <= 0xffffffffll)
      sch.segs = static_cast<uint32_t>(S);
  }
  return sch;
}

// ---- tile width -----------------------------------------------------------

// 0: automatic; 16 or 32: elements per consumer thread forced wherever both
// kernels exist (tests and tuning; ascan_set_tile_width).
extern int g_tile_width;  // defined in ascan.cu (process-wide)

// Whether a launch runs 8192-element tiles (32 elements per thread) rather
// than 4096-element ones.  Wide tiles halve the consumer warps' fixed
// per-tile chain (fold, warp scan, hand-offs, carry) per byte.  Measured on
// B200 (fwd / bwd, us): B=8, C=1536, fp32 T=4096 fwd 143 -> 106, T=65536
// 2267 -> 1481; bf16 T=4096 139/173 -> 99/130; fp16 T=2048 76/92 -> 55/69;
// C=256, T=2^20 fwd 868 -> 559; 16-bit varlen rows (bf16, C=2048) fwd
// 1127 -> 800.  They lose when they would turn a row order into a flat one
// for the fp32 forward (varlen C=2048: 1150 -> 1196), and gain nothing when
// the tiles are too few to fill the SMs twice.  Rows fewer than the CTAs
// would put a tile's predecessor in its own wave.
static bool use_wide(int64_t N, int64_t BL, int64_t S, bool allow_ragged, bool forward,
                     bool narrow_type = false, bool* row_hint = nullptr) {
  if (row_hint) *row_hint = false;
  tma::TileSched wide = make_sched(tma::Geo<32>::kTileElems, N, BL, S, allow_ragged);
  // fp32 ragged rows at the wide width would need a 257-row TMA box, one
  // more than a box may hold: those launches keep the narrow tiles
  const bool box_ok = !forward || narrow_type || !wide.ragged;
  if (g_tile_width != 0) return g_tile_width == 32 && box_ok;
  if (forward) {
    // keep the narrow row order unless sequences average a whole wide tile
    // (then the wide flat tiles mostly start at sequence heads); 16-bit
    // types keep it with wide tiles (ragged rows included)
    const tma::TileSched narrow = make_sched(tma::Geo<16>::kTileElems, N, BL, S, allow_ragged);
    if (narrow.row_mode && !wide.row_mode && BL < S * tma::Geo<32>::kTileElems) {
      if (!narrow_type || !row_hint) return false;
      wide = make_sched(tma::Geo<32>::kTileElems, N, BL, S, allow_ragged, true);
      if (!wide.row_mode) return false;
      *row_hint = true;
    }
    if (!box_ok) return false;
  }
  const uint32_t sms = static_cast<uint32_t>(sm_count());
  if (sms == 0 || wide.num_tiles < 2 * sms) return false;
  if (wide.row_mode && wide.rows < sms) return false;
  return true;
}

// 1: launched, 0: not applicable (caller falls back to the plain kernel), <0: error
template <typename T, typename IdxT, bool REV, bool GOUT, int P, bool RG>
static int launch_fwd_tma_sched(const FwdArgs<T, IdxT>& a, const tma::TileSched& sch0, bool io,
                                cudaStream_t s) {
  using F = tma::Fmt<T, P>;
  constexpr int NOUT = GOUT ? 2 : 1;
  constexpr int NS = ring_depth<T, 2, NOUT, P, RG>();
  constexpr size_t smem = tma::smem_bytes<2, NOUT, NS, T, P, RG>();
  static_assert(smem <= kSmemBudget, "TMA forward ring does not fit in shared memory");
  const int64_t rows = a.N / F::kElemsPerRow;
  CUtensorMap mg, mx, my, mgo;
  constexpr int kPart = F::kRows / tma::kConsumerWarps;  // stores: one warp's slice
  constexpr int kInRows = F::kRows + (RG ? 1 : 0);     // ragged: one more row
  // an aggregate-only pass stores nothing: its output map is a never-used view of g
  if (!make_map<T>(&mg, a.g, rows, kInRows) || !make_map<T>(&mx, a.x, rows, kInRows) ||
      !make_map<T>(&my, a.y ? a.y : a.g, rows, kPart))
    return 0;
  if (GOUT) {
    if (!make_map<T>(&mgo, a.gout, rows, kPart)) return 0;
  } else {
    mgo = my;
  }
  const void* kern;
  if constexpr (RG)  // slab I/O exists in the staged kernels only
    kern = reinterpret_cast<const void*>(scan_fwd_tma_kernel<T, IdxT, REV, GOUT, NS, false, P, RG>);
  else
    kern = io ? reinterpret_cast<const void*>(scan_fwd_tma_kernel<T, IdxT, REV, GOUT, NS, true, P, false>)
              : reinterpret_cast<const void*>(scan_fwd_tma_kernel<T, IdxT, REV, GOUT, NS, false, P, false>);
  int64_t n_tma_total = rows * F::kElemsPerRow;
  FwdArgs<T, IdxT> b = a;
  tma::TileSched sch = sch0;
  b.num_tiles = sch.num_tiles;
  uint32_t* err_host = g_err_host;
  void* params[] = {&mg, &mx, &my, &mgo, &b, &n_tma_total, &sch, &err_host};
  return launch_cooperative(kern, smem, b.num_tiles, params, s);
}

template <typename T, typename IdxT, bool REV, bool GOUT, int P>
static int launch_fwd_tma_p(const FwdArgs<T, IdxT>& a, bool allow_ragged, bool io,
                            cudaStream_t s, bool row_hint = false) {
  // ragged rows need the shifted-tile kernels, which exist without slab I/O only
  const tma::TileSched sch =
      make_sched(tma::Geo<P>::kTileElems, a.N, a.BL, a.S, allow_ragged && !io, row_hint);
  constexpr bool kStaged = staged_fits<T, 2, GOUT ? 2 : 1, P>();
  if (sch.ragged || !kStaged) {
    if (io) return 0;  // slab I/O exists in the staged kernels only
    return launch_fwd_tma_sched<T, IdxT, REV, GOUT, P, true>(a, sch, io, s);
  }
  // rows of whole tiles in row order, outputs written, no aggregate: the
  // producers of the plain kernels turn the row carry into the tiles'
  // carry-in, so the slab kernels (row I/O in the consumers) are not needed
  const bool meta_io = io && sch.row_mode && !sch.ragged && a.io.agg == nullptr && a.y != nullptr;
  if constexpr (kStaged)
    return launch_fwd_tma_sched<T, IdxT, REV, GOUT, P, false>(a, sch, io && !meta_io, s);
  return 0;
}

// allow_ragged is passed beside the kernel arguments, not inside them: the
// argument structs are what the kernels receive.
template <typename T, typename IdxT, bool REV, bool GOUT>
static int launch_fwd_tma(const FwdArgs<T, IdxT>& a, bool allow_ragged, cudaStream_t s) {
  const bool io = a.io.carry || a.io.halo || a.io.agg || !a.y;
  // wide tiles for the plain forward (the gate-product output stays narrow)
  if constexpr (!GOUT) {
    bool row_hint = false;
    if (use_wide(a.N, a.BL, a.S, allow_ragged && !io, /*forward=*/true, sizeof(T) == 2,
                 &row_hint))
      return launch_fwd_tma_p<T, IdxT, REV, GOUT, 32>(a, allow_ragged, io, s, row_hint);
  }
  return launch_fwd_tma_p<T, IdxT, REV, GOUT, 16>(a, allow_ragged, io, s);
}

template <typename T, typename IdxT, bool CAUSAL, int P, bool RG>
static int launch_bwd_tma_sched(const BwdArgs<T, IdxT>& a, const tma::TileSched& sch0, bool io,
                                cudaStream_t s) {
  using F = tma::Fmt<T, P>;
  constexpr int NS = ring_depth<T, 3, 2, P, RG>();
  constexpr size_t smem = tma::smem_bytes<3, 2, NS, T, P, RG>();
  static_assert(smem <= kSmemBudget, "TMA backward ring does not fit in shared memory");
  const int64_t rows = a.N / F::kElemsPerRow;
  CUtensorMap mdy, mg, mh, mdx, mdg;
  constexpr int kPart = F::kRows / tma::kConsumerWarps;  // stores: one warp's slice
  constexpr int kInRows = F::kRows + (RG ? 1 : 0);     // ragged: one more row
  if (!make_map<T>(&mdy, a.dy, rows, kInRows) || !make_map<T>(&mg, a.g, rows, kInRows) ||
      !make_map<T>(&mh, a.h, rows, kInRows) ||
      !make_map<T>(&mdx, a.dx ? a.dx : a.dy, rows, kPart) ||
      !make_map<T>(&mdg, a.dg ? a.dg : a.dy, rows, kPart))
    return 0;
  const void* kern;
  if constexpr (RG)
    kern = reinterpret_cast<const void*>(scan_bwd_tma_kernel<T, IdxT, CAUSAL, NS, false, P, RG>);
  else
    kern = io ? reinterpret_cast<const void*>(scan_bwd_tma_kernel<T, IdxT, CAUSAL, NS, true, P, false>)
              : reinterpret_cast<const void*>(scan_bwd_tma_kernel<T, IdxT, CAUSAL, NS, false, P, false>);
  int64_t n_tma_total = rows * F::kElemsPerRow;
  BwdArgs<T, IdxT> b = a;
  tma::TileSched sch = sch0;
  b.num_tiles = sch.num_tiles;
  uint32_t* err_host = g_err_host;
  void* params[] = {&mdy, &mg, &mh, &mdx, &mdg, &b, &n_tma_total, &sch, &err_host};
  return launch_cooperative(kern, smem, b.num_tiles, params, s);
}

template <typename T, typename IdxT, bool CAUSAL, int P>
static int launch_bwd_tma_p(const BwdArgs<T, IdxT>& a, bool allow_ragged, bool io,
                            cudaStream_t s) {
  const tma::TileSched sch =
      make_sched(tma::Geo<P>::kTileElems, a.N, a.BL, a.S, allow_ragged && !io);
  constexpr bool kStaged = staged_fits<T, 3, 2, P>();
  if (sch.ragged || !kStaged) {
    if (io) return 0;  // slab I/O exists in the staged kernels only
    return launch_bwd_tma_sched<T, IdxT, CAUSAL, P, true>(a, sch, io, s);
  }
  // rows of whole tiles in row order, outputs written, no aggregate: the
  // producers of the plain kernels carry the row I/O (see the forward)
  const bool meta_io = io && sch.row_mode && !sch.ragged && a.io.agg == nullptr &&
                       a.dx != nullptr;
  if constexpr (kStaged)
    return launch_bwd_tma_sched<T, IdxT, CAUSAL, P, false>(a, sch, io && !meta_io, s);
  return 0;
}

// 16-bit types take wide tiles in the backward too (the same bytes per tile
// as fp32 at 16 elements per thread); fp32 keeps 4096-element tiles, whose
// three inputs and two staged outputs fill the shared memory.
template <typename T>
constexpr bool kWideBwd = sizeof(T) == 2;

template <typename T, typename IdxT, bool CAUSAL>
static int launch_bwd_tma(const BwdArgs<T, IdxT>& a, bool allow_ragged, cudaStream_t s) {
  const bool io = a.io.carry || a.io.halo || a.io.agg || !a.dx;
  if constexpr (kWideBwd<T>) {
    if (use_wide(a.N, a.BL, a.S, allow_ragged && !io, /*forward=*/false))
      return launch_bwd_tma_p<T, IdxT, CAUSAL, 32>(a, allow_ragged, io, s);
  }
  return launch_bwd_tma_p<T, IdxT, CAUSAL, 16>(a, allow_ragged, io, s);
}

template <typename T, typename IdxT, int VEC>
static void fwd_dispatch(const FwdArgs<T, IdxT>& a, bool reverse, bool gout, cudaStream_t s) {
  const dim3 grid(a.num_tiles), block(kThreads);
  if (reverse) {
    if (gout)
      scan_fwd_kernel<T, IdxT, VEC, true, true><<<grid, block, 0, s>>>(a, g_err_host);
    else
      scan_fwd_kernel<T, IdxT, VEC, true, false><<<grid, block, 0, s>>>(a, g_err_host);
  } else {
    if (gout)
      scan_fwd_kernel<T, IdxT, VEC, false, true><<<grid, block, 0, s>>>(a, g_err_host);
    else
      scan_fwd_kernel<T, IdxT, VEC, false, false><<<grid, block, 0, s>>>(a, g_err_host);
  }
}

template <typename T, typename IdxT>
int fwd_typed(const void* g, const void* x, void* y, void* gout, const void* cu,
                     int64_t S, int64_t C, int64_t BL, int reverse, const Workspace& w,
                     cudaStream_t s, const RowIO& io = RowIO{nullptr, nullptr, nullptr}) {
  FwdArgs<T, IdxT> a;
  a.g = static_cast<const T*>(g);
  a.x = static_cast<const T*>(x);
  a.y = static_cast<T*>(y);
  a.gout = static_cast<T*>(gout);
  a.cu = static_cast<const IdxT*>(cu);
  a.S = S;
  a.BL = BL;
  a.N = C * BL;
  a.num_tiles = static_cast<uint32_t>(tiles_of(a.N));
  a.ticket = w.ticket;
  a.st = w.st;
  a.io = io;
  const bool vec = aligned16(g) && aligned16(x) && aligned16(y) && (!gout || aligned16(gout));
  constexpr int kVec = 16 / sizeof(T);
  // row I/O and absent outputs exist only in the persistent TMA kernels
  const bool slab = io.carry || io.halo || io.agg || !y;
  if (slab) {
    if (!vec || a.N < tma::Fmt<T>::kElemsPerRow) return ASCAN_EINVAL;
    if (!y)  // aggregate-only pass: a row reduction, no scan
      return launch_slab_aggregate<T, IdxT, false>(a.g, a.x, a.cu, S, C, BL, reverse != 0,
                                                   io.carry, io.agg, w, s);
    int rc;
    if (reverse)
      rc = gout ? launch_fwd_tma<T, IdxT, true, true>(a, w.allow_ragged, s) : launch_fwd_tma<T, IdxT, true, false>(a, w.allow_ragged, s);
    else
      rc = gout ? launch_fwd_tma<T, IdxT, false, true>(a, w.allow_ragged, s) : launch_fwd_tma<T, IdxT, false, false>(a, w.allow_ragged, s);
    return rc > 0 ? ASCAN_OK : (rc == 0 ? ASCAN_EINVAL : rc);
  }
  if (vec && use_tma() && a.N >= tma::Fmt<T>::kElemsPerRow) {
    int rc;
    if (reverse)
      rc = gout ? launch_fwd_tma<T, IdxT, true, true>(a, w.allow_ragged, s) : launch_fwd_tma<T, IdxT, true, false>(a, w.allow_ragged, s);
    else
      rc = gout ? launch_fwd_tma<T, IdxT, false, true>(a, w.allow_ragged, s) : launch_fwd_tma<T, IdxT, false, false>(a, w.allow_ragged, s);
    if (rc != 0) return rc > 0 ? ASCAN_OK : rc;
  }
  if (vec)
    fwd_dispatch<T, IdxT, kVec>(a, reverse != 0, gout != nullptr, s);
  else
    fwd_dispatch<T, IdxT, 1>(a, reverse != 0, gout != nullptr, s);
  return launch_status();
}

template <typename T, typename IdxT, int VEC>
static void bwd_dispatch(const BwdArgs<T, IdxT>& a, bool causal, cudaStream_t s) {
  const dim3 grid(a.num_tiles), block(kThreads);
  if (causal)
    scan_bwd_kernel<T, IdxT, VEC, true><<<grid, block, 0, s>>>(a, g_err_host);
  else
    scan_bwd_kernel<T, IdxT, VEC, false><<<grid, block, 0, s>>>(a, g_err_host);
}

template <typename T, typename IdxT>
int bwd_typed(const void* dy, const void* g, const void* h, void* dx, void* dg,
                     const void* cu, int64_t S, int64_t C, int64_t BL, int causal,
                     const Workspace& w, cudaStream_t s,
                     const RowIO& io = RowIO{nullptr, nullptr, nullptr}) {
  BwdArgs<T, IdxT> a;
  a.dy = static_cast<const T*>(dy);
  a.g = static_cast<const T*>(g);
  a.h = static_cast<const T*>(h);
  a.dx = static_cast<T*>(dx);
  a.dg = static_cast<T*>(dg);
  a.cu = static_cast<const IdxT*>(cu);
  a.S = S;
  a.BL = BL;
  a.N = C * BL;
  a.num_tiles = static_cast<uint32_t>(tiles_of(a.N));
  a.ticket = w.ticket;
  a.st = w.st;
  a.io = io;
  const bool vec = aligned16(dy) && aligned16(g) && aligned16(h) && aligned16(dx) && aligned16(dg);
  constexpr int kVec = 16 / sizeof(T);
  // row I/O and absent outputs exist only in the persistent TMA kernels
  const bool slab = io.carry || io.halo || io.agg || !dx;
  if (slab) {
    if (!vec || a.N < tma::Fmt<T>::kElemsPerRow) return ASCAN_EINVAL;
    if (!dx)  // aggregate-only pass: a row reduction, no scan (the states are not read)
      return launch_slab_aggregate<T, IdxT, true>(a.g, a.dy, a.cu, S, C, BL, causal != 0,
                                                  io.carry, io.agg, w, s);
    const int rc = causal ? launch_bwd_tma<T, IdxT, true>(a, w.allow_ragged, s) : launch_bwd_tma<T, IdxT, false>(a, w.allow_ragged, s);
    return rc > 0 ? ASCAN_OK : (rc == 0 ? ASCAN_EINVAL : rc);
  }
  if (vec && use_tma() && a.N >= tma::Fmt<T>::kElemsPerRow) {
    const int rc = causal ? launch_bwd_tma<T, IdxT, true>(a, w.allow_ragged, s) : launch_bwd_tma<T, IdxT, false>(a, w.allow_ragged, s);
    if (rc != 0) return rc > 0 ? ASCAN_OK : rc;
  }
  if (vec)
    bwd_dispatch<T, IdxT, kVec>(a, causal != 0, s);
  else
    bwd_dispatch<T, IdxT, 1>(a, causal != 0, s);
  return launch_status();
}

// ---- bidirectional pairs --------------------------------------------------

// One cooperative launch for the two scans of a bidirectional pair (same
// geometry and cu_seqlens, independent data).  1: launched, 0: not possible
// here (the caller runs the two scans one after the other), <0: error.
template <typename T, typename IdxT, int P, bool RG>
static int launch_fwd_bidi_sched(const FwdArgs<T, IdxT>& fa, const FwdArgs<T, IdxT>& ba,
                                 tma::TileSched fs, tma::TileSched bs, cudaStream_t s) {
  constexpr int NS = ring_depth<T, 2, 1, P, RG>();
  constexpr size_t smem = tma::smem_bytes<2, 1, NS, T, P, RG>();
  static_assert(smem <= kSmemBudget, "TMA forward ring does not fit in shared memory");
  const int64_t rows = fa.N / tma::Fmt<T, P>::kElemsPerRow;
  constexpr int kPart = tma::Fmt<T, P>::kRows / tma::kConsumerWarps;
  constexpr int kInRows = tma::Fmt<T, P>::kRows + (RG ? 1 : 0);
  CUtensorMap fg, fx, fy, bg, bx, by;
  if (!make_map<T>(&fg, fa.g, rows, kInRows) || !make_map<T>(&fx, fa.x, rows, kInRows) ||
      !make_map<T>(&fy, fa.y, rows, kPart) || !make_map<T>(&bg, ba.g, rows, kInRows) ||
      !make_map<T>(&bx, ba.x, rows, kInRows) || !make_map<T>(&by, ba.y, rows, kPart))
    return 0;
  const void* kern = reinterpret_cast<const void*>(scan_fwd_bidi_tma_kernel<T, IdxT, NS, P, RG>);
  const int cap = coop_capacity(kern, smem);
  if (cap <= 0) return cap;
  uint32_t grid = 0;
  if (!split_bidi(cap, fs, bs, grid)) return 0;
  int64_t n_tma_total = rows * tma::Fmt<T, P>::kElemsPerRow;
  FwdArgs<T, IdxT> f = fa, b = ba;
  f.num_tiles = fs.num_tiles;
  b.num_tiles = bs.num_tiles;
  uint32_t* err_host = g_err_host;
  void* params[] = {&fg, &fx, &fy, &bg, &bx, &by, &f, &b, &n_tma_total, &fs, &bs, &err_host};
  return launch_coop_grid(kern, smem, grid, params, s);
}

template <typename T, typename IdxT, int P, bool RG>
static int launch_bwd_bidi_sched(const BwdArgs<T, IdxT>& fa, const BwdArgs<T, IdxT>& ba,
                                 tma::TileSched fs, tma::TileSched bs, cudaStream_t s) {
  constexpr int NS = ring_depth<T, 3, 2, P, RG>();
  constexpr size_t smem = tma::smem_bytes<3, 2, NS, T, P, RG>();
  static_assert(smem <= kSmemBudget, "TMA backward ring does not fit in shared memory");
  const int64_t rows = fa.N / tma::Fmt<T, P>::kElemsPerRow;
  constexpr int kPart = tma::Fmt<T, P>::kRows / tma::kConsumerWarps;
  constexpr int kInRows = tma::Fmt<T, P>::kRows + (RG ? 1 : 0);
  CUtensorMap m[10];
  const BwdArgs<T, IdxT>* both[2] = {&fa, &ba};
  for (int d = 0; d < 2; ++d) {
    const BwdArgs<T, IdxT>& a = *both[d];
    CUtensorMap* md = m + 5 * d;
    if (!make_map<T>(&md[0], a.dy, rows, kInRows) || !make_map<T>(&md[1], a.g, rows, kInRows) ||
        !make_map<T>(&md[2], a.h, rows, kInRows) || !make_map<T>(&md[3], a.dx, rows, kPart) ||
        !make_map<T>(&md[4], a.dg, rows, kPart))
      return 0;
  }
  const void* kern = reinterpret_cast<const void*>(scan_bwd_bidi_tma_kernel<T, IdxT, NS, P, RG>);
  const int cap = coop_capacity(kern, smem);
  if (cap <= 0) return cap;
  uint32_t grid = 0;
  if (!split_bidi(cap, fs, bs, grid)) return 0;
  int64_t n_tma_total = rows * tma::Fmt<T, P>::kElemsPerRow;
  BwdArgs<T, IdxT> f = fa, b = ba;
  f.num_tiles = fs.num_tiles;
  b.num_tiles = bs.num_tiles;
  uint32_t* err_host = g_err_host;
  void* params[] = {&m[0], &m[1], &m[2], &m[3], &m[4], &m[5], &m[6], &m[7], &m[8], &m[9],
                    &f,    &b,    &n_tma_total, &fs, &bs, &err_host};
  return launch_coop_grid(kern, smem, grid, params, s);
}

// Tile order and kernel variant of a bidirectional launch at tile width P.
template <typename T, typename IdxT, int P>
static int launch_fwd_bidi_p(const FwdArgs<T, IdxT>& fa, const FwdArgs<T, IdxT>& ba,
                             bool allow_ragged, cudaStream_t s, bool row_hint = false) {
  const tma::TileSched sch =
      make_sched(tma::Geo<P>::kTileElems, fa.N, fa.BL, fa.S, allow_ragged, row_hint);
  if constexpr (staged_fits<T, 2, 1, P>()) {
    if (!sch.ragged) return launch_fwd_bidi_sched<T, IdxT, P, false>(fa, ba, sch, sch, s);
  }
  return launch_fwd_bidi_sched<T, IdxT, P, true>(fa, ba, sch, sch, s);
}

template <typename T, typename IdxT, int P>
static int launch_bwd_bidi_p(const BwdArgs<T, IdxT>& fa, const BwdArgs<T, IdxT>& ba,
                             bool allow_ragged, cudaStream_t s) {
  const tma::TileSched sch = make_sched(tma::Geo<P>::kTileElems, fa.N, fa.BL, fa.S, allow_ragged);
  if constexpr (staged_fits<T, 3, 2, P>()) {
    if (!sch.ragged) return launch_bwd_bidi_sched<T, IdxT, P, false>(fa, ba, sch, sch, s);
  }
  return launch_bwd_bidi_sched<T, IdxT, P, true>(fa, ba, sch, sch, s);
}

// Causal scan of (gf, xf) and reverse scan of (gb, xb): one launch when the
// persistent kernels apply, else the two scans one after the other.
template <typename T, typename IdxT>
int fwd_bidi_typed(const void* gf, const void* xf, void* yf, const void* gb,
                          const void* xb, void* yb, const void* cu, int64_t S, int64_t C,
                          int64_t BL, const Workspace& wf, const Workspace& wb, cudaStream_t s) {
  const int64_t N = C * BL;
  const bool vec = aligned16(gf) && aligned16(xf) && aligned16(yf) && aligned16(gb) &&
                   aligned16(xb) && aligned16(yb);
  if (vec && use_tma() && N >= tma::Fmt<T>::kElemsPerRow) {
    FwdArgs<T, IdxT> fa{}, ba{};
    const void* in[2][2] = {{gf, xf}, {gb, xb}};
    void* out[2] = {yf, yb};
    const Workspace* ws[2] = {&wf, &wb};
    FwdArgs<T, IdxT>* args[2] = {&fa, &ba};
    for (int d = 0; d < 2; ++d) {
      FwdArgs<T, IdxT>& a = *args[d];
      a.g = static_cast<const T*>(in[d][0]);
      a.x = static_cast<const T*>(in[d][1]);
      a.y = static_cast<T*>(out[d]);
      a.gout = nullptr;
      a.cu = static_cast<const IdxT*>(cu);
      a.S = S;
      a.BL = BL;
      a.N = N;
      a.ticket = ws[d]->ticket;
      a.st = ws[d]->st;
      a.io = RowIO{nullptr, nullptr, nullptr};
    }
    const bool ragged_ok = wf.allow_ragged && wb.allow_ragged;
    bool row_hint = false;
    const int rc = use_wide(N, BL, S, ragged_ok, /*forward=*/true, sizeof(T) == 2, &row_hint)
                       ? launch_fwd_bidi_p<T, IdxT, 32>(fa, ba, ragged_ok, s, row_hint)
                       : launch_fwd_bidi_p<T, IdxT, 16>(fa, ba, ragged_ok, s);
    if (rc != 0) return rc > 0 ? ASCAN_OK : rc;
  }
  const int rc = fwd_typed<T, IdxT>(gf, xf, yf, nullptr, cu, S, C, BL, 0, wf, s);
  if (rc != ASCAN_OK) return rc;
  return fwd_typed<T, IdxT>(gb, xb, yb, nullptr, cu, S, C, BL, 1, wb, s);
}

// Causal adjoint of (dyf, gf, hf) and reverse adjoint of (dyb, gb, hb).
template <typename T, typename IdxT>
int bwd_bidi_typed(const void* const (&in)[2][3], void* const (&out)[2][2], const void* cu,
                          int64_t S, int64_t C, int64_t BL, const Workspace& wf,
                          const Workspace& wb, cudaStream_t s) {
  const int64_t N = C * BL;
  bool vec = true;
  for (int d = 0; d < 2; ++d) {
    for (int k = 0; k < 3; ++k) vec = vec && aligned16(in[d][k]);
    for (int k = 0; k < 2; ++k) vec = vec && aligned16(out[d][k]);
  }
  if (vec && use_tma() && N >= tma::Fmt<T>::kElemsPerRow) {
    BwdArgs<T, IdxT> fa{}, ba{};
    const Workspace* ws[2] = {&wf, &wb};
    BwdArgs<T, IdxT>* args[2] = {&fa, &ba};
    for (int d = 0; d < 2; ++d) {
      BwdArgs<T, IdxT>& a = *args[d];
      a.dy = static_cast<const T*>(in[d][0]);
      a.g = static_cast<const T*>(in[d][1]);
      a.h = static_cast<const T*>(in[d][2]);
      a.dx = static_cast<T*>(out[d][0]);
      a.dg = static_cast<T*>(out[d][1]);
      a.cu = static_cast<const IdxT*>(cu);
      a.S = S;
      a.BL = BL;
      a.N = N;
      a.ticket = ws[d]->ticket;
      a.st = ws[d]->st;
      a.io = RowIO{nullptr, nullptr, nullptr};
    }
    const bool ragged_ok = wf.allow_ragged && wb.allow_ragged;
    int rc;
    if constexpr (kWideBwd<T>)
      rc = use_wide(N, BL, S, ragged_ok, /*forward=*/false)
               ? launch_bwd_bidi_p<T, IdxT, 32>(fa, ba, ragged_ok, s)
               : launch_bwd_bidi_p<T, IdxT, 16>(fa, ba, ragged_ok, s);
    else
      rc = launch_bwd_bidi_p<T, IdxT, 16>(fa, ba, ragged_ok, s);
    if (rc != 0) return rc > 0 ? ASCAN_OK : rc;
  }
  const int rc = bwd_typed<T, IdxT>(in[0][0], in[0][1], in[0][2], out[0][0], out[0][1], cu, S, C,
                                    BL, 1, wf, s);
  if (rc != ASCAN_OK) return rc;
  return bwd_typed<T, IdxT>(in[1][0], in[1][1], in[1][2], out[1][0], out[1][1], cu, S, C, BL, 0,
                            wb, s);
}

template <typename T, typename IdxT>
int shift_pad_typed(const void* data, void* out, const void* cu, int64_t S, int64_t C,
                           int64_t BL, double pad, int backward, int wrap, cudaStream_t s) {
  const int64_t N = C * BL;
  int64_t blocks = (N + kThreads - 1) / kThreads;
  if (blocks > 148 * 64) blocks = 148 * 64;
  shift_pad_kernel<T, IdxT><<<static_cast<unsigned>(blocks), kThreads, 0, s>>>(
      static_cast<const T*>(data), static_cast<T*>(out), static_cast<const IdxT*>(cu), S, BL, N,
      static_cast<float>(pad), backward, wrap);
  return launch_status();
}

static int check_common(const void* cu, int cu_type, int64_t S, int64_t C, int64_t BL, int dtype) {
  if (!cu || S < 0 || C < 0 || BL < 0) return ASCAN_EINVAL;
  if (cu_type != ASCAN_I32 && cu_type != ASCAN_I64) return ASCAN_EINVAL;
  if (dtype != ASCAN_F32 && dtype != ASCAN_F16 && dtype != ASCAN_BF16) return ASCAN_EINVAL;
  if (BL > 0 && C > INT64_MAX / BL) return ASCAN_EINVAL;
  // tile indices are 32-bit
  if (status_slots(C, BL, false) > 0xffffffffull) return ASCAN_EINVAL;
  return ASCAN_OK;
}

}  // namespace ascan

// ---------------------------------------------------------------------------
// Launchers compiled by the units (explicit instantiations live there), and
// the per-unit error-word accessors
// ---------------------------------------------------------------------------

namespace ascan {

#define ASCAN_FOR_EACH_TYPE_PAIR(X)                                                           \
  X(float, int32_t)                                                                           \
  X(float, int64_t)                                                                           \
  X(__half, int32_t)                                                                          \
  X(__half, int64_t)                                                                          \
  X(__nv_bfloat16, int32_t)                                                                   \
  X(__nv_bfloat16, int64_t)

#define ASCAN_DECL_FWD(T, I)                                                                  \
  template int fwd_typed<T, I>(const void*, const void*, void*, void*, const void*, int64_t,  \
                               int64_t, int64_t, int, const Workspace&, cudaStream_t,         \
                               const RowIO&);
#define ASCAN_DECL_BWD(T, I)                                                                  \
  template int bwd_typed<T, I>(const void*, const void*, const void*, void*, void*,           \
                               const void*, int64_t, int64_t, int64_t, int, const Workspace&, \
                               cudaStream_t, const RowIO&);
#define ASCAN_DECL_FWD_BIDI(T, I)                                                             \
  template int fwd_bidi_typed<T, I>(const void*, const void*, void*, const void*,             \
                                    const void*, void*, const void*, int64_t, int64_t,        \
                                    int64_t, const Workspace&, const Workspace&,              \
                                    cudaStream_t);
#define ASCAN_DECL_BWD_BIDI(T, I)                                                             \
  template int bwd_bidi_typed<T, I>(const void* const (&)[2][3], void* const (&)[2][2],       \
                                    const void*, int64_t, int64_t, int64_t, const Workspace&, \
                                    const Workspace&, cudaStream_t);
#define ASCAN_DECL_SHIFT_PAD(T, I)                                                            \
  template int shift_pad_typed<T, I>(const void*, void*, const void*, int64_t, int64_t,       \
                                     int64_t, double, int, int, cudaStream_t);

// Every unit that does not define a launcher sees only its declaration.
#define ASCAN_EXTERN(DECL) extern DECL
#define ASCAN_EXTERN_FWD(T, I) ASCAN_EXTERN(ASCAN_DECL_FWD(T, I))
#define ASCAN_EXTERN_BWD(T, I) ASCAN_EXTERN(ASCAN_DECL_BWD(T, I))
#define ASCAN_EXTERN_FWD_BIDI(T, I) ASCAN_EXTERN(ASCAN_DECL_FWD_BIDI(T, I))
#define ASCAN_EXTERN_BWD_BIDI(T, I) ASCAN_EXTERN(ASCAN_DECL_BWD_BIDI(T, I))
#define ASCAN_EXTERN_SHIFT_PAD(T, I) ASCAN_EXTERN(ASCAN_DECL_SHIFT_PAD(T, I))
ASCAN_FOR_EACH_TYPE_PAIR(ASCAN_EXTERN_FWD)
ASCAN_FOR_EACH_TYPE_PAIR(ASCAN_EXTERN_BWD)
ASCAN_FOR_EACH_TYPE_PAIR(ASCAN_EXTERN_FWD_BIDI)
ASCAN_FOR_EACH_TYPE_PAIR(ASCAN_EXTERN_BWD_BIDI)
ASCAN_FOR_EACH_TYPE_PAIR(ASCAN_EXTERN_SHIFT_PAD)

// The units with kernels, each with its own error word: op 0 reads it into
// (*code, *detail), op 1 clears it (current device; no synchronisation).
#define ASCAN_UNITS(X) X(fwd_f32) X(fwd_f16) X(fwd_bf16) X(bwd_f32) X(bwd_f16) X(bwd_bf16) X(bidi) X(misc)
#define ASCAN_DECL_UNIT_ERR(NAME) int unit_err_##NAME(int op, unsigned int* code, unsigned long long* detail);
ASCAN_UNITS(ASCAN_DECL_UNIT_ERR)

#define ASCAN_UNIT_ERROR_ACCESSORS(NAME)                                                      \
  int unit_err_##NAME(int op, unsigned int* code, unsigned long long* detail) {               \
    if (op == 0) {                                                                            \
      if (cudaMemcpyFromSymbol(code, g_err_code, sizeof(*code)) != cudaSuccess ||             \
          cudaMemcpyFromSymbol(detail, g_err_detail, sizeof(*detail)) != cudaSuccess)         \
        return ASCAN_ECUDA;                                                                   \
      return ASCAN_OK;                                                                        \
    }                                                                                         \
    const unsigned int zc = 0;                                                                \
    const unsigned long long zd = 0;                                                          \
    if (cudaMemcpyToSymbol(g_err_code, &zc, sizeof(zc)) != cudaSuccess ||                     \
        cudaMemcpyToSymbol(g_err_detail, &zd, sizeof(zd)) != cudaSuccess)                     \
      return ASCAN_ECUDA;                                                                     \
    return ASCAN_OK;                                                                          \
  }

}  // namespace ascan

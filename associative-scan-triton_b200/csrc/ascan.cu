// ascan.cu -- sm_100a kernels and C ABI of the packed-varlen linear scan.
//
// Design (one kernel per direction, every sequence length):
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
#include <stdio.h>

#include "../../include/ascan.h"
#include "ascan_device.cuh"

namespace ascan {

// Sticky per-device error word (ASCAN_DEV_ERR_* bits) and a detail value.
__device__ unsigned int g_err_code = 0;
__device__ unsigned long long g_err_detail = 0;

__device__ __forceinline__ void report(unsigned int bits, unsigned long long detail) {
  if (atomicOr(&g_err_code, bits) == 0u) atomicExch(&g_err_detail, detail);
}

// The first tile checks cu_seqlens once per launch.  Every other tile only
// clamps what it reads (cu_at), so a bad array can never move an access.
template <typename IdxT>
__device__ void validate_cu(const IdxT* __restrict__ cu, int64_t S, int64_t BL) {
  unsigned bits = 0u;
  for (int64_t i = threadIdx.x; i <= S; i += kThreads) {
    const int64_t v = static_cast<int64_t>(__ldg(cu + i));
    if (v < 0 || v > BL) bits |= ASCAN_DEV_ERR_CU_ORDER;
    if (i < S && static_cast<int64_t>(__ldg(cu + i + 1)) < v) bits |= ASCAN_DEV_ERR_CU_ORDER;
    if (i == S && v != BL) bits |= ASCAN_DEV_ERR_CU_END;
  }
  if (bits) report(bits, 0ull);
}

// Tile-level tail shared by the forward and backward kernels: chains the warp
// totals, publishes this tile's status, looks back when the tile's first
// element does not start a sequence, and returns the prefix that precedes
// this warp's first element in scan order.
template <bool REV>
__device__ __forceinline__ Pfx tile_prefix(Pfx warp_total, bool first_is_head, uint32_t ticket,
                                           const TileStatus& st, int warp, int lane) {
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
            timed_out = true;  // treated as an empty inclusive prefix
          }
        }
        const unsigned incmask = __ballot_sync(kFull, inc);
        const int stop = incmask ? (__ffs(incmask) - 1) : 31;
        if (lane > stop) x = pfx_empty();
        // x_stop o ... o x_1 o x_0 (a higher lane is an earlier tile)
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
      if (__any_sync(kFull, timed_out) && lane == 0) report(ASCAN_DEV_ERR_LOOKBACK, ticket);
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

template <typename T, typename IdxT>
struct FwdArgs {
  const T* g;
  const T* x;
  T* y;
  T* gout;
  const IdxT* cu;
  int64_t S, BL, N;
  uint32_t num_tiles;
  uint32_t* ticket;
  TileStatus st;
};

// Row position of flat index p.
__device__ __forceinline__ int64_t row_pos(int64_t p, int64_t BL, bool small) {
  return small ? static_cast<int64_t>(static_cast<uint32_t>(p) % static_cast<uint32_t>(BL))
               : p % BL;
}

template <typename T, typename IdxT, int VEC, bool REV, bool GATES_OUT>
__global__ void __launch_bounds__(kThreads) scan_fwd_kernel(const FwdArgs<T, IdxT> args) {
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
  if (ticket == 0) validate_cu(args.cu, S, BL);

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
  const Pfx wpre = tile_prefix<REV>(carry, first_is_head, ticket, args.st, warp, lane);

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
  T* dx;
  T* dg;
  const IdxT* cu;
  int64_t S, BL, N;
  uint32_t num_tiles;
  uint32_t* ticket;
  TileStatus st;
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
__global__ void __launch_bounds__(kThreads) scan_bwd_kernel(const BwdArgs<T, IdxT> args) {
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
  if (ticket == 0) validate_cu(args.cu, S, BL);

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
  const Pfx wpre = tile_prefix<REV>(carry, first_is_head, ticket, args.st, warp, lane);

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

struct Workspace {
  uint32_t* ticket;
  TileStatus st;
  size_t clear_bytes;
};

static size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

static size_t tiles_of(int64_t n) { return static_cast<size_t>((n + kTile - 1) / kTile); }

static size_t workspace_bytes_for(int64_t n) {
  const size_t tiles = tiles_of(n);
  return 256 + align256(tiles * sizeof(uint32_t)) + tiles * sizeof(float4);
}

static int carve(void* ws, size_t ws_bytes, int64_t n, Workspace& out) {
  if (!ws || (reinterpret_cast<uintptr_t>(ws) & 255u) != 0) return ASCAN_EWORKSPACE;
  if (ws_bytes < workspace_bytes_for(n)) return ASCAN_EWORKSPACE;
  char* base = static_cast<char*>(ws);
  const size_t tiles = tiles_of(n);
  out.ticket = reinterpret_cast<uint32_t*>(base);
  out.st.flags = reinterpret_cast<uint32_t*>(base + 256);
  out.st.vals = reinterpret_cast<float4*>(base + 256 + align256(tiles * sizeof(uint32_t)));
  out.clear_bytes = 256 + align256(tiles * sizeof(uint32_t));
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

template <typename T, typename IdxT, int VEC>
static void fwd_dispatch(const FwdArgs<T, IdxT>& a, bool reverse, bool gout, cudaStream_t s) {
  const dim3 grid(a.num_tiles), block(kThreads);
  if (reverse) {
    if (gout)
      scan_fwd_kernel<T, IdxT, VEC, true, true><<<grid, block, 0, s>>>(a);
    else
      scan_fwd_kernel<T, IdxT, VEC, true, false><<<grid, block, 0, s>>>(a);
  } else {
    if (gout)
      scan_fwd_kernel<T, IdxT, VEC, false, true><<<grid, block, 0, s>>>(a);
    else
      scan_fwd_kernel<T, IdxT, VEC, false, false><<<grid, block, 0, s>>>(a);
  }
}

template <typename T, typename IdxT>
static int fwd_typed(const void* g, const void* x, void* y, void* gout, const void* cu,
                     int64_t S, int64_t C, int64_t BL, int reverse, const Workspace& w,
                     cudaStream_t s) {
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
  const bool vec = aligned16(g) && aligned16(x) && aligned16(y) && (!gout || aligned16(gout));
  constexpr int kVec = 16 / sizeof(T);
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
    scan_bwd_kernel<T, IdxT, VEC, true><<<grid, block, 0, s>>>(a);
  else
    scan_bwd_kernel<T, IdxT, VEC, false><<<grid, block, 0, s>>>(a);
}

template <typename T, typename IdxT>
static int bwd_typed(const void* dy, const void* g, const void* h, void* dx, void* dg,
                     const void* cu, int64_t S, int64_t C, int64_t BL, int causal,
                     const Workspace& w, cudaStream_t s) {
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
  const bool vec = aligned16(dy) && aligned16(g) && aligned16(h) && aligned16(dx) && aligned16(dg);
  constexpr int kVec = 16 / sizeof(T);
  if (vec)
    bwd_dispatch<T, IdxT, kVec>(a, causal != 0, s);
  else
    bwd_dispatch<T, IdxT, 1>(a, causal != 0, s);
  return launch_status();
}

template <typename T, typename IdxT>
static int shift_pad_typed(const void* data, void* out, const void* cu, int64_t S, int64_t C,
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
  if (tiles_of(C * BL) > 0xffffffffull) return ASCAN_EINVAL;
  return ASCAN_OK;
}

}  // namespace ascan

using namespace ascan;

extern "C" {

int ascan_abi_version(void) { return ASCAN_ABI_VERSION; }

const char* ascan_build_info(void) {
  return "ascan sm_100a: decoupled look-back tile scan, 4096-element tiles, 256 threads, "
         "128-bit vector IO, fp32 accumulation";
}

const char* ascan_strerror(int status) {
  switch (status) {
    case ASCAN_OK: return "ok";
    case ASCAN_EINVAL: return "invalid argument (size, dtype, flag or null pointer)";
    case ASCAN_EWORKSPACE: return "workspace missing, not 256-byte aligned or too small";
    case ASCAN_ECUDA: return "CUDA launch or memset failed";
    case ASCAN_EDEVICE: return "no usable CUDA device";
    default: return "unknown ascan status";
  }
}

size_t ascan_workspace_size(int64_t num_channels, int64_t seq_total, int dtype) {
  (void)dtype;
  if (num_channels <= 0 || seq_total <= 0) return 256;
  return workspace_bytes_for(num_channels * seq_total);
}

#define ASCAN_DISPATCH_TYPES(DTYPE, CUT, CALL)                                         \
  do {                                                                                 \
    if ((DTYPE) == ASCAN_F32) {                                                        \
      if ((CUT) == ASCAN_I32) return CALL(float, int32_t);                             \
      return CALL(float, int64_t);                                                     \
    } else if ((DTYPE) == ASCAN_F16) {                                                 \
      if ((CUT) == ASCAN_I32) return CALL(__half, int32_t);                            \
      return CALL(__half, int64_t);                                                    \
    } else {                                                                           \
      if ((CUT) == ASCAN_I32) return CALL(__nv_bfloat16, int32_t);                     \
      return CALL(__nv_bfloat16, int64_t);                                             \
    }                                                                                  \
  } while (0)

int ascan_forward(const void* gates, const void* tokens, void* tokens_out, void* gates_out,
                  const void* cu_seqlens, int cu_index_type, int64_t num_seq,
                  int64_t num_channels, int64_t seq_total, int dtype, int reverse,
                  void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_common(cu_seqlens, cu_index_type, num_seq, num_channels, seq_total, dtype);
  if (rc != ASCAN_OK) return rc;
  if (!gates || !tokens || !tokens_out) return ASCAN_EINVAL;
  const int64_t n = num_channels * seq_total;
  if (n == 0 || num_seq == 0) return ASCAN_OK;
  Workspace w;
  rc = carve(workspace, workspace_bytes, n, w);
  if (rc != ASCAN_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(w.ticket, 0, w.clear_bytes, s) != cudaSuccess) return ASCAN_ECUDA;
#define ASCAN_FWD_CALL(T, I)                                                                   \
  fwd_typed<T, I>(gates, tokens, tokens_out, gates_out, cu_seqlens, num_seq, num_channels,     \
                  seq_total, reverse, w, s)
  ASCAN_DISPATCH_TYPES(dtype, cu_index_type, ASCAN_FWD_CALL);
#undef ASCAN_FWD_CALL
}

int ascan_backward(const void* grad, const void* gates, const void* states, void* d_tokens,
                   void* d_gates, const void* cu_seqlens, int cu_index_type, int64_t num_seq,
                   int64_t num_channels, int64_t seq_total, int dtype, int causal,
                   void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_common(cu_seqlens, cu_index_type, num_seq, num_channels, seq_total, dtype);
  if (rc != ASCAN_OK) return rc;
  if (!grad || !gates || !states || !d_tokens || !d_gates) return ASCAN_EINVAL;
  // The shifted reads of gates and states cross thread boundaries, so the
  // outputs must not overwrite them.
  if (d_gates == gates || d_gates == states || d_tokens == gates || d_tokens == states ||
      d_tokens == d_gates)
    return ASCAN_EINVAL;
  const int64_t n = num_channels * seq_total;
  if (n == 0 || num_seq == 0) return ASCAN_OK;
  Workspace w;
  rc = carve(workspace, workspace_bytes, n, w);
  if (rc != ASCAN_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(w.ticket, 0, w.clear_bytes, s) != cudaSuccess) return ASCAN_ECUDA;
#define ASCAN_BWD_CALL(T, I)                                                                    \
  bwd_typed<T, I>(grad, gates, states, d_tokens, d_gates, cu_seqlens, num_seq, num_channels,    \
                  seq_total, causal, w, s)
  ASCAN_DISPATCH_TYPES(dtype, cu_index_type, ASCAN_BWD_CALL);
#undef ASCAN_BWD_CALL
}

int ascan_shift_pad(const void* data, void* out, const void* cu_seqlens, int cu_index_type,
                    int64_t num_seq, int64_t num_channels, int64_t seq_total, int dtype,
                    double pad_value, int backward, int wrap, void* stream) {
  int rc = check_common(cu_seqlens, cu_index_type, num_seq, num_channels, seq_total, dtype);
  if (rc != ASCAN_OK) return rc;
  if (!data || !out || data == out) return ASCAN_EINVAL;
  if (num_channels * seq_total == 0 || num_seq == 0) return ASCAN_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define ASCAN_SP_CALL(T, I)                                                                    \
  shift_pad_typed<T, I>(data, out, cu_seqlens, num_seq, num_channels, seq_total, pad_value,    \
                        backward, wrap, s)
  ASCAN_DISPATCH_TYPES(dtype, cu_index_type, ASCAN_SP_CALL);
#undef ASCAN_SP_CALL
}

int ascan_get_device_error(int device, unsigned int* code, long long* detail) {
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) return ASCAN_EDEVICE;
  if (cudaSetDevice(device) != cudaSuccess) return ASCAN_EDEVICE;
  int rc = ASCAN_OK;
  unsigned int c = 0;
  unsigned long long d = 0;
  if (cudaDeviceSynchronize() != cudaSuccess ||
      cudaMemcpyFromSymbol(&c, g_err_code, sizeof(c)) != cudaSuccess ||
      cudaMemcpyFromSymbol(&d, g_err_detail, sizeof(d)) != cudaSuccess)
    rc = ASCAN_ECUDA;
  cudaSetDevice(prev);
  if (code) *code = c;
  if (detail) *detail = static_cast<long long>(d);
  return rc;
}

int ascan_clear_device_error(int device) {
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) return ASCAN_EDEVICE;
  if (cudaSetDevice(device) != cudaSuccess) return ASCAN_EDEVICE;
  const unsigned int zc = 0;
  const unsigned long long zd = 0;
  int rc = ASCAN_OK;
  if (cudaMemcpyToSymbol(g_err_code, &zc, sizeof(zc)) != cudaSuccess ||
      cudaMemcpyToSymbol(g_err_detail, &zd, sizeof(zd)) != cudaSuccess)
    rc = ASCAN_ECUDA;
  cudaSetDevice(prev);
  return rc;
}

}  // extern "C"

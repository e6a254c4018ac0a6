// ascan_slab.cuh -- per-row aggregates of a time slab by a bandwidth-bound row
// reduction: the aggregate-only passes of ascan_forward_slab (tokens_out ==
// NULL) and ascan_backward_slab (d_tokens == d_gates == NULL).
//
// A time-sharded run only needs, per row, the inclusive (product, value) of
// the slab's last sequence piece in scan order.  That is a reduction with the
// scan's (associative, not commutative) operator, so it needs no look-back, no
// carry and no stores: warps stream contiguous ranges with 16-byte loads,
// fold their lanes' vectors, combine the 32 lanes in order by a shuffle tree
// and chain their tiles.  Work is balanced over warps, not rows: the rows'
// pieces are laid end to end and every warp of a grid of resident CTAs takes
// one contiguous, equal share (which may cross a row end), so no warp idles
// while another finishes a long part.  Each warp leaves one partial per row
// it touched in the workspace, and the last warp to finish a row combines
// that row's partials in order (no warp ever waits for another).
//
// The pieces, with lo = the last sequence start before L and hi = the first
// sequence end after 0 (cu[0] = 0 for a slab):
//   forward, causal     fold (g, x) left to right over [lo, L)
//   forward, reverse    fold (g, x) right to left over [0, hi)
//   backward, causal    dh[t] = dy[t] + g[t+1] dh[t+1] at column 0: with
//                       w_u = g[u] (dy[u] + w_{u+1}), dh[0] = dy[0] + w_1, so
//                       fold (g, g dy) right to left over [1, hi), no shifted
//                       operand; the product also takes g[hi] when hi < L (the
//                       sequence end's own coefficient, as the scan kernels
//                       count it) and 1 for the row's last column
//   backward, reverse   the mirror image: fold (g, g dy) left to right over
//                       [lo, L-1), dh[L-1] = dy[L-1] + w_{L-2}, product times
//                       g[lo-1] when lo > 0
// The row carry enters only when the piece starts at the row's first element
// in scan order (the forward composes (product, state); the backward adds
// product x carry to the adjoint).  Results equal the scan kernels' aggregates
// up to fp32 reassociation.
#pragma once

namespace ascan {
namespace slab {

constexpr int kAggThreads = 256;
constexpr int kAggWarps = kAggThreads / 32;
constexpr int kAggUnroll = 8;       // 16-byte loads of each input per lane in flight
constexpr int kAggCtasPerSm = 2;    // 128 KB in flight per SM; up to 128 registers: no spills
constexpr int64_t kAggMinShare = 32 * kAggUnroll;  // vectors: a warp's share is at least one round

template <typename T, typename IdxT>
struct AggArgs {
  const T* a;          // gates
  const T* b;          // tokens (forward) or grad (backward)
  const IdxT* cu;
  int64_t S, L, C;
  const float* carry;  // nullable: forward [C][2], backward [C]
  float* agg;          // [C][2]
  uint32_t* counters;  // [C], zeroed
  float2* partials;    // [C][per_row]: one per warp that touches the row
  uint32_t per_row;    // >= ceil(warps / C) + 1, the most warps one row can span
  uint32_t* err_host;  // nullable pinned host error flag
};

struct Pair {
  float p, y;  // product of the coefficients, value from a zero start
};

// "l then r" in scan order
__device__ __forceinline__ Pair seq(const Pair& l, const Pair& r) {
  return Pair{l.p * r.p, fmaf(r.p, l.y, r.y)};
}

// Piece boundary of the row (same for every row): L2R needs lo (the last
// sequence start below L), R2L needs hi (the first sequence end above 0).
// Called by all threads; returns the same value in all of them.
template <typename IdxT, bool R2L>
__device__ __forceinline__ int64_t piece_edge(const IdxT* cu, int64_t S, int64_t L) {
  __shared__ unsigned long long s_edge;
  if (threadIdx.x == 0) s_edge = R2L ? static_cast<unsigned long long>(L) : 0ull;
  __syncthreads();
  if (S + 1 <= 4096) {
    unsigned long long best = R2L ? static_cast<unsigned long long>(L) : 0ull;
    for (int64_t i = threadIdx.x; i <= S; i += kAggThreads) {
      const int64_t v = cu_at(cu, i, L);
      if (!R2L && i < S && v < L && static_cast<unsigned long long>(v) > best) best = v;
      if (R2L && i >= 1 && v > 0 && static_cast<unsigned long long>(v) < best) best = v;
    }
    if (R2L)
      atomicMin(&s_edge, best);
    else
      atomicMax(&s_edge, best);
  } else if (threadIdx.x == 0) {
    // sorted entries: binary search (any input gives an index in range)
    int64_t lo = 0, hi = S + 1;
    if (!R2L) {  // first index with cu >= L, then the entry before it
      while (lo < hi) {
        const int64_t m = (lo + hi) >> 1;
        if (cu_at(cu, m, L) < L) lo = m + 1; else hi = m;
      }
      s_edge = lo > 0 ? static_cast<unsigned long long>(cu_at(cu, lo - 1, L)) : 0ull;
    } else {  // first index >= 1 with cu > 0
      lo = 1;
      while (lo < hi) {
        const int64_t m = (lo + hi) >> 1;
        if (cu_at(cu, m, L) > 0) hi = m; else lo = m + 1;
      }
      s_edge = lo <= S ? static_cast<unsigned long long>(cu_at(cu, lo, L)) : L;
    }
  }
  __syncthreads();
  return static_cast<int64_t>(s_edge);
}

// VEC elements of vector v of both arrays as (coefficient, value) pairs;
// elements outside [q0, q1) (flat indices) are identities.
template <typename T, int VEC, bool BWD>
__device__ __forceinline__ void load_pairs(const T* a, const T* b, int64_t v, int64_t q0, int64_t q1,
                                           int64_t N, float (&pa)[VEC], float (&pb)[VEC]) {
  const int64_t e0 = v * VEC;
  if (e0 >= q0 && e0 + VEC <= q1 && e0 + VEC <= N) {
    unpack16<T>(ld_stream_v4(a + e0), pa);
    unpack16<T>(ld_stream_v4(b + e0), pb);
  } else {
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      const int64_t q = e0 + j;
      const bool in = q >= q0 && q < q1;
      pa[j] = in ? Cvt<T>::to(a[q]) : 1.f;
      pb[j] = in ? Cvt<T>::to(b[q]) : 0.f;
    }
  }
  if constexpr (BWD) {
#pragma unroll
    for (int j = 0; j < VEC; ++j) pb[j] *= pa[j];  // g dy (identity stays 0)
  }
}

template <int VEC, bool R2L>
__device__ __forceinline__ Pair fold_lane(const float (&pa)[VEC], const float (&pb)[VEC]) {
  Pair r{1.f, 0.f};
#pragma unroll
  for (int jj = 0; jj < VEC; ++jj) {
    const int j = R2L ? VEC - 1 - jj : jj;
    r.y = fmaf(pa[j], r.y, pb[j]);
    r.p *= pa[j];
  }
  return r;
}

// Ordered combination of the 32 lanes' pairs (lane 0 gets the warp's total).
template <bool R2L>
__device__ __forceinline__ Pair warp_total(Pair x, int lane) {
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const Pair o{__shfl_down_sync(kFull, x.p, off), __shfl_down_sync(kFull, x.y, off)};
    if (lane + off < 32) x = R2L ? seq(o, x) : seq(x, o);
  }
  return x;
}

// The 16-byte word of p holding elements [e0, e0 + VEC), with `ident` in
// place of every element outside [q0, q1) (only those inside are read).
template <typename T>
__device__ __noinline__ uint4 masked_word(const T* p, int64_t e0, int64_t q0, int64_t q1, float ident) {
  constexpr int VEC = 16 / sizeof(T);
  union {
    uint4 w;
    T v[VEC];
  } r;
#pragma unroll
  for (int j = 0; j < VEC; ++j) {
    const int64_t q = e0 + j;
    r.v[j] = q >= q0 && q < q1 ? p[q] : Cvt<T>::from(ident);
  }
  return r.w;
}

// Ordered fold of one row's vectors [f0, f1) (flat vector indices) by one
// warp; elements outside [q0, q1) are identities.  Each round issues all its
// loads (raw 16-byte words, unpacked only when folded) before folding any.
// Lane 0's result counts.
template <typename T, bool R2L, bool BWD>
__device__ __forceinline__ Pair fold_range(const T* a, const T* b, int64_t f0, int64_t f1,
                                           int64_t q0, int64_t q1, int64_t N, int lane) {
  constexpr int VEC = 16 / sizeof(T);
  const int64_t qe = q1 < N ? q1 : N;
  Pair acc{1.f, 0.f};
  for (int64_t t0 = f0; t0 < f1; t0 += 32 * kAggUnroll) {
    uint4 ra[kAggUnroll], rb[kAggUnroll];
#pragma unroll
    for (int u = 0; u < kAggUnroll; ++u) {
      const int64_t v = t0 + 32 * u + lane, e0 = v * VEC;
      if (v < f1 && e0 >= q0 && e0 + VEC <= qe) {
        ra[u] = ld_stream_v4(a + e0);
        rb[u] = ld_stream_v4(b + e0);
      } else {  // a piece edge, or past this warp's range: identities
        const int64_t hi = v < f1 ? qe : q0;
        ra[u] = masked_word<T>(a, e0, q0, hi, 1.f);
        rb[u] = masked_word<T>(b, e0, q0, hi, 0.f);
      }
    }
#pragma unroll
    for (int u = 0; u < kAggUnroll; ++u) {
      float pa[VEC], pb[VEC];
      unpack16<T>(ra[u], pa);
      unpack16<T>(rb[u], pb);
      if constexpr (BWD) {
#pragma unroll
        for (int j = 0; j < VEC; ++j) pb[j] *= pa[j];  // g dy (identity stays 0)
      }
      const Pair tile = warp_total<R2L>(fold_lane<VEC, R2L>(pa, pb), lane);
      acc = R2L ? seq(tile, acc) : seq(acc, tile);
    }
  }
  return acc;
}

template <typename T, typename IdxT, bool R2L, bool BWD>
__global__ void __launch_bounds__(kAggThreads, kAggCtasPerSm)
    slab_aggregate_kernel(const AggArgs<T, IdxT> args) {
  constexpr int VEC = 16 / sizeof(T);
  const int64_t L = args.L, C = args.C, N = C * L;
  if (blockIdx.x == 0) validate_cu(args.cu, args.S, L, args.err_host);
  const int64_t edge = piece_edge<IdxT, R2L>(args.cu, args.S, L);
  // the piece [rs, re) of every row, in row positions
  int64_t rs, re;
  if (!BWD) {
    rs = R2L ? 0 : edge;
    re = R2L ? edge : L;
  } else {
    rs = R2L ? 1 : edge;
    re = R2L ? edge : L - 1;
  }
  if (re < rs) re = rs;
  const bool whole = R2L ? edge == L : edge == 0;  // the piece starts at the row's first element in scan order
  // vectors per row: the piece's span, plus one when rows or the piece do not
  // start on a vector (a fully masked vector reads nothing); at least one, so
  // every row gets a partial and a finishing warp
  const bool aligned = L % VEC == 0 && rs % VEC == 0;
  int64_t nv = aligned ? (re - rs + VEC - 1) / VEC : (re - rs + 2 * VEC - 2) / VEC;
  if (nv < 1) nv = 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * kAggWarps;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * kAggWarps + warp;
  const int64_t total = C * nv;
  // per_row == 0 (a workspace too small for two partials per row): whole
  // rows per warp, no partials
  const int64_t share = args.per_row != 0u ? (total + warps - 1) / warps
                                           : ((C + warps - 1) / warps) * nv;
  int64_t j0 = gw * share;
  const int64_t j1 = j0 + share < total ? j0 + share : total;
  while (j0 < j1) {
    const int64_t row = j0 / nv;
    const int64_t row_end = (row + 1) * nv < j1 ? (row + 1) * nv : j1;
    const int64_t q0 = row * L + rs, q1 = row * L + re;
    const int64_t f = q0 / VEC;  // the row piece's first vector
    const Pair part = fold_range<T, R2L, BWD>(args.a, args.b, f + (j0 - row * nv),
                                              f + (row_end - row * nv), q0, q1, N, lane);
    // warps [first, last] share this row; this one is number gw - first
    const int64_t first = (row * nv) / share;
    const int64_t last = ((row + 1) * nv - 1) / share;
    // a row inside this warp's share is finished here; otherwise the last
    // of its warps to arrive combines the partials
    Pair tot = part;
    bool finish = first == last;
    if (!finish) {
      float2* slots = args.partials + row * args.per_row;
      if (lane == 0) {
        slots[gw - first] = make_float2(part.p, part.y);
        __threadfence();
        finish = atomicAdd(&args.counters[row], 1u) == static_cast<uint32_t>(last - first);
      }
      finish = __shfl_sync(kFull, finish, 0);
      if (finish) {
        __threadfence();
        // ordered combination of the row's partials: each lane folds a
        // contiguous run, the shuffle tree joins the runs
        const int n = static_cast<int>(last - first + 1);
        const int per = (n + 31) / 32;
        Pair acc{1.f, 0.f};
        for (int k = lane * per; k < n && k < (lane + 1) * per; ++k) {
          const float2 pk = __ldcg(&slots[k]);
          const Pair pr{pk.x, pk.y};
          acc = R2L ? seq(pr, acc) : seq(acc, pr);
        }
        tot = warp_total<R2L>(acc, lane);
      }
    }
    if (finish) {
      if (lane == 0) {
        const int64_t base = row * L;
        float P = tot.p, Y = tot.y;
        if (!BWD) {
          if (args.carry && whole) {
            Y = fmaf(P, args.carry[2 * row + 1], Y);
            P *= args.carry[2 * row];
          }
        } else {
          // the element the adjoint is read at, and the sequence end's own coefficient
          const int64_t at = R2L ? 0 : L - 1;
          float D = Cvt<T>::to(args.b[base + at]) + Y;
          if (args.carry && whole) D = fmaf(P, args.carry[row], D);
          if (R2L && edge < L) P *= Cvt<T>::to(args.a[base + edge]);
          if (!R2L && edge > 0) P *= Cvt<T>::to(args.a[base + edge - 1]);
          Y = D;
        }
        args.agg[2 * row] = P;
        args.agg[2 * row + 1] = Y;
      }
    }
    j0 = row_end;
  }
}

}  // namespace slab
}  // namespace ascan

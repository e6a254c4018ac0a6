// ascan_slab.cuh -- per-row aggregates of a time slab by a bandwidth-bound row
// reduction: the aggregate-only passes of ascan_forward_slab (tokens_out ==
// NULL) and ascan_backward_slab (d_tokens == d_gates == NULL).
//
// A time-sharded run only needs, per row, the inclusive (product, value) of
// the slab's last sequence piece in scan order.  That is a reduction with the
// scan's (associative, not commutative) operator, so it needs no look-back, no
// carry and no stores: warps stream contiguous ranges with 16-byte loads,
// fold their lanes' vectors, combine the 32 lanes in order by a shuffle tree,
// chain their tiles, and the CTAs of a row combine their parts in order
// through the workspace (the last CTA of a row to finish does it; no CTA ever
// waits for another).
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
constexpr int kAggUnroll = 4;       // 32-vector tiles per warp in flight
constexpr int kAggCtasPerSm = 4;    // 64 registers per thread: no spills
constexpr int64_t kAggPart = 16384; // elements of a row per CTA (many short waves, small tail)

template <typename T, typename IdxT>
struct AggArgs {
  const T* a;          // gates
  const T* b;          // tokens (forward) or grad (backward)
  const IdxT* cu;
  int64_t S, L, C;
  const float* carry;  // nullable: forward [C][2], backward [C]
  float* agg;          // [C][2]
  uint32_t* counters;  // [C], zeroed (splits > 1)
  float2* partials;    // [C][splits] (splits > 1)
  uint32_t splits;
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

template <typename T, typename IdxT, bool R2L, bool BWD>
__global__ void __launch_bounds__(kAggThreads, kAggCtasPerSm)
    slab_aggregate_kernel(const AggArgs<T, IdxT> args) {
  constexpr int VEC = 16 / sizeof(T);
  const int64_t L = args.L, N = args.C * L;
  const uint32_t splits = args.splits;
  const int64_t row = blockIdx.x / splits;
  const uint32_t part = blockIdx.x - static_cast<uint32_t>(row) * splits;
  if (blockIdx.x == 0) validate_cu(args.cu, args.S, L, args.err_host);
  const int64_t edge = piece_edge<IdxT, R2L>(args.cu, args.S, L);
  // the piece [rs, re) of the row, in row positions
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
  // this CTA's part, in whole vectors of the flat array (elements outside the
  // piece are masked)
  const int64_t q0 = row * L + rs, q1 = row * L + re;
  const int64_t v_lo = q0 / VEC, v_hi = (q1 + VEC - 1) / VEC;
  const int64_t per_part = (v_hi - v_lo + splits - 1) / splits;
  const int64_t pv0 = v_lo + per_part * part;
  const int64_t pv1 = pv0 + per_part < v_hi ? pv0 + per_part : v_hi;
  // this warp's contiguous slice of the part
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n_part = pv1 > pv0 ? pv1 - pv0 : 0;
  const int64_t per_warp = (n_part + kAggWarps - 1) / kAggWarps;
  const int64_t wv0 = pv0 + per_warp * warp;
  const int64_t wv1 = wv0 + per_warp < pv1 ? wv0 + per_warp : pv1;
  Pair acc{1.f, 0.f};
  for (int64_t t0 = wv0; t0 < wv1; t0 += 32 * kAggUnroll) {
    float pa[kAggUnroll][VEC], pb[kAggUnroll][VEC];
#pragma unroll
    for (int u = 0; u < kAggUnroll; ++u) {
      const int64_t v = t0 + 32 * u + lane;
      if (v < wv1) {
        load_pairs<T, VEC, BWD>(args.a, args.b, v, q0, q1, N, pa[u], pb[u]);
      } else {
#pragma unroll
        for (int j = 0; j < VEC; ++j) pa[u][j] = 1.f, pb[u][j] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < kAggUnroll; ++u) {
      const Pair tile = warp_total<R2L>(fold_lane<VEC, R2L>(pa[u], pb[u]), lane);
      acc = R2L ? seq(tile, acc) : seq(acc, tile);  // lane 0's is the one that counts
    }
  }
  __shared__ Pair s_warp[kAggWarps];
  __shared__ bool s_last;
  if (lane == 0) s_warp[warp] = acc;
  __syncthreads();
  if (threadIdx.x != 0) return;
  Pair tot{1.f, 0.f};
#pragma unroll
  for (int w = 0; w < kAggWarps; ++w) tot = R2L ? seq(s_warp[w], tot) : seq(tot, s_warp[w]);
  if (splits > 1) {
    args.partials[row * splits + part] = make_float2(tot.p, tot.y);
    __threadfence();
    s_last = atomicAdd(&args.counters[row], 1u) == splits - 1u;
    if (!s_last) return;
    __threadfence();
    tot = Pair{1.f, 0.f};
    for (uint32_t k = 0; k < splits; ++k) {
      const float2 pk = __ldcg(&args.partials[row * splits + k]);
      const Pair pr{pk.x, pk.y};
      tot = R2L ? seq(pr, tot) : seq(tot, pr);
    }
  }
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

}  // namespace slab
}  // namespace ascan

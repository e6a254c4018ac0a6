// ascan_device.cuh -- device building blocks of the sm_100a scan kernels.
//
// The scan element is the pair (a, b) of the first-order recurrence
// h[t] = a[t] * h[t-1] + b[t]; composing "l then r" gives
// (l.a * r.a, r.a * l.b + r.b), which is the reference's combine operator
// `op` (src/associative_scan_triton/_kernels.py:6-16) with the operands
// named by scan order.  Sequence boundaries from cu_seqlens are carried as a
// HEAD flag: composing anything with a right operand that contains a head
// returns the right operand unchanged (the left one is discarded by select,
// never multiplied by zero), so no value -- not even a NaN or Inf -- crosses
// a document boundary, and the first element of every sequence is stored
// exactly as its input token.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ascan {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr unsigned kFull = 0xffffffffu;
// Every thread owns 16 elements per tile, so a tile is 4096 elements for
// every dtype and load width.
constexpr int kElemsPerThread = 16;
constexpr int kTile = kThreads * kElemsPerThread;

// Prefix flags.
constexpr int kHead = 1;   // a sequence head lies inside the span
constexpr int kValid = 2;  // the span is non-empty

// Tile status values in the lookback workspace.
constexpr uint32_t kStatusNone = 0;
constexpr uint32_t kStatusAggregate = 1;
constexpr uint32_t kStatusInclusive = 2;

// Bounded wait for a predecessor tile (nanoseconds of %globaltimer).
constexpr unsigned long long kLookbackTimeoutNs = 2000000000ull;

struct Pfx {
  float a, b;
  int f;
};

__device__ __forceinline__ Pfx pfx_empty() { return Pfx{1.f, 0.f, 0}; }

// "l then r"; either side may be empty.
__device__ __forceinline__ Pfx compose(const Pfx& l, const Pfx& r) {
  if (!(r.f & kValid)) return l;
  if (!(l.f & kValid) || (r.f & kHead)) return r;
  return Pfx{l.a * r.a, fmaf(r.a, l.b, r.b), l.f | r.f};
}

// "l then r" for two non-empty operands.
__device__ __forceinline__ Pfx compose_nonempty(const Pfx& l, const Pfx& r) {
  if (r.f & kHead) return r;
  return Pfx{l.a * r.a, fmaf(r.a, l.b, r.b), l.f | r.f};
}

// ---------------------------------------------------------------------------
// dtype conversion and 128-bit vector IO
// ---------------------------------------------------------------------------

template <typename T>
struct Cvt;
template <>
struct Cvt<float> {
  static __device__ __forceinline__ float to(float v) { return v; }
  static __device__ __forceinline__ float from(float v) { return v; }
};
template <>
struct Cvt<__half> {
  static __device__ __forceinline__ float to(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from(float v) { return __float2half_rn(v); }
};
template <>
struct Cvt<__nv_bfloat16> {
  static __device__ __forceinline__ float to(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from(float v) { return __float2bfloat16_rn(v); }
};

__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ void st_v4(void* p, uint4 v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

template <typename T>
__device__ __forceinline__ void unpack16(uint4 raw, float* v);
template <>
__device__ __forceinline__ void unpack16<float>(uint4 raw, float* v) {
  v[0] = __uint_as_float(raw.x);
  v[1] = __uint_as_float(raw.y);
  v[2] = __uint_as_float(raw.z);
  v[3] = __uint_as_float(raw.w);
}
template <>
__device__ __forceinline__ void unpack16<__half>(uint4 raw, float* v) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h2 = *reinterpret_cast<const __half2*>(&w[i]);
    float2 f = __half22float2(h2);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void unpack16<__nv_bfloat16>(uint4 raw, float* v) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h2 = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
    float2 f = __bfloat1622float2(h2);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

template <typename T>
__device__ __forceinline__ uint4 pack16(const float* v);
template <>
__device__ __forceinline__ uint4 pack16<float>(const float* v) {
  return make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]),
                    __float_as_uint(v[3]));
}
template <>
__device__ __forceinline__ uint4 pack16<__half>(const float* v) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h2 = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&h2);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}
template <>
__device__ __forceinline__ uint4 pack16<__nv_bfloat16>(const float* v) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h2 = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&h2);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Load VEC consecutive elements starting at flat index p (p >= 0).  With
// VEC*sizeof(T) == 16 the caller guarantees 16-byte alignment of base + p.
// Elements at or past n read as `fill`.
template <typename T, int VEC>
__device__ __forceinline__ void load_vec(const T* __restrict__ base, int64_t p, int64_t n,
                                         float fill, float (&v)[VEC]) {
  if constexpr (VEC * sizeof(T) == 16) {
    if (p + VEC <= n) {
      unpack16<T>(ld_stream_v4(base + p), v);
      return;
    }
  }
#pragma unroll
  for (int j = 0; j < VEC; ++j) v[j] = (p + j < n) ? Cvt<T>::to(base[p + j]) : fill;
}

// Store the elements of v whose bit is set in `mask` (bits beyond n are
// never set by the callers).
template <typename T, int VEC>
__device__ __forceinline__ void store_vec(T* __restrict__ base, int64_t p, unsigned mask,
                                          const float (&v)[VEC]) {
  constexpr unsigned kAll = (VEC >= 32) ? 0xffffffffu : ((1u << VEC) - 1u);
  if constexpr (VEC * sizeof(T) == 16) {
    if (mask == kAll) {
      st_v4(base + p, pack16<T>(v));
      return;
    }
  }
#pragma unroll
  for (int j = 0; j < VEC; ++j)
    if ((mask >> j) & 1u) base[p + j] = Cvt<T>::from(v[j]);
}

// ---------------------------------------------------------------------------
// Sequence boundaries: a cursor over cu_seqlens for one row position t
// ---------------------------------------------------------------------------

// Values read from cu_seqlens are clamped to [0, BL], so a malformed array
// can only change which positions count as boundaries, never an address.
template <typename IdxT>
__device__ __forceinline__ int64_t cu_at(const IdxT* __restrict__ cu, int64_t i, int64_t BL) {
  int64_t v = static_cast<int64_t>(__ldg(cu + i));
  return v < 0 ? 0 : (v > BL ? BL : v);
}

// seg: index of the sequence holding t (-1: t lies before cu[0]);
// [lo, hi): that sequence's extent within the row.
struct Cursor {
  int64_t seg, lo, hi;
};

template <typename IdxT>
__device__ __forceinline__ void cursor_seek(Cursor& c, const IdxT* __restrict__ cu, int64_t S,
                                            int64_t BL, int64_t t) {
  int64_t a = 0, b = S;  // count of cu[0..S-1] entries <= t
  while (a < b) {
    int64_t m = (a + b) >> 1;
    if (cu_at(cu, m, BL) <= t)
      a = m + 1;
    else
      b = m;
  }
  c.seg = a - 1;
  c.lo = (a > 0) ? cu_at(cu, a - 1, BL) : -1;
  c.hi = cu_at(cu, a, BL);
}

template <typename IdxT>
__device__ __forceinline__ void cursor_advance(Cursor& c, const IdxT* __restrict__ cu, int64_t S,
                                               int64_t BL, int64_t t) {
  while (t >= c.hi && c.seg + 1 < S) {
    ++c.seg;
    c.lo = c.hi;
    c.hi = cu_at(cu, c.seg + 1, BL);
  }
}

// Boundary masks of VEC consecutive elements whose first element sits at row
// position t and flat index p.  Bit j of
//   smask: element j starts a sequence (or belongs to none, or is past n)
//   emask: element j ends a sequence   (same exceptions)
//   wmask: element j belongs to a sequence and lies below n (it is written)
// `cur` describes position t and is left unchanged.
template <typename IdxT, int VEC>
__device__ __forceinline__ void vec_bounds(const Cursor& cur, int64_t t, int64_t p, int64_t n,
                                           const IdxT* __restrict__ cu, int64_t S, int64_t BL,
                                           unsigned& smask, unsigned& emask, unsigned& wmask) {
  constexpr unsigned kAll = (VEC >= 32) ? 0xffffffffu : ((1u << VEC) - 1u);
  if (cur.seg >= 0 && t > cur.lo && t + VEC < cur.hi && p + VEC <= n) {
    smask = 0u;
    emask = 0u;
    wmask = kAll;
    return;
  }
  Cursor c = cur;
  int64_t tt = t;
  unsigned s = 0u, e = 0u, w = 0u;
#pragma unroll
  for (int j = 0; j < VEC; ++j) {
    if (j > 0) {
      ++tt;
      if (tt >= BL) {
        tt = 0;
        cursor_seek(c, cu, S, BL, 0);
      } else {
        cursor_advance(c, cu, S, BL, tt);
      }
    }
    const bool in_seq = (c.seg >= 0) && (p + j < n);
    if (!in_seq || tt == c.lo) s |= 1u << j;
    if (!in_seq || tt == c.hi - 1) e |= 1u << j;
    if (in_seq) w |= 1u << j;
  }
  smask = s;
  emask = e;
  wmask = w;
}

// Move a cursor from row position t forward by `step` elements.
template <typename IdxT>
__device__ __forceinline__ void cursor_step(Cursor& c, int64_t& t, int64_t step,
                                            const IdxT* __restrict__ cu, int64_t S, int64_t BL) {
  t += step;
  if (t >= BL) {
    t = (BL > step) ? t - BL : t % BL;
    cursor_seek(c, cu, S, BL, t);
  } else {
    cursor_advance(c, cu, S, BL, t);
  }
}

// ---------------------------------------------------------------------------
// Scans
// ---------------------------------------------------------------------------

// Aggregate of one thread's VEC elements in scan order (REV: descending).
template <int VEC, bool REV>
__device__ __forceinline__ Pfx vec_aggregate(const float (&a)[VEC], const float (&b)[VEC],
                                             unsigned head) {
  constexpr int j0 = REV ? VEC - 1 : 0;
  Pfx p{a[j0], b[j0], kValid | (int)((head >> j0) & 1u)};
#pragma unroll
  for (int jj = 1; jj < VEC; ++jj) {
    const int j = REV ? VEC - 1 - jj : jj;
    if ((head >> j) & 1u) {
      p.a = a[j];
      p.b = b[j];
      p.f |= kHead;
    } else {
      p.b = fmaf(a[j], p.b, b[j]);
      p.a = p.a * a[j];
    }
  }
  return p;
}

template <bool REV>
__device__ __forceinline__ float shfl_prev(float v, int d) {
  return REV ? __shfl_down_sync(kFull, v, d) : __shfl_up_sync(kFull, v, d);
}
template <bool REV>
__device__ __forceinline__ int shfl_prev(int v, int d) {
  return REV ? __shfl_down_sync(kFull, v, d) : __shfl_up_sync(kFull, v, d);
}

// Warp-wide scan of one non-empty value per lane in scan order (REV: lane 31
// first).  Returns the exclusive prefix of this lane (empty for the first
// lane) and the warp total.
template <bool REV>
__device__ __forceinline__ void warp_scan(Pfx v, int lane, Pfx& excl, Pfx& total) {
  const int ll = REV ? 31 - lane : lane;
  const bool any_head = __any_sync(kFull, v.f & kHead);
  Pfx inc = v;
  if (any_head) {
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      Pfx o{shfl_prev<REV>(inc.a, d), shfl_prev<REV>(inc.b, d), shfl_prev<REV>(inc.f, d)};
      if (ll >= d) inc = compose_nonempty(o, inc);
    }
  } else {
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const float oa = shfl_prev<REV>(inc.a, d);
      const float ob = shfl_prev<REV>(inc.b, d);
      if (ll >= d) {
        inc.b = fmaf(inc.a, ob, inc.b);
        inc.a = oa * inc.a;
      }
    }
  }
  const float ea = shfl_prev<REV>(inc.a, 1);
  const float eb = shfl_prev<REV>(inc.b, 1);
  const int ef = shfl_prev<REV>(inc.f, 1);
  excl = (ll == 0) ? pfx_empty() : Pfx{ea, eb, ef};
  const int last = REV ? 0 : 31;
  total = Pfx{__shfl_sync(kFull, inc.a, last), __shfl_sync(kFull, inc.b, last),
              __shfl_sync(kFull, inc.f, last)};
}

// ---------------------------------------------------------------------------
// Decoupled look-back across tiles (Merrill & Garland, "Single-pass Parallel
// Prefix Scan with Decoupled Look-back", 2016), indexed by dynamic ticket.
// ---------------------------------------------------------------------------

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// True once more than `limit_ns` (default kLookbackTimeoutNs) have passed
// since t0.  The difference is taken signed, so a timer reading that steps
// back never counts as an expired wait.
__device__ __forceinline__ bool wait_expired(unsigned long long t0,
                                             unsigned long long limit_ns = kLookbackTimeoutNs) {
  return static_cast<long long>(globaltimer() - t0) > static_cast<long long>(limit_ns);
}

// Tile status records, one 16-byte slot per ticket: two 64-bit words
// {a, state} and {b, state} written by one relaxed vector store.  Each
// aligned 64-bit word is single-copy atomic, states only grow
// (none -> aggregate -> inclusive), and a reader accepts a slot only when
// both words carry the same state -- so no fence orders the value before the
// flag, and publishing never stalls the publishing warp.
// `abort` is a per-launch word: once any wait of the launch has given up,
// every other wait returns at once, so a lost predecessor costs one timeout,
// not one per tile.
struct TileStatus {
  uint4* slots;
  uint32_t* abort;
};

__device__ __forceinline__ uint32_t ld_volatile_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ bool launch_aborted(const TileStatus& st) {
  return ld_volatile_u32(st.abort) != 0u;
}

__device__ __forceinline__ void set_aborted(const TileStatus& st) { atomicExch(st.abort, 1u); }

__device__ __forceinline__ void publish(const TileStatus& st, uint32_t ticket, uint32_t kind,
                                        float a, float b) {
  asm volatile("st.relaxed.gpu.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(st.slots + ticket),
               "r"(__float_as_uint(a)), "r"(kind), "r"(__float_as_uint(b)), "r"(kind)
               : "memory");
}

// One read of a slot; returns its state (kStatusNone when empty or torn).
__device__ __forceinline__ uint32_t read_status(const TileStatus& st, uint32_t ticket, float& a,
                                                float& b) {
  uint32_t w0, w1, w2, w3;
  asm volatile("ld.relaxed.gpu.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(w0), "=r"(w1), "=r"(w2), "=r"(w3)
               : "l"(st.slots + ticket)
               : "memory");
  a = __uint_as_float(w0);
  b = __uint_as_float(w2);
  return (w1 == w3) ? w1 : kStatusNone;
}

// Wait (bounded) until the status of `ticket` is published; kStatusNone on
// timeout or when the launch has been aborted.
__device__ __forceinline__ uint32_t wait_status(const TileStatus& st, uint32_t ticket, float& a,
                                                float& b) {
  uint32_t s = read_status(st, ticket, a, b);
  if (s != kStatusNone) return s;
  const unsigned long long t0 = globaltimer();
  unsigned ns = 16;
  while (true) {
    __nanosleep(ns);
    if (ns < 256) ns <<= 1;
    s = read_status(st, ticket, a, b);
    if (s != kStatusNone) return s;
    if (launch_aborted(st)) return kStatusNone;
    if (wait_expired(t0)) {
      set_aborted(st);
      return kStatusNone;
    }
  }
}

// Warp-parallel decoupled look-back (all 32 lanes).  The window covers the
// 32*K tiles before `ticket` in scan order, whose tickets are `stride` apart
// (1 when tiles follow each other in the flat array, the number of rows when
// they are dealt tile-major across rows): lane l owns the K consecutive
// predecessors at distance K*l+1 .. K*l+K (slot i = 0 is the nearest).  Each
// poll reads the whole window in one round trip, finds the nearest inclusive
// record and is satisfied once every slot nearer than it holds at least an
// aggregate -- slots beyond it are never waited for.  A window without an
// inclusive record is composed whole and the window slides back.  Returns the
// exclusive prefix of `ticket`; *timed_out is set when a needed predecessor
// was not published within the bounded wait (it then counts as empty).
template <int K>
__device__ __forceinline__ Pfx lookback_warp(const TileStatus& st, uint32_t ticket, int lane,
                                             bool* timed_out, uint32_t stride = 1u,
                                             unsigned long long limit_ns = kLookbackTimeoutNs) {
  Pfx te = pfx_empty();
  int64_t base = 0;  // distance (in predecessors) of this window's nearest slot, minus one
  bool lost = false;
  while (true) {
    uint32_t sk[K];
    float va[K], vb[K];
    int my_inc = K;   // nearest inclusive slot of this lane (K: none)
    int stop = 32;    // first lane holding an inclusive slot (32: none)
    unsigned long long t0 = 0;
    unsigned ns = 16;
    for (int poll = 0;; ++poll) {
#pragma unroll
      for (int i = 0; i < K; ++i) {
        const int64_t q = static_cast<int64_t>(ticket) -
                          (base + static_cast<int64_t>(K) * lane + i + 1) * stride;
        if (q < 0) {
          sk[i] = kStatusInclusive;  // nothing precedes ticket 0: a zero state
          va[i] = 1.f;
          vb[i] = 0.f;
        } else {
          sk[i] = read_status(st, static_cast<uint32_t>(q), va[i], vb[i]);
        }
      }
      my_inc = K;
#pragma unroll
      for (int i = K - 1; i >= 0; --i)
        if (sk[i] == kStatusInclusive) my_inc = i;
      const unsigned incmask = __ballot_sync(kFull, my_inc < K);
      stop = incmask ? (__ffs(incmask) - 1) : 32;
      bool missing = false;
#pragma unroll
      for (int i = 0; i < K; ++i) {
        const bool needed = lane < stop || (lane == stop && i < my_inc);
        if (needed && sk[i] == kStatusNone) missing = true;
      }
      if (!__any_sync(kFull, missing)) break;
      if (poll == 0) t0 = globaltimer();
      __nanosleep(ns);
      if (ns < 256) ns <<= 1;
      const bool give_up = launch_aborted(st) || wait_expired(t0, limit_ns);
      if (__any_sync(kFull, give_up)) {
        if (lane == 0) set_aborted(st);
        lost = true;  // unpublished slots count as empty records
        break;
      }
    }
    Pfx x = pfx_empty();
    if (lane <= stop) {
#pragma unroll
      for (int i = K - 1; i >= 0; --i) {  // earliest first
        if (lane == stop && i > my_inc) continue;
        if (sk[i] == kStatusInclusive)
          x = Pfx{va[i], vb[i], kValid | kHead};
        else if (sk[i] == kStatusAggregate)
          x = compose(x, Pfx{va[i], vb[i], kValid});
      }
    }
    // x_31 o ... o x_1 o x_0 (a higher lane holds earlier tiles)
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const Pfx o{__shfl_down_sync(kFull, x.a, off), __shfl_down_sync(kFull, x.b, off),
                  __shfl_down_sync(kFull, x.f, off)};
      if (lane + off < 32) x = compose(o, x);
    }
    const Pfx part{__shfl_sync(kFull, x.a, 0), __shfl_sync(kFull, x.b, 0),
                   __shfl_sync(kFull, x.f, 0)};
    te = compose(part, te);
    if (stop < 32 || lost) break;
    base += 32 * K;
  }
  *timed_out = __any_sync(kFull, lost);
  te.f &= ~kHead;
  return te;
}

constexpr int kLookbackPerLane = 8;  // window of 256 predecessors per round trip

}  // namespace ascan

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

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ float2 ld_relaxed_f2(const float* p) {
  float2 v;
  asm volatile("ld.relaxed.gpu.global.v2.f32 {%0,%1}, [%2];" : "=f"(v.x), "=f"(v.y) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_relaxed_f2(float* p, float a, float b) {
  asm volatile("st.relaxed.gpu.global.v2.f32 [%0], {%1,%2};" ::"l"(p), "f"(a), "f"(b) : "memory");
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Status slot of a ticket: flag word plus (aggregate a, b, inclusive a, b).
// `abort` is a per-launch word: once any wait of the launch has given up, every
// other wait returns at once, so a lost predecessor costs one timeout, not one
// per tile.
struct TileStatus {
  uint32_t* flags;
  float4* vals;
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
  float* dst = reinterpret_cast<float*>(st.vals + ticket) + (kind == kStatusInclusive ? 2 : 0);
  st_relaxed_f2(dst, a, b);
  st_release(st.flags + ticket, kind);
}

// Wait (bounded) until the status of `ticket` is published; 0 on timeout or
// when the launch has been aborted.
__device__ __forceinline__ uint32_t wait_status(const TileStatus& st, uint32_t ticket) {
  uint32_t s = ld_acquire(st.flags + ticket);
  if (s != kStatusNone) return s;
  const unsigned long long t0 = globaltimer();
  unsigned ns = 16;
  while (true) {
    __nanosleep(ns);
    if (ns < 256) ns <<= 1;
    s = ld_acquire(st.flags + ticket);
    if (s != kStatusNone) return s;
    if (launch_aborted(st)) return kStatusNone;
    if (globaltimer() - t0 > kLookbackTimeoutNs) {
      set_aborted(st);
      return kStatusNone;
    }
  }
}

}  // namespace ascan

// ascan_exchange.cuh -- the carry exchange of a time-sharded run over peer
// memory: one kernel per direction publishes this rank's per-row record in its
// own exchange buffer, waits (bounded) for the records of the ranks whose
// slabs it depends on, reads them straight from those ranks' buffers over
// NVLink and folds them into this rank's carry.  It replaces an all-gather of
// the records plus the fold launch (time_shard_fold_kernel computes the same
// fold from a gathered [world][record] array).
//
// Exchange buffer of one rank (device memory from cudaMalloc, shared with the
// other ranks through a CUDA IPC handle; zeroed at creation):
//   [0, 128)     epoch[2]     exchanges this rank has finished, per direction
//   [128, 256)   flag[2]      e + 1 once this rank's record of exchange e is out
//   [256, 384)   consumed[2]  e + 1 once this rank has read everything of exchange e
//   [512, ...)   ring[2 directions][2 slots][4 C] floats: the record of exchange e
//                sits in slot e % 2 (forward [0, 2C): (gate product, state) per
//                row; backward [0, 2C): (coefficient product, adjoint), [2C, 3C):
//                the slab's first gate column, [3C, 4C): its last state column)
// Every rank runs the same sequence of exchanges per direction, so e agrees
// across ranks.  Before a rank overwrites slot e % 2 (last used by exchange
// e - 2) it waits until every peer has consumed exchange e - 2; a rank never
// runs more than one exchange ahead of a peer it waits on, so two slots are
// enough and no record is overwritten while a peer still reads it.
//
// Memory ordering: the record goes out with plain stores, then a system-scope
// fence and a release store of the flag; readers take the flag with an
// acquire load at system scope and read the record with relaxed system-scope
// loads (never from a stale cache line).  No multicast, no TMA: plain peer
// loads only.  Every wait polls %globaltimer and gives up after `timeout_ns`
// (ASCAN_DEV_ERR_EXCHANGE; the kernel then finishes with what it has, so the
// stream and the context stay usable).
#pragma once

namespace ascan {
namespace xchg {

constexpr int kThreads = 512;
constexpr size_t kHeaderBytes = 512;

__device__ __forceinline__ uint32_t* epoch_word(char* buf, int dir) {
  return reinterpret_cast<uint32_t*>(buf) + dir;
}
__device__ __forceinline__ uint32_t* flag_word(char* buf, int dir) {
  return reinterpret_cast<uint32_t*>(buf + 128) + dir;
}
__device__ __forceinline__ uint32_t* consumed_word(char* buf, int dir) {
  return reinterpret_cast<uint32_t*>(buf + 256) + dir;
}
__device__ __forceinline__ float* ring_slot(char* buf, int64_t C, int dir, uint32_t e) {
  return reinterpret_cast<float*>(buf + kHeaderBytes) + ((2 * dir + (e & 1u)) * 4) * C;
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ float ld_relaxed_sys(const float* p) {
  float v;
  asm volatile("ld.relaxed.sys.global.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
  return v;
}

// Waits until *p >= want (a word of another rank's buffer, or this rank's);
// false if `timeout_ns` passed first.
__device__ __forceinline__ bool wait_at_least(const uint32_t* p, uint32_t want,
                                              unsigned long long timeout_ns) {
  if (ld_acquire_sys(p) >= want) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
    __nanosleep(200);
    if (ld_acquire_sys(p) >= want) return true;
    if (wait_expired(t0, timeout_ns)) return false;
  }
}

constexpr int kPublish = 1, kFold = 2;

template <typename T>
struct XArgs {
  char* own;                 // this rank's exchange buffer
  const uint64_t* bufs;      // [world] exchange buffers as this process maps them (own at rank)
  int world, rank, dir, mode;
  int64_t C, L;
  int parts;                 // H: every row scanned as H parts of L / H columns
  const float* aggregate;    // [H C][2] this rank's aggregate of every row part
  const T* first;            // backward: gates [C][L] (the parts' first columns)
  const T* last;             // backward: states [C][L] (the parts' last columns)
  uint32_t new_mask, inner_mask;
  float* carry;              // fold: forward [H C][2], backward [H C]
  float* halo;               // fold, backward: [H C] or NULL
  unsigned long long timeout_ns;
  uint32_t* err_host;
};

// Whether this rank's fold reads rank j's record.
__device__ __forceinline__ bool needs(int j, int rank, int dir, bool halo) {
  if (j == rank) return false;
  return dir == 0 ? j < rank : (j > rank || (halo && j == rank - 1));
}

template <typename T>
__global__ void __launch_bounds__(kThreads) time_shard_exchange_kernel(const XArgs<T> a) {
  __shared__ uint32_t s_e;
  const int tid = threadIdx.x;
  const int64_t C = a.C;
  if (tid == 0) s_e = ld_volatile_u32(epoch_word(a.own, a.dir));
  __syncthreads();
  const uint32_t e = s_e;
  if (a.mode & kPublish) {
    // the slot was last used by exchange e - 2: every peer must be done with it
    if (e >= 2 && tid < a.world && tid != a.rank) {
      char* peer = reinterpret_cast<char*>(a.bufs[tid]);
      if (!wait_at_least(consumed_word(peer, a.dir), e - 1, a.timeout_ns))
        report(ASCAN_DEV_ERR_EXCHANGE, (static_cast<unsigned long long>(tid) << 32) | e, a.err_host);
    }
    __syncthreads();
    // the record of each row: its parts' aggregates composed in scan order
    float* slot = ring_slot(a.own, C, a.dir, e);
    const int H = a.parts;
    const int64_t lp = a.L / H;
    for (int64_t r = tid; r < C; r += kThreads) {
      const float* ag = a.aggregate + 2 * H * r;
      if (a.dir == 0) {  // h at the row end = P h_in + Y, part after part
        float P = 1.f, Y = 0.f;
        for (int k = 0; k < H; ++k) {
          Y = fmaf(ag[2 * k], Y, ag[2 * k + 1]);
          P *= ag[2 * k];
        }
        slot[2 * r] = P;
        slot[2 * r + 1] = Y;
      } else {  // dh at the row start = Q c_in + D, part after part from the right
        float Q = ag[2 * (H - 1)], D = ag[2 * (H - 1) + 1];
        for (int k = H - 2; k >= 0; --k) {
          const float qg = ag[2 * k] * Cvt<T>::to(a.first[r * a.L + (k + 1) * lp]);
          D = fmaf(qg, D, ag[2 * k + 1]);
          Q *= qg;
        }
        slot[2 * r] = Q;
        slot[2 * r + 1] = D;
        slot[2 * C + r] = Cvt<T>::to(a.first[r * a.L]);
        slot[3 * C + r] = Cvt<T>::to(a.last[r * a.L + a.L - 1]);
      }
    }
    __syncthreads();
    if (tid == 0) {
      __threadfence_system();
      st_release_sys(flag_word(a.own, a.dir), e + 1u);
    }
  }
  if (a.mode & kFold) {
    const bool halo = a.halo != nullptr;
    if (tid < a.world && needs(tid, a.rank, a.dir, halo)) {
      char* peer = reinterpret_cast<char*>(a.bufs[tid]);
      if (!wait_at_least(flag_word(peer, a.dir), e + 1u, a.timeout_ns))
        report(ASCAN_DEV_ERR_EXCHANGE, (static_cast<unsigned long long>(tid) << 32) | e, a.err_host);
    }
    __syncthreads();
    const int world = a.world, rank = a.rank;
    // one thread per row; the peers' values of a group of kGroup ranks are
    // all requested before any is used, so a group costs one round trip
    constexpr int kGroup = 8;
    for (int64_t r = tid; r < C; r += kThreads) {
      if (a.dir == 0) {
        float prod = 1.f, state = 0.f;
        for (int j0 = 0; j0 < rank; j0 += kGroup) {
          float P[kGroup], Y[kGroup];
#pragma unroll
          for (int k = 0; k < kGroup; ++k) {
            if (j0 + k < rank) {
              const float* rec = ring_slot(reinterpret_cast<char*>(a.bufs[j0 + k]), C, 0, e);
              P[k] = ld_relaxed_sys(rec + 2 * r);
              Y[k] = ld_relaxed_sys(rec + 2 * r + 1);
            }
          }
#pragma unroll
          for (int k = 0; k < kGroup; ++k) {
            const int j = j0 + k;
            if (j < rank) {
              const bool cont = !((a.new_mask >> j) & 1u) && !((a.inner_mask >> j) & 1u);
              state = cont ? fmaf(P[k], state, Y[k]) : Y[k];
              prod = cont ? P[k] * prod : P[k];
            }
          }
        }
        const bool fresh = (a.new_mask >> rank) & 1u;
        // the carry entering each part of the row (the parts continue one
        // another: the slab has no sequence boundary inside when H > 1)
        prod = fresh ? 1.f : prod;
        state = fresh ? 0.f : state;
        const float* ag = a.aggregate + 2 * a.parts * r;
        float* out = a.carry + 2 * a.parts * r;
        for (int k = 0; k < a.parts; ++k) {
          out[2 * k] = prod;
          out[2 * k + 1] = state;
          if (k + 1 < a.parts) {
            state = fmaf(ag[2 * k], state, ag[2 * k + 1]);
            prod *= ag[2 * k];
          }
        }
      } else {
        float c = 0.f;
        // ranks world-1 down to rank+1, kGroup at a time
        for (int j0 = world - 1; j0 > rank; j0 -= kGroup) {
          float Q[kGroup], D[kGroup], G[kGroup];
#pragma unroll
          for (int k = 0; k < kGroup; ++k) {
            if (j0 - k > rank) {
              const float* rec = ring_slot(reinterpret_cast<char*>(a.bufs[j0 - k]), C, 1, e);
              Q[k] = ld_relaxed_sys(rec + 2 * r);
              D[k] = ld_relaxed_sys(rec + 2 * r + 1);
              G[k] = ld_relaxed_sys(rec + 2 * C + r);
            }
          }
#pragma unroll
          for (int k = 0; k < kGroup; ++k) {
            const int j = j0 - k;
            if (j > rank) {
              const float dh = ((a.inner_mask >> j) & 1u) ? D[k] : fmaf(Q[k], c, D[k]);
              c = ((a.new_mask >> j) & 1u) ? 0.f : G[k] * dh;
            }
          }
        }
        // the carry entering each part's last column, from the right, and
        // each part's state halo (the previous part's last state)
        const int H = a.parts;
        const int64_t lp = a.L / H;
        const float* ag = a.aggregate + 2 * H * r;
        for (int k = H - 1; k >= 0; --k) {
          a.carry[H * r + k] = c;
          if (k > 0) c = Cvt<T>::to(a.first[r * a.L + k * lp]) * fmaf(ag[2 * k], c, ag[2 * k + 1]);
        }
        if (halo) {
          float h = 0.f;
          if (rank > 0 && !((a.new_mask >> rank) & 1u)) {
            const float* rec = ring_slot(reinterpret_cast<char*>(a.bufs[rank - 1]), C, 1, e);
            h = ld_relaxed_sys(rec + 3 * C + r);
          }
          a.halo[H * r] = h;
          for (int k = 1; k < H; ++k) a.halo[H * r + k] = Cvt<T>::to(a.last[r * a.L + k * lp - 1]);
        }
      }
    }
    __syncthreads();  // every read of the peers' slots has returned
    if (tid == 0) {
      __threadfence_system();
      st_release_sys(consumed_word(a.own, a.dir), e + 1u);
      *epoch_word(a.own, a.dir) = e + 1u;
    }
  }
}

}  // namespace xchg
}  // namespace ascan

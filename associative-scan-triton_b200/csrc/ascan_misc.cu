// ascan_misc.cu -- compilation unit of the scan library: shift_pad for every
// dtype and the self-test of the kernels' bounded waits.
// The kernels and launchers are defined in ascan_impl.cuh.
#define ASCAN_UNIT_MISC
#include "ascan_impl.cuh"
#include "ascan_exchange.cuh"

namespace ascan {

ASCAN_FOR_EACH_TYPE_PAIR(ASCAN_DECL_SHIFT_PAD)

// Runs selftest_waits_kernel on `s` and copies its four results to the host
// (synchronises `s`).  `workspace`: 512 bytes of device memory, 256-aligned.
int selftest_waits_run(void* workspace, long long limit_ns, long long* results, cudaStream_t s) {
  char* base = static_cast<char*>(workspace);
  auto* out = reinterpret_cast<unsigned long long*>(base);  // 4 words
  auto* abort_word = reinterpret_cast<uint32_t*>(base + 64);
  auto* slots = reinterpret_cast<uint4*>(base + 256);       // 16 slots
  if (cudaMemsetAsync(workspace, 0, 512, s) != cudaSuccess) return ASCAN_ECUDA;
  selftest_waits_kernel<<<1, 32, 0, s>>>(slots, abort_word,
                                         static_cast<unsigned long long>(limit_ns), out);
  if (cudaGetLastError() != cudaSuccess) return ASCAN_ECUDA;
  unsigned long long host[4] = {0, 0, 0, 0};
  if (cudaMemcpyAsync(host, out, sizeof(host), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return ASCAN_ECUDA;
  for (int i = 0; i < 4; ++i) results[i] = static_cast<long long>(host[i]);
  return ASCAN_OK;
}

// Carry fold of a time-sharded run (ascan_time_shard_fold): one thread per
// row walks the records of the other slabs in scan order.  Forward: the
// (gate product, state) entering slab `rank`, composed from the aggregates of
// the slabs before it -- a slab whose last piece continues a sequence from
// before it composes onto the carry, any other slab restarts it.  Backward:
// the adjoint term entering slab `rank`'s last column, walked from the last
// slab, and the state halo h[t0 - 1] (the previous slab's last state).
__global__ void __launch_bounds__(256)
    time_shard_fold_kernel(const float* __restrict__ rec, int64_t rf, int world, int rank,
                           int64_t C, uint32_t new_mask, uint32_t inner_mask, int direction,
                           float* __restrict__ carry, float* __restrict__ halo) {
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x; r < C;
       r += static_cast<int64_t>(gridDim.x) * 256) {
    if (direction == 0) {
      float prod = 1.f, state = 0.f;
      for (int j = 0; j < rank; ++j) {
        const float P = rec[j * rf + 2 * r], Y = rec[j * rf + 2 * r + 1];
        const bool cont = !((new_mask >> j) & 1u) && !((inner_mask >> j) & 1u);
        state = cont ? fmaf(P, state, Y) : Y;
        prod = cont ? P * prod : P;
      }
      const bool fresh = (new_mask >> rank) & 1u;
      carry[2 * r] = fresh ? 1.f : prod;
      carry[2 * r + 1] = fresh ? 0.f : state;
    } else {
      float c = 0.f;
      for (int j = world - 1; j > rank; --j) {
        const float Q = rec[j * rf + 2 * r], D = rec[j * rf + 2 * r + 1];
        const float g_first = rec[j * rf + 2 * C + r];
        const float dh = ((inner_mask >> j) & 1u) ? D : fmaf(Q, c, D);
        c = ((new_mask >> j) & 1u) ? 0.f : g_first * dh;
      }
      carry[r] = c;
      if (halo)
        halo[r] = (rank == 0 || ((new_mask >> rank) & 1u)) ? 0.f : rec[(rank - 1) * rf + 3 * C + r];
    }
  }
}

int time_shard_fold_run(const float* records, int64_t record_floats, int world, int rank,
                        int64_t C, uint32_t new_mask, uint32_t inner_mask, int direction,
                        float* carry, float* halo, cudaStream_t s) {
  int64_t blocks = (C + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  time_shard_fold_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(
      records, record_floats, world, rank, C, new_mask, inner_mask, direction, carry, halo);
  return launch_status();
}

// The carry exchange of a time-sharded run over peer memory
// (ascan_time_shard_exchange): one CTA on `s`.
int time_shard_exchange_run(void* own, const uint64_t* bufs, int world, int rank, int dir, int mode,
                            int64_t C, int64_t L, int parts, const float* aggregate, const void* first,
                            const void* last, int dtype, uint32_t new_mask, uint32_t inner_mask,
                            float* carry, float* halo, unsigned long long timeout_ns,
                            cudaStream_t s) {
  auto launch = [&](auto tag) {
    using T = decltype(tag);
    const xchg::XArgs<T> a{static_cast<char*>(own), bufs, world, rank, dir, mode, C, L, parts, aggregate,
                           static_cast<const T*>(first), static_cast<const T*>(last), new_mask,
                           inner_mask, carry, halo, timeout_ns, g_err_host};
    xchg::time_shard_exchange_kernel<T><<<1, xchg::kThreads, 0, s>>>(a);
  };
  switch (dtype) {
    case ASCAN_F32: launch(float{}); break;
    case ASCAN_F16: launch(__half{}); break;
    case ASCAN_BF16: launch(__nv_bfloat16{}); break;
    default: return ASCAN_EINVAL;
  }
  return launch_status();
}

ASCAN_UNIT_ERROR_ACCESSORS(misc)

}  // namespace ascan

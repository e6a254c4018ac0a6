// ascan_misc.cu -- compilation unit of the scan library: shift_pad for every
// dtype and the self-test of the kernels' bounded waits.
// The kernels and launchers are defined in ascan_impl.cuh.
#define ASCAN_UNIT_MISC
#include "ascan_impl.cuh"

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

ASCAN_UNIT_ERROR_ACCESSORS(misc)

}  // namespace ascan

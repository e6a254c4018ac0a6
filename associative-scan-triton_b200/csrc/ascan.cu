// ascan.cu -- C ABI of the B200 (sm_100a) packed-varlen linear scan.
//
// The kernels and their launchers live in ascan_impl.cuh and are compiled by
// the units ascan_fwd_*.cu, ascan_bwd_*.cu, ascan_bidi.cu and ascan_misc.cu;
// this file checks arguments, carves workspaces and dispatches on dtype and
// index type (include/ascan.h documents every entry point).
#include <cstring>

#include "ascan_impl.cuh"

namespace ascan {

// Process-wide switches (ascan_set_implementation / ascan_set_tile_width).
int g_impl = -1;
int g_tile_width = 0;
uint32_t* g_err_host = nullptr;
static uint32_t* g_err_host_ptr = nullptr;  // host address of the same word

// Fixed scratch of ascan_forward_noalloc: the look-back workspace for callers
// that cannot allocate device memory.  Every device that loads this library
// holds these bytes until the process exits; all calls share them.
constexpr size_t kNoAllocScratchBytes = ASCAN_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

int selftest_waits_run(void* workspace, long long limit_ns, long long* results, cudaStream_t s);
int time_shard_fold_run(const float* records, int64_t record_floats, int world, int rank,
                        int64_t C, uint32_t new_mask, uint32_t inner_mask, int direction,
                        float* carry, float* halo, cudaStream_t s);
int time_shard_exchange_run(void* own, const uint64_t* bufs, int world, int rank, int dir, int mode,
                            int64_t C, int64_t L, int parts, const float* aggregate, const void* first,
                            const void* last, int dtype, uint32_t new_mask, uint32_t inner_mask,
                            float* carry, float* halo, unsigned long long timeout_ns,
                            cudaStream_t s);

}  // namespace ascan

using namespace ascan;


extern "C" {

int ascan_abi_version(void) { return ASCAN_ABI_VERSION; }

const char* ascan_build_info(void) {
  return "ascan sm_100a: persistent TMA-pipelined decoupled look-back scan (one CTA of 8 "
         "consumer warps + 1 producer warp per SM, 288 threads, 4096- or 8192-element tiles "
         "chosen per launch, 128B-swizzled TMA loads and stores); plain one-CTA-per-tile "
         "kernels with 128-bit vector IO for misaligned views; fp32 accumulation";
}

const char* ascan_strerror(int status) {
  switch (status) {
    case ASCAN_OK: return "ok";
    case ASCAN_EINVAL: return "invalid argument (size, dtype, flag or null pointer)";
    case ASCAN_EWORKSPACE: return "workspace missing, not 256-byte aligned or too small";
    case ASCAN_ECUDA: return "CUDA launch or memset failed";
    case ASCAN_EDEVICE: return "no usable CUDA device";
    case ASCAN_ETOOLARGE:
      return "problem too large for the fixed scratch of ascan_forward_noalloc "
             "(num_channels * seq_total must be <= ASCAN_NOALLOC_MAX_ELEMENTS)";
    default: return "unknown ascan status";
  }
}

size_t ascan_workspace_size(int64_t num_channels, int64_t seq_total, int dtype) {
  (void)dtype;
  if (num_channels <= 0 || seq_total <= 0) return 256;
  return workspace_bytes_for(num_channels, seq_total, true);
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
  rc = carve(workspace, workspace_bytes, num_channels, seq_total, w);
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
  rc = carve(workspace, workspace_bytes, num_channels, seq_total, w);
  if (rc != ASCAN_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(w.ticket, 0, w.clear_bytes, s) != cudaSuccess) return ASCAN_ECUDA;
#define ASCAN_BWD_CALL(T, I)                                                                    \
  bwd_typed<T, I>(grad, gates, states, d_tokens, d_gates, cu_seqlens, num_seq, num_channels,    \
                  seq_total, causal, w, s)
  ASCAN_DISPATCH_TYPES(dtype, cu_index_type, ASCAN_BWD_CALL);
#undef ASCAN_BWD_CALL
}

int ascan_forward_slab(const void* gates, const void* tokens, void* tokens_out, void* gates_out,
                       const void* cu_seqlens, int cu_index_type, int64_t num_seq,
                       int64_t num_channels, int64_t seq_total, int dtype, int reverse,
                       const float* row_carry, float* row_aggregate, void* workspace,
                       size_t workspace_bytes, void* stream) {
  int rc = check_common(cu_seqlens, cu_index_type, num_seq, num_channels, seq_total, dtype);
  if (rc != ASCAN_OK) return rc;
  if (!gates || !tokens) return ASCAN_EINVAL;
  if (!tokens_out && (gates_out || !row_aggregate)) return ASCAN_EINVAL;
  const int64_t n = num_channels * seq_total;
  if (n == 0 || num_seq == 0) return ASCAN_OK;
  Workspace w;
  rc = carve(workspace, workspace_bytes, num_channels, seq_total, w);
  if (rc != ASCAN_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(w.ticket, 0, w.clear_bytes, s) != cudaSuccess) return ASCAN_ECUDA;
  const RowIO io{row_carry, nullptr, row_aggregate};
#define ASCAN_FWD_CALL(T, I)                                                                   \
  fwd_typed<T, I>(gates, tokens, tokens_out, gates_out, cu_seqlens, num_seq, num_channels,     \
                  seq_total, reverse, w, s, io)
  ASCAN_DISPATCH_TYPES(dtype, cu_index_type, ASCAN_FWD_CALL);
#undef ASCAN_FWD_CALL
}

int ascan_backward_slab(const void* grad, const void* gates, const void* states, void* d_tokens,
                        void* d_gates, const void* cu_seqlens, int cu_index_type, int64_t num_seq,
                        int64_t num_channels, int64_t seq_total, int dtype, int causal,
                        const float* row_carry, const float* row_state_halo, float* row_aggregate,
                        void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_common(cu_seqlens, cu_index_type, num_seq, num_channels, seq_total, dtype);
  if (rc != ASCAN_OK) return rc;
  if (!grad || !gates || !states) return ASCAN_EINVAL;
  if ((d_tokens == nullptr) != (d_gates == nullptr)) return ASCAN_EINVAL;
  if (!d_tokens && !row_aggregate) return ASCAN_EINVAL;
  if (d_tokens && (d_gates == gates || d_gates == states || d_tokens == gates ||
                   d_tokens == states || d_tokens == d_gates))
    return ASCAN_EINVAL;
  const int64_t n = num_channels * seq_total;
  if (n == 0 || num_seq == 0) return ASCAN_OK;
  Workspace w;
  rc = carve(workspace, workspace_bytes, num_channels, seq_total, w);
  if (rc != ASCAN_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(w.ticket, 0, w.clear_bytes, s) != cudaSuccess) return ASCAN_ECUDA;
  const RowIO io{row_carry, row_state_halo, row_aggregate};
#define ASCAN_BWD_CALL(T, I)                                                                    \
  bwd_typed<T, I>(grad, gates, states, d_tokens, d_gates, cu_seqlens, num_seq, num_channels,    \
                  seq_total, causal, w, s, io)
  ASCAN_DISPATCH_TYPES(dtype, cu_index_type, ASCAN_BWD_CALL);
#undef ASCAN_BWD_CALL
}

int ascan_time_shard_fold(const float* records, int64_t record_floats, int world, int rank,
                          int64_t num_channels, uint32_t starts_new_mask,
                          uint32_t inner_boundary_mask, int direction, float* carry_out,
                          float* halo_out, void* stream) {
  if (!records || !carry_out || world < 1 || world > 32 || rank < 0 || rank >= world ||
      num_channels <= 0 || (direction != 0 && direction != 1))
    return ASCAN_EINVAL;
  if (record_floats < (direction == 0 ? 2 : 4) * num_channels) return ASCAN_EINVAL;
  if (direction == 0 && halo_out) return ASCAN_EINVAL;
  return time_shard_fold_run(records, record_floats, world, rank, num_channels, starts_new_mask,
                             inner_boundary_mask, direction, carry_out, halo_out,
                             static_cast<cudaStream_t>(stream));
}

// Exchange buffers of ascan_time_shard_exchange: a 512-byte header (epoch,
// flag and consumed words per direction) and two directions x two slots of
// 4 C floats.
size_t ascan_exchange_bytes(int64_t num_channels) {
  if (num_channels <= 0) return 0;
  return 512 + 2 * 2 * 4 * static_cast<size_t>(num_channels) * sizeof(float);
}

int ascan_exchange_create(int64_t num_channels, void** buffer_out) {
  if (!buffer_out || num_channels <= 0) return ASCAN_EINVAL;
  *buffer_out = nullptr;
  const size_t bytes = ascan_exchange_bytes(num_channels);
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return ASCAN_ECUDA;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(p);
    return ASCAN_ECUDA;
  }
  *buffer_out = p;
  return ASCAN_OK;
}

int ascan_exchange_export(void* buffer, void* handle_out) {
  static_assert(sizeof(cudaIpcMemHandle_t) == ASCAN_IPC_HANDLE_BYTES, "IPC handle size");
  if (!buffer || !handle_out) return ASCAN_EINVAL;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, buffer) != cudaSuccess) return ASCAN_ECUDA;
  memcpy(handle_out, &h, sizeof(h));
  return ASCAN_OK;
}

int ascan_exchange_import(const void* handle, void** peer_buffer_out) {
  if (!handle || !peer_buffer_out) return ASCAN_EINVAL;
  *peer_buffer_out = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return ASCAN_ECUDA;
  *peer_buffer_out = p;
  return ASCAN_OK;
}

int ascan_exchange_close(void* peer_buffer) {
  if (!peer_buffer) return ASCAN_EINVAL;
  return cudaIpcCloseMemHandle(peer_buffer) == cudaSuccess ? ASCAN_OK : ASCAN_ECUDA;
}

int ascan_exchange_destroy(void* buffer) {
  if (!buffer) return ASCAN_EINVAL;
  return cudaFree(buffer) == cudaSuccess ? ASCAN_OK : ASCAN_ECUDA;
}

int ascan_time_shard_exchange(void* buffer, const void* buffers, int world, int rank,
                              int64_t num_channels, int64_t seq_total, int parts,
                              const float* aggregate, const void* gates, const void* states,
                              int dtype, uint32_t starts_new_mask, uint32_t inner_boundary_mask,
                              int direction, int mode, float* carry_out, float* halo_out,
                              long long timeout_ns, void* stream) {
  if (!buffer || !buffers || world < 1 || world > 32 || rank < 0 || rank >= world ||
      num_channels <= 0 || (direction != 0 && direction != 1) || mode < 1 || mode > 3 ||
      timeout_ns <= 0 || parts < 1)
    return ASCAN_EINVAL;
  if (dtype != ASCAN_F32 && dtype != ASCAN_F16 && dtype != ASCAN_BF16) return ASCAN_EINVAL;
  // parts > 1: the slab must have no sequence boundary inside, the parts are
  // whole columns, and the fold needs the parts' aggregates (and columns)
  if (parts > 1 && ((inner_boundary_mask >> rank) & 1u)) return ASCAN_EINVAL;
  if (parts > 1 && direction == 1 && (seq_total <= 0 || seq_total % parts != 0))
    return ASCAN_EINVAL;
  const bool needs_aggregate = (mode & 1) || parts > 1;
  const bool needs_columns = direction == 1 && ((mode & 1) || parts > 1);
  if (needs_aggregate && !aggregate) return ASCAN_EINVAL;
  if (needs_columns && (!gates || !states || seq_total <= 0)) return ASCAN_EINVAL;
  if ((mode & 2) && !carry_out) return ASCAN_EINVAL;
  if (direction == 0 && halo_out) return ASCAN_EINVAL;
  return time_shard_exchange_run(buffer, static_cast<const uint64_t*>(buffers), world, rank,
                                 direction, mode, num_channels, seq_total, parts, aggregate, gates,
                                 states, dtype, starts_new_mask, inner_boundary_mask, carry_out,
                                 halo_out, static_cast<unsigned long long>(timeout_ns),
                                 static_cast<cudaStream_t>(stream));
}

// Workspace of a bidirectional pair: two halves, one per scan, each a
// multiple of 256 bytes.
static size_t bidi_half_bytes(int64_t C, int64_t BL) {
  const size_t b = (C <= 0 || BL <= 0) ? 256 : workspace_bytes_for(C, BL, true);
  return (b + 255) & ~static_cast<size_t>(255);
}

size_t ascan_workspace_size_bidi(int64_t num_channels, int64_t seq_total, int dtype) {
  (void)dtype;
  return 2 * bidi_half_bytes(num_channels, seq_total);
}

// Splits and clears the workspace of a bidirectional pair.
static int carve_bidi(void* ws, size_t ws_bytes, int64_t C, int64_t BL, Workspace& wf,
                      Workspace& wb, cudaStream_t s) {
  if (!ws || (reinterpret_cast<uintptr_t>(ws) & 255u) != 0) return ASCAN_EWORKSPACE;
  const size_t half = (ws_bytes / 2) & ~static_cast<size_t>(255);
  int rc = carve(ws, half, C, BL, wf);
  if (rc != ASCAN_OK) return rc;
  rc = carve(static_cast<char*>(ws) + half, half, C, BL, wb);
  if (rc != ASCAN_OK) return rc;
  if (cudaMemsetAsync(ws, 0, half + wb.clear_bytes, s) != cudaSuccess) return ASCAN_ECUDA;
  return ASCAN_OK;
}

int ascan_forward_bidi(const void* gates_fwd, const void* tokens_fwd, void* tokens_out_fwd,
                       const void* gates_bwd, const void* tokens_bwd, void* tokens_out_bwd,
                       const void* cu_seqlens, int cu_index_type, int64_t num_seq,
                       int64_t num_channels, int64_t seq_total, int dtype, void* workspace,
                       size_t workspace_bytes, void* stream) {
  int rc = check_common(cu_seqlens, cu_index_type, num_seq, num_channels, seq_total, dtype);
  if (rc != ASCAN_OK) return rc;
  if (!gates_fwd || !tokens_fwd || !tokens_out_fwd || !gates_bwd || !tokens_bwd ||
      !tokens_out_bwd)
    return ASCAN_EINVAL;
  // the two scans run at the same time: neither output may be the other's input
  if (tokens_out_fwd == tokens_out_bwd || tokens_out_fwd == gates_bwd ||
      tokens_out_fwd == tokens_bwd || tokens_out_bwd == gates_fwd || tokens_out_bwd == tokens_fwd)
    return ASCAN_EINVAL;
  const int64_t n = num_channels * seq_total;
  if (n == 0 || num_seq == 0) return ASCAN_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  Workspace wf, wb;
  rc = carve_bidi(workspace, workspace_bytes, num_channels, seq_total, wf, wb, s);
  if (rc != ASCAN_OK) return rc;
#define ASCAN_FWD_BIDI_CALL(T, I)                                                               \
  fwd_bidi_typed<T, I>(gates_fwd, tokens_fwd, tokens_out_fwd, gates_bwd, tokens_bwd,            \
                       tokens_out_bwd, cu_seqlens, num_seq, num_channels, seq_total, wf, wb, s)
  ASCAN_DISPATCH_TYPES(dtype, cu_index_type, ASCAN_FWD_BIDI_CALL);
#undef ASCAN_FWD_BIDI_CALL
}

int ascan_backward_bidi(const void* grad_fwd, const void* gates_fwd, const void* states_fwd,
                        void* d_tokens_fwd, void* d_gates_fwd, const void* grad_bwd,
                        const void* gates_bwd, const void* states_bwd, void* d_tokens_bwd,
                        void* d_gates_bwd, const void* cu_seqlens, int cu_index_type,
                        int64_t num_seq, int64_t num_channels, int64_t seq_total, int dtype,
                        void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_common(cu_seqlens, cu_index_type, num_seq, num_channels, seq_total, dtype);
  if (rc != ASCAN_OK) return rc;
  const void* const in[2][3] = {{grad_fwd, gates_fwd, states_fwd},
                                {grad_bwd, gates_bwd, states_bwd}};
  void* const out[2][2] = {{d_tokens_fwd, d_gates_fwd}, {d_tokens_bwd, d_gates_bwd}};
  for (int d = 0; d < 2; ++d) {
    for (int k = 0; k < 3; ++k)
      if (!in[d][k]) return ASCAN_EINVAL;
    for (int k = 0; k < 2; ++k)
      if (!out[d][k]) return ASCAN_EINVAL;
  }
  // every output distinct from the other outputs and from the gates and states
  // of both directions (the shifted reads cross thread boundaries, and the two
  // adjoints run at the same time)
  for (int d = 0; d < 2; ++d)
    for (int k = 0; k < 2; ++k) {
      const void* o = out[d][k];
      for (int e = 0; e < 2; ++e) {
        if (o == in[e][1] || o == in[e][2]) return ASCAN_EINVAL;
        if (e != d && o == in[e][0]) return ASCAN_EINVAL;
        for (int j = 0; j < 2; ++j)
          if ((e != d || j != k) && o == out[e][j]) return ASCAN_EINVAL;
      }
    }
  const int64_t n = num_channels * seq_total;
  if (n == 0 || num_seq == 0) return ASCAN_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  Workspace wf, wb;
  rc = carve_bidi(workspace, workspace_bytes, num_channels, seq_total, wf, wb, s);
  if (rc != ASCAN_OK) return rc;
#define ASCAN_BWD_BIDI_CALL(T, I)                                                               \
  bwd_bidi_typed<T, I>(in, out, cu_seqlens, num_seq, num_channels, seq_total, wf, wb, s)
  ASCAN_DISPATCH_TYPES(dtype, cu_index_type, ASCAN_BWD_BIDI_CALL);
#undef ASCAN_BWD_BIDI_CALL
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

// Device address of g_noalloc_scratch in the calling thread's current CUDA
// context.  In host code the symbol is only a host-side stand-in, so the
// address is looked up with cudaGetSymbolAddress (with the device current)
// once per context and cached under the context's unique ID
// (cuCtxGetId): a module global belongs to a context, not to a device, and a
// foreign binding may run in a context it created itself, or in a primary
// context re-created after cudaDeviceReset -- each gets its own lookup.
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

static bool current_context_id(unsigned long long* id) {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
  });
  CUcontext ctx = nullptr;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return false;
  return get_id(ctx, id) == CUDA_SUCCESS;
}

static void* noalloc_scratch(int* status) {
  struct Entry {
    unsigned long long ctx_id;
    void* ptr;
  };
  constexpr int kEntries = 64;
  static std::mutex mu;
  static Entry cache[kEntries] = {};
  static int next = 0;
  unsigned long long id = 0;
  if (!current_context_id(&id)) {
    // no context is current yet: the lookup below makes the device's primary
    // context current (runtime semantics), after which it has an ID
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr ||
        !current_context_id(&id)) {
      *status = ASCAN_ECUDA;
      return nullptr;
    }
  }
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < kEntries; ++i)
    if (cache[i].ptr != nullptr && cache[i].ctx_id == id) return cache[i].ptr;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) {
    *status = ASCAN_ECUDA;
    return nullptr;
  }
  cache[next] = Entry{id, p};
  next = (next + 1) % kEntries;
  return p;
}

int ascan_forward_noalloc(const void* gates, const void* tokens, void* tokens_out,
                          void* gates_out, const void* cu_seqlens, int cu_index_type,
                          int64_t num_seq, int64_t num_channels, int64_t seq_total, int dtype,
                          int reverse, void* stream) {
  int rc = check_common(cu_seqlens, cu_index_type, num_seq, num_channels, seq_total, dtype);
  if (rc != ASCAN_OK) return rc;
  const int64_t n = num_channels * seq_total;
  if (n == 0 || num_seq == 0) return ASCAN_OK;
  // the size limit is checked first, so that an oversized call is refused on
  // the host whatever else is wrong with it
  if (workspace_bytes_for(num_channels, seq_total, false) > kNoAllocScratchBytes)
    return ASCAN_ETOOLARGE;
  if (!gates || !tokens || !tokens_out) return ASCAN_EINVAL;
  void* ws = noalloc_scratch(&rc);
  if (ws == nullptr) return rc;
  Workspace w;
  rc = carve(ws, kNoAllocScratchBytes, num_channels, seq_total, w);
  if (rc != ASCAN_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the previous call's tickets and tile flags are still in the array
  if (cudaMemsetAsync(w.ticket, 0, w.clear_bytes, s) != cudaSuccess) return ASCAN_ECUDA;
#define ASCAN_FWD_NA_CALL(T, I)                                                                \
  fwd_typed<T, I>(gates, tokens, tokens_out, gates_out, cu_seqlens, num_seq, num_channels,     \
                  seq_total, reverse, w, s)
  ASCAN_DISPATCH_TYPES(dtype, cu_index_type, ASCAN_FWD_NA_CALL);
#undef ASCAN_FWD_NA_CALL
}

int ascan_set_implementation(int impl) {
  if (impl < 0 || impl > 4) return ASCAN_EINVAL;
  g_impl = impl;
  return ASCAN_OK;
}

int ascan_get_implementation(void) { return impl_mode(); }

int ascan_set_tile_width(int elems_per_thread) {
  if (elems_per_thread != 0 && elems_per_thread != 16 && elems_per_thread != 32)
    return ASCAN_EINVAL;
  g_tile_width = elems_per_thread;
  return ASCAN_OK;
}

int ascan_get_tile_width(void) { return g_tile_width; }

int ascan_get_device_error(int device, unsigned int* code, long long* detail) {
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) return ASCAN_EDEVICE;
  if (cudaSetDevice(device) != cudaSuccess) return ASCAN_EDEVICE;
  int rc = cudaDeviceSynchronize() == cudaSuccess ? ASCAN_OK : ASCAN_ECUDA;
  unsigned int c = 0;
  unsigned long long d = 0;
  // every compilation unit's module has its own word: OR the bits, keep the
  // first non-zero detail
#define ASCAN_READ_UNIT(NAME)                                                                 \
  if (rc == ASCAN_OK) {                                                                       \
    unsigned int uc = 0;                                                                      \
    unsigned long long ud = 0;                                                                \
    rc = unit_err_##NAME(0, &uc, &ud);                                                        \
    if (uc != 0u && c == 0u) d = ud;                                                          \
    c |= uc;                                                                                  \
  }
  ASCAN_UNITS(ASCAN_READ_UNIT)
#undef ASCAN_READ_UNIT
  cudaSetDevice(prev);
  if (code) *code = c;
  if (detail) *detail = static_cast<long long>(d);
  return rc;
}

int ascan_selftest_waits(void* workspace, size_t workspace_bytes, long long limit_ns,
                         long long* results, void* stream) {
  if (!workspace || !results || workspace_bytes < 512 ||
      (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return ASCAN_EINVAL;
  if (limit_ns < 1000000ll) limit_ns = 1000000ll;  // 1 ms .. the production limit
  if (limit_ns > static_cast<long long>(kLookbackTimeoutNs))
    limit_ns = static_cast<long long>(kLookbackTimeoutNs);
  return selftest_waits_run(workspace, limit_ns, results, static_cast<cudaStream_t>(stream));
}

volatile unsigned int* ascan_error_flag(void) {
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = nullptr;
    if (cudaHostAlloc(&h, 64, cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) {
      cudaGetLastError();
      return;
    }
    memset(h, 0, 64);
    void* d = nullptr;
    if (cudaHostGetDevicePointer(&d, h, 0) != cudaSuccess || d == nullptr) {
      cudaGetLastError();
      cudaFreeHost(h);
      return;
    }
    g_err_host_ptr = static_cast<uint32_t*>(h);
    g_err_host = static_cast<uint32_t*>(d);  // kernels launched from now on write it
  });
  return g_err_host_ptr;
}

int ascan_clear_device_error(int device) {
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) return ASCAN_EDEVICE;
  if (cudaSetDevice(device) != cudaSuccess) return ASCAN_EDEVICE;
  int rc = ASCAN_OK;
#define ASCAN_CLEAR_UNIT(NAME) \
  if (rc == ASCAN_OK) rc = unit_err_##NAME(1, nullptr, nullptr);
  ASCAN_UNITS(ASCAN_CLEAR_UNIT)
#undef ASCAN_CLEAR_UNIT
  if (g_err_host_ptr) *reinterpret_cast<volatile uint32_t*>(g_err_host_ptr) = 0u;
  cudaSetDevice(prev);
  return rc;
}

}  // extern "C"

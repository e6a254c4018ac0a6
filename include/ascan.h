/*
 * ascan.h -- C ABI of the B200 (sm_100a) first-order linear-recurrence scan.
 *
 *   h[t] = g[t] * h[t-1] + x[t]        (causal; reverse: h[t+1] on the right)
 *
 * over the packed varlen layout of the reference project: every tensor is
 * [C, BL] row-major and contiguous, sequence i of channel c occupies
 * [c*BL + cu[i], c*BL + cu[i+1]), and BL == cu[num_seq]
 * (reference src/associative_scan_triton/scan_eager.py:74-83,
 * _kernels.py:49-52).
 *
 * Conventions shared by every entry point
 *   - All data pointers are caller-owned DEVICE memory on the current device.
 *   - dtype is one of ASCAN_F32 / ASCAN_F16 / ASCAN_BF16; every floating-point
 *     tensor of one call has that dtype.  Arithmetic is float32 for all three.
 *   - cu_seqlens is int32 (ASCAN_I32) or int64 (ASCAN_I64) with num_seq + 1
 *     entries, monotone, cu[num_seq] == seq_total.  Positions of a row before
 *     cu[0] belong to no sequence and are not written.
 *   - stream is a cudaStream_t passed as void*; work is enqueued on it and
 *     the call does not synchronise.
 *   - workspace: scratch of at least ascan_workspace_size(...) bytes, 256-byte
 *     aligned, used by one call at a time (two calls in flight at once need two
 *     workspaces).  Its contents need no initialisation.
 *   - Return value: ASCAN_OK (0) or a negative ASCAN_E* code describing a bad
 *     argument or a CUDA launch failure.  Problems only visible on the device
 *     (a cu_seqlens that is not monotone or does not end at seq_total, a tile
 *     whose predecessor never published) set a sticky per-device error word
 *     read by ascan_get_device_error(), and the host-visible flag of
 *     ascan_error_flag() once it is enabled.  No device-side condition can
 *     make a kernel trap, hang or touch memory outside the arrays it was given.
 */
#ifndef ASCAN_H_
#define ASCAN_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ASCAN_API __attribute__((visibility("default")))
#else
#define ASCAN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define ASCAN_ABI_VERSION 1

enum ascan_dtype { ASCAN_F32 = 0, ASCAN_F16 = 1, ASCAN_BF16 = 2 };
enum ascan_index { ASCAN_I32 = 0, ASCAN_I64 = 1 };

enum ascan_status {
  ASCAN_OK = 0,
  ASCAN_EINVAL = -1,         /* bad size, dtype, flag or null pointer */
  ASCAN_EWORKSPACE = -2,     /* workspace missing, misaligned or too small */
  ASCAN_ECUDA = -3,          /* a CUDA call failed (launch, memset) */
  ASCAN_EDEVICE = -4,        /* no usable CUDA device */
  ASCAN_ETOOLARGE = -5,      /* problem exceeds the fixed scratch of ascan_forward_noalloc */
};

/* Bits of the sticky per-device error word. */
#define ASCAN_DEV_ERR_CU_END 0x1u       /* cu_seqlens[num_seq] != seq_total */
#define ASCAN_DEV_ERR_CU_ORDER 0x2u     /* cu_seqlens not monotone / out of [0, seq_total] */
#define ASCAN_DEV_ERR_LOOKBACK 0x4u     /* a tile predecessor never published (bounded wait expired) */
#define ASCAN_DEV_ERR_EXCHANGE 0x8u     /* a peer rank's record or release never came (bounded wait expired) */

/* Library identification. */
ASCAN_API int ascan_abi_version(void);
ASCAN_API const char* ascan_build_info(void);

/* Human-readable text for an ascan_status value. */
ASCAN_API const char* ascan_strerror(int status);

/*
 * Bytes of workspace that ascan_forward / ascan_backward need for
 * num_channels * seq_total elements of dtype.
 */
ASCAN_API size_t ascan_workspace_size(int64_t num_channels, int64_t seq_total, int dtype);

/*
 * Forward scan.  Replaces the reference's two forward kernels and their
 * dispatcher:
 *   forward_scan_chunked            src/associative_scan_triton/_kernels.py:19-81
 *   forward_scan_onepass_pipelined  src/associative_scan_triton/_kernels.py:84-168
 *   forward_scan_full (routing)     src/associative_scan_triton/_dispatcher.py:12-70
 * One kernel covers every sequence length; chunk_size / NUM_STAGES have no
 * equivalent here.
 *
 *   gates, tokens      inputs [C, BL]
 *   tokens_out         output [C, BL]; may equal tokens (in place, INPLACE=True)
 *   gates_out          NULL, or output [C, BL] receiving the cumulative gate
 *                      product from each sequence's first element (the
 *                      reference's TESTING=True write-back); may equal gates
 *   reverse            0: h[t] = g[t]h[t-1] + x[t];  1: h[t] = g[t]h[t+1] + x[t]
 */
ASCAN_API int ascan_forward(const void* gates, const void* tokens, void* tokens_out, void* gates_out,
                  const void* cu_seqlens, int cu_index_type, int64_t num_seq,
                  int64_t num_channels, int64_t seq_total, int dtype, int reverse,
                  void* workspace, size_t workspace_bytes, void* stream);

/*
 * Fused backward.  Replaces the reference's two backward kernels and their
 * dispatcher:
 *   backward_scan_fused               src/associative_scan_triton/_kernels.py:171-287
 *   backward_scan_fused_single_chunk  src/associative_scan_triton/_kernels.py:290-374
 *   backward_scan_fused_full          src/associative_scan_triton/_dispatcher.py:73-117
 *
 *   grad      dL/dh, [C, BL]
 *   gates     the forward's gates
 *   states    the forward's outputs h
 *   d_tokens  output dL/dx = dh
 *   d_gates   output dL/dg = dh[t] * h[t-1]   (causal; h[t+1] when causal == 0)
 *   causal    1: adjoint of the causal scan (dh runs right to left);
 *             0: adjoint of the reverse scan.
 * Sequence boundaries: g past the end reads as 1, h before the start as 0.
 */
ASCAN_API int ascan_backward(const void* grad, const void* gates, const void* states, void* d_tokens,
                   void* d_gates, const void* cu_seqlens, int cu_index_type, int64_t num_seq,
                   int64_t num_channels, int64_t seq_total, int dtype, int causal,
                   void* workspace, size_t workspace_bytes, void* stream);

/*
 * Forward scan that allocates nothing: ascan_forward without the workspace
 * arguments.  No counterpart in the reference.
 *
 * For callers that cannot allocate device memory when they call the scan --
 * for example a serving loop that runs under a fixed memory budget and owns
 * no allocator, a plugin whose host application hands it only the input and
 * output buffers, or a foreign-language binding of this C ABI that has no
 * access to torch's caching allocator.  They still pass their inputs and
 * outputs; the look-back scratch (tile tickets and status records) lives in
 * a fixed array of ASCAN_NOALLOC_SCRATCH_BYTES inside this library, which
 * every GPU that loads the library holds until the process exits.
 *
 * Limits and rules:
 *   - num_channels * seq_total <= ASCAN_NOALLOC_MAX_ELEMENTS, otherwise
 *     ASCAN_ETOOLARGE is returned and nothing is launched;
 *   - every call on a device uses the same array: calls that overlap on the
 *     GPU (two streams, two threads) race and corrupt each other's results --
 *     serialise them, or use ascan_forward with separate workspaces;
 *   - the array keeps the previous call's contents; each call clears the part
 *     that must start at zero before its kernel runs (stream-ordered);
 *   - the first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress, with that device current) and caches it; make
 *     that first call before any stream capture begins;
 *   - no cudaMalloc, cudaFree or other allocating routine is called.
 * Arguments, results and other return codes are those of ascan_forward.
 */
#define ASCAN_NOALLOC_SCRATCH_BYTES (2u << 20)
#define ASCAN_NOALLOC_MAX_ELEMENTS 536805376ll /* 131056 status slots of 4096 elements */
ASCAN_API int ascan_forward_noalloc(const void* gates, const void* tokens, void* tokens_out,
                                    void* gates_out, const void* cu_seqlens, int cu_index_type,
                                    int64_t num_seq, int64_t num_channels, int64_t seq_total,
                                    int dtype, int reverse, void* stream);

/*
 * Time slabs: the scan of columns [t0, t1) of every row when the sequence
 * axis of a longer problem is split across devices (the rest of each row
 * lives on other GPUs).  No counterpart in the reference, whose kernels see
 * whole rows; these entry points serve a time-sharded run (reduce, exchange a
 * few floats per row, scan again), see associative_scan_triton/time_shard.py.
 *
 * cu_seqlens are the slab's own boundaries rebased to the slab (cu[0] = 0,
 * cu[S] = seq_total): the slab's first piece may continue a sequence that
 * started on an earlier device, and its last piece may go on after it.
 * All pointers must be 16-byte aligned and the slab must hold at least one
 * 128-byte row; otherwise ASCAN_EINVAL.  Per-row arrays are float32, indexed
 * by channel, in device memory.
 *
 * ascan_forward_slab: ascan_forward plus
 *   row_carry     [C][2] (gate product, state) that enters each row's first
 *                 element in scan order (NULL: none, as ascan_forward);
 *   row_aggregate [C][2] output: the inclusive (gate product, state) at each
 *                 row's last element in scan order (NULL: not written).
 *   tokens_out may be NULL together with gates_out for an aggregate-only pass
 *   (reads gates and tokens, writes only row_aggregate): a row reduction over
 *   the row's last sequence piece in scan order, no scan.
 * ascan_backward_slab: ascan_backward plus
 *   row_carry      [C] additive term for the adjoint at each row's first
 *                  element in scan order (causal: the slab's last column):
 *                  the successor gate times the successor adjoint, both from
 *                  the neighbouring slab (NULL: none);
 *   row_state_halo [C] state neighbour of the element whose neighbour lies
 *                  outside the slab (causal: h[t0-1], anti-causal: h[t1]);
 *                  that element's gate gradient uses it instead of being
 *                  zero at a sequence start (NULL: as ascan_backward);
 *   row_aggregate  [C][2] output: inclusive (coefficient product, adjoint) at
 *                  each row's last element in scan order, where the product
 *                  leaves out the first element's coefficient (it lives in
 *                  row_carry).
 *   d_tokens and d_gates may both be NULL for an aggregate-only pass (a row
 *   reduction over the row's first sequence piece in array order for the
 *   causal adjoint; the states are not read).
 */
ASCAN_API int ascan_forward_slab(const void* gates, const void* tokens, void* tokens_out,
                                 void* gates_out, const void* cu_seqlens, int cu_index_type,
                                 int64_t num_seq, int64_t num_channels, int64_t seq_total,
                                 int dtype, int reverse, const float* row_carry,
                                 float* row_aggregate, void* workspace, size_t workspace_bytes,
                                 void* stream);
ASCAN_API int ascan_backward_slab(const void* grad, const void* gates, const void* states,
                                  void* d_tokens, void* d_gates, const void* cu_seqlens,
                                  int cu_index_type, int64_t num_seq, int64_t num_channels,
                                  int64_t seq_total, int dtype, int causal, const float* row_carry,
                                  const float* row_state_halo, float* row_aggregate,
                                  void* workspace, size_t workspace_bytes, void* stream);

/*
 * Carry fold of a time-sharded run (no counterpart in the reference): the
 * carry that enters slab `rank` of `world` (world <= 32), from the records all
 * ranks contributed to one all-gather -- record j (record_floats floats,
 * device memory) is rank j's:
 *   direction 0 (forward):  [0, 2C)  ascan_forward_slab's row_aggregate of
 *                                    slab j (gate product, state) per row
 *      -> carry_out [C][2]: row_carry for ascan_forward_slab; halo_out NULL
 *   direction 1 (backward): [0, 2C)  ascan_backward_slab's row_aggregate of
 *                                    slab j (from a zero row_carry)
 *                           [2C, 3C) slab j's first gate column g[t0_j]
 *                           [3C, 4C) slab j's last state column h[t1_j - 1]
 *      -> carry_out [C]: row_carry for ascan_backward_slab; halo_out [C]
 *         (nullable): row_state_halo, h[t0 - 1] or 0 at a sequence start
 * starts_new_mask bit j: a sequence starts at slab j's first column;
 * inner_boundary_mask bit j: a sequence boundary lies strictly inside slab j.
 * One small kernel on `stream`; replaces a host loop over the ranks
 * (associative_scan_triton/time_shard.py: forward_carry, backward_carry,
 * state_halo restate it).
 */
ASCAN_API int ascan_time_shard_fold(const float* records, int64_t record_floats, int world,
                                    int rank, int64_t num_channels, uint32_t starts_new_mask,
                                    uint32_t inner_boundary_mask, int direction,
                                    float* carry_out, float* halo_out, void* stream);

/*
 * The same carry exchange without a collective (no counterpart in the
 * reference): every rank owns an exchange buffer in its own device memory,
 * maps the other ranks' buffers through CUDA IPC, and one kernel per
 * direction publishes this rank's record in its buffer, waits for the records
 * of the ranks its slab depends on and reads them over NVLink, folding them
 * exactly as ascan_time_shard_fold does.
 *
 * ascan_exchange_bytes(C)         bytes of one exchange buffer
 * ascan_exchange_create(C, &buf)  cudaMalloc + zero on the current device
 * ascan_exchange_export(buf, h)   its IPC handle, ASCAN_IPC_HANDLE_BYTES bytes
 * ascan_exchange_import(h, &peer) map another process's buffer (never this
 *                                 process's own: use its pointer directly)
 * ascan_exchange_close(peer)      unmap it
 * ascan_exchange_destroy(buf)     free this process's buffer (every peer must
 *                                 have closed its mapping first)
 *
 * ascan_time_shard_exchange: buffers = device array [world] of the buffers as
 * this process addresses them (own buffer at `rank`); aggregate = this rank's
 * [C][2] row_aggregate (ascan_forward_slab / ascan_backward_slab); gates and
 * states ([C][seq_total], `dtype`) give the backward record's first gate and
 * last state columns (direction 1; NULL for direction 0); masks, carry_out
 * and halo_out as for ascan_time_shard_fold.  parts = H > 1 (only for a slab
 * with no sequence boundary inside, seq_total a multiple of H): the slab was
 * scanned as [H C][seq_total / H] (every row cut into H parts), aggregate is
 * [H C][2] (one record per part), the record sent is each row's parts
 * composed, and carry_out ([H C][2] forward, [H C] backward) and halo_out
 * ([H C]) hold one carry / halo per part -- so the seeded pass runs on the
 * same [H C][seq_total / H] view, with H times more rows in its tile order.
 * The fold then also needs aggregate and (backward) gates and states.
 * mode: 1 publish only, 2 wait
 * and fold only, 3 both in one kernel (the normal case: one rank per GPU).
 * Modes 1 then 2 let one process emulate all ranks on one device (publish
 * every rank first, then fold every rank), so that no kernel waits for a
 * kernel launched after it.  Every rank must run the same sequence of
 * exchanges per direction.  Every wait gives up after timeout_ns
 * (ASCAN_DEV_ERR_EXCHANGE); the kernel then completes and the stream stays
 * usable.
 */
#define ASCAN_IPC_HANDLE_BYTES 64
ASCAN_API size_t ascan_exchange_bytes(int64_t num_channels);
ASCAN_API int ascan_exchange_create(int64_t num_channels, void** buffer_out);
ASCAN_API int ascan_exchange_export(void* buffer, void* handle_out);
ASCAN_API int ascan_exchange_import(const void* handle, void** peer_buffer_out);
ASCAN_API int ascan_exchange_close(void* peer_buffer);
ASCAN_API int ascan_exchange_destroy(void* buffer);
ASCAN_API int ascan_time_shard_exchange(void* buffer, const void* buffers, int world, int rank,
                                        int64_t num_channels, int64_t seq_total, int parts,
                                        const float* aggregate, const void* gates,
                                        const void* states, int dtype, uint32_t starts_new_mask,
                                        uint32_t inner_boundary_mask, int direction, int mode,
                                        float* carry_out, float* halo_out, long long timeout_ns,
                                        void* stream);

/*
 * Bidirectional pair in one launch: the causal scan of (gates_fwd,
 * tokens_fwd) and the reverse scan of (gates_bwd, tokens_bwd), same
 * cu_seqlens and shape.  Replaces the two forward_scan_full calls of
 * ScanBidirectionalBranched.forward
 * (src/associative_scan_triton/scan_eager.py:122-131) and of the
 * scan_bidi_fwd triton_op (src/associative_scan_triton/scan_compiled.py:208-240).
 * When the persistent kernels apply, the launch's CTAs are split in two
 * groups, one per scan; otherwise the two scans run one after the other.
 * The outputs may equal their own direction's tokens (in place) but no
 * buffer of the other direction.  workspace: ascan_workspace_size_bidi bytes.
 */
ASCAN_API size_t ascan_workspace_size_bidi(int64_t num_channels, int64_t seq_total, int dtype);
ASCAN_API int ascan_forward_bidi(const void* gates_fwd, const void* tokens_fwd,
                                 void* tokens_out_fwd, const void* gates_bwd,
                                 const void* tokens_bwd, void* tokens_out_bwd,
                                 const void* cu_seqlens, int cu_index_type, int64_t num_seq,
                                 int64_t num_channels, int64_t seq_total, int dtype,
                                 void* workspace, size_t workspace_bytes, void* stream);

/*
 * Adjoint of ascan_forward_bidi in one launch: ascan_backward with causal = 1
 * on the *_fwd buffers and with causal = 0 on the *_bwd buffers.  Replaces
 * the two backward_scan_fused_full calls of
 * ScanBidirectionalBranched.backward
 * (src/associative_scan_triton/scan_eager.py:160-169) and the scan_bidi_bwd
 * triton_op (src/associative_scan_triton/scan_compiled.py:243-279).  Every output must
 * differ from every other output and from the gates and states of both
 * directions; d_tokens may equal its own direction's grad.
 */
ASCAN_API int ascan_backward_bidi(const void* grad_fwd, const void* gates_fwd,
                                  const void* states_fwd, void* d_tokens_fwd, void* d_gates_fwd,
                                  const void* grad_bwd, const void* gates_bwd,
                                  const void* states_bwd, void* d_tokens_bwd, void* d_gates_bwd,
                                  const void* cu_seqlens, int cu_index_type, int64_t num_seq,
                                  int64_t num_channels, int64_t seq_total, int dtype,
                                  void* workspace, size_t workspace_bytes, void* stream);

/*
 * Shift by one position inside every sequence and pad the vacated slot.
 * Replaces _shift_pad_kernel / shift_pad_compiled
 * (src/associative_scan_triton/_shift_pad.py:63-165) and the torch.roll
 * variant shift_pad (_shift_pad.py:18-55).
 *   backward 1: out[t] = data[t-1], pad at sequence starts cu[0..S-1]
 *            0: out[t] = data[t+1], pad at sequence ends cu[1..S]-1
 *   wrap     1: source index wraps around the row (torch.roll variant)
 *            0: source index is clamped to [0, BL-1] (kernel variant)
 * out must not overlap data.
 */
ASCAN_API int ascan_shift_pad(const void* data, void* out, const void* cu_seqlens, int cu_index_type,
                    int64_t num_seq, int64_t num_channels, int64_t seq_total, int dtype,
                    double pad_value, int backward, int wrap, void* stream);

/*
 * Kernel family used by the calls that follow (process-wide):
 *   0  automatic (the default; env ASCAN_IMPL=simple|tma|tma-flat|tma-row
 *      overrides it): the persistent TMA-pipelined kernels whenever
 *      possible (as 2), the plain kernels otherwise
 *   1  always the plain kernels (128-bit loads, one CTA per tile)
 *   2  the persistent TMA-pipelined kernels whenever every pointer is
 *      16-byte aligned and the array holds at least one 128-byte row,
 *      the plain kernels otherwise
 *   3  as 2, tiles always dealt in flat order (a tile's predecessor is the
 *      tile before it in memory)
 *   4  as 2, tiles dealt tile-major across rows whenever every row is a
 *      whole number of tiles (a tile's predecessor is in the same row)
 * Both families compute the same results; the switch exists for testing
 * and measurement.  No counterpart in the reference, which has one
 * Triton kernel per case.
 */
ASCAN_API int ascan_set_implementation(int impl);
ASCAN_API int ascan_get_implementation(void);

/*
 * Tile width of the persistent kernels, for tests and tuning (no
 * counterpart in the reference): 0 (default) chooses per launch, 16 or 32
 * forces 4096- or 8192-element tiles (16 or 32 elements per consumer
 * thread) wherever the library has both kernels -- the forward of every
 * dtype without gates_out (fp32 ragged rows excepted: their shifted load
 * would exceed a TMA box), and the backward of fp16/bf16 (time slabs
 * included); other launches always use 16.  Process-wide; results agree up
 * to rounding.
 */
ASCAN_API int ascan_set_tile_width(int elems_per_thread);
ASCAN_API int ascan_get_tile_width(void);

/*
 * Read the sticky error word of `device` (ASCAN_DEV_ERR_* bits; 0 = none).
 * Synchronises that device first.  *detail, if non-NULL, receives an
 * implementation-defined integer about the first error (e.g. a tile index).
 * Returns ASCAN_OK or a negative status.
 */
ASCAN_API int ascan_get_device_error(int device, unsigned int* code, long long* detail);

/*
 * Self-test of the kernels' bounded waits (no counterpart in the reference):
 * one warp waits on a stage barrier nobody arrives on, on a hand-off slot
 * nobody tags and on a look-back predecessor that never publishes, each with
 * the limit `limit_ns` (clamped to 1 ms .. 2 s).  Every wait must give up and
 * the context stay usable.  `workspace`: device memory of at least 512 bytes,
 * 256-byte aligned (cleared here).  results[4] (host): barrier wait
 * succeeded, slot wait succeeded, look-back gave up, elapsed nanoseconds.
 * Synchronises `stream`.  Does not touch the sticky device error word.
 */
ASCAN_API int ascan_selftest_waits(void* workspace, size_t workspace_bytes, long long limit_ns,
                                   long long* results, void* stream);

/*
 * Host-visible error flag (no counterpart in the reference): the address of a
 * word of pinned, mapped host memory that every kernel which sets a bit of
 * the sticky device error word also writes (with that error's bits), so a
 * caller can poll for device-side errors after each call without
 * synchronising.  The first call allocates the word (cudaHostAlloc, mapped
 * and portable; make it before any stream capture) and enables it for every
 * launch that follows, in every thread and on every device of the process.
 * Concurrent reports may overwrite each other's bits in this word; the sticky
 * word (ascan_get_device_error) keeps all of them.  ascan_clear_device_error
 * zeroes it.  Returns NULL when it cannot be allocated (no device).
 */
ASCAN_API volatile unsigned int* ascan_error_flag(void);

/* Reset the sticky error word of `device` (and the host-visible flag). */
ASCAN_API int ascan_clear_device_error(int device);

#ifdef __cplusplus
}
#endif

#endif /* ASCAN_H_ */

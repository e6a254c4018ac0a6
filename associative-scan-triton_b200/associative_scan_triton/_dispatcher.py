"""Forward / backward dispatchers with the reference's signatures.

Reference: src/associative_scan_triton/_dispatcher.py:12-117.  The reference
routes single-chunk and multi-chunk launches to different Triton kernels; the
B200 library has one kernel per direction for every length, so both routes
end in the same native call.  Argument checking and defaults are kept:
``grid[0]`` must equal ``len(cu_seqlens) - 1``, ``tokens_out=None`` means in
place, and ``TESTING`` (default True) writes the cumulative gate products back
into ``gates``.
"""

from __future__ import annotations

from . import _lib


def forward_scan_full(
  gates,
  tokens,
  cu_seqlens,
  grid: tuple,
  REVERSE,
  CHUNK_SIZE,
  TESTING=True,
  NUM_STAGES=None,
  tokens_out=None,
) -> None:
  """Forward scan of every (sequence, channel) pair.

  Args:
    gates, tokens: [C, BL] (or [BL] with C = grid[2]) CUDA tensors.
    cu_seqlens: [num_seq + 1] int32/int64 CUDA tensor, cu_seqlens[-1] == BL.
    grid: (num_seq, num_chunks, C) as built by ``get_grid``.
    REVERSE: scan right to left (h[t] = g[t] h[t+1] + x[t]).
    CHUNK_SIZE, NUM_STAGES: accepted for compatibility; unused.
    TESTING: also write the cumulative gate products into ``gates``.
    tokens_out: output tensor; None writes the result into ``tokens``.
  """
  assert len(cu_seqlens) - 1 == grid[0], "cu_seqlens do not match grid configuration"
  out = tokens if tokens_out is None else tokens_out
  _lib.forward(gates, tokens, out, gates if TESTING else None, cu_seqlens,
               num_seq=grid[0], num_channels=grid[2], reverse=bool(REVERSE))


def backward_scan_fused_full(
  grad,
  gates,
  states,
  d_tokens_out,
  d_gates_out,
  cu_seqlens,
  grid: tuple,
  CHUNK_SIZE,
  CAUSAL,
  NUM_STAGES=None,
) -> None:
  """Fused backward: d_tokens = dh, d_gates = dh * (shifted states).

  CAUSAL=True is the adjoint of the causal scan (dh[t] = dy[t] + g[t+1] dh[t+1],
  d_gates[t] = dh[t] h[t-1]); CAUSAL=False the adjoint of the reverse scan.
  """
  num_seq, _num_chunks, no_channels = grid
  _lib.backward(grad, gates, states, d_tokens_out, d_gates_out, cu_seqlens,
                num_seq=num_seq, num_channels=no_channels, causal=bool(CAUSAL))


def forward_scan_full_bidi(gates_fwd, tokens_fwd, out_fwd, gates_bwd, tokens_bwd, out_bwd,
                           cu_seqlens, grid: tuple, CHUNK_SIZE, NUM_STAGES=None) -> None:
  """``forward_scan_full(REVERSE=False, TESTING=False)`` on the *_fwd pair and
  ``forward_scan_full(REVERSE=True, TESTING=False)`` on the *_bwd pair, as
  one launch (the two calls of the reference's
  ``ScanBidirectionalBranched.forward``, scan_eager.py:122-131)."""
  assert len(cu_seqlens) - 1 == grid[0], "cu_seqlens do not match grid configuration"
  _lib.forward_bidi(gates_fwd, tokens_fwd, out_fwd, gates_bwd, tokens_bwd, out_bwd, cu_seqlens,
                    num_seq=grid[0], num_channels=grid[2])


def backward_scan_fused_full_bidi(grad_fwd, gates_fwd, states_fwd, d_tokens_fwd, d_gates_fwd,
                                  grad_bwd, gates_bwd, states_bwd, d_tokens_bwd, d_gates_bwd,
                                  cu_seqlens, grid: tuple, CHUNK_SIZE, NUM_STAGES=None) -> None:
  """``backward_scan_fused_full(CAUSAL=True)`` on the *_fwd buffers and
  ``backward_scan_fused_full(CAUSAL=False)`` on the *_bwd buffers, as one
  launch (scan_eager.py:160-169 of the reference)."""
  num_seq, _num_chunks, no_channels = grid
  _lib.backward_bidi(grad_fwd, gates_fwd, states_fwd, d_tokens_fwd, d_gates_fwd, grad_bwd,
                     gates_bwd, states_bwd, d_tokens_bwd, d_gates_bwd, cu_seqlens,
                     num_seq=num_seq, num_channels=no_channels)

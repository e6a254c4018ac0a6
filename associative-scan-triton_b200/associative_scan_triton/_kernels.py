"""Kernel-level entry points with the reference's launch syntax.

The reference exposes four Triton kernels that callers launch directly as
``kernel[grid](name=tensor, ..., CONSTEXPR=value)`` (reference
src/associative_scan_triton/_kernels.py:19-374, launched that way in
tests/test_scan_kernels.py:74-83 and bench/bench_kernels.py:89-136).  Here the
same four names are launcher objects with the same keyword arguments; each one
calls the native library, which runs a single sm_100a kernel per direction for
every sequence length.  ``CHUNK_SIZE``, ``NUM_CHUNKS`` and ``NUM_STAGES`` are
accepted and ignored: the B200 kernels tile by 4096 elements and always
process whole sequences.
"""

from __future__ import annotations

from . import _lib


def op(fl, xl, fr, xr):
  """The first-order recurrence combine: (fl, xl) then (fr, xr).

  Returns ``(fr * fl, fr * xl + xr)``; works on Python numbers and tensors.
  Reference: src/associative_scan_triton/_kernels.py:6-16.
  """
  f = fr * fl
  x = fr * xl + xr
  return f, x


class _Launcher:
  """``launcher[grid](**kwargs)`` -> native call; grid = (num_seq, ..., channels)."""

  def __init__(self, name: str, fn, doc: str):
    self.__name__ = name
    self._fn = fn
    self.__doc__ = doc

  def __getitem__(self, grid):
    grid = tuple(int(v) for v in grid)
    if len(grid) < 2:
      raise ValueError(f"{self.__name__}: grid must be (num_seq, ..., num_channels), got {grid}")

    def launch(**kwargs):
      return self._fn(grid, **kwargs)

    return launch

  def __repr__(self) -> str:
    return f"<associative_scan_triton kernel {self.__name__} (sm_100a native)>"


def _forward(grid, gates_ptr, tokens_ptr, tokens_out_ptr, cu_seqlens_ptr, REVERSE, TESTING,
             INPLACE, CHUNK_SIZE=None, NUM_CHUNKS=None, NUM_STAGES=None):
  out = tokens_ptr if INPLACE else tokens_out_ptr
  gates_out = gates_ptr if TESTING else None
  _lib.forward(gates_ptr, tokens_ptr, out, gates_out, cu_seqlens_ptr, num_seq=grid[0],
               num_channels=grid[-1], reverse=bool(REVERSE))


def _backward(grid, grad_ptr, gates_ptr, states_ptr, d_tokens_ptr, d_gates_ptr, cu_seqlens_ptr,
              CAUSAL, CHUNK_SIZE=None, NUM_CHUNKS=None, NUM_STAGES=None):
  _lib.backward(grad_ptr, gates_ptr, states_ptr, d_tokens_ptr, d_gates_ptr, cu_seqlens_ptr,
                num_seq=grid[0], num_channels=grid[-1], causal=bool(CAUSAL))


forward_scan_chunked = _Launcher(
  "forward_scan_chunked", _forward,
  """Forward scan; grid (num_seq, 1, C).  Reference _kernels.py:19-81.

  kwargs: gates_ptr, tokens_ptr, tokens_out_ptr, cu_seqlens_ptr, REVERSE,
  CHUNK_SIZE, TESTING (write cumulative gate products into gates), INPLACE
  (write the scan into tokens instead of tokens_out).""")

forward_scan_onepass_pipelined = _Launcher(
  "forward_scan_onepass_pipelined", _forward,
  """Forward scan; grid (num_seq, C).  Reference _kernels.py:84-168.

  kwargs as forward_scan_chunked plus NUM_CHUNKS and NUM_STAGES (ignored).""")

backward_scan_fused = _Launcher(
  "backward_scan_fused", _backward,
  """Fused backward; grid (num_seq, C).  Reference _kernels.py:171-287.

  kwargs: grad_ptr, gates_ptr, states_ptr, d_tokens_ptr, d_gates_ptr,
  cu_seqlens_ptr, CHUNK_SIZE, NUM_CHUNKS, NUM_STAGES, CAUSAL.""")

backward_scan_fused_single_chunk = _Launcher(
  "backward_scan_fused_single_chunk", _backward,
  """Fused backward; grid (num_seq, 1, C).  Reference _kernels.py:290-374.

  kwargs: grad_ptr, gates_ptr, states_ptr, d_tokens_ptr, d_gates_ptr,
  cu_seqlens_ptr, CHUNK_SIZE, CAUSAL.""")

"""torch.compile-safe scans: custom ops under the ``associative_scan_triton::`` namespace.

Reference: src/associative_scan_triton/scan_compiled.py:33-371 registers four
``triton_op``s.  Here they are ``torch.library.custom_op``s whose bodies call
the native library, with fake (meta) kernels for tracing and
``register_autograd`` for the backward.

* ``scan_causal_fwd``, ``scan_causal_bwd``, ``scan_bidi_fwd``,
  ``scan_bidi_bwd`` keep the reference's names and schemas exactly, so code or
  exported graphs that call ``torch.ops.associative_scan_triton.*`` directly
  see the same outputs -- including the ``gates.clone()`` that the
  reference's forward ops return (scan_compiled.py:113, :240).
* ``scan_causal_compiled`` / ``scan_bidirectional_branched_compiled`` call
  ``scan_causal_fwd_noclone`` / ``scan_bidi_fwd_noclone`` instead: they
  return only the scanned tokens and save the gates for the backward straight
  from the op's inputs, which removes that clone (one full read + write of
  every gate tensor).
"""

from __future__ import annotations

import torch

from . import _lib

_NS = "associative_scan_triton"


def _num_seq(cu_seqlens: torch.Tensor) -> int:
  return int(cu_seqlens.shape[0]) - 1


# ---------------------------------------------------------------------------
# causal
# ---------------------------------------------------------------------------


def _causal_fwd(gates, tokens, cu_seqlens, no_channels):
  out = torch.empty_like(tokens)
  _lib.forward(gates, tokens, out, None, cu_seqlens, _num_seq(cu_seqlens), no_channels, False)
  return out


@torch.library.custom_op(f"{_NS}::scan_causal_fwd_noclone", mutates_args=())
def scan_causal_fwd_noclone_op(gates: torch.Tensor, tokens: torch.Tensor,
                               cu_seqlens: torch.Tensor, num_chunks: int, no_channels: int,
                               chunk_size: int) -> torch.Tensor:
  """Causal scan forward; gates and tokens are read-only; returns the states."""
  return _causal_fwd(gates, tokens, cu_seqlens, no_channels)


@scan_causal_fwd_noclone_op.register_fake
def _scan_causal_fwd_noclone_fake(gates, tokens, cu_seqlens, num_chunks, no_channels, chunk_size):
  return torch.empty_like(tokens)


@torch.library.custom_op(f"{_NS}::scan_causal_fwd", mutates_args=())
def scan_causal_fwd_op(gates: torch.Tensor, tokens: torch.Tensor, cu_seqlens: torch.Tensor,
                       num_chunks: int, no_channels: int,
                       chunk_size: int) -> tuple[torch.Tensor, torch.Tensor]:
  """The reference's op schema: returns (states, gates.clone())."""
  return _causal_fwd(gates, tokens, cu_seqlens, no_channels), gates.clone()


@scan_causal_fwd_op.register_fake
def _scan_causal_fwd_fake(gates, tokens, cu_seqlens, num_chunks, no_channels, chunk_size):
  return torch.empty_like(tokens), torch.empty_like(gates)


@torch.library.custom_op(f"{_NS}::scan_causal_bwd", mutates_args=())
def scan_causal_bwd_op(grad: torch.Tensor, gates: torch.Tensor, states: torch.Tensor,
                       cu_seqlens: torch.Tensor, num_chunks: int, no_channels: int,
                       chunk_size: int) -> tuple[torch.Tensor, torch.Tensor]:
  """Causal scan backward; returns (d_gates, d_tokens)."""
  grad = grad.contiguous()
  d_tokens = torch.empty_like(grad)
  d_gates = torch.empty_like(gates)
  _lib.backward(grad, gates, states, d_tokens, d_gates, cu_seqlens, _num_seq(cu_seqlens),
                no_channels, True)
  return d_gates, d_tokens


@scan_causal_bwd_op.register_fake
def _scan_causal_bwd_fake(grad, gates, states, cu_seqlens, num_chunks, no_channels, chunk_size):
  return torch.empty_like(gates), torch.empty_like(grad)


def _scan_causal_setup_context(ctx, inputs, output) -> None:
  gates, _tokens, cu_seqlens, num_chunks, no_channels, chunk_size = inputs
  states = output[0] if isinstance(output, tuple) else output
  ctx.save_for_backward(states, gates, cu_seqlens)
  ctx.num_chunks = num_chunks
  ctx.no_channels = no_channels
  ctx.chunk_size = chunk_size


def _scan_causal_backward(ctx, grad, *_grad_gates_copy):
  states, gates, cu_seqlens = ctx.saved_tensors
  if grad is None:
    grad = torch.zeros_like(states)
  d_gates, d_tokens = scan_causal_bwd_op(grad, gates, states, cu_seqlens, ctx.num_chunks,
                                         ctx.no_channels, ctx.chunk_size)
  return d_gates, d_tokens, None, None, None, None


for _op in (scan_causal_fwd_noclone_op, scan_causal_fwd_op):
  _op.register_autograd(_scan_causal_backward, setup_context=_scan_causal_setup_context)


# ---------------------------------------------------------------------------
# bidirectional, branched
# ---------------------------------------------------------------------------


def _bidi_fwd(gates_fwd, tokens_fwd, gates_bwd, tokens_bwd, cu_seqlens, no_channels):
  out_fwd = torch.empty_like(tokens_fwd)
  out_bwd = torch.empty_like(tokens_bwd)
  # both branches in one launch (ascan_forward_bidi)
  _lib.forward_bidi(gates_fwd, tokens_fwd, out_fwd, gates_bwd, tokens_bwd, out_bwd, cu_seqlens,
                    _num_seq(cu_seqlens), no_channels)
  return out_fwd, out_bwd


@torch.library.custom_op(f"{_NS}::scan_bidi_fwd_noclone", mutates_args=())
def scan_bidi_fwd_noclone_op(gates_fwd: torch.Tensor, tokens_fwd: torch.Tensor,
                             gates_bwd: torch.Tensor, tokens_bwd: torch.Tensor,
                             cu_seqlens: torch.Tensor, num_chunks: int, no_channels: int,
                             chunk_size: int) -> tuple[torch.Tensor, torch.Tensor]:
  """Causal branch over the *_fwd pair and reverse branch over the *_bwd pair."""
  return _bidi_fwd(gates_fwd, tokens_fwd, gates_bwd, tokens_bwd, cu_seqlens, no_channels)


@scan_bidi_fwd_noclone_op.register_fake
def _scan_bidi_fwd_noclone_fake(gates_fwd, tokens_fwd, gates_bwd, tokens_bwd, cu_seqlens,
                                num_chunks, no_channels, chunk_size):
  return torch.empty_like(tokens_fwd), torch.empty_like(tokens_bwd)


@torch.library.custom_op(f"{_NS}::scan_bidi_fwd", mutates_args=())
def scan_bidi_fwd_op(gates_fwd: torch.Tensor, tokens_fwd: torch.Tensor, gates_bwd: torch.Tensor,
                     tokens_bwd: torch.Tensor, cu_seqlens: torch.Tensor, num_chunks: int,
                     no_channels: int, chunk_size: int
                     ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
  """The reference's op schema: (out_fwd, out_bwd, gates_fwd.clone(), gates_bwd.clone())."""
  out_fwd, out_bwd = _bidi_fwd(gates_fwd, tokens_fwd, gates_bwd, tokens_bwd, cu_seqlens,
                               no_channels)
  return out_fwd, out_bwd, gates_fwd.clone(), gates_bwd.clone()


@scan_bidi_fwd_op.register_fake
def _scan_bidi_fwd_fake(gates_fwd, tokens_fwd, gates_bwd, tokens_bwd, cu_seqlens, num_chunks,
                        no_channels, chunk_size):
  return (torch.empty_like(tokens_fwd), torch.empty_like(tokens_bwd),
          torch.empty_like(gates_fwd), torch.empty_like(gates_bwd))


@torch.library.custom_op(f"{_NS}::scan_bidi_bwd", mutates_args=())
def scan_bidi_bwd_op(grad_fwd: torch.Tensor, grad_bwd: torch.Tensor, states_fwd: torch.Tensor,
                     states_bwd: torch.Tensor, gates_fwd: torch.Tensor, gates_bwd: torch.Tensor,
                     cu_seqlens: torch.Tensor, num_chunks: int, no_channels: int,
                     chunk_size: int
                     ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
  """Backward of both branches; returns (d_gates_fwd, d_tokens_fwd, d_gates_bwd, d_tokens_bwd)."""
  grad_fwd = grad_fwd.contiguous()
  grad_bwd = grad_bwd.contiguous()
  d_tokens_fwd = torch.empty_like(grad_fwd)
  d_gates_fwd = torch.empty_like(gates_fwd)
  d_tokens_bwd = torch.empty_like(grad_bwd)
  d_gates_bwd = torch.empty_like(gates_bwd)
  n = _num_seq(cu_seqlens)
  # both adjoints in one launch (ascan_backward_bidi)
  _lib.backward_bidi(grad_fwd, gates_fwd, states_fwd, d_tokens_fwd, d_gates_fwd, grad_bwd,
                     gates_bwd, states_bwd, d_tokens_bwd, d_gates_bwd, cu_seqlens, n, no_channels)
  return d_gates_fwd, d_tokens_fwd, d_gates_bwd, d_tokens_bwd


@scan_bidi_bwd_op.register_fake
def _scan_bidi_bwd_fake(grad_fwd, grad_bwd, states_fwd, states_bwd, gates_fwd, gates_bwd,
                        cu_seqlens, num_chunks, no_channels, chunk_size):
  return (torch.empty_like(gates_fwd), torch.empty_like(grad_fwd), torch.empty_like(gates_bwd),
          torch.empty_like(grad_bwd))


def _scan_bidi_setup_context(ctx, inputs, output) -> None:
  gates_fwd, _tf, gates_bwd, _tb, cu_seqlens, num_chunks, no_channels, chunk_size = inputs
  out_fwd, out_bwd = output[0], output[1]
  ctx.save_for_backward(out_fwd, out_bwd, gates_fwd, gates_bwd, cu_seqlens)
  ctx.num_chunks = num_chunks
  ctx.no_channels = no_channels
  ctx.chunk_size = chunk_size


def _scan_bidi_backward(ctx, grad_fwd, grad_bwd, *_grad_gates_copies):
  states_fwd, states_bwd, gates_fwd, gates_bwd, cu_seqlens = ctx.saved_tensors
  if grad_fwd is None:
    grad_fwd = torch.zeros_like(states_fwd)
  if grad_bwd is None:
    grad_bwd = torch.zeros_like(states_bwd)
  d_gates_fwd, d_tokens_fwd, d_gates_bwd, d_tokens_bwd = scan_bidi_bwd_op(
    grad_fwd, grad_bwd, states_fwd, states_bwd, gates_fwd, gates_bwd, cu_seqlens,
    ctx.num_chunks, ctx.no_channels, ctx.chunk_size)
  return d_gates_fwd, d_tokens_fwd, d_gates_bwd, d_tokens_bwd, None, None, None, None


for _op in (scan_bidi_fwd_noclone_op, scan_bidi_fwd_op):
  _op.register_autograd(_scan_bidi_backward, setup_context=_scan_bidi_setup_context)


# ---------------------------------------------------------------------------
# public API (same signatures as the eager functions)
# ---------------------------------------------------------------------------


def scan_causal_compiled(gates: torch.Tensor, tokens: torch.Tensor, args: dict) -> torch.Tensor:
  """Drop-in replacement for ``scan_causal`` that torch.compile can trace."""
  _num_seq_grid, num_chunks, no_channels = args["grid"]
  return scan_causal_fwd_noclone_op(gates, tokens, args["cu_seqlens"], num_chunks, no_channels,
                                    args["chunk_size"])


def scan_bidirectional_branched_compiled(
  gates_fwd: torch.Tensor,
  tokens_fwd: torch.Tensor,
  gates_bwd: torch.Tensor,
  tokens_bwd: torch.Tensor,
  args: dict,
  testing: bool = True,
) -> tuple[torch.Tensor, torch.Tensor]:
  """Drop-in replacement for ``scan_bidirectional_branched`` that torch.compile can trace."""
  _num_seq_grid, num_chunks, no_channels = args["grid"]
  return scan_bidi_fwd_noclone_op(gates_fwd, tokens_fwd, gates_bwd, tokens_bwd,
                                  args["cu_seqlens"], num_chunks, no_channels,
                                  args["chunk_size"])

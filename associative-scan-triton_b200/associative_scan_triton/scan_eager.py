"""Autograd functions: causal and bidirectional-branched scans.

Reference: src/associative_scan_triton/scan_eager.py:20-210.  Same classes,
functions, argument checks and saved tensors; the forward and backward run the
native sm_100a kernels through the dispatchers.
"""

from __future__ import annotations

import torch

from ._dispatcher import (
  backward_scan_fused_full,
  backward_scan_fused_full_bidi,
  forward_scan_full,
  forward_scan_full_bidi,
)


class ScanCausal(torch.autograd.Function):
  """Causal scan h[t] = g[t] h[t-1] + x[t] with a fused backward."""

  @staticmethod
  def forward(ctx, gates, tokens, args) -> torch.Tensor:
    shape = gates.shape
    assert tokens.shape == shape
    assert gates.is_contiguous()
    assert tokens.is_contiguous()
    cu_seqlens, chunk_size, grid = args["cu_seqlens"], args["chunk_size"], args["grid"]
    need_backward = gates.requires_grad or tokens.requires_grad

    out_tokens = torch.empty_like(tokens)
    forward_scan_full(gates, tokens, cu_seqlens, grid, REVERSE=False, CHUNK_SIZE=chunk_size,
                      TESTING=False, tokens_out=out_tokens)
    if need_backward:
      ctx.grid = grid
      ctx.cu_seqlens = cu_seqlens
      ctx.chunk_size = chunk_size
      ctx.save_for_backward(out_tokens, gates)
    return out_tokens

  @staticmethod
  def backward(ctx, grad_output):
    states, gates = ctx.saved_tensors
    grad_output = grad_output.contiguous()
    d_tokens = torch.empty_like(grad_output)
    d_gates = torch.empty_like(gates)
    backward_scan_fused_full(grad_output, gates, states, d_tokens, d_gates, ctx.cu_seqlens,
                             ctx.grid, CHUNK_SIZE=ctx.chunk_size, CAUSAL=True)
    return d_gates, d_tokens, None


def scan_causal(gates: torch.Tensor, tokens: torch.Tensor, args: dict) -> torch.Tensor:
  """Causal (unidirectional) scan.

  Args:
    gates, tokens: [C, B*L] CUDA tensors (float32 / float16 / bfloat16).
    args: {"cu_seqlens": [B+1] int tensor, "chunk_size": int,
           "grid": (num_seq, num_chunks, C)}.
  Returns:
    the scanned tokens, [C, B*L].
  """
  return ScanCausal.apply(gates, tokens, args)


class ScanBidirectionalBranched(torch.autograd.Function):
  """A causal branch over (gates_fwd, tokens_fwd) and a reverse branch over
  (gates_bwd, tokens_bwd)."""

  @staticmethod
  def forward(ctx, gates_fwd, tokens_fwd, gates_bwd, tokens_bwd, args, testing=False):
    shape = gates_fwd.shape
    assert tokens_fwd.shape == shape
    assert tokens_bwd.shape == shape
    assert gates_fwd.is_contiguous()
    assert gates_bwd.is_contiguous()
    assert tokens_fwd.is_contiguous()
    assert tokens_bwd.is_contiguous()
    cu_seqlens, chunk_size, grid = args["cu_seqlens"], args["chunk_size"], args["grid"]
    need_backward = (gates_fwd.requires_grad or tokens_fwd.requires_grad
                     or gates_bwd.requires_grad or tokens_bwd.requires_grad)

    out_fwd = torch.empty_like(tokens_fwd)
    out_bwd = torch.empty_like(tokens_bwd)
    # the reference's two forward_scan_full calls (scan_eager.py:122-131), as
    # one launch for both branches
    forward_scan_full_bidi(gates_fwd, tokens_fwd, out_fwd, gates_bwd, tokens_bwd, out_bwd,
                           cu_seqlens, grid, CHUNK_SIZE=chunk_size)
    if need_backward:
      ctx.grid = grid
      ctx.cu_seqlens = cu_seqlens
      ctx.chunk_size = chunk_size
      ctx.testing = testing
      ctx.save_for_backward(out_fwd, out_bwd, gates_fwd, gates_bwd)
    return out_fwd, out_bwd

  @staticmethod
  def backward(ctx, grad_output_fwd, grad_output_bwd):
    states_fwd, states_bwd, gates_fwd, gates_bwd = ctx.saved_tensors
    grad_output_fwd = grad_output_fwd.contiguous()
    grad_output_bwd = grad_output_bwd.contiguous()
    d_tokens_fwd = torch.empty_like(grad_output_fwd)
    d_gates_fwd = torch.empty_like(gates_fwd)
    d_tokens_bwd = torch.empty_like(grad_output_bwd)
    d_gates_bwd = torch.empty_like(gates_bwd)
    # the reference's two backward_scan_fused_full calls (scan_eager.py:160-169),
    # as one launch for both adjoints
    backward_scan_fused_full_bidi(grad_output_fwd, gates_fwd, states_fwd, d_tokens_fwd,
                                  d_gates_fwd, grad_output_bwd, gates_bwd, states_bwd,
                                  d_tokens_bwd, d_gates_bwd, ctx.cu_seqlens, ctx.grid,
                                  CHUNK_SIZE=ctx.chunk_size)
    return d_gates_fwd, d_tokens_fwd, d_gates_bwd, d_tokens_bwd, None, None


def scan_bidirectional_branched(
  gates_fwd: torch.Tensor,
  tokens_fwd: torch.Tensor,
  gates_bwd: torch.Tensor,
  tokens_bwd: torch.Tensor,
  args: dict,
  testing: bool = True,
) -> tuple[torch.Tensor, torch.Tensor]:
  """Causal scan of (gates_fwd, tokens_fwd) and reverse scan of (gates_bwd, tokens_bwd).

  ``testing`` is accepted for compatibility; as in the reference it does not
  change what is computed.
  """
  return ScanBidirectionalBranched.apply(gates_fwd, tokens_fwd, gates_bwd, tokens_bwd, args,
                                         testing)

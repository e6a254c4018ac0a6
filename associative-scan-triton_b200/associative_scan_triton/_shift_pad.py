"""shift_pad: shift every sequence by one position and pad the vacated slot.

Reference: src/associative_scan_triton/_shift_pad.py:18-165.  Both variants
run the native ``ascan_shift_pad`` kernel:

* ``shift_pad`` keeps the reference's eager semantics -- the source index wraps
  around the row like ``torch.roll`` -- and its zero-length-segment assertion;
* ``shift_pad_compiled`` is the ``associative_scan_triton::shift_pad`` custom
  op (torch.compile-safe) with the reference kernel's clamped source index.

The two differ only for rows whose first sequence does not start at 0.
"""

from __future__ import annotations

import torch

from . import _lib


def shift_pad(
  data: torch.Tensor,
  cu_seqlens: torch.Tensor,
  pad_value: float = 0.0,
  backward: bool = True,
) -> torch.Tensor:
  """Shift right (``backward=True``, pad at sequence starts) or left (pad at ends).

  Args:
    data: [C, BL] CUDA tensor.
    cu_seqlens: cumulative sequence lengths on the same device.
    pad_value: value written into the vacated slots.
    backward: True shifts right, False shifts left.
  """
  _C, _BL = data.shape
  assert not (cu_seqlens[1:] == cu_seqlens[:-1]).any(), "can't shift_pad zero-length seqments"
  out = torch.empty_like(data)
  _lib.shift_pad(data.contiguous(), out, cu_seqlens.contiguous(), pad_value, backward, wrap=True)
  return out


@torch.library.custom_op("associative_scan_triton::shift_pad", mutates_args=())
def shift_pad_compiled(
  data: torch.Tensor,
  cu_seqlens: torch.Tensor,
  pad_value: float,
  backward: bool,
) -> torch.Tensor:
  """torch.compile-safe shift_pad (clamped source index at row edges)."""
  out = torch.empty_like(data)
  _lib.shift_pad(data.contiguous(), out, cu_seqlens.contiguous(), pad_value, backward, wrap=False)
  return out


@shift_pad_compiled.register_fake
def _shift_pad_fake(data, cu_seqlens, pad_value, backward):
  return torch.empty_like(data)

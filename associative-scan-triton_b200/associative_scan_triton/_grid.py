"""Launch-geometry helpers, kept with the reference's names and results.

Reference: src/associative_scan_triton/_grid.py:4-70.  The B200 kernels size
their own launches from the tensors (4096-element tiles), so the grid tuple
only carries (number of sequences, -, number of channels) into them; these
helpers exist so that code written against the reference keeps working and
builds identical ``args["grid"]`` tuples.
"""

from __future__ import annotations


def next_power_of_2(n: int) -> int:
  """Smallest power of two >= n; 0 for n <= 0.

  Same results as the reference's bit-smearing version for n <= 2**64.
  """
  n = int(n)
  if n <= 0:
    return 0
  return 1 << (n - 1).bit_length()


def get_grid(no_seq: int, max_seqlen: int, chunk_size: int,
             no_channels: int) -> tuple[int, int, int]:
  """(num_seq, num_chunks, no_channels) as the reference computes it.

  Args:
    no_seq: len(cu_seqlens), i.e. number of sequences + 1
    max_seqlen: longest sequence in the batch
    chunk_size: chunk length of the reference kernels (must be even)
    no_channels: number of channels
  """
  assert chunk_size % 2 == 0, "chunk size must be divisible by 2"
  num_chunks = next_power_of_2(-(-max_seqlen // chunk_size))
  return (no_seq - 1, num_chunks, no_channels)


def get_num_stages(num_chunks: int, kernel: str = "fwd") -> int:
  """The reference's software-pipelining depth table (H100-tuned).

  Accepted for API compatibility; the B200 kernels take no stage count.
  """
  if num_chunks <= 1:
    return 1
  if kernel == "fwd":
    return 1 if num_chunks <= 4 else 3
  return 2 if num_chunks <= 4 else 3


def get_static_grid(max_seqlen: int, chunk_size: int,
                    no_channels: int) -> tuple[int, int]:
  """The batch-independent part (num_chunks, no_channels) of get_grid."""
  return get_grid(2, max_seqlen, chunk_size, no_channels)[1:]

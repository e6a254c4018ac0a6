"""First-order linear-recurrence scan for NVIDIA B200 (sm_100a).

Drop-in for the Python API of the reference package of the same name
(reference src/associative_scan_triton/__init__.py:1-36): the same modules,
functions, launcher objects, argument dicts and custom-op names.  Every op runs
hand-written CUDA kernels from the native library ``libascan_b200.so`` (C ABI
in include/ascan.h); CUDA tensors only, no CPU fallback.
"""

__version__ = "1.0.0"

from associative_scan_triton import _lib

_lib.try_load()

from associative_scan_triton._kernels import (  # noqa: E402
  op,
  forward_scan_chunked,
  forward_scan_onepass_pipelined,
  backward_scan_fused,
  backward_scan_fused_single_chunk,
)
from associative_scan_triton._dispatcher import forward_scan_full, backward_scan_fused_full  # noqa: E402
from associative_scan_triton._shift_pad import shift_pad, shift_pad_compiled  # noqa: E402
from associative_scan_triton._grid import (  # noqa: E402
  next_power_of_2,
  get_grid,
  get_static_grid,
  get_num_stages,
)
from associative_scan_triton.scan_eager import scan_causal, scan_bidirectional_branched  # noqa: E402
from associative_scan_triton.scan_compiled import (  # noqa: E402
  scan_causal_compiled,
  scan_bidirectional_branched_compiled,
)
from associative_scan_triton._lib import (  # noqa: E402
  ScanError,
  check_device_error,
  set_sync_check,
)

__all__ = [
  # Kernels
  "op",
  "forward_scan_chunked",
  "forward_scan_onepass_pipelined",
  "forward_scan_full",
  "backward_scan_fused",
  "backward_scan_fused_single_chunk",
  "backward_scan_fused_full",
  # Shift-pad
  "shift_pad",
  "shift_pad_compiled",
  # Grid utilities
  "next_power_of_2",
  "get_grid",
  "get_static_grid",
  # High-level API
  "scan_causal",
  "scan_causal_compiled",
  "scan_bidirectional_branched",
  "scan_bidirectional_branched_compiled",
]

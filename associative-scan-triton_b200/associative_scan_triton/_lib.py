"""ctypes binding of the native library ``libascan_b200.so`` (C ABI: include/ascan.h).

Every op of this package reaches the GPU through the entry points bound here --
``ascan_forward``, ``ascan_backward``, ``ascan_shift_pad``, the bidirectional
pairs and, for time slabs, ``ascan_forward_slab`` / ``ascan_backward_slab`` /
``ascan_time_shard_fold`` -- with raw device pointers, sizes and torch's
current CUDA stream.  There is no CPU
path: a missing library, a CPU tensor or a machine without CUDA raises.

Device-side checks (malformed ``cu_seqlens``, a look-back that gave up) set a
sticky error word on the device and a pinned host word (``ascan_error_flag``,
enabled by the first op).  After every op the host word is read -- a plain
memory read, no synchronisation -- and a set flag raises :class:`ScanError`
(with the exact bits, read after a synchronisation) from that op or a later
one, once the failing kernel has run.  With sync checking on
(``set_sync_check(True)`` or ``ASCAN_SYNC_CHECK=1``) every op synchronises and
reports its own error; :func:`check_device_error` does the same on demand.
"""

from __future__ import annotations

import ctypes
import os
import warnings
from pathlib import Path

import torch

LIB_NAME = "libascan_b200.so"
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

ASCAN_OK = 0
DEV_ERR_CU_END = 0x1
DEV_ERR_CU_ORDER = 0x2
DEV_ERR_LOOKBACK = 0x4
DEV_ERR_EXCHANGE = 0x8

DTYPE_CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
INDEX_CODES = {torch.int32: 0, torch.int64: 1}

# Symbols declared in include/ascan.h.
EXPORTED_SYMBOLS = (
  "ascan_abi_version",
  "ascan_build_info",
  "ascan_strerror",
  "ascan_workspace_size",
  "ascan_forward",
  "ascan_forward_noalloc",
  "ascan_backward",
  "ascan_forward_slab",
  "ascan_backward_slab",
  "ascan_time_shard_fold",
  "ascan_exchange_bytes",
  "ascan_exchange_create",
  "ascan_exchange_export",
  "ascan_exchange_import",
  "ascan_exchange_close",
  "ascan_exchange_destroy",
  "ascan_time_shard_exchange",
  "ascan_workspace_size_bidi",
  "ascan_forward_bidi",
  "ascan_backward_bidi",
  "ascan_shift_pad",
  "ascan_set_implementation",
  "ascan_get_implementation",
  "ascan_set_tile_width",
  "ascan_get_tile_width",
  "ascan_get_device_error",
  "ascan_clear_device_error",
  "ascan_error_flag",
  "ascan_selftest_waits",
)

IMPLEMENTATIONS = {"auto": 0, "simple": 1, "tma": 2, "tma-flat": 3, "tma-row": 4}


class ScanError(RuntimeError):
  """An error reported by the native library or detected on the device."""


_lib = None
_load_error: Exception | None = None
_sync_check = os.environ.get("ASCAN_SYNC_CHECK", "0") not in ("", "0")
_flag: ctypes.c_uint | None = None  # the library's pinned host error flag, once enabled


def _bind(lib) -> None:
  p, i64, ci, sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t
  lib.ascan_abi_version.restype = ci
  lib.ascan_abi_version.argtypes = []
  lib.ascan_build_info.restype = ctypes.c_char_p
  lib.ascan_build_info.argtypes = []
  lib.ascan_strerror.restype = ctypes.c_char_p
  lib.ascan_strerror.argtypes = [ci]
  lib.ascan_workspace_size.restype = sz
  lib.ascan_workspace_size.argtypes = [i64, i64, ci]
  lib.ascan_forward.restype = ci
  lib.ascan_forward.argtypes = [p, p, p, p, p, ci, i64, i64, i64, ci, ci, p, sz, p]
  lib.ascan_backward.restype = ci
  lib.ascan_backward.argtypes = [p, p, p, p, p, p, ci, i64, i64, i64, ci, ci, p, sz, p]
  lib.ascan_forward_slab.restype = ci
  lib.ascan_forward_slab.argtypes = [p, p, p, p, p, ci, i64, i64, i64, ci, ci, p, p, p, sz, p]
  lib.ascan_backward_slab.restype = ci
  lib.ascan_backward_slab.argtypes = [p, p, p, p, p, p, ci, i64, i64, i64, ci, ci, p, p, p, p,
                                      sz, p]
  lib.ascan_time_shard_fold.restype = ci
  lib.ascan_time_shard_fold.argtypes = [p, i64, ci, ci, i64, ctypes.c_uint32, ctypes.c_uint32, ci,
                                        p, p, p]
  lib.ascan_exchange_bytes.restype = sz
  lib.ascan_exchange_bytes.argtypes = [i64]
  lib.ascan_exchange_create.restype = ci
  lib.ascan_exchange_create.argtypes = [i64, ctypes.POINTER(p)]
  lib.ascan_exchange_export.restype = ci
  lib.ascan_exchange_export.argtypes = [p, p]
  lib.ascan_exchange_import.restype = ci
  lib.ascan_exchange_import.argtypes = [p, ctypes.POINTER(p)]
  lib.ascan_exchange_close.restype = ci
  lib.ascan_exchange_close.argtypes = [p]
  lib.ascan_exchange_destroy.restype = ci
  lib.ascan_exchange_destroy.argtypes = [p]
  lib.ascan_time_shard_exchange.restype = ci
  lib.ascan_time_shard_exchange.argtypes = [p, p, ci, ci, i64, i64, ci, p, p, p, ci,
                                            ctypes.c_uint32, ctypes.c_uint32, ci, ci, p, p,
                                            ctypes.c_longlong, p]
  lib.ascan_workspace_size_bidi.restype = sz
  lib.ascan_workspace_size_bidi.argtypes = [i64, i64, ci]
  lib.ascan_forward_bidi.restype = ci
  lib.ascan_forward_bidi.argtypes = [p, p, p, p, p, p, p, ci, i64, i64, i64, ci, p, sz, p]
  lib.ascan_backward_bidi.restype = ci
  lib.ascan_backward_bidi.argtypes = [p, p, p, p, p, p, p, p, p, p, p, ci, i64, i64, i64, ci,
                                      p, sz, p]
  lib.ascan_shift_pad.restype = ci
  lib.ascan_shift_pad.argtypes = [p, p, p, ci, i64, i64, i64, ci, ctypes.c_double, ci, ci, p]
  lib.ascan_set_implementation.restype = ci
  lib.ascan_set_implementation.argtypes = [ci]
  lib.ascan_get_implementation.restype = ci
  lib.ascan_get_implementation.argtypes = []
  lib.ascan_set_tile_width.restype = ci
  lib.ascan_set_tile_width.argtypes = [ci]
  lib.ascan_get_tile_width.restype = ci
  lib.ascan_get_tile_width.argtypes = []
  lib.ascan_get_device_error.restype = ci
  lib.ascan_get_device_error.argtypes = [ci, ctypes.POINTER(ctypes.c_uint),
                                         ctypes.POINTER(ctypes.c_longlong)]
  lib.ascan_clear_device_error.restype = ci
  lib.ascan_clear_device_error.argtypes = [ci]
  lib.ascan_error_flag.restype = p
  lib.ascan_error_flag.argtypes = []
  lib.ascan_selftest_waits.restype = ci
  lib.ascan_selftest_waits.argtypes = [p, sz, ctypes.c_longlong,
                                       ctypes.POINTER(ctypes.c_longlong), p]


def load(path: str | os.PathLike | None = None):
  """Load (once) and return the native library; raise if it is missing."""
  global _lib, _load_error
  if _lib is not None:
    return _lib
  target = Path(path) if path is not None else LIB_PATH
  if not target.exists():
    _load_error = ScanError(
      f"native library {target} is missing; build it with "
      "`python associative-scan-triton_b200/build_native.py` (needs nvcc)")
    raise _load_error
  lib = ctypes.CDLL(str(target))
  _bind(lib)
  _lib = lib
  _load_error = None
  return lib


def try_load() -> bool:
  """Load the library if it exists; warn (do not raise) when it does not."""
  global _lib
  try:
    load()
    return True
  except (ScanError, OSError, AttributeError) as e:  # raised again by the first op
    _lib = None
    warnings.warn(f"associative_scan_triton native library unusable: {e}", RuntimeWarning,
                  stacklevel=2)
    return False


def library_path() -> Path:
  return LIB_PATH


def set_sync_check(enabled: bool) -> None:
  """Synchronise after every op and raise on a device-side error."""
  global _sync_check
  _sync_check = bool(enabled)


def sync_check_enabled() -> bool:
  return _sync_check


def set_implementation(name: str) -> None:
  """Kernel family for the following calls: "auto" (the default choice),
  "simple" (always the plain one-CTA-per-tile kernels), "tma" (the
  persistent TMA-pipelined kernels whenever pointers are 16-byte aligned),
  "tma-flat" / "tma-row" (the TMA kernels with the tile order forced)."""
  rc = load().ascan_set_implementation(IMPLEMENTATIONS[name])
  if rc != ASCAN_OK:
    raise ScanError(f"ascan_set_implementation: {strerror(rc)}")


def set_tile_width(elems_per_thread: int) -> None:
  """Tile width of the persistent kernels: 0 chooses per launch, 16 or 32
  forces 4096- or 8192-element tiles where both kernels exist."""
  rc = load().ascan_set_tile_width(int(elems_per_thread))
  if rc != ASCAN_OK:
    raise ValueError(f"tile width must be 0, 16 or 32, got {elems_per_thread}")


def get_tile_width() -> int:
  return int(load().ascan_get_tile_width())


def get_implementation() -> str:
  code = load().ascan_get_implementation()
  return {v: k for k, v in IMPLEMENTATIONS.items()}[int(code)]


def strerror(status: int) -> str:
  return load().ascan_strerror(int(status)).decode()


def describe_device_error(code: int) -> str:
  parts = []
  if code & DEV_ERR_CU_END:
    parts.append("cu_seqlens[-1] does not equal the packed length of the tensors")
  if code & DEV_ERR_CU_ORDER:
    parts.append("cu_seqlens is not monotone or lies outside [0, packed length]")
  if code & DEV_ERR_LOOKBACK:
    parts.append("a tile's predecessor did not publish within the bounded wait")
  if code & DEV_ERR_EXCHANGE:
    parts.append("a peer rank's time-shard record or release did not arrive within the "
                 "bounded wait")
  return "; ".join(parts) or f"device error {code:#x}"


def get_device_error(device: int | torch.device | None = None) -> tuple[int, int]:
  """Synchronise ``device`` and return its sticky (error bits, detail)."""
  dev = _device_index(device)
  code, detail = ctypes.c_uint(0), ctypes.c_longlong(0)
  rc = load().ascan_get_device_error(dev, ctypes.byref(code), ctypes.byref(detail))
  if rc != ASCAN_OK:
    raise ScanError(f"ascan_get_device_error: {strerror(rc)}")
  return int(code.value), int(detail.value)


def clear_device_error(device: int | torch.device | None = None) -> None:
  rc = load().ascan_clear_device_error(_device_index(device))
  if rc != ASCAN_OK:
    raise ScanError(f"ascan_clear_device_error: {strerror(rc)}")


def check_device_error(device: int | torch.device | None = None) -> None:
  """Raise (and clear) if a kernel on ``device`` reported an error."""
  code, detail = get_device_error(device)
  if code:
    clear_device_error(device)
    raise ScanError(f"device-side error: {describe_device_error(code)} (detail {detail})")


def _device_index(device) -> int:
  if device is None:
    return torch.cuda.current_device()
  if isinstance(device, torch.device):
    return device.index if device.index is not None else torch.cuda.current_device()
  return int(device)


# ---------------------------------------------------------------------------
# argument checking
# ---------------------------------------------------------------------------


def _require_cuda(name: str, t: torch.Tensor, device: torch.device | None) -> None:
  if not isinstance(t, torch.Tensor):
    raise TypeError(f"{name} must be a torch.Tensor, got {type(t).__name__}")
  if t.device.type != "cuda":
    raise ValueError(
      f"{name} is on {t.device}; associative_scan_triton (B200) runs on CUDA tensors only")
  if device is not None and t.device != device:
    raise ValueError(f"{name} is on {t.device}, expected {device}")


def _layout(t: torch.Tensor, num_channels: int) -> tuple[int, int]:
  """(C, BL) of a packed tensor given the channel count of the launch grid."""
  if num_channels <= 0:
    raise ValueError(f"number of channels must be positive, got {num_channels}")
  if t.dim() == 2:
    if num_channels > t.shape[0]:
      raise ValueError(f"grid asks for {num_channels} channels, tensor has {t.shape[0]}")
    return int(num_channels), int(t.shape[1])
  if t.numel() % num_channels:
    raise ValueError(f"{t.numel()} elements are not {num_channels} equal channels")
  return int(num_channels), int(t.numel() // num_channels)


def _workspace(n_channels: int, seq_total: int, dtype_code: int, device) -> torch.Tensor:
  nbytes = int(load().ascan_workspace_size(n_channels, seq_total, dtype_code))
  return torch.empty(nbytes, dtype=torch.uint8, device=device)


def _stream_ptr(device: torch.device) -> int:
  return torch.cuda.current_stream(device).cuda_stream


def _enable_error_flag() -> None:
  """Enable the library's pinned host error flag (once, outside any stream
  capture: its first use allocates pinned host memory)."""
  global _flag
  if _flag is None and not torch.cuda.is_current_stream_capturing():
    ptr = load().ascan_error_flag()
    if ptr:
      _flag = ctypes.c_uint.from_address(ptr)


def error_flag() -> int:
  """The host error flag's current bits (0: no device error seen yet), read
  without synchronising."""
  _enable_error_flag()
  return int(_flag.value) if _flag is not None else 0


def _finish(rc: int, what: str, device: torch.device) -> None:
  if rc != ASCAN_OK:
    raise ScanError(f"{what}: {strerror(rc)}")
  if _sync_check or (_flag is not None and _flag.value):
    check_device_error(device)


def _check_inputs(names_tensors, cu_seqlens, num_seq):
  first = names_tensors[0][1]
  device = first.device
  for name, t in names_tensors:
    _require_cuda(name, t, device if name != names_tensors[0][0] else None)
    if not t.is_contiguous():
      raise ValueError(f"{name} must be contiguous")
    if t.dtype != first.dtype:
      raise TypeError(f"{name} has dtype {t.dtype}, expected {first.dtype}")
  if first.dtype not in DTYPE_CODES:
    raise TypeError(f"unsupported dtype {first.dtype}; use float32, float16 or bfloat16")
  _require_cuda("cu_seqlens", cu_seqlens, device)
  if cu_seqlens.dtype not in INDEX_CODES:
    raise TypeError(f"cu_seqlens must be int32 or int64, got {cu_seqlens.dtype}")
  if not cu_seqlens.is_contiguous():
    raise ValueError("cu_seqlens must be contiguous")
  if cu_seqlens.numel() != num_seq + 1:
    raise ValueError(f"cu_seqlens has {cu_seqlens.numel()} entries, expected {num_seq + 1}")
  _enable_error_flag()  # the inputs are CUDA tensors: a device exists
  return device


# ---------------------------------------------------------------------------
# the three native entry points
# ---------------------------------------------------------------------------


def forward(gates: torch.Tensor, tokens: torch.Tensor, tokens_out: torch.Tensor,
            gates_out: torch.Tensor | None, cu_seqlens: torch.Tensor, num_seq: int,
            num_channels: int, reverse: bool) -> None:
  """ascan_forward on torch tensors (tokens_out may be tokens; gates_out may be gates)."""
  tensors = [("gates", gates), ("tokens", tokens), ("tokens_out", tokens_out)]
  if gates_out is not None:
    tensors.append(("gates_out", gates_out))
  device = _check_inputs(tensors, cu_seqlens, num_seq)
  C, BL = _layout(tokens, num_channels)
  for name, t in tensors:
    if _layout(t, num_channels) != (C, BL):
      raise ValueError(f"{name} shape {tuple(t.shape)} does not match tokens {tuple(tokens.shape)}")
  lib = load()
  dcode = DTYPE_CODES[tokens.dtype]
  with torch.cuda.device(device):
    ws = _workspace(C, BL, dcode, device)
    rc = lib.ascan_forward(
      gates.data_ptr(), tokens.data_ptr(), tokens_out.data_ptr(),
      gates_out.data_ptr() if gates_out is not None else None,
      cu_seqlens.data_ptr(), INDEX_CODES[cu_seqlens.dtype], int(num_seq), C, BL, dcode,
      int(bool(reverse)), ws.data_ptr(), ws.numel(), _stream_ptr(device))
  _finish(rc, "ascan_forward", device)


def backward(grad: torch.Tensor, gates: torch.Tensor, states: torch.Tensor,
             d_tokens: torch.Tensor, d_gates: torch.Tensor, cu_seqlens: torch.Tensor,
             num_seq: int, num_channels: int, causal: bool) -> None:
  """ascan_backward on torch tensors."""
  tensors = [("grad", grad), ("gates", gates), ("states", states), ("d_tokens", d_tokens),
             ("d_gates", d_gates)]
  device = _check_inputs(tensors, cu_seqlens, num_seq)
  C, BL = _layout(grad, num_channels)
  for name, t in tensors:
    if _layout(t, num_channels) != (C, BL):
      raise ValueError(f"{name} shape {tuple(t.shape)} does not match grad {tuple(grad.shape)}")
  lib = load()
  dcode = DTYPE_CODES[grad.dtype]
  with torch.cuda.device(device):
    ws = _workspace(C, BL, dcode, device)
    rc = lib.ascan_backward(
      grad.data_ptr(), gates.data_ptr(), states.data_ptr(), d_tokens.data_ptr(),
      d_gates.data_ptr(), cu_seqlens.data_ptr(), INDEX_CODES[cu_seqlens.dtype], int(num_seq),
      C, BL, dcode, int(bool(causal)), ws.data_ptr(), ws.numel(), _stream_ptr(device))
  _finish(rc, "ascan_backward", device)


def _check_pair(names_tensors, cu_seqlens, num_seq, num_channels):
  device = _check_inputs(names_tensors, cu_seqlens, num_seq)
  first_name, first = names_tensors[0]
  C, BL = _layout(first, num_channels)
  for name, t in names_tensors:
    if _layout(t, num_channels) != (C, BL):
      raise ValueError(f"{name} shape {tuple(t.shape)} does not match {first_name} "
                       f"{tuple(first.shape)}")
  return device, C, BL


def _bidi_workspace(C: int, BL: int, dtype_code: int, device) -> torch.Tensor:
  nbytes = int(load().ascan_workspace_size_bidi(C, BL, dtype_code))
  return torch.empty(nbytes, dtype=torch.uint8, device=device)


def forward_bidi(gates_fwd: torch.Tensor, tokens_fwd: torch.Tensor, out_fwd: torch.Tensor,
                 gates_bwd: torch.Tensor, tokens_bwd: torch.Tensor, out_bwd: torch.Tensor,
                 cu_seqlens: torch.Tensor, num_seq: int, num_channels: int) -> None:
  """ascan_forward_bidi: causal scan of the *_fwd pair and reverse scan of the
  *_bwd pair in one launch."""
  tensors = [("gates_fwd", gates_fwd), ("tokens_fwd", tokens_fwd), ("out_fwd", out_fwd),
             ("gates_bwd", gates_bwd), ("tokens_bwd", tokens_bwd), ("out_bwd", out_bwd)]
  device, C, BL = _check_pair(tensors, cu_seqlens, num_seq, num_channels)
  lib = load()
  dcode = DTYPE_CODES[tokens_fwd.dtype]
  with torch.cuda.device(device):
    ws = _bidi_workspace(C, BL, dcode, device)
    rc = lib.ascan_forward_bidi(
      gates_fwd.data_ptr(), tokens_fwd.data_ptr(), out_fwd.data_ptr(), gates_bwd.data_ptr(),
      tokens_bwd.data_ptr(), out_bwd.data_ptr(), cu_seqlens.data_ptr(),
      INDEX_CODES[cu_seqlens.dtype], int(num_seq), C, BL, dcode, ws.data_ptr(), ws.numel(),
      _stream_ptr(device))
  _finish(rc, "ascan_forward_bidi", device)


def backward_bidi(grad_fwd: torch.Tensor, gates_fwd: torch.Tensor, states_fwd: torch.Tensor,
                  d_tokens_fwd: torch.Tensor, d_gates_fwd: torch.Tensor,
                  grad_bwd: torch.Tensor, gates_bwd: torch.Tensor, states_bwd: torch.Tensor,
                  d_tokens_bwd: torch.Tensor, d_gates_bwd: torch.Tensor,
                  cu_seqlens: torch.Tensor, num_seq: int, num_channels: int) -> None:
  """ascan_backward_bidi: causal adjoint of the *_fwd buffers and reverse
  adjoint of the *_bwd buffers in one launch."""
  tensors = [("grad_fwd", grad_fwd), ("gates_fwd", gates_fwd), ("states_fwd", states_fwd),
             ("d_tokens_fwd", d_tokens_fwd), ("d_gates_fwd", d_gates_fwd),
             ("grad_bwd", grad_bwd), ("gates_bwd", gates_bwd), ("states_bwd", states_bwd),
             ("d_tokens_bwd", d_tokens_bwd), ("d_gates_bwd", d_gates_bwd)]
  device, C, BL = _check_pair(tensors, cu_seqlens, num_seq, num_channels)
  lib = load()
  dcode = DTYPE_CODES[grad_fwd.dtype]
  with torch.cuda.device(device):
    ws = _bidi_workspace(C, BL, dcode, device)
    rc = lib.ascan_backward_bidi(
      *[t.data_ptr() for _, t in tensors], cu_seqlens.data_ptr(),
      INDEX_CODES[cu_seqlens.dtype], int(num_seq), C, BL, dcode, ws.data_ptr(), ws.numel(),
      _stream_ptr(device))
  _finish(rc, "ascan_backward_bidi", device)


def _row_array(name: str, t: torch.Tensor | None, C: int, width: int, device) -> int | None:
  """Pointer of a per-row float32 array [C] (width 1) or [C, 2] (width 2)."""
  if t is None:
    return None
  _require_cuda(name, t, device)
  if t.dtype != torch.float32 or not t.is_contiguous() or t.numel() != C * width:
    raise ValueError(f"{name} must be a contiguous float32 tensor of {C * width} elements")
  return t.data_ptr()


def forward_slab(gates: torch.Tensor, tokens: torch.Tensor, tokens_out: torch.Tensor | None,
                 gates_out: torch.Tensor | None, cu_seqlens: torch.Tensor, num_seq: int,
                 num_channels: int, reverse: bool, row_carry: torch.Tensor | None = None,
                 row_aggregate: torch.Tensor | None = None) -> None:
  """ascan_forward_slab: the forward over one time slab of every row, with an
  optional carried (gate product, state) per row and an optional per-row
  aggregate output; ``tokens_out=None`` makes it an aggregate-only pass."""
  tensors = [("gates", gates), ("tokens", tokens)]
  if tokens_out is not None:
    tensors.append(("tokens_out", tokens_out))
  if gates_out is not None:
    tensors.append(("gates_out", gates_out))
  device = _check_inputs(tensors, cu_seqlens, num_seq)
  C, BL = _layout(tokens, num_channels)
  for name, t in tensors:
    if _layout(t, num_channels) != (C, BL):
      raise ValueError(f"{name} shape {tuple(t.shape)} does not match tokens {tuple(tokens.shape)}")
  carry = _row_array("row_carry", row_carry, C, 2, device)
  agg = _row_array("row_aggregate", row_aggregate, C, 2, device)
  lib = load()
  dcode = DTYPE_CODES[tokens.dtype]
  with torch.cuda.device(device):
    ws = _workspace(C, BL, dcode, device)
    rc = lib.ascan_forward_slab(
      gates.data_ptr(), tokens.data_ptr(),
      tokens_out.data_ptr() if tokens_out is not None else None,
      gates_out.data_ptr() if gates_out is not None else None,
      cu_seqlens.data_ptr(), INDEX_CODES[cu_seqlens.dtype], int(num_seq), C, BL, dcode,
      int(bool(reverse)), carry, agg, ws.data_ptr(), ws.numel(), _stream_ptr(device))
  _finish(rc, "ascan_forward_slab", device)


def backward_slab(grad: torch.Tensor, gates: torch.Tensor, states: torch.Tensor,
                  d_tokens: torch.Tensor | None, d_gates: torch.Tensor | None,
                  cu_seqlens: torch.Tensor, num_seq: int, num_channels: int, causal: bool,
                  row_carry: torch.Tensor | None = None,
                  row_state_halo: torch.Tensor | None = None,
                  row_aggregate: torch.Tensor | None = None) -> None:
  """ascan_backward_slab: the fused backward over one time slab of every row,
  with an optional additive adjoint term per row, the state neighbour from
  the adjacent slab and an optional per-row aggregate output; ``d_tokens`` and
  ``d_gates`` both None make it an aggregate-only pass."""
  tensors = [("grad", grad), ("gates", gates), ("states", states)]
  if (d_tokens is None) != (d_gates is None):
    raise ValueError("d_tokens and d_gates are given together or not at all")
  if d_tokens is not None:
    tensors += [("d_tokens", d_tokens), ("d_gates", d_gates)]
  device = _check_inputs(tensors, cu_seqlens, num_seq)
  C, BL = _layout(grad, num_channels)
  for name, t in tensors:
    if _layout(t, num_channels) != (C, BL):
      raise ValueError(f"{name} shape {tuple(t.shape)} does not match grad {tuple(grad.shape)}")
  carry = _row_array("row_carry", row_carry, C, 1, device)
  halo = _row_array("row_state_halo", row_state_halo, C, 1, device)
  agg = _row_array("row_aggregate", row_aggregate, C, 2, device)
  lib = load()
  dcode = DTYPE_CODES[grad.dtype]
  with torch.cuda.device(device):
    ws = _workspace(C, BL, dcode, device)
    rc = lib.ascan_backward_slab(
      grad.data_ptr(), gates.data_ptr(), states.data_ptr(),
      d_tokens.data_ptr() if d_tokens is not None else None,
      d_gates.data_ptr() if d_gates is not None else None,
      cu_seqlens.data_ptr(), INDEX_CODES[cu_seqlens.dtype], int(num_seq), C, BL, dcode,
      int(bool(causal)), carry, halo, agg, ws.data_ptr(), ws.numel(), _stream_ptr(device))
  _finish(rc, "ascan_backward_slab", device)


def time_shard_fold(records: torch.Tensor, world: int, rank: int, num_channels: int,
                    starts_new_mask: int, inner_boundary_mask: int, direction: int,
                    carry_out: torch.Tensor, halo_out: torch.Tensor | None = None) -> None:
  """ascan_time_shard_fold: the carry entering slab ``rank`` from the gathered
  records ``[world, record_floats]`` (float32, contiguous, CUDA)."""
  _require_cuda("records", records, None)
  device = records.device
  if records.dtype != torch.float32 or not records.is_contiguous() or records.dim() != 2 \
      or records.shape[0] != world:
    raise ValueError(f"records must be a contiguous float32 [{world}, k] tensor")
  C = int(num_channels)
  carry = _row_array("carry_out", carry_out, C, 2 if direction == 0 else 1, device)
  halo = _row_array("halo_out", halo_out, C, 1, device)
  with torch.cuda.device(device):
    rc = load().ascan_time_shard_fold(
      records.data_ptr(), int(records.shape[1]), int(world), int(rank), C,
      int(starts_new_mask), int(inner_boundary_mask), int(direction), carry, halo,
      _stream_ptr(device))
  _finish(rc, "ascan_time_shard_fold", device)


IPC_HANDLE_BYTES = 64
EXCHANGE_PUBLISH, EXCHANGE_FOLD, EXCHANGE_BOTH = 1, 2, 3


def exchange_create(num_channels: int, device) -> int:
  """ascan_exchange_create on ``device``: a zeroed exchange buffer (its
  device address; free it with :func:`exchange_destroy`)."""
  buf = ctypes.c_void_p(0)
  with torch.cuda.device(torch.device(device)):
    rc = load().ascan_exchange_create(int(num_channels), ctypes.byref(buf))
  if rc != ASCAN_OK:
    raise ScanError(f"ascan_exchange_create: {strerror(rc)}")
  return int(buf.value)


def exchange_export(buffer: int) -> bytes:
  """The CUDA IPC handle of an exchange buffer of this process."""
  h = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
  rc = load().ascan_exchange_export(ctypes.c_void_p(buffer), h)
  if rc != ASCAN_OK:
    raise ScanError(f"ascan_exchange_export: {strerror(rc)}")
  return h.raw


def exchange_import(handle: bytes, device) -> int:
  """Maps another process's exchange buffer on ``device``; its address here."""
  if len(handle) != IPC_HANDLE_BYTES:
    raise ValueError(f"an IPC handle has {IPC_HANDLE_BYTES} bytes, got {len(handle)}")
  peer = ctypes.c_void_p(0)
  with torch.cuda.device(torch.device(device)):
    rc = load().ascan_exchange_import(ctypes.create_string_buffer(handle, IPC_HANDLE_BYTES),
                                      ctypes.byref(peer))
  if rc != ASCAN_OK:
    raise ScanError(f"ascan_exchange_import: {strerror(rc)}")
  return int(peer.value)


def exchange_close(peer_buffer: int) -> None:
  rc = load().ascan_exchange_close(ctypes.c_void_p(peer_buffer))
  if rc != ASCAN_OK:
    raise ScanError(f"ascan_exchange_close: {strerror(rc)}")


def exchange_destroy(buffer: int) -> None:
  rc = load().ascan_exchange_destroy(ctypes.c_void_p(buffer))
  if rc != ASCAN_OK:
    raise ScanError(f"ascan_exchange_destroy: {strerror(rc)}")


def time_shard_exchange(buffer: int, buffers: torch.Tensor, world: int, rank: int,
                        num_channels: int, aggregate: torch.Tensor | None,
                        starts_new_mask: int, inner_boundary_mask: int, direction: int,
                        mode: int, carry_out: torch.Tensor | None,
                        halo_out: torch.Tensor | None = None, gates: torch.Tensor | None = None,
                        states: torch.Tensor | None = None, timeout_s: float = 2.0,
                        parts: int = 1) -> None:
  """ascan_time_shard_exchange on the current stream of ``buffers``' device.
  ``buffers``: int64 [world] device tensor of the exchange buffers as this
  process addresses them (its own at ``rank``); ``aggregate`` [parts * C, 2]
  float32; ``gates``/``states`` [C, L] for the backward record's edge columns
  (and, with ``parts`` > 1, the parts' edge columns); ``carry_out`` /
  ``halo_out`` hold one entry per row part."""
  _require_cuda("buffers", buffers, None)
  device = buffers.device
  if buffers.dtype != torch.int64 or buffers.numel() != world:
    raise ValueError(f"buffers must be an int64 tensor of {world} addresses")
  C, H = int(num_channels), int(parts)
  agg = _row_array("aggregate", aggregate, H * C, 2, device)
  carry = _row_array("carry_out", carry_out, H * C, 2 if direction == 0 else 1, device)
  halo = _row_array("halo_out", halo_out, H * C, 1, device)
  L, dcode, gp, sp = 0, DTYPE_CODES[torch.float32], None, None
  if direction == 1 and (mode & EXCHANGE_PUBLISH or H > 1):
    for name, t in (("gates", gates), ("states", states)):
      if t is None:
        raise ValueError(f"the backward record needs {name}")
      _require_cuda(name, t, device)
      if t.dim() != 2 or t.shape[0] != C or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous [{C}, L] tensor")
    if gates.shape != states.shape or gates.dtype != states.dtype:
      raise ValueError("gates and states must have one shape and dtype")
    L, dcode, gp, sp = int(gates.shape[1]), DTYPE_CODES[gates.dtype], gates.data_ptr(), \
        states.data_ptr()
  with torch.cuda.device(device):
    rc = load().ascan_time_shard_exchange(
      ctypes.c_void_p(buffer), buffers.data_ptr(), int(world), int(rank), C, L, H, agg, gp, sp,
      dcode, int(starts_new_mask), int(inner_boundary_mask), int(direction), int(mode), carry,
      halo, int(timeout_s * 1e9), _stream_ptr(device))
  _finish(rc, "ascan_time_shard_exchange", device)


def shift_pad(data: torch.Tensor, out: torch.Tensor, cu_seqlens: torch.Tensor,
              pad_value: float, backward: bool, wrap: bool) -> None:
  """ascan_shift_pad on a 2-D [C, BL] tensor."""
  if data.dim() != 2:
    raise ValueError(f"shift_pad expects a [C, BL] tensor, got shape {tuple(data.shape)}")
  num_seq = cu_seqlens.numel() - 1
  device = _check_inputs([("data", data), ("out", out)], cu_seqlens, num_seq)
  C, BL = int(data.shape[0]), int(data.shape[1])
  lib = load()
  with torch.cuda.device(device):
    rc = lib.ascan_shift_pad(
      data.data_ptr(), out.data_ptr(), cu_seqlens.data_ptr(), INDEX_CODES[cu_seqlens.dtype],
      num_seq, C, BL, DTYPE_CODES[data.dtype], float(pad_value), int(bool(backward)),
      int(bool(wrap)), _stream_ptr(device))
  _finish(rc, "ascan_shift_pad", device)

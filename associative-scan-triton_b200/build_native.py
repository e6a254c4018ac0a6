"""Build the native library (CUDA for sm_100a) in place.

    python associative-scan-triton_b200/build_native.py [--force] [--verbose]

nvcc cross-compiles without a GPU, so this runs on a CPU-only host too.  The
result, ``associative_scan_triton/libascan_b200.so``, sits inside the package;
it links the CUDA runtime statically so it loads on any host with an NVIDIA
driver.  This module lives outside the package so that building never loads a
(possibly stale) copy of the library into the process.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

DIST_DIR = Path(__file__).resolve().parent
PKG_DIR = DIST_DIR / "associative_scan_triton"
REPO_DIR = DIST_DIR.parent
CSRC_DIR = DIST_DIR / "csrc"
INCLUDE_DIR = REPO_DIR / "include"
LIB_NAME = "libascan_b200.so"
LIB_PATH = PKG_DIR / LIB_NAME

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
  for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
    if cand and Path(cand).exists():
      return cand
  raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def sources() -> list[Path]:
  return sorted(CSRC_DIR.glob("*.cu"))


def _inputs() -> list[Path]:
  return sources() + sorted(CSRC_DIR.glob("*.cuh")) + sorted(INCLUDE_DIR.glob("*.h"))


def up_to_date() -> bool:
  if not LIB_PATH.exists():
    return False
  mtime = LIB_PATH.stat().st_mtime
  return all(p.stat().st_mtime <= mtime for p in _inputs())


def build(force: bool = False, verbose: bool = False) -> Path:
  """Compile csrc/*.cu into libascan_b200.so (skipped when up to date)."""
  if not force and up_to_date():
    return LIB_PATH
  tmp = LIB_PATH.with_name(f".{LIB_NAME}.{os.getpid()}.tmp")
  cmd = [
    _nvcc(), *ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC,-fvisibility=hidden", "-shared", "-cudart", "static",
    f"-I{INCLUDE_DIR}", "-o", str(tmp), *map(str, sources()),
  ]
  if verbose:
    cmd.insert(1, "-Xptxas=-v")
    print(" ".join(cmd), flush=True)
  try:
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
  finally:
    if tmp.exists():
      tmp.unlink()
  return LIB_PATH


def main(argv: list[str] | None = None) -> int:
  ap = argparse.ArgumentParser(description=__doc__)
  ap.add_argument("--force", action="store_true")
  ap.add_argument("--verbose", action="store_true")
  a = ap.parse_args(argv)
  print(build(force=a.force, verbose=a.verbose))
  return 0


if __name__ == "__main__":
  sys.exit(main())

"""Build the native library (CUDA for sm_100a) in place.

    python associative-scan-triton_b200/build_native.py [--force] [--verbose]

nvcc cross-compiles without a GPU, so this runs on a CPU-only host too.  The
result, ``associative_scan_triton/libascan_b200.so``, sits inside the package;
it links the CUDA runtime statically so it loads on any host with an NVIDIA
driver.  Every ``csrc/*.cu`` unit compiles to its own object in ``_build/``
in parallel (the kernels are split across units by dtype and direction), and
the objects are linked into the library.  This module lives outside the
package so that building never loads a (possibly stale) copy of the library
into the process.
"""

from __future__ import annotations

import argparse
import concurrent.futures
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
OBJ_DIR = DIST_DIR / "_build"

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


def _compile_flags(verbose: bool) -> list[str]:
  flags = [*ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17",
           "-Xcompiler", "-fPIC,-fvisibility=hidden", f"-I{INCLUDE_DIR}"]
  if verbose:
    flags.insert(0, "-Xptxas=-v")
  return flags


def _compile(src: Path, obj: Path, verbose: bool) -> tuple[Path, int, str]:
  tmp = obj.with_name(f".{obj.name}.{os.getpid()}.tmp")
  cmd = [_nvcc(), *_compile_flags(verbose), "-c", "-o", str(tmp), str(src)]
  if verbose:
    print(" ".join(cmd), flush=True)
  proc = subprocess.run(cmd, capture_output=True, text=True)
  if proc.returncode == 0:
    os.replace(tmp, obj)
  elif tmp.exists():
    tmp.unlink()
  return src, proc.returncode, proc.stdout + proc.stderr


def _headers_mtime() -> float:
  hdrs = sorted(CSRC_DIR.glob("*.cuh")) + sorted(INCLUDE_DIR.glob("*.h"))
  return max((p.stat().st_mtime for p in hdrs), default=0.0)


def build(force: bool = False, verbose: bool = False, jobs: int | None = None) -> Path:
  """Compile csrc/*.cu into libascan_b200.so (skipped when up to date).

  Units whose object is newer than the unit and every header are reused."""
  if not force and up_to_date():
    return LIB_PATH
  OBJ_DIR.mkdir(exist_ok=True)
  hdr_mtime = _headers_mtime()
  todo, objs = [], []
  for src in sources():
    obj = OBJ_DIR / (src.stem + ".o")
    objs.append(obj)
    stale = force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr_mtime)
    if stale:
      todo.append((src, obj))
  jobs = jobs or min(len(todo), os.cpu_count() or 1) or 1
  failures = []
  with concurrent.futures.ThreadPoolExecutor(max_workers=jobs) as pool:
    for src, rc, out in pool.map(lambda so: _compile(so[0], so[1], verbose), todo):
      if out.strip() and (verbose or rc != 0):
        print(out, end="", flush=True)
      if rc != 0:
        failures.append(src.name)
  if failures:
    raise RuntimeError(f"nvcc failed for {', '.join(failures)}")
  tmp = LIB_PATH.with_name(f".{LIB_NAME}.{os.getpid()}.tmp")
  cmd = [_nvcc(), *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
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
  ap.add_argument("--jobs", type=int, default=None)
  a = ap.parse_args(argv)
  print(build(force=a.force, verbose=a.verbose, jobs=a.jobs))
  return 0


if __name__ == "__main__":
  sys.exit(main())

"""Build ``libsparsefold_b200.so`` in-tree with nvcc for sm_100a.

    python -m sparsefold_b200.build [--force] [-j N]

Every ``csrc/*.cu`` is compiled to an object under ``_build/`` (skipped when
newer than its sources), then linked into ``sparsefold_b200/libsparsefold_b200.so``.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(REPO, "_build")
LIB = os.path.join(PKG, "libsparsefold_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def nvcc() -> str:
  for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
    if cand and os.path.exists(cand):
      return cand
  raise RuntimeError("nvcc not found")


def _deps() -> list[str]:
  return glob.glob(os.path.join(CSRC, "*.cuh")) + [os.path.join(REPO, "include", "sparsefold_b200.h")]


def _stale(target: str, sources: list[str]) -> bool:
  if not os.path.exists(target):
    return True
  t = os.path.getmtime(target)
  return any(os.path.getmtime(s) > t for s in sources)


def _compile(src: str, extra: list[str]) -> str:
  obj = os.path.join(BUILD, os.path.basename(src).replace(".cu", ".o"))
  if _stale(obj, [src] + _deps()):
    cmd = [nvcc(), *ARCH, *FLAGS, *extra, "-I", os.path.join(REPO, "include"), "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
      raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip():
      sys.stderr.write(r.stderr)
  return obj


def build(force: bool = False, jobs: int | None = None, verbose_ptxas: bool = False) -> str:
  os.makedirs(BUILD, exist_ok=True)
  sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
  if force:
    for o in glob.glob(os.path.join(BUILD, "*.o")):
      os.remove(o)
  extra = ["-Xptxas", "-v"] if verbose_ptxas else []
  with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as ex:
    objs = list(ex.map(lambda s: _compile(s, extra), sources))
  if force or _stale(LIB, objs):
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *ARCH, "-shared", "-o", tmp, *objs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
      raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
  return LIB


if __name__ == "__main__":
  ap = argparse.ArgumentParser()
  ap.add_argument("--force", action="store_true")
  ap.add_argument("-j", type=int, default=None)
  ap.add_argument("--ptxas-v", action="store_true")
  args = ap.parse_args()
  print(build(force=args.force, jobs=args.j, verbose_ptxas=args.ptxas_v))

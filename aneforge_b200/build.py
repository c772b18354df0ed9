"""Build libaf_cuda.so (every CUDA source of the package) for sm_100a, in-tree.

    python -m aneforge_b200.build        # or aneforge_b200.build.build()

The library lands in aneforge_b200/_lib/ so it travels with the source tree; nothing is installed
into site-packages and no JIT cache is used.
"""
from __future__ import annotations

import hashlib
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "libaf_cuda.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def sources():
  return sorted(CSRC.glob("*.cu"))


def _fingerprint() -> str:
  h = hashlib.sha256()
  for p in sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))
                  + [ROOT / "include" / "af_cuda.h"]):
    h.update(p.name.encode()); h.update(p.read_bytes())
  h.update(" ".join(ARCH).encode())
  return h.hexdigest()


def nvcc() -> str:
  for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
    if c and (os.path.sep not in c or os.path.exists(c)):
      return c
  return "nvcc"


def build(force: bool = False, verbose: bool = False) -> Path:
  """Compile all sources into one shared library (parallel per-file objects, then link)."""
  LIB_DIR.mkdir(exist_ok=True)
  stamp = LIB_DIR / "libaf_cuda.sha256"
  fp = _fingerprint()
  if not force and LIB.exists() and stamp.exists() and stamp.read_text() == fp:
    return LIB
  objs, procs = [], []
  flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr",
                  "-I", str(ROOT / "include")]
  for src in sources():
    obj = LIB_DIR / (src.stem + ".o")
    objs.append(obj)
    cmd = [nvcc(), "-c", str(src), "-o", str(obj)] + flags
    if verbose:
      print(" ".join(cmd))
    procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
  failed = []
  for src, p in procs:
    out, _ = p.communicate()
    if p.returncode != 0:
      failed.append((src, out.decode(errors="replace")))
    elif verbose and out:
      print(out.decode(errors="replace"))
  if failed:
    msg = "\n".join(f"--- {s.name}\n{o}" for s, o in failed)
    raise RuntimeError(f"nvcc failed:\n{msg}")
  tmp = LIB.with_suffix(".so.tmp")
  link = [nvcc(), "-shared", "-o", str(tmp)] + [str(o) for o in objs] + ARCH + ["-lcudart"]
  r = subprocess.run(link, capture_output=True, text=True)
  if r.returncode != 0:
    raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
  os.replace(tmp, LIB)
  for o in objs:
    o.unlink(missing_ok=True)
  stamp.write_text(fp)
  return LIB


if __name__ == "__main__":
  print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))

"""Build libcfk_b200.so in-tree with nvcc for sm_100a (no GPU needed: nvcc cross-compiles).

  python colabfold-kernels_b200/build.py [--force] [--verbose]

Objects go to colabfold-kernels_b200/build/, the library to colabfold-kernels_b200/lib/.
"""
import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "build")
LIB = os.path.join(HERE, "lib", "libcfk_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-lineinfo", "--use_fast_math",
         "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr"]
# fp32-accurate files: no fast-math (exp2f/log2f/div must stay IEEE-grade for the 1e-4 float32 bound)
PRECISE = {"attention_simt.cu", "layer_norm.cu"}


def _stale(src, obj, headers):
  if not os.path.exists(obj):
    return True
  t = os.path.getmtime(obj)
  return any(os.path.getmtime(f) > t for f in [src] + headers)


def _compile(src, verbose):
  obj = os.path.join(OBJ, os.path.basename(src)[:-3] + ".o")
  flags = [f for f in FLAGS if not (f == "--use_fast_math" and os.path.basename(src) in PRECISE)]
  cmd = [NVCC, *flags, "-I", os.path.join(HERE, "..", "include"), "-c", src, "-o", obj]
  if verbose:
    cmd.insert(1, "-Xptxas=-v")
  r = subprocess.run(cmd, capture_output=True, text=True)
  return src, r.returncode, r.stdout + r.stderr


def build(force=False, verbose=False):
  os.makedirs(OBJ, exist_ok=True)
  os.makedirs(os.path.dirname(LIB), exist_ok=True)
  srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
  headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(HERE, "..", "include", "*.h"))
  todo = [s for s in srcs if force or _stale(s, os.path.join(OBJ, os.path.basename(s)[:-3] + ".o"), headers)]
  with cf.ThreadPoolExecutor(max_workers=min(8, max(1, len(todo)))) as ex:
    for src, rc, out in ex.map(lambda s: _compile(s, verbose), todo):
      if out.strip() and (verbose or rc != 0):
        print(f"--- {os.path.basename(src)}\n{out}", file=sys.stderr)
      if rc != 0:
        raise RuntimeError(f"nvcc failed on {src}")
  objs = [os.path.join(OBJ, os.path.basename(s)[:-3] + ".o") for s in srcs]
  if todo or not os.path.exists(LIB):
    cmd = [NVCC, "-shared", "-o", LIB, *objs, "-Xlinker", "--no-undefined", "-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
      raise RuntimeError("link failed:\n" + r.stdout + r.stderr)
  return LIB


if __name__ == "__main__":
  ap = argparse.ArgumentParser()
  ap.add_argument("--force", action="store_true")
  ap.add_argument("--verbose", action="store_true")
  a = ap.parse_args()
  print(build(a.force, a.verbose))

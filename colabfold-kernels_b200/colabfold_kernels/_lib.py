"""ctypes binding of libcfk_b200.so.

The prototypes are read from include/cfk_b200.h, so the binding cannot drift from the C ABI.
There is no CPU fallback: a missing library or symbol raises.  `COLABFOLD_KERNELS_B200_LIB`
overrides the library path (as COLABFOLD_CUDA_KERNELS_LIB does in the reference, contract.py:27-28).
"""
import ctypes
import os
import re

_HERE = os.path.dirname(os.path.abspath(__file__))
_PKG = os.path.dirname(_HERE)
HEADER = os.path.join(os.path.dirname(_PKG), "include", "cfk_b200.h")
DEFAULT_LIB = os.path.join(_PKG, "lib", "libcfk_b200.so")

OK = 0
F32, BF16, E4M3 = 0, 1, 2

_CTYPES = {
    "int": ctypes.c_int, "float": ctypes.c_float, "int64_t": ctypes.c_int64, "size_t": ctypes.c_size_t,
    "int32_t": ctypes.c_int32, "long long": ctypes.c_longlong, "uint8_t": ctypes.c_uint8, "void": None,
}


class CfkError(RuntimeError):
  def __init__(self, name, code):
    super().__init__(f"{name} failed with status {code} ({STATUS_NAMES.get(code, '?')})")
    self.code = code


def _parse_header(path):
  text = open(path).read()
  text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
  status = {int(v): k for k, v in re.findall(r"(CFK_[A-Z_]+)\s*=\s*(-?\d+)", text)}
  protos = {}
  for ret, name, args in re.findall(r"CFK_API\s+([\w\s\*]+?)\s*\b(cfk_\w+)\s*\(([^)]*)\)\s*;", text):
    argt = []
    for a in [a.strip() for a in args.split(",") if a.strip() and a.strip() != "void"]:
      if "*" in a:
        argt.append(ctypes.c_char_p if a.startswith("const char") else ctypes.c_void_p)
      else:
        argt.append(_CTYPES[a.replace("const ", "").split()[0]])
    ret = " ".join(ret.split())
    rt = ctypes.c_char_p if ret == "const char*" else _CTYPES[ret]
    protos[name] = (rt, argt)
  return protos, status


PROTOTYPES, STATUS_NAMES = _parse_header(HEADER)
_lib = None


def library_path():
  return os.environ.get("COLABFOLD_KERNELS_B200_LIB") or DEFAULT_LIB


def load():
  """dlopen the library (once) and bind every prototype of the header; raises if anything is missing."""
  global _lib
  if _lib is not None:
    return _lib
  path = library_path()
  if not os.path.exists(path):
    raise FileNotFoundError(f"{path} not found: build it with `python colabfold-kernels_b200/build.py` "
                            "(there is no CPU fallback)")
  lib = ctypes.CDLL(path)
  for name, (rt, argt) in PROTOTYPES.items():
    fn = getattr(lib, name)  # AttributeError if the symbol is missing
    fn.restype, fn.argtypes = rt, argt
  _lib = lib
  return lib


def available():
  try:
    load()
    return True
  except (OSError, AttributeError):
    return False


def call(name, *args):
  """Call an int-returning entry and raise CfkError on a non-zero status."""
  rc = getattr(load(), name)(*args)
  if rc != OK:
    raise CfkError(name, rc)

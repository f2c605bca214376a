"""The C-ABI library loads and exports every symbol include/cfk_b200.h declares (no compute calls: CPU only)."""
import os
import re

import pytest


def test_header_symbols_exported():
  from colabfold_kernels import _lib
  assert os.path.exists(_lib.library_path()), "build the library first: python colabfold-kernels_b200/build.py"
  lib = _lib.load()
  text = open(_lib.HEADER).read()
  declared = set(re.findall(r"\b(cfk_\w+)\s*\(", re.sub(r"/\*.*?\*/", "", text, flags=re.S)))
  assert declared == set(_lib.PROTOTYPES), declared ^ set(_lib.PROTOTYPES)
  for name in declared:
    assert hasattr(lib, name), name
  assert lib.cfk_version().startswith(b"cfk_b200")


def test_bad_arguments_return_status_without_a_gpu():
  """Argument checks come before any CUDA call, so they can be exercised on a CPU-only host."""
  from colabfold_kernels import _lib
  lib = _lib.load()
  assert lib.cfk_layer_norm(None, None, None, None, 4, 8, _lib.BF16, 1e-5, None) == -4   # CFK_ERR_NULL
  assert lib.cfk_attention_fwd(None, None, None, None, None, None, None, 1, 1, 1, 1, 1, _lib.BF16, 0, 1.0, None) == -4
  assert lib.cfk_trim_limits(None, None, 1, 1, None) == -4
  # the entries whose stores are the exchange of the row-sharded triangle multiplication: null arrays of peer pointers
  assert lib.cfk_ln_gated_dual_proj_peer(None, None, None, None, None, None, None, None, None, None, 0, 2, 128, 128, 128, 256,
                                         0, 1, 1e-5, None) == -4
  assert lib.cfk_contract_exchanged_peer(None, None, None, 0, 64, 256, 256, 256, _lib.BF16, 1.0, 2, 0, None) == -4


def test_cpu_tensors_are_refused():
  import torch
  from colabfold_kernels import ops
  with pytest.raises(ValueError):
    ops.layer_norm(torch.zeros(4, 8), torch.ones(8), torch.zeros(8))

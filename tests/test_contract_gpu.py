"""Triangle-multiplication contraction on the GPU against the CPU oracle: bf16 and e4m3 operands,
ragged I/J/K, both einsum orders of tests/test_ln_fusions.py:216-222."""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [(4, 128, 256, 64), (3, 200, 264, 136), (2, 512, 512, 512), (5, 24, 16, 32),
                                   (1, 1000, 1000, 1000), (128, 128, 128, 128)])
def test_contract_bf16(shape):
  from colabfold_kernels import ops
  c, i, j, k = shape
  rng = np.random.default_rng(0)
  a = torch.from_numpy(rng.standard_normal((c, i, k)).astype(np.float32)).to(torch.bfloat16)
  b = torch.from_numpy(rng.standard_normal((c, j, k)).astype(np.float32)).to(torch.bfloat16)
  out = ops.contract(a.cuda(), b.cuda())
  assert ops.device_status() == 0
  ref = O.ref_contract(a, b)
  # fp32 accumulation, one rounding to bf16 on store
  assert O.rel_err(out.cpu().float(), ref) <= 8e-3


@pytest.mark.parametrize("shape", [(4, 128, 256, 128), (3, 200, 264, 144), (2, 24, 16, 32)])
def test_contract_e4m3(shape, golden):
  from colabfold_kernels import ops
  c, i, j, k = shape
  rng = np.random.default_rng(1)
  a = O.e4m3(torch.from_numpy(rng.standard_normal((c, i, k)).astype(np.float32) * 2))
  b = O.e4m3(torch.from_numpy(rng.standard_normal((c, j, k)).astype(np.float32) * 2))
  out = ops.contract(a.cuda(), b.cuda())
  assert ops.device_status() == 0
  ref = O.ref_fp8_contract(a.float(), b.float())
  assert O.rel_err(out.cpu().float(), ref) <= 1e-2   # the reference's own bound, tests/test_ln_fusions.py:211
  g = golden("fp8_contract")
  out = ops.contract(O.e4m3(torch.from_numpy(g["a"])).cuda(), O.e4m3(torch.from_numpy(g["b"])).cuda())
  assert O.rel_err(out.cpu().float(), torch.from_numpy(g["out"])) <= 1e-2


def test_triangle_einsum_orders():
  """outgoing 'ikc,jkc->ijc' and incoming 'kjc,kic->ijc' through channel-major operands."""
  from colabfold_kernels import ops
  rng = np.random.default_rng(2)
  n, c = 72, 16
  l = torch.from_numpy(rng.standard_normal((n, n, c)).astype(np.float32)).to(torch.bfloat16)
  r = torch.from_numpy(rng.standard_normal((n, n, c)).astype(np.float32)).to(torch.bfloat16)
  out = ops.contract(l.permute(2, 0, 1).contiguous().cuda(), r.permute(2, 0, 1).contiguous().cuda())
  ref = torch.einsum("ikc,jkc->cij", l.float(), r.float())
  assert O.rel_err(out.cpu().float(), ref) <= 8e-3
  out = ops.contract(r.permute(2, 1, 0).contiguous().cuda(), l.permute(2, 1, 0).contiguous().cuda())
  ref = torch.einsum("kjc,kic->cij", l.float(), r.float())
  assert O.rel_err(out.cpu().float(), ref) <= 8e-3

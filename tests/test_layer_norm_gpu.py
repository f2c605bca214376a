"""LayerNorm forward/backward on the GPU through the C ABI against the CPU oracle
(shapes of tests/test_ln_gdp_grad.py:40 plus ragged and wide rows)."""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,c", [(4096, 128), (777, 64), (1024, 256), (1, 128), (33, 512), (50, 96), (7, 20)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_layer_norm(m, c, dtype):
  from colabfold_kernels import ops
  rng = np.random.default_rng(0)
  x = torch.from_numpy((rng.standard_normal((m, c)) * .5).astype(np.float32)).to(dtype)
  sc = torch.from_numpy(rng.standard_normal(c).astype(np.float32))
  of = torch.from_numpy(rng.standard_normal(c).astype(np.float32))
  dy = torch.from_numpy((rng.standard_normal((m, c)) * .5).astype(np.float32)).to(dtype)
  ref = O.ref_layer_norm(x, sc, of, 1e-5)
  y = ops.layer_norm(x.cuda(), sc.cuda(), of.cuda(), 1e-5)
  if dtype == torch.float32:
    assert float((y.cpu() - ref).abs().max()) <= 1e-4
  else:
    assert O.rel_err(y.cpu().float(), ref) <= 2e-2
    assert torch.equal(y.cpu(), ref.to(dtype)) or O.rel_err(y.cpu().float(), ref.to(dtype).float()) <= 8e-3
  rdx, rds, rdo = O.layer_norm_bwd(x, sc, dy, 1e-5)
  dx, ds, do = ops.layer_norm_bwd(x.cuda(), sc.cuda(), dy.cuda(), 1e-5)
  tol = 1e-4 if dtype == torch.float32 else 2e-2
  assert O.rel_err(dx.cpu().float(), rdx) <= tol
  assert O.rel_err(ds.cpu(), rds) <= max(tol, 2e-4)
  assert O.rel_err(do.cpu(), rdo) <= max(tol, 2e-4)

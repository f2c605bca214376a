"""The allocation-free LayerNorm backward entry (built-in scratch) against the workspace entry, through the C ABI.

Collected last on purpose: the entry's first call on a device does its set-up, and it must work both when this file
runs on its own and after every other kernel of the library has run in the same process."""
import pytest
import torch

from colabfold_kernels import _lib, ops

pytestmark = pytest.mark.gpu


def _static_bwd(x, scale, dy, eps):
  c = x.shape[-1]
  m = x.numel() // c
  dx = torch.empty_like(x)
  dscale = torch.empty(c, dtype=torch.float32, device=x.device)
  doffset = torch.empty(c, dtype=torch.float32, device=x.device)
  _lib.call("cfk_layer_norm_bwd_static", x.data_ptr(), scale.data_ptr(), dy.data_ptr(), dx.data_ptr(), dscale.data_ptr(),
            doffset.data_ptr(), m, c, ops.tag(x.dtype), float(eps), torch.cuda.current_stream().cuda_stream)
  return dx, dscale, doffset


@pytest.mark.parametrize("m,c,dtype", [(4099, 128, torch.bfloat16), (1000, 256, torch.float32), (7, 96, torch.bfloat16)])
def test_matches_workspace_entry_twice(m, c, dtype):
  g = torch.Generator().manual_seed(11)
  x = torch.randn(m, c, generator=g).to(dtype).cuda()
  dy = torch.randn(m, c, generator=g).to(dtype).cuda()
  scale = (1 + 0.1 * torch.randn(c, generator=g)).cuda()
  want = ops.layer_norm_bwd(x, scale, dy, 1e-5)
  for _ in range(2):  # the second call reuses the scratch the first one left behind
    got = _static_bwd(x, scale, dy, 1e-5)
    torch.cuda.synchronize()
    for a, b in zip(got, want):
      assert torch.equal(a, b)
  assert ops.device_status() == 0


def test_rejects_rows_wider_than_the_scratch():
  x = torch.randn(64, 512, device="cuda", dtype=torch.bfloat16)
  scale = torch.ones(512, device="cuda")
  ops.layer_norm_bwd(x, scale, x, 1e-5)  # the workspace entry takes this width
  with pytest.raises(_lib.CfkError) as err:
    _static_bwd(x, scale, x, 1e-5)
  assert err.value.code == -5  # CFK_ERR_WORKSPACE


def test_second_call_allocates_nothing():
  """After the first call on the device has done its set-up, a call with caller-owned outputs leaves the driver's free
  memory (cudaMemGetInfo) and torch's allocator counters exactly where they were: no allocation by any route."""
  g = torch.Generator().manual_seed(12)
  m, c = 2048, 128
  x = torch.randn(m, c, generator=g).to(torch.bfloat16).cuda()
  dy = torch.randn(m, c, generator=g).to(torch.bfloat16).cuda()
  scale = torch.ones(c, device="cuda")
  dx = torch.empty_like(x)
  dscale = torch.empty(c, dtype=torch.float32, device="cuda")
  doffset = torch.empty(c, dtype=torch.float32, device="cuda")
  stream = torch.cuda.current_stream().cuda_stream

  def call():
    _lib.call("cfk_layer_norm_bwd_static", x.data_ptr(), scale.data_ptr(), dy.data_ptr(), dx.data_ptr(), dscale.data_ptr(),
              doffset.data_ptr(), m, c, ops.tag(x.dtype), 1e-5, stream)

  call()  # set-up, if this is the first call on the device
  torch.cuda.synchronize()
  free0, _ = torch.cuda.mem_get_info()
  alloc0, reserved0 = torch.cuda.memory_allocated(), torch.cuda.memory_reserved()
  call()
  torch.cuda.synchronize()
  free1, _ = torch.cuda.mem_get_info()
  assert free1 == free0
  assert torch.cuda.memory_allocated() == alloc0 and torch.cuda.memory_reserved() == reserved0
  want = ops.layer_norm_bwd(x, scale, dy, 1e-5)
  assert torch.equal(dx, want[0]) and torch.equal(dscale, want[1]) and torch.equal(doffset, want[2])
  assert ops.device_status() == 0

"""One Evoformer block on the GPU (every op a kernel of the library except the transitions' GEMMs) against the
same composition on the CPU oracle.  bf16 through nine residual updates: rel <= 2e-2 on both representations."""
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("s,r", [(16, 64), (24, 136)])
def test_block_matches_oracle(s, r):
  from colabfold_kernels import evoformer, ops
  from oracle.evoformer_ref import oracle_kernels
  g = torch.Generator().manual_seed(0)
  bf = torch.bfloat16
  msa, pair = torch.randn(s, r, 256, generator=g).to(bf), torch.randn(r, r, 128, generator=g).to(bf)
  msa_mask = (torch.rand(s, r, generator=g) < 0.95).float()
  pair_mask = (torch.rand(r, r, generator=g) < 0.95).float()
  params = evoformer.init_params(seed=3)
  ref_m, ref_p = evoformer.block(oracle_kernels(), msa, pair, msa_mask, pair_mask, params)
  cu = lambda t: t.cuda() if torch.is_tensor(t) else t
  def to_cuda(d):
    return {k: (to_cuda(v) if isinstance(v, dict) else tuple(cu(x) for x in v) if isinstance(v, tuple) else cu(v))
            for k, v in d.items()}
  m, p = evoformer.block(evoformer.cuda_kernels(), msa.cuda(), pair.cuda(), msa_mask.cuda(), pair_mask.cuda(),
                         to_cuda(params))
  assert ops.device_status() == 0
  assert O.rel_err(m.cpu().float(), ref_m) <= 2e-2
  assert O.rel_err(p.cpu().float(), ref_p) <= 2e-2


def test_block_with_e4m3_triangle_operands():
  """The opt-in e4m3 triangle multiplication inside the block against the bf16 block: FP8 tolerance (6e-2)."""
  from colabfold_kernels import evoformer, ops
  g = torch.Generator().manual_seed(1)
  bf = torch.bfloat16
  s, r = 16, 128
  msa, pair = torch.randn(s, r, 256, generator=g).to(bf).cuda(), torch.randn(r, r, 128, generator=g).to(bf).cuda()
  msa_mask = (torch.rand(s, r, generator=g) < 0.95).float().cuda()
  pair_mask = (torch.rand(r, r, generator=g) < 0.95).float().cuda()
  params = evoformer.init_params(seed=3, device="cuda")
  K = evoformer.cuda_kernels()
  m0, p0 = evoformer.block(K, msa, pair, msa_mask, pair_mask, params)
  m1, p1 = evoformer.block(K, msa, pair, msa_mask, pair_mask, params, fp8_trimul=True)
  assert ops.device_status() == 0
  assert O.rel_err(m1.cpu().float(), m0.cpu().float()) <= 6e-2
  assert O.rel_err(p1.cpu().float(), p0.cpu().float()) <= 6e-2
  assert not torch.equal(p0, p1)  # the e4m3 path really ran


def test_block_replayed_as_a_cuda_graph_matches_the_eager_block():
  """The whole block recorded once into a CUDA graph: a replay writes the same bits as launching op by op, and
  follows new input values written into the captured input tensors."""
  from colabfold_kernels import evoformer, ops
  g = torch.Generator().manual_seed(2)
  bf = torch.bfloat16
  s, r = 16, 64
  msa, pair = torch.randn(s, r, 256, generator=g).to(bf).cuda(), torch.randn(r, r, 128, generator=g).to(bf).cuda()
  msa_mask = (torch.rand(s, r, generator=g) < 0.9).float().cuda()
  pair_mask = (torch.rand(r, r, generator=g) < 0.9).float().cuda()
  params = evoformer.init_params(seed=4, device="cuda")
  K = evoformer.cuda_kernels()
  run = lambda: evoformer.block(K, msa, pair, msa_mask, pair_mask, params)
  m0, p0 = run()
  replay, (mg, pg) = evoformer.capture(run)
  replay()
  torch.cuda.synchronize()
  assert torch.equal(mg, m0) and torch.equal(pg, p0)
  msa.copy_(torch.randn(s, r, 256, generator=g).to(bf))
  m1, p1 = run()
  replay()
  torch.cuda.synchronize()
  assert ops.device_status() == 0
  assert torch.equal(mg, m1) and torch.equal(pg, p1) and not torch.equal(m1, m0)


def test_block_with_e4m3_attention_scores():
  """The FP8 attention opt-in inside the block (q and k in e4m3 in all four attentions) against the bf16 block: the
  reference's criterion for its FP8 attention, relative RMS < 0.08 (tests/test_ln_fusions.py:161,181)."""
  from colabfold_kernels import evoformer, ops
  g = torch.Generator().manual_seed(5)
  bf = torch.bfloat16
  s, r = 16, 128
  msa, pair = torch.randn(s, r, 256, generator=g).to(bf).cuda(), torch.randn(r, r, 128, generator=g).to(bf).cuda()
  msa_mask = (torch.rand(s, r, generator=g) < 0.95).float().cuda()
  pair_mask = (torch.rand(r, r, generator=g) < 0.95).float().cuda()
  params = evoformer.init_params(seed=6, device="cuda")
  K = evoformer.cuda_kernels()
  m0, p0 = evoformer.block(K, msa, pair, msa_mask, pair_mask, params)
  m1, p1 = evoformer.block(K, msa, pair, msa_mask, pair_mask, params, fp8_attention=True)
  assert ops.device_status() == 0
  assert O.rms_err(m1.cpu().float(), m0.cpu().float()) < 0.08
  assert O.rms_err(p1.cpu().float(), p0.cpu().float()) < 0.08
  assert not torch.equal(m0, m1) and not torch.equal(p0, p1)  # the e4m3 path really ran

"""The sharded Evoformer block on two GPUs (NCCL, one process per GPU) against the single-device block, both on the
CUDA kernels.  Skipped on a box with one GPU.  NVLS is switched off and the ranks only leave between steps."""
import os
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu


def _inputs(s=64, r=256):
  g = torch.Generator().manual_seed(0)
  msa, pair = torch.randn(s, r, 256, generator=g), torch.randn(r, r, 128, generator=g)
  msa_mask = (torch.rand(s, r, generator=g) < 0.9).float()
  pair_mask = (torch.rand(r, r, generator=g) < 0.9).float()
  return msa.bfloat16(), pair.bfloat16(), msa_mask, pair_mask


def _worker(rank, world, port, out, peer=False):
  for p in (ROOT, os.path.join(ROOT, "colabfold-kernels_b200")):
    sys.path.insert(0, p)
  from colabfold_kernels import evoformer, ops
  os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
  torch.cuda.set_device(rank)
  dev = torch.device("cuda", rank)
  dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
  msa, pair, msa_mask, pair_mask = _inputs()
  params = evoformer.init_params(seed=1, device=dev)
  # peer: the all-to-alls as the library's kernels over NVLink peer memory (and the triangle multiplication in its
  # exchanged form, so that every kind of all-to-all of the block runs); twice, so that receive buffers and the barrier
  # counter are reused
  kw = dict(exchange_triangle=True, peer_exchange=evoformer.PeerExchange(None, dev)) if peer else {}
  blk = evoformer.ShardedBlock(evoformer.cuda_kernels(), params, **kw)
  s, r = msa_mask.shape
  for _ in range(2 if peer else 1):
    m, p = blk(msa[blk.shard(s)].to(dev), pair[blk.shard(r)].to(dev), msa_mask.to(dev), pair_mask.to(dev))
  torch.cuda.synchronize()
  torch.save((m.cpu(), p.cpu(), ops.device_status()), os.path.join(out, f"rank{rank}.pt"))
  dist.barrier()
  dist.destroy_process_group()


@pytest.mark.timeout(600)
@pytest.mark.parametrize("peer", [False, True])
def test_two_gpu_block_matches_single_gpu(tmp_path, peer):
  if torch.cuda.device_count() < 2:
    pytest.skip("needs two GPUs")
  from colabfold_kernels import evoformer
  world, port = 2, 29711 + os.getpid() % 200 + (300 if peer else 0)
  mp.spawn(_worker, args=(world, port, str(tmp_path), peer), nprocs=world, join=True)
  msa, pair, msa_mask, pair_mask = _inputs()
  params = evoformer.init_params(seed=1, device="cuda")
  ref_m, ref_p = evoformer.block(evoformer.cuda_kernels(), msa.cuda(), pair.cuda(), msa_mask.cuda(), pair_mask.cuda(), params)
  got = [torch.load(os.path.join(tmp_path, f"rank{r}.pt")) for r in range(world)]
  assert all(g[2] == 0 for g in got)
  m = torch.cat([g[0] for g in got], 0).float()
  p = torch.cat([g[1] for g in got], 0).float()
  ref_m, ref_p = ref_m.float().cpu(), ref_p.float().cpu()
  # bf16 kernels; the sharded run sums the same terms in the same order, so the match is far inside the bf16 tolerance
  assert float((m - ref_m).abs().max()) <= 2e-2 * float(ref_m.abs().max())
  assert float((p - ref_p).abs().max()) <= 2e-2 * float(ref_p.abs().max())

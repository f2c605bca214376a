"""Host logic of the sharded Evoformer block on CPU: two gloo ranks with oracle-backed ops must reproduce the
single-device block exactly (the collectives only move data)."""
import os
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _inputs(s=8, r=16):
  g = torch.Generator().manual_seed(0)
  msa, pair = torch.randn(s, r, 256, generator=g), torch.randn(r, r, 128, generator=g)
  msa_mask = (torch.rand(s, r, generator=g) < 0.9).float()
  pair_mask = (torch.rand(r, r, generator=g) < 0.9).float()
  return msa, pair, msa_mask, pair_mask


def _worker(rank, world, port, out):
  for p in (ROOT, os.path.join(ROOT, "colabfold-kernels_b200")):
    sys.path.insert(0, p)
  from colabfold_kernels import evoformer
  from oracle.evoformer_ref import oracle_kernels
  os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
  dist.init_process_group("gloo", rank=rank, world_size=world)
  torch.set_num_threads(2)
  msa, pair, msa_mask, pair_mask = _inputs()
  params = evoformer.init_params(dtype=torch.float32, seed=1)
  blk = evoformer.ShardedBlock(oracle_kernels(), params)
  s, r = msa_mask.shape
  m, p = blk(msa[blk.shard(s)].contiguous(), pair[blk.shard(r)].contiguous(), msa_mask, pair_mask)
  torch.save((m, p), os.path.join(out, f"rank{rank}.pt"))
  dist.destroy_process_group()


@pytest.mark.timeout(600)
def test_two_rank_block_matches_single_device(tmp_path):
  from colabfold_kernels import evoformer
  from oracle.evoformer_ref import oracle_kernels
  world, port = 2, 29611 + os.getpid() % 200
  mp.spawn(_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True)
  msa, pair, msa_mask, pair_mask = _inputs()
  params = evoformer.init_params(dtype=torch.float32, seed=1)
  ref_m, ref_p = evoformer.block(oracle_kernels(), msa, pair, msa_mask, pair_mask, params)
  got = [torch.load(os.path.join(tmp_path, f"rank{r}.pt")) for r in range(world)]
  m = torch.cat([g[0] for g in got], 0)
  p = torch.cat([g[1] for g in got], 0)
  assert float((m - ref_m).abs().max()) <= 1e-4 * float(ref_m.abs().max())
  assert float((p - ref_p).abs().max()) <= 1e-4 * float(ref_p.abs().max())

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


def _worker(rank, world, port, out, s_r=(8, 16)):
  for p in (ROOT, os.path.join(ROOT, "colabfold-kernels_b200")):
    sys.path.insert(0, p)
  from colabfold_kernels import evoformer
  from oracle.evoformer_ref import oracle_kernels
  os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
  dist.init_process_group("gloo", rank=rank, world_size=world)
  torch.set_num_threads(2)
  msa, pair, msa_mask, pair_mask = _inputs(*s_r)
  params = evoformer.init_params(dtype=torch.float32, seed=1)
  blk = evoformer.ShardedBlock(oracle_kernels(), params, exchange_triangle=True)
  blk.validate(msa[blk.shard(s_r[0])], pair[blk.shard(s_r[1])], msa_mask, pair_mask, across_ranks=True)
  s, r = msa_mask.shape
  m, p = blk(msa[blk.shard(s)].contiguous(), pair[blk.shard(r)].contiguous(), msa_mask, pair_mask)
  torch.save((m, p), os.path.join(out, f"rank{rank}.pt"))
  dist.destroy_process_group()


@pytest.mark.timeout(900)
@pytest.mark.parametrize("s_r", [(8, 16), (4, 256)])
def test_two_rank_block_matches_single_device(tmp_path, s_r):
  """(8, 16): the gathered form of the triangle multiplication; (4, 256): shards of whole 128-row tiles, which take the
  exchanged form (all-to-all over channels, contraction of whole channels, all-to-all back)."""
  from colabfold_kernels import evoformer
  from oracle.evoformer_ref import oracle_kernels
  world, port = 2, 29611 + os.getpid() % 200
  mp.spawn(_worker, args=(world, port, str(tmp_path), s_r), nprocs=world, join=True)
  msa, pair, msa_mask, pair_mask = _inputs(*s_r)
  params = evoformer.init_params(dtype=torch.float32, seed=1)
  ref_m, ref_p = evoformer.block(oracle_kernels(), msa, pair, msa_mask, pair_mask, params)
  got = [torch.load(os.path.join(tmp_path, f"rank{r}.pt")) for r in range(world)]
  m = torch.cat([g[0] for g in got], 0)
  p = torch.cat([g[1] for g in got], 0)
  assert float((m - ref_m).abs().max()) <= 1e-4 * float(ref_m.abs().max())
  assert float((p - ref_p).abs().max()) <= 1e-4 * float(ref_p.abs().max())


class _FakePeer:
  """Stands in for evoformer.PeerExchange on CPU: the receive buffers are local tensors, the "addresses" handed to the
  kernels are the site numbers (every rank names a site the same way), the barrier is the process group's."""

  def __init__(self, world):
    self.P, self.bufs = world, {}

  def receive_buffer(self, site, shape, dtype):
    self.bufs[site] = torch.empty(shape, dtype=dtype)
    return self.bufs[site], [site] * self.P

  def barrier(self):
    dist.barrier()


def _fused_worker(rank, world, port, out):
  """The block with the triangle multiplication's exchanges done by the producing kernels' stores
  (ShardedBlock.projected_triangle_product): the two "peer" kernels are emulated by the oracle's kernels followed by the
  all-to-all that their stores amount to, so the wiring (buffer shapes, operand roles of the incoming update, site
  numbering, barriers) runs on CPU."""
  for p in (ROOT, os.path.join(ROOT, "colabfold-kernels_b200")):
    sys.path.insert(0, p)
  import types
  from colabfold_kernels import evoformer
  from oracle.evoformer_ref import oracle_kernels
  os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
  dist.init_process_group("gloo", rank=rank, world_size=world)
  torch.set_num_threads(2)
  K0, fake, calls = oracle_kernels(), _FakePeer(world), []

  def ln_gated_dual_proj_peer(x, sc, of, wp, bp, wg, bg, mask, lptrs, rptrs, my_rank, transpose=False):
    assert my_rank == rank and len(lptrs) == world
    l, r = K0.ln_gated_dual_proj(x, sc, of, wp, bp, wg, bg, mask, transpose=transpose)
    for t, site in ((l, lptrs[0]), (r, rptrs[0])):
      send = t.reshape((world, t.shape[0] // world) + tuple(t.shape[1:])).contiguous()
      assert tuple(fake.bufs[site].shape) == tuple(send.shape)
      dist.all_to_all_single(fake.bufs[site], send)
    calls.append("projection")

  def contract_exchanged_peer(ap, bp, optrs, my_rank, split_k=False):
    send = K0.contract_exchanged(ap, bp, split_k=split_k).contiguous()
    assert tuple(fake.bufs[optrs[0]].shape) == tuple(send.shape)
    dist.all_to_all_single(fake.bufs[optrs[0]], send)
    calls.append("contraction")

  K = types.SimpleNamespace(**vars(K0), ln_gated_dual_proj_peer=ln_gated_dual_proj_peer,
                            contract_exchanged_peer=contract_exchanged_peer)
  msa, pair, msa_mask, pair_mask = _inputs(4, 256)
  params = evoformer.init_params(dtype=torch.float32, seed=1)
  blk = evoformer.ShardedBlock(K, params)
  inner = blk.projected_triangle_product

  def with_peer(*a, **k):  # only this step sees the peer exchange: every other collective stays on the process group
    blk.peer = fake
    try:
      return inner(*a, **k)
    finally:
      blk.peer = None

  blk.projected_triangle_product = with_peer
  m, p = blk(msa[blk.shard(4)].contiguous(), pair[blk.shard(256)].contiguous(), msa_mask, pair_mask)
  torch.save((m, p, calls), os.path.join(out, f"rank{rank}.pt"))
  dist.destroy_process_group()


@pytest.mark.timeout(900)
def test_two_rank_block_with_the_exchanges_in_the_kernels_stores(tmp_path):
  from colabfold_kernels import evoformer
  from oracle.evoformer_ref import oracle_kernels
  world, port = 2, 29011 + os.getpid() % 200
  mp.spawn(_fused_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True)
  msa, pair, msa_mask, pair_mask = _inputs(4, 256)
  params = evoformer.init_params(dtype=torch.float32, seed=1)
  ref_m, ref_p = evoformer.block(oracle_kernels(), msa, pair, msa_mask, pair_mask, params)
  got = [torch.load(os.path.join(tmp_path, f"rank{r}.pt")) for r in range(world)]
  assert all(g[2] == ["projection", "contraction"] * 2 for g in got)  # outgoing and incoming update, both fused
  m = torch.cat([g[0] for g in got], 0)
  p = torch.cat([g[1] for g in got], 0)
  assert float((m - ref_m).abs().max()) <= 1e-4 * float(ref_m.abs().max())
  assert float((p - ref_p).abs().max()) <= 1e-4 * float(ref_p.abs().max())


def _bad_shard_worker(rank, world, port, out):
  for p in (ROOT, os.path.join(ROOT, "colabfold-kernels_b200")):
    sys.path.insert(0, p)
  from colabfold_kernels import evoformer
  from oracle.evoformer_ref import oracle_kernels
  os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
  dist.init_process_group("gloo", rank=rank, world_size=world)
  params = evoformer.init_params(dtype=torch.float32, seed=1)
  blk = evoformer.ShardedBlock(oracle_kernels(), params)
  found = []
  # sizes not divisible by the ranks, a shard of the wrong height, and ranks that disagree on n_res
  msa, pair, mm, pm = _inputs(7, 16)
  for args in ((msa[:3], pair[:8], mm, pm), ):
    try:
      blk(*args)
    except evoformer.ShardError as e:
      found.append(str(e))
  msa, pair, mm, pm = _inputs(8, 16)
  try:
    blk(msa[:4], pair[:5], mm, pm)
  except evoformer.ShardError as e:
    found.append(str(e))
  r = 16 if rank == 0 else 32
  msa, pair, mm, pm = _inputs(8, r)
  try:
    blk.validate(msa[:4], pair[:r // 2], mm, pm, across_ranks=True)
  except evoformer.ShardError as e:
    found.append(str(e))
  torch.save(found, os.path.join(out, f"err{rank}.pt"))
  dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_shard_errors_are_raised_before_any_work(tmp_path):
  world, port = 2, 29411 + os.getpid() % 200
  mp.spawn(_bad_shard_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True)
  for r in range(world):
    found = torch.load(os.path.join(tmp_path, f"err{r}.pt"))
    assert len(found) == 3, found
    assert "divisible" in found[0] and "pair shard" in found[1] and "disagree" in found[2]


def _stuck_worker(rank, world, port, out):
  import datetime
  for p in (ROOT, os.path.join(ROOT, "colabfold-kernels_b200")):
    sys.path.insert(0, p)
  from colabfold_kernels import evoformer
  from oracle.evoformer_ref import oracle_kernels
  os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
  dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
  blk = evoformer.ShardedBlock(oracle_kernels(), evoformer.init_params(dtype=torch.float32, seed=1))
  result = "peer"
  if rank == 0:  # rank 1 never joins this collective: the watchdog turns the stuck call into an error
    x = torch.ones(4)
    try:
      blk.guarded(lambda: dist.all_reduce(x))
      result = "no error"
    except evoformer.CollectiveTimeout as e:
      result = "timeout: " + str(e)[:80]
  torch.save(result, os.path.join(out, f"stuck{rank}.pt"))
  if rank == 1:
    import time
    time.sleep(8)  # stays away from the collective, leaves between steps


@pytest.mark.timeout(300)
def test_missing_peer_becomes_an_error_not_a_hang(tmp_path):
  world, port = 2, 29211 + os.getpid() % 200
  mp.spawn(_stuck_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True)
  assert torch.load(os.path.join(tmp_path, "stuck0.pt")).startswith("timeout")

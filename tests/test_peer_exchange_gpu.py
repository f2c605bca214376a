"""cfk_peer_alltoall on ONE GPU: the ranks are emulated one after the other (every "peer" buffer is a local one and the
flags the barrier waits for are set beforehand, so no kernel ever waits on another), which checks the strided copy
forms against torch; and the barrier's bounded wait: a flag nobody sets makes it give up after about a second and
leave its code in the status word.  The real exchange between GPUs is tests/test_evoformer_sharding_gpu.py."""
import pytest
import torch

pytestmark = pytest.mark.gpu
bf = torch.bfloat16


def ptrs(tensors):
  return torch.tensor([t.data_ptr() for t in tensors], dtype=torch.int64, device="cuda")


def emulate(P, sends, recv_bytes, **strides):
  """Run rank 0 .. P-1's call in turn; returns the P receive buffers (uint8)."""
  from colabfold_kernels import ops
  recvs = [torch.zeros(recv_bytes, dtype=torch.uint8, device="cuda") for _ in range(P)]
  flags = [torch.full((P,), 1 << 20, dtype=torch.int32, device="cuda") for _ in range(P)]  # already past any barrier number
  rp, fp = ptrs(recvs), ptrs(flags)
  for r in range(P):
    counter = torch.zeros(2, dtype=torch.int32, device="cuda")
    ops.peer_alltoall(sends[r], rp, fp, counter, r, P, **strides)
    assert int(counter[0]) == 1 and int(counter[1]) == 0
  torch.cuda.synchronize()
  assert ops.device_status() == 0
  return recvs


@pytest.mark.parametrize("P", [1, 2, 4, 8])
def test_plain_and_strided_forms(P):
  g = torch.Generator().manual_seed(P)
  n0, n1, c = 6, 8 * P, 16   # local [n0, n1, c]
  xs = [torch.randn(n0, n1, c, generator=g).to(bf).cuda() for _ in range(P)]
  es = 2
  # plain: part p of rank r's [P, chunk] lands as part r of rank p
  sends = [x.reshape(P, -1).contiguous() for x in xs]
  got = emulate(P, sends, sends[0].numel() * es)
  for p in range(P):
    want = torch.stack([sends[r][p] for r in range(P)])
    assert torch.equal(got[p].view(bf).view(want.shape), want)
  # rows -> columns: [n0, n1, c] per rank (rows sharded) -> [P n0, n1 / P, c] (columns sharded)
  run = n1 // P * c * es
  got = emulate(P, xs, xs[0].numel() * es, rows=n0, run_bytes=run, src_part=run, src_row=P * run, dst_part=n0 * run, dst_row=run)
  whole = torch.cat(xs, 0)                                   # [P n0, n1, c]
  for p in range(P):
    assert torch.equal(got[p].view(bf).view(P * n0, n1 // P, c), whole[:, p * (n1 // P):(p + 1) * (n1 // P)])
  # columns -> rows: [P n0', n1', c] per rank (columns sharded) -> [n0', P n1', c]
  ys = [torch.randn(P * 4, 8, c, generator=g).to(bf).cuda() for _ in range(P)]
  run = 8 * c * es
  got = emulate(P, ys, ys[0].numel() * es, rows=4, run_bytes=run, src_part=4 * run, src_row=run, dst_part=run, dst_row=P * run)
  whole = torch.cat(ys, 1)                                   # [P n0', P n1', c]
  for p in range(P):
    assert torch.equal(got[p].view(bf).view(4, P * 8, c), whole[p * 4:(p + 1) * 4])
  # all-gather along axis 1: the same source for every peer, strided destination
  zs = [torch.randn(3, 8, c, generator=g).to(bf).cuda() for _ in range(P)]
  run = 8 * c * es
  got = emulate(P, zs, P * zs[0].numel() * es, rows=3, run_bytes=run, src_part=0, src_row=run, dst_part=run, dst_row=P * run)
  for p in range(P):
    assert torch.equal(got[p].view(bf).view(3, P * 8, c), torch.cat(zs, 1))


def test_missing_peer_times_out_instead_of_hanging():
  from colabfold_kernels import _lib, ops
  send = torch.randn(2, 1024, device="cuda").to(bf)
  recvs = [torch.zeros(send.numel() * 2, dtype=torch.uint8, device="cuda") for _ in range(2)]
  flags = [torch.zeros(2, dtype=torch.int32, device="cuda") for _ in range(2)]   # rank 1 never arrives
  counter = torch.zeros(2, dtype=torch.int32, device="cuda")
  ops.peer_alltoall(send, ptrs(recvs), ptrs(flags), counter, 0, 2)
  torch.cuda.synchronize()                                    # the kernel gave up by itself (about a second)
  assert int(flags[1][0]) == 1                                # it did tell the peer
  assert ops.device_status(reset=False) == 1901
  with pytest.raises(_lib.CfkError):                          # and the library refuses further work until the status is read
    ops.layer_norm(send, torch.ones(1024, device="cuda"), torch.zeros(1024, device="cuda"))
  assert ops.device_status() == 1901 and ops.device_status() == 0
  ops.layer_norm(send, torch.ones(1024, device="cuda"), torch.zeros(1024, device="cuda"))


@pytest.mark.parametrize("P", [2, 4, 8])
@pytest.mark.parametrize("transpose", [False, True])
def test_projection_whose_stores_are_the_exchange(P, transpose):
  """ops.ln_gated_dual_proj_peer with the ranks emulated in turn on one GPU (every "peer" buffer is a local one):
  channel part q of rank r's left / right must land at index r of buffer q, bit-identical to the same kernel's
  ordinary outputs (the all-to-all over channels of the row-sharded triangle multiplication, evoformer.py
  ShardedBlock.projected_triangle_product; tri_mul.py:222-283 for the projection itself)."""
  from colabfold_kernels import ops
  g = torch.Generator().manual_seed(7 * P + int(transpose))
  a, b, k, p = (40, 256, 128, 256) if not transpose else (64, 136, 128, 256)
  rn = lambda *s, sc=1.0: (torch.randn(*s, generator=g) * sc).to(bf).cuda()
  wp, bp_, wg, bg = rn(k, p, sc=k ** -.5), rn(p, sc=.1), rn(k, p, sc=k ** -.5), rn(p, sc=.1)
  scale, offset = (1 + 0.1 * torch.randn(k, generator=g)).cuda(), (0.1 * torch.randn(k, generator=g)).cuda()
  outer, inner = (b, a) if transpose else (a, b)
  cp = 128 // P
  lbufs = [torch.zeros(P, cp, outer, inner, dtype=bf, device="cuda") for _ in range(P)]
  rbufs = [torch.zeros(P, cp, outer, inner, dtype=bf, device="cuda") for _ in range(P)]
  want = []
  for r in range(P):
    x = rn(a, b, k)
    mask = (torch.rand(a, b, generator=g) > .1).to(bf).cuda()
    want.append(ops.ln_gated_dual_proj(x, scale, offset, wp, bp_, wg, bg, mask, transpose=transpose))
    ops.ln_gated_dual_proj_peer(x, scale, offset, wp, bp_, wg, bg, mask, [t.data_ptr() for t in lbufs],
                                [t.data_ptr() for t in rbufs], r, transpose=transpose)
  torch.cuda.synchronize()
  assert ops.device_status() == 0
  for q in range(P):
    for r in range(P):
      assert torch.equal(lbufs[q][r], want[r][0][q * cp:(q + 1) * cp])
      assert torch.equal(rbufs[q][r], want[r][1][q * cp:(q + 1) * cp])


@pytest.mark.parametrize("P", [2, 4])
@pytest.mark.parametrize("split_k", [False, True])
def test_contraction_whose_stores_are_the_exchange(P, split_k):
  """ops.contract_exchanged_peer with the ranks emulated in turn on one GPU: rows [q i/P, (q+1) i/P) of rank r's
  product must land at index r of buffer q, bit-identical to ops.contract_exchanged's send buffer (the all-to-all of
  the triangle product back to row shards, evoformer.py ShardedBlock.projected_triangle_product)."""
  from colabfold_kernels import ops
  g = torch.Generator().manual_seed(11 * P + int(split_k))
  c, n, k = 3, 128 * P, 64 * P
  shape = (P, c, n, k // P) if split_k else (P, c, n // P, k)
  obufs = [torch.zeros(P, c, n // P, n, dtype=bf, device="cuda") for _ in range(P)]
  want = []
  for r in range(P):
    a, b = torch.randn(shape, generator=g).to(bf).cuda(), torch.randn(shape, generator=g).to(bf).cuda()
    want.append(ops.contract_exchanged(a, b, split_k=split_k))
    ops.contract_exchanged_peer(a, b, [t.data_ptr() for t in obufs], r, split_k=split_k)
  torch.cuda.synchronize()
  assert ops.device_status() == 0
  for q in range(P):
    for r in range(P):
      assert torch.equal(obufs[q][r], want[r][q])

"""One AlphaFold2 Evoformer block composed from the fused ops, on one GPU or row-sharded over P GPUs.

The block wiring is not part of colabfold-kernels (it lives in ColabFold/AlphaFold); this module composes the
reference's ops in the published Evoformer order - MSA row attention with pair bias, MSA column attention, MSA
transition, outer product mean, triangle multiplication outgoing and incoming, triangle attention starting and
ending node, pair transition - each a residual update, inference mode (no dropout).

`block(...)` runs on one device.  `ShardedBlock` keeps the MSA sharded over sequences (or residues) and the pair
representation sharded over rows, one process per GPU: every op works on its local shard, all-to-all switches an
operand between row and column sharding, all-gather supplies what every rank needs whole (the shared attention
biases, the right-hand operand of the triangle contraction, the right outer-product projection).  The kernels
only ever read local memory.

Every function takes the namespace `K` that supplies the ops: `cuda_kernels()` (the C library) in production; the
CPU tests pass one built on the oracle so that the sharding logic can be checked with the gloo backend.
"""
import math
import types

import torch


def init_params(c_m=256, c_z=128, heads_msa=8, heads_pair=4, d_head=32, c_opm=32, c_tri=128, factor=4, seed=0,
                dtype=torch.bfloat16, device="cpu"):
  """Random-init weights of one block (Xavier-normal matrices, zero biases, LayerNorm scale 1 / offset 0)."""
  g = torch.Generator().manual_seed(seed)

  def xav(*shape):
    fan_in, fan_out = shape[-2], shape[-1]
    return (torch.randn(*shape, generator=g) * math.sqrt(2.0 / (fan_in + fan_out))).to(dtype).to(device)

  def zeros(*shape):
    return torch.zeros(*shape, dtype=dtype, device=device)

  def ln(c):
    return torch.ones(c, dtype=torch.float32, device=device), torch.zeros(c, dtype=torch.float32, device=device)

  def attn(c, heads, bias_from=None):
    d = {"ln": ln(c), "w": xav(4, c, heads * d_head), "gate_bias": zeros(heads, d_head).add_(1.0),
         "wo": xav(heads * d_head, c), "bo": zeros(c), "heads": heads}
    if bias_from is not None:
      d["bias_ln"], d["wb"] = ln(bias_from), xav(bias_from, heads)
    return d

  def trans(c):
    return {"ln": ln(c), "w1": xav(c, factor * c), "b1": zeros(factor * c), "w2": xav(factor * c, c), "b2": zeros(c)}

  def trimul():
    return {"ln": ln(c_z), "wp": xav(c_z, 2 * c_tri), "bp": zeros(2 * c_tri), "wg": xav(c_z, 2 * c_tri),
            "bg": zeros(2 * c_tri).add_(1.0), "center_ln": ln(c_tri), "wo": xav(c_tri, c_z), "bo": zeros(c_z),
            "wgo": xav(c_z, c_z), "bgo": zeros(c_z).add_(1.0)}

  return {
      "row_attn": attn(c_m, heads_msa, bias_from=c_z), "col_attn": attn(c_m, heads_msa), "msa_transition": trans(c_m),
      "opm": {"ln": ln(c_m), "lw": xav(c_m, c_opm), "lb": zeros(c_opm), "rw": xav(c_m, c_opm), "rb": zeros(c_opm),
              "w": xav(c_opm * c_opm, c_z), "b": zeros(c_z)},
      "tri_out": trimul(), "tri_in": trimul(),
      "tri_attn_start": attn(c_z, heads_pair, bias_from=c_z), "tri_attn_end": attn(c_z, heads_pair, bias_from=c_z),
      "pair_transition": trans(c_z), "d_head": d_head,
  }


def cuda_kernels():
  """The production namespace: every op is a kernel of libcfk_b200."""
  from colabfold_kernels import ops

  def transition(x, ln, w1, b1, w2, b2):
    return ops.transition(x, ln[0], ln[1], w1, b1, w2, b2, add_input=True)

  return types.SimpleNamespace(
      ln_projection=ops.ln_projection, packed_attention=ops.packed_attention_fwd, output_projection=ops.output_projection,
      opm_projection=ops.opm_projection, outer_product_mean=ops.outer_product_mean,
      opm_projection_cm=ops.opm_projection_cm, outer_product_mean_cm=ops.outer_product_mean_cm,
      ln_gated_dual_proj=ops.ln_gated_dual_proj, ln_gated_dual_proj_peer=ops.ln_gated_dual_proj_peer,
      contract=ops.contract, contract_gathered=ops.contract_gathered,
      contract_exchanged=ops.contract_exchanged, contract_exchanged_peer=ops.contract_exchanged_peer,
      trimul_epilogue=ops.trimul_epilogue,
      transition=transition)


# ------------------------------------------------------------------------------------------ building blocks
def head_bias(K, x, prm):
  """Per-head attention bias from a (shard of the) pair representation x [a, b, c] -> [h, a, b]."""
  a, b, c = x.shape
  _, bias = K.ln_projection(x.reshape(a * b, c), prm["bias_ln"][0], prm["bias_ln"][1], None, prm["wb"])
  return bias.reshape(-1, a, b)


def attend(K, x, prm, bias, kmask, column, d_head, fp8=False):
  """Gated self-attention along axis 1 (rows) or axis 0 (columns) of x [X, Y, c] with residual update.
  fp8: the projection writes q (times sm_scale * log2 e) and k in e4m3 and the scores run on the 8-bit tensor-core
  path (the reference's opt-in, fused_ops.py:83-97); v, the gate and the output stay bf16."""
  X, Y, c = x.shape
  h = prm["heads"]
  if fp8:
    scales = (d_head ** -0.5 * 1.4426950408889634, 1.0)
    p, _, p8 = K.ln_projection(x.reshape(X * Y, c), prm["ln"][0], prm["ln"][1], prm["w"], None, f8_slots=(0, 1), f8_scales=scales)
    o = K.packed_attention(p.reshape(X, Y, 2, h, d_head), bias, kmask, prm["gate_bias"], d_head ** -0.5, column=column,
                           p8=p8.reshape(X, Y, 2, h, d_head))
    return K.output_projection(o.reshape(X * Y, h * d_head), prm["wo"], prm["bo"], x.reshape(X * Y, c)).reshape(X, Y, c)
  p, _ = K.ln_projection(x.reshape(X * Y, c), prm["ln"][0], prm["ln"][1], prm["w"], None)
  o = K.packed_attention(p.reshape(X, Y, 4, h, d_head), bias, kmask, prm["gate_bias"], d_head ** -0.5, column=column)
  return K.output_projection(o.reshape(X * Y, h * d_head), prm["wo"], prm["bo"], x.reshape(X * Y, c)).reshape(X, Y, c)


def triangle_update(K, pair_rows, x_cm, prm):
  """Center LayerNorm, output projection, sigmoid gate from the re-normed input, residual add (one kernel)."""
  a, b, c = pair_rows.shape
  out = K.trimul_epilogue(x_cm.reshape(x_cm.shape[0], a * b), pair_rows.reshape(a * b, c), prm["center_ln"][0],
                          prm["center_ln"][1], prm["wo"], prm["bo"], prm["wgo"], prm["bgo"], in_scale=prm["ln"][0],
                          in_offset=prm["ln"][1], add_input=True)
  return out.reshape(a, b, c)


def transition(K, x, prm):
  shape = x.shape
  return K.transition(x.reshape(-1, shape[-1]), prm["ln"], prm["w1"], prm["b1"], prm["w2"], prm["b2"]).reshape(shape)


def block(K, msa, pair, msa_mask, pair_mask, params, fp8_trimul=False, fp8_attention=False, fp8_opm=False):
  """One Evoformer block on one device.  msa [s, r, c_m], pair [r, r, c_z], msa_mask [s, r], pair_mask [r, r] (0/1).
  fp8_trimul: the triangle-multiplication operands are written and contracted in e4m3 (the reference's opt-in
  fp8_contraction, fused_ops.py:262-275): half the operand bytes, 1.7x the contraction rate, FP8 tolerance."""
  f8 = {"fp8": True} if fp8_trimul else {}
  fa = {"fp8": True} if fp8_attention else {}  # e4m3 q and k in the four attentions (forward only)
  d = params["d_head"]
  mm, pm = msa_mask > 0, pair_mask > 0
  msa = attend(K, msa, params["row_attn"], head_bias(K, pair, params["row_attn"]), mm, False, d, **fa)
  msa = attend(K, msa, params["col_attn"], None, mm.t().contiguous(), True, d, **fa)
  msa = transition(K, msa, params["msa_transition"])
  o = params["opm"]
  if fp8_opm:  # the e4m3 outer product keeps the three-kernel form
    left, right = K.opm_projection(msa, o["ln"][0], o["ln"][1], o["lw"], o["lb"], o["rw"], o["rb"], msa_mask.to(msa.dtype))
    pair = K.outer_product_mean(left, right, msa_mask, msa_mask, o["w"], o["b"], residual=pair, fp8=True)
  else:  # projections channel-major with the depth contiguous, then one kernel with the outer product on chip
    left, right = K.opm_projection_cm(msa, o["ln"][0], o["ln"][1], o["lw"], o["lb"], o["rw"], o["rb"], msa_mask.to(msa.dtype))
    pair = K.outer_product_mean_cm(left, right, msa_mask, msa_mask, o["w"], o["b"], residual=pair)
  for name, incoming in (("tri_out", False), ("tri_in", True)):
    t = params[name]
    l, r = K.ln_gated_dual_proj(pair, t["ln"][0], t["ln"][1], t["wp"], t["bp"], t["wg"], t["bg"], pair_mask.to(pair.dtype),
                                transpose=incoming, **f8)
    pair = triangle_update(K, pair, K.contract(r, l) if incoming else K.contract(l, r), t)
  pair = attend(K, pair, params["tri_attn_start"], head_bias(K, pair, params["tri_attn_start"]), pm, False, d, **fa)
  bias_end = head_bias(K, pair, params["tri_attn_end"]).transpose(1, 2).contiguous()
  pair = attend(K, pair, params["tri_attn_end"], bias_end, pm.t().contiguous(), True, d, **fa)
  pair = transition(K, pair, params["pair_transition"])
  return msa, pair


# ------------------------------------------------------------------------------------------ sharded over P ranks
class ShardError(ValueError):
  """The shards handed to the sharded block do not fit its partitioning (raised before anything is launched)."""


class CollectiveTimeout(RuntimeError):
  """A collective of the sharded block did not complete in time (a peer is missing or stuck)."""


class PeerExchange:
  """All-to-all over NVLink peer memory for the sharded block: receive buffers and flags in symmetric memory
  (torch.distributed._symmetric_memory supplies the allocation and the exchange of device pointers, nothing else),
  the transfers and the barrier are kernels of the library (cfk_peer_alltoall: plain stores into the peers' buffers, a
  flag barrier with a bounded wait).  Every call site of the block has its own receive buffer, allocated the first time
  the site runs (a collective rendezvous: run the block once eagerly before recording it into a CUDA graph); what a site
  received stays valid until the same site runs again."""

  def __init__(self, group, device):
    import os
    import torch.distributed as dist
    # plain peer mappings are all this needs: no NVLink multicast object is bound to the buffers
    os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
    import torch.distributed._symmetric_memory as symm
    self.symm, self.group, self.device = symm, group if group is not None else dist.group.WORLD, device
    self.P, self.rank = dist.get_world_size(group), dist.get_rank(group)
    self.flags = symm.empty(64, dtype=torch.int32, device=device)
    self.flags.zero_()
    torch.cuda.synchronize(device)
    self._handles = [symm.rendezvous(self.flags, self.group)]
    self.flag_ptrs = torch.tensor([int(p) for p in self._handles[0].buffer_ptrs], dtype=torch.int64, device=device)
    self.counter = torch.zeros(2, dtype=torch.int32, device=device)  # barrier number, finished blocks
    self.sites, self._retired = {}, []
    dist.barrier(group)  # every rank's flags are zero before any peer counts on them

  def _site(self, site, nbytes):
    if site not in self.sites or self.sites[site][0].numel() < nbytes:
      if site in self.sites:
        self._retired.append(self.sites[site])  # a recorded graph may still write there: never handed back
      buf = self.symm.empty(nbytes, dtype=torch.uint8, device=self.device)
      h = self.symm.rendezvous(buf, self.group)
      self._handles.append(h)
      host = [int(p) for p in h.buffer_ptrs]
      self.sites[site] = (buf, torch.tensor(host, dtype=torch.int64, device=self.device), host)
    return self.sites[site]

  def receive_buffer(self, site, shape, dtype):
    """The site's receive buffer as a tensor of this shape, and every rank's address of it (for a kernel whose own
    stores are the exchange, ops.ln_gated_dual_proj_peer); barrier() goes between those stores and the first read."""
    nbytes = torch.empty((), dtype=dtype).element_size()
    for d in shape:
      nbytes *= d
    buf, _, host = self._site(site, nbytes)
    return buf[:nbytes].view(dtype).view(shape), host

  def barrier(self):
    """The flag barrier alone (bounded wait, code 1901): every rank's earlier kernels on this stream have completed."""
    from colabfold_kernels import ops
    ops.peer_alltoall(self.flags, self.flag_ptrs, self.flag_ptrs, self.counter, self.rank, self.P, rows=0, run_bytes=0,
                      src_part=0, dst_part=0)

  def all_gather(self, site, x, dim):
    """Every rank's x concatenated along dim (0 or any later axis) -> a view of the site's receive buffer: each rank writes
    its shard straight to where it belongs in every peer's result, so no concatenation copy follows."""
    from colabfold_kernels import ops
    x = x.contiguous()
    es, P = x.element_size(), self.P
    lead = 1
    for d in x.shape[:dim]:
      lead *= d
    run = x.numel() // lead * es          # bytes of one leading-index slice of the local shard
    buf, ptrs, _ = self._site(site, P * x.numel() * es)
    ops.peer_alltoall(x, ptrs, self.flag_ptrs, self.counter, self.rank, P, rows=lead, run_bytes=run, src_part=0, src_row=run,
                      dst_part=run, dst_row=P * run)
    shape = list(x.shape)
    shape[dim] *= P
    return buf[:P * x.numel() * es].view(x.dtype).view(shape)

  def all_to_all(self, site, x, out_shape=None, **strides):
    """x [P, ...] contiguous: part p goes to rank p -> [P, ...] with part q what rank q sent here (a view of the site's
    receive buffer).  With strides (ops.peer_alltoall) x is any contiguous tensor whose parts are strided runs, and
    out_shape the shape of what arrives."""
    from colabfold_kernels import ops
    nbytes = x.numel() * x.element_size()
    buf, ptrs, _ = self._site(site, nbytes)
    ops.peer_alltoall(x, ptrs, self.flag_ptrs, self.counter, self.rank, self.P, **strides)
    return buf[:nbytes].view(x.dtype).view(x.shape if out_shape is None else out_shape)


class ShardedBlock:
  """The same block with the MSA sharded over sequences and the pair over rows, one rank per GPU.

  Inputs and outputs of `__call__` are the local shards msa [s/P, r, c_m] and pair [r/P, r, c_z]; the masks are
  replicated.  s and r must be divisible by the world size."""

  def __init__(self, K, params, group=None, fp8_trimul=False, fp8_attention=False, fp8_opm=False, exchange_triangle=None,
               peer_exchange=None):
    import torch.distributed as dist
    self.exchange_triangle = exchange_triangle  # None: by rank count; True / False: force the exchanged / gathered form
    self.K, self.params, self.dist, self.group = K, params, dist, group
    self.f8 = {"fp8": True} if fp8_trimul else {}  # e4m3 triangle operands: the gathered operand is half the bytes
    self.fa = {"fp8": True} if fp8_attention else {}  # e4m3 q and k in the attentions
    self.fo = {"fp8": True} if fp8_opm else {}  # e4m3 outer product of the MSA projections
    self.P = dist.get_world_size(group)
    self.rank = dist.get_rank(group)
    # a PeerExchange: the all-to-alls run as the library's kernels over NVLink peer memory instead of NCCL's
    self.peer, self._site_no = peer_exchange, 0

  def _all_to_all(self, send):
    """send [P, ...] contiguous -> what every rank sent here, [P, ...]."""
    self._site_no += 1
    if self.peer is not None:
      return self.peer.all_to_all(self._site_no, send)
    recv = torch.empty_like(send)
    if send.element_size() == 1:  # e4m3 operands travel as bytes
      self.dist.all_to_all_single(recv.view(torch.uint8), send.view(torch.uint8), group=self.group)
    else:
      self.dist.all_to_all_single(recv, send, group=self.group)
    return recv

  # dim 0 sharded -> dim 1 sharded: [n0/P, n1, c] -> [n0, n1/P, c]
  def rows_to_cols(self, x):
    P = self.P
    n0, n1, c = x.shape
    if self.peer is not None and (n1 // P * c * x.element_size()) % 16 == 0:
      # part p = columns [p n1/P, (p+1) n1/P) of every local row, read in place; it lands as rows [rank n0, (rank+1) n0)
      self._site_no += 1
      run = n1 // P * c * x.element_size()
      return self.peer.all_to_all(self._site_no, x.contiguous(), (P * n0, n1 // P, c), rows=n0, run_bytes=run, src_part=run,
                                  src_row=P * run, dst_part=n0 * run, dst_row=run)
    send = x.reshape(n0, P, n1 // P, c).permute(1, 0, 2, 3).contiguous()
    return self._all_to_all(send).reshape(P * n0, n1 // P, c)

  # dim 1 sharded -> dim 0 sharded: [n0, n1/P, c] -> [n0/P, n1, c]
  def cols_to_rows(self, x):
    P = self.P
    n0, n1, c = x.shape
    if self.peer is not None and (n1 * c * x.element_size()) % 16 == 0:
      # part p = rows [p n0/P, (p+1) n0/P), contiguous; it lands as columns [rank n1, (rank+1) n1) of the receiver's rows
      self._site_no += 1
      run = n1 * c * x.element_size()
      return self.peer.all_to_all(self._site_no, x.contiguous(), (n0 // P, P * n1, c), rows=n0 // P, run_bytes=run,
                                  src_part=n0 // P * run, src_row=run, dst_part=run, dst_row=P * run)
    send = x.reshape(P, n0 // P, n1, c).contiguous()
    return self._all_to_all(send).permute(1, 0, 2, 3).reshape(n0 // P, P * n1, c)

  def gather(self, x, dim):
    x = x.contiguous()
    if self.peer is not None and (x.numel() // max(1, math.prod(x.shape[:dim])) * x.element_size()) % 16 == 0:
      self._site_no += 1
      return self.peer.all_gather(self._site_no, x, dim)
    out = torch.empty((self.P * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    if x.element_size() == 1:  # e4m3 operands travel as bytes
      self.dist.all_gather_into_tensor(out.view(torch.uint8), x.view(torch.uint8), group=self.group)
    else:
      self.dist.all_gather_into_tensor(out, x, group=self.group)
    return out if dim == 0 else torch.cat(list(out.view((self.P,) + tuple(x.shape)).unbind(0)), dim=dim)

  def contract_all(self, a, b_local):
    """contract(a, every rank's b_local stacked on the row axis).  The gathered operand is read where the all-gather
    wrote it ([P, c, rows/P, k]) when its parts are whole 128-row tiles; otherwise it is re-laid out first."""
    if b_local.shape[1] % 128 == 0:
      return self.K.contract_gathered(a, self.gather(b_local, 0).view((self.P,) + tuple(b_local.shape)))
    return self.K.contract(a, self.gather(b_local, 1))

  def exchange(self, x):
    """All-to-all of x [P, ...] along its leading axis (part p goes to rank p), no re-layout on either side."""
    return self._all_to_all(x.contiguous())

  def triangle_product(self, a, b, split_k):
    """x_cm [c, rows/P, r] of a triangle multiplication from this rank's channel-major operands, or None when the
    shard sizes do not take the exchanged form.  Instead of gathering the right operand of every channel (P - 1 parts
    of [c, r/P, r] received per rank), the ranks swap to channel shards: an all-to-all of each operand over the
    channel axis, the contraction of c/P whole channels, and an all-to-all of the product back to row shards.  Each
    moves (P - 1)/P of one [c, r/P, r] tensor; the operands leave the projection kernel and the product leaves the
    contraction kernel in the layout the all-to-all sends, and what arrives is read in place.
    split_k False (outgoing edges): a, b [c, r/P, r], this rank's rows.  True (incoming edges): a, b [c, r, r/P], this
    rank's slice of the contracted axis."""
    P = self.P
    c = a.shape[0]
    rows, k_local = (a.shape[1], a.shape[2]) if split_k else (a.shape[1] * P, a.shape[2])
    unit = 128 // a.element_size()  # elements of a 128-byte slice
    if c % P or rows % (128 * P) or (split_k and k_local % unit) or not hasattr(self.K, "contract_exchanged"):
      return None
    if not self.exchange_triangle if self.exchange_triangle is not None else P < 4:
      return None  # three all-to-alls move 3 (P - 1) / P operand shards, the all-gather P - 1: a gain from 4 ranks on
    a, b = a.contiguous(), b.contiguous()
    ap = self.exchange(a.view((P, c // P) + tuple(a.shape[1:])))
    bp = self.exchange(b.view((P, c // P) + tuple(b.shape[1:])))
    out = self.exchange(self.K.contract_exchanged(ap, bp, split_k=split_k))  # [P, c/P, rows/P, r] = [c, rows/P, r]
    return out.view(c, out.shape[2], out.shape[3])

  def projected_triangle_product(self, pair_r, t, mask, incoming):
    """triangle_product with the two operand all-to-alls done by the projection kernel's own stores
    (ops.ln_gated_dual_proj_peer: channel part q of this rank's left and right go straight into rank q's receive
    buffers over NVLink peer memory), then one flag barrier; None when that form does not apply (no peer exchange,
    e4m3 operands, shard sizes outside the exchanged form)."""
    P, K = self.P, self.K
    a, b, c = pair_r.shape[0], pair_r.shape[1], 128
    outer, inner = (b, a) if incoming else (a, b)
    rows, k_local = (outer, inner) if incoming else (outer * P, inner)
    unit = 128 // pair_r.element_size()
    if self.peer is None or self.f8 or not hasattr(K, "ln_gated_dual_proj_peer") or not hasattr(K, "contract_exchanged"):
      return None
    if pair_r.shape[2] != 128 or t["wp"].shape[1] != 256 or 16 % P or P > 8:
      return None
    if pair_r.dtype not in getattr(K.ln_gated_dual_proj_peer, "dtypes", (pair_r.dtype,)):  # the CUDA kernel: bf16 only
      return None
    if rows % (128 * P) or (incoming and k_local % unit) or (inner * pair_r.element_size()) % 16:
      return None
    # with the operands' exchange inside the projection's stores the exchanged form wins from two ranks on (8.11 against
    # 8.26 ms for the gathered form at N_res 1024 on 2 GPUs)
    if not self.exchange_triangle if self.exchange_triangle is not None else P < 2:
      return None
    shape = (P, c // P, outer, inner)
    self._site_no += 1
    lbuf, lptrs = self.peer.receive_buffer(self._site_no, shape, pair_r.dtype)
    self._site_no += 1
    rbuf, rptrs = self.peer.receive_buffer(self._site_no, shape, pair_r.dtype)
    K.ln_gated_dual_proj_peer(pair_r, t["ln"][0], t["ln"][1], t["wp"], t["bp"], t["wg"], t["bg"], mask, lptrs, rptrs,
                              self.rank, transpose=incoming)
    self.peer.barrier()
    ap, bp = (rbuf, lbuf) if incoming else (lbuf, rbuf)
    if hasattr(K, "contract_exchanged_peer"):  # the product's way back likewise: stores into the peers' buffers, a barrier
      self._site_no += 1
      out, optrs = self.peer.receive_buffer(self._site_no, (P, c // P, rows // P, rows), pair_r.dtype)
      K.contract_exchanged_peer(ap, bp, optrs, self.rank, split_k=incoming)
      self.peer.barrier()
    else:
      out = self.exchange(K.contract_exchanged(ap, bp, split_k=incoming))
    return out.view(c, out.shape[2], out.shape[3])

  def shard(self, n):
    step = n // self.P
    return slice(self.rank * step, (self.rank + 1) * step)

  def validate(self, msa_s, pair_r, msa_mask, pair_mask, across_ranks=False):
    """Shape checks of one call's arguments; raises ShardError.  across_ranks also compares the sizes with every other
    rank's (one small all-reduce: call it outside a CUDA-graph capture)."""
    P = self.P
    if msa_mask.ndim != 2 or pair_mask.ndim != 2 or pair_mask.shape[0] != pair_mask.shape[1]:
      raise ShardError(f"masks must be [s, r] and [r, r], got {tuple(msa_mask.shape)} and {tuple(pair_mask.shape)}")
    s, r = msa_mask.shape
    if pair_mask.shape[0] != r:
      raise ShardError(f"msa_mask has {r} residues, pair_mask {pair_mask.shape[0]}")
    if s % P or r % P:
      raise ShardError(f"n_seq = {s} and n_res = {r} must both be divisible by the {P} ranks")
    if msa_s.ndim != 3 or tuple(msa_s.shape[:2]) != (s // P, r):
      raise ShardError(f"msa shard must be [n_seq / P, n_res, c] = [{s // P}, {r}, c], got {tuple(msa_s.shape)}")
    if pair_r.ndim != 3 or tuple(pair_r.shape[:2]) != (r // P, r):
      raise ShardError(f"pair shard must be [n_res / P, n_res, c] = [{r // P}, {r}, c], got {tuple(pair_r.shape)}")
    if across_ranks:
      sizes = torch.tensor([s, r, msa_s.shape[2], pair_r.shape[2]], dtype=torch.int64, device=msa_s.device)
      lo, hi = sizes.clone(), sizes.clone()
      self.guarded(lambda: (self.dist.all_reduce(lo, op=self.dist.ReduceOp.MIN, group=self.group),
                            self.dist.all_reduce(hi, op=self.dist.ReduceOp.MAX, group=self.group)))
      if not torch.equal(lo.cpu(), hi.cpu()):
        raise ShardError(f"ranks disagree on (n_seq, n_res, c_m, c_z): min {lo.tolist()}, max {hi.tolist()}")

  def guarded(self, fn, timeout_s=60.0):
    """Run fn() (which enqueues collectives) under a host-side watchdog: an error the process group raises (its own
    timeout when a peer never joins, a peer that went away) and device work that has not finished after timeout_s
    both become CollectiveTimeout, so the caller sees an error instead of a stuck rank."""
    import time
    try:
      out = fn()
      if torch.cuda.is_available() and torch.cuda.is_initialized():
        done = torch.cuda.Event()
        done.record()
        deadline = time.monotonic() + timeout_s
        while not done.query():
          if time.monotonic() > deadline:
            raise CollectiveTimeout(f"device work of rank {self.rank} still pending after {timeout_s:.0f} s")
          time.sleep(0.001)
      return out
    except CollectiveTimeout:
      raise
    except (RuntimeError, self.dist.DistBackendError) as e:
      raise CollectiveTimeout(f"collective failed on rank {self.rank}: {e}") from e

  def __call__(self, msa_s, pair_r, msa_mask, pair_mask):
    self.validate(msa_s, pair_r, msa_mask, pair_mask)
    self._site_no = 0
    K, prm, d = self.K, self.params, self.params["d_head"]
    s, r = msa_mask.shape
    ss, rs = self.shard(s), self.shard(r)
    mm, pm = msa_mask > 0, pair_mask > 0
    # 1 MSA row attention: sequences are independent; the pair bias is assembled from every rank's rows
    bias = self.gather(head_bias(K, pair_r, prm["row_attn"]), 1)
    msa_s = attend(K, msa_s, prm["row_attn"], bias, mm[ss].contiguous(), False, d, **self.fa)
    # 2-3 column attention and transition on the residue-sharded MSA
    msa_c = self.rows_to_cols(msa_s)
    msa_c = attend(K, msa_c, prm["col_attn"], None, mm.t()[rs].contiguous(), True, d, **self.fa)
    msa_c = transition(K, msa_c, prm["msa_transition"])
    # 4 outer product mean: local left projection against everyone's right projection -> local pair rows
    o = prm["opm"]
    mloc = msa_mask[:, rs].contiguous()
    if self.fo:
      left, right = K.opm_projection(msa_c, o["ln"][0], o["ln"][1], o["lw"], o["lb"], o["rw"], o["rb"], mloc.to(msa_c.dtype))
      pair_r = K.outer_product_mean(left, self.gather(right, 1), mloc, msa_mask, o["w"], o["b"], residual=pair_r, **self.fo)
    else:
      left, right = K.opm_projection_cm(msa_c, o["ln"][0], o["ln"][1], o["lw"], o["lb"], o["rw"], o["rb"], mloc.to(msa_c.dtype))
      pair_r = K.outer_product_mean_cm(left, self.gather(right, 1), mloc, msa_mask, o["w"], o["b"], residual=pair_r)
    msa_s = self.cols_to_rows(msa_c)
    # 5 triangle multiplication, outgoing edges: local rows of the left operand, all rows of the right
    t = prm["tri_out"]
    x_cm = self.projected_triangle_product(pair_r, t, pair_mask[rs].contiguous().to(pair_r.dtype), False)
    if x_cm is None:
      l, rr = K.ln_gated_dual_proj(pair_r, t["ln"][0], t["ln"][1], t["wp"], t["bp"], t["wg"], t["bg"],
                                   pair_mask[rs].contiguous().to(pair_r.dtype), **self.f8)
      x_cm = self.triangle_product(l, rr, False)
      if x_cm is None:
        x_cm = self.contract_all(l, rr)
    pair_r = triangle_update(K, pair_r, x_cm, t)
    # 6 incoming edges: out[i, j] = sum_k r[k, i] l[k, j].  Read transposed, this rank's pair rows give every (i, j)'s
    # operands for its own k: a slice of the contracted axis
    t = prm["tri_in"]
    l, rr = None, None
    x_cm = self.projected_triangle_product(pair_r, t, pair_mask[rs].contiguous().to(pair_r.dtype), True)
    if x_cm is None and r % (128 * self.P) == 0 and (self.exchange_triangle if self.exchange_triangle is not None else self.P >= 4):
      l, rr = K.ln_gated_dual_proj(pair_r, t["ln"][0], t["ln"][1], t["wp"], t["bp"], t["wg"], t["bg"],
                                   pair_mask[rs].contiguous().to(pair_r.dtype), transpose=True, **self.f8)
      x_cm = self.triangle_product(rr, l, True)
    if x_cm is None:  # shard sizes outside the exchanged form: operands from the column-sharded pair, gathered
      pair_c = self.rows_to_cols(pair_r)
      l, rr = K.ln_gated_dual_proj(pair_c, t["ln"][0], t["ln"][1], t["wp"], t["bp"], t["wg"], t["bg"],
                                   pair_mask[:, rs].contiguous().to(pair_r.dtype), transpose=True, **self.f8)
      x_cm = self.contract_all(rr, l)
    pair_r = triangle_update(K, pair_r, x_cm, t)
    # 7 triangle attention, starting node
    bias = self.gather(head_bias(K, pair_r, prm["tri_attn_start"]), 1)
    pair_r = attend(K, pair_r, prm["tri_attn_start"], bias, pm[rs].contiguous(), False, d, **self.fa)
    # 8 ending node on the column-sharded pair
    pair_c = self.rows_to_cols(pair_r)
    bias_end = self.gather(head_bias(K, pair_c, prm["tri_attn_end"]), 2).transpose(1, 2).contiguous()
    pair_c = attend(K, pair_c, prm["tri_attn_end"], bias_end, pm.t()[rs].contiguous(), True, d, **self.fa)
    pair_r = self.cols_to_rows(pair_c)
    # 9 pair transition
    pair_r = transition(K, pair_r, prm["pair_transition"])
    return msa_s, pair_r


def capture(fn):
  """Record one call of fn() (kernels, copies and NCCL collectives alike) into a CUDA graph on a side stream and
  return (replay, outputs): replay() launches the whole recorded block with one host call, writing into the same
  output tensors.  fn must have run before (extension attributes set, communicators built) and its inputs must stay
  where they are; every rank of a sharded block captures and replays together."""
  side = torch.cuda.Stream()
  side.wait_stream(torch.cuda.current_stream())
  with torch.cuda.stream(side):
    fn()  # once on the capturing stream: allocator pools and lazy state settle before the recording
  torch.cuda.current_stream().wait_stream(side)
  torch.cuda.synchronize()
  graph = torch.cuda.CUDAGraph()
  with torch.cuda.graph(graph, stream=side):
    outputs = fn()
  return graph.replay, outputs


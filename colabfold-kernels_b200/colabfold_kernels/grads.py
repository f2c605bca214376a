"""Differentiation glue: torch.autograd wrappers with the semantics of the reference's custom VJPs
(src/colabfold_kernels/grads.py and tri_flash.py:421-449).  Forward and backward both run in the C library."""
import torch

from colabfold_kernels import ops


class _Attention(torch.autograd.Function):
  """tri_flash.py:421-446: forward with lse, backward through the flash backward; the boolean mask gets no
  gradient and dbias is cast to the bias dtype."""

  @staticmethod
  def forward(ctx, q, k, v, bias, kmask, scale, seq_major):
    out, lse = ops.attention_fwd(q, k, v, bias, kmask, scale, seq_major=seq_major, want_lse=True)
    ctx.save_for_backward(q, k, v, bias if bias is not None else torch.empty(0, device=q.device), kmask, out, lse)
    ctx.scale, ctx.seq_major, ctx.has_bias = scale, seq_major, bias is not None
    return out

  @staticmethod
  def backward(ctx, dout):
    q, k, v, bias, kmask, out, lse = ctx.saved_tensors
    bias = bias if ctx.has_bias else None
    want_dbias = ctx.has_bias and ctx.needs_input_grad[3]
    dq, dk, dv, dbias = ops.attention_bwd(q, k, v, bias, kmask, out, dout, lse, ctx.scale, seq_major=ctx.seq_major,
                                          want_dbias=want_dbias)
    return dq, dk, dv, (dbias.to(bias.dtype) if want_dbias else None), None, None, None


def attention(q, k, v, mask_bias, nonbatched_bias, scale, *, seq_major=False):
  """pallas_attention's contract (tri_flash.py:452-478): mask_bias [b|1,1,1,Sk] additive (about -1e9 = masked),
  nonbatched_bias [h,Sq,Sk] or None, key_dim == value_dim; returns q's layout and dtype."""
  assert q.shape[-1] == v.shape[-1], f"attention needs key_dim == value_dim, got {q.shape[-1]} vs {v.shape[-1]}"
  b = q.shape[0]
  sk = k.shape[1] if seq_major else k.shape[2]
  kmask = (mask_bias[:, 0, 0, :] > -1e3).expand(b, sk).contiguous()
  bias = None if nonbatched_bias is None else nonbatched_bias.to(q.dtype)
  return _Attention.apply(q, k, v, bias, kmask, float(scale), bool(seq_major))


class _LayerNorm(torch.autograd.Function):
  """grads.py:16-50."""

  @staticmethod
  def forward(ctx, x, scale, offset, eps):
    ctx.save_for_backward(x, scale, offset)
    ctx.eps = eps
    return ops.layer_norm(x, scale, offset, eps)

  @staticmethod
  def backward(ctx, dy):
    x, scale, offset = ctx.saved_tensors
    dx, dscale, doffset = ops.layer_norm_bwd(x, scale, dy, ctx.eps)
    return dx, dscale.to(scale.dtype), doffset.to(offset.dtype), None


def layer_norm(x, scale, offset, *, eps=1e-5):
  return _LayerNorm.apply(x, scale, offset, float(eps))


# ---- forward-only kernels, backward through the differentiable reference (grads.py:106-143) -----------------
def differentiable_via(fwd, ref, nondiff=()):
  """fwd's forward with the gradient of ref, which recomputes in the backward.  fwd and ref take the same
  arguments; keyword arguments must be named in `nondiff` (they are static); integral or absent positional
  inputs get no gradient."""

  def call(*args, **kwargs):
    extra = set(kwargs) - set(nondiff)
    if extra:
      raise TypeError(f"{getattr(fwd, '__name__', fwd)}: pass {sorted(extra)} positionally")
    diff = [i for i, a in enumerate(args) if torch.is_tensor(a) and a.is_floating_point() and a.requires_grad]
    if not diff or not torch.is_grad_enabled():
      return fwd(*args, **kwargs)
    return _Via.apply(fwd, ref, kwargs, diff, len(args), *args)

  call.__name__ = getattr(fwd, "__name__", "fused")
  call.__doc__ = fwd.__doc__
  return call


class _Via(torch.autograd.Function):

  @staticmethod
  def forward(ctx, fwd, ref, kwargs, diff, nargs, *args):
    ctx.ref, ctx.kwargs, ctx.diff = ref, kwargs, diff
    ctx.args = args
    out = fwd(*[a.detach() if torch.is_tensor(a) else a for a in args], **kwargs)
    ctx.tuple_out = isinstance(out, (tuple, list))
    return tuple(out) if ctx.tuple_out else out

  @staticmethod
  def backward(ctx, *douts):
    args = list(ctx.args)
    leaves = []
    for i in ctx.diff:
      leaf = args[i].detach().requires_grad_(True)
      args[i] = leaf
      leaves.append(leaf)
    with torch.enable_grad():
      out = ctx.ref(*args, **ctx.kwargs)
      outs = out if isinstance(out, (tuple, list)) else (out,)
      pairs = [(o, d) for o, d in zip(outs, douts) if o is not None and d is not None]
      loss = sum((o.float() * d.float()).sum() for o, d in pairs)
    grads = torch.autograd.grad(loss, leaves, allow_unused=True)
    full = [None] * len(ctx.args)
    for i, g in zip(ctx.diff, grads):
      full[i] = None if g is None else g.to(ctx.args[i].dtype)
    return (None, None, None, None, None, *full)


# ---- gated dual projection (grads.py:56-102): the two projections are recomputed in the backward -------------
class _Gdp(torch.autograd.Function):

  @staticmethod
  def forward(ctx, x, wp, bp, wg, bg, mask, split, channel_major, activation):
    ctx.save_for_backward(x, wp, bp, wg, bg, mask)
    ctx.cfg = (split, channel_major, activation)
    out = ops.gated_dual_proj(x, wp, bp, wg, bg, mask, split=split, channel_major=channel_major, activation=activation)
    return out

  @staticmethod
  def backward(ctx, *dys):
    x, wp, bp, wg, bg, mask = ctx.saved_tensors
    split, channel_major, activation = ctx.cfg
    if split:
      left, right = (t.T for t in dys) if channel_major else dys
      dy = torch.cat([left, right], dim=-1)
    else:
      dy = dys[0]
    xf, dyf = x.float(), dy.float()
    proj = xf @ wp.float() + bp.float()
    gate = (xf @ wg.float() + bg.float()).detach().requires_grad_(True)
    with torch.enable_grad():
      act = torch.nn.functional.silu(gate) if activation == 1 else torch.sigmoid(gate)
    m = mask.float()[:, None]
    dproj = dyf * m * act.detach()
    dgate, = torch.autograd.grad(act, gate, dyf * m * proj)
    dx = dproj @ wp.float().T + dgate @ wg.float().T
    dmask = (dyf * proj * act.detach()).sum(-1).to(mask.dtype) if mask.is_floating_point() else None
    return (dx.to(x.dtype), (xf.T @ dproj).to(wp.dtype), dproj.sum(0).to(bp.dtype), (xf.T @ dgate).to(wg.dtype),
            dgate.sum(0).to(bg.dtype), dmask, None, None, None)


def gated_dual_proj(x, wp, bp, wg, bg, mask, *, split=False, channel_major=False, activation=0):
  return _Gdp.apply(x, wp, bp, wg, bg, mask, bool(split), bool(channel_major), int(activation))


# ---- packed attention: forward reads p in place, backward is the flash backward on the unpacked slots ----------
class _PackedAttention(torch.autograd.Function):
  """packed_attn.py:163-177 `attention_via`: the VJP is that of attention on the unpacked slots followed by the gate."""

  @staticmethod
  def forward(ctx, p, bias, kmask, gate_bias, sm_scale, column, trim):
    ctx.save_for_backward(p, bias if bias is not None else torch.empty(0, device=p.device), kmask,
                          gate_bias if gate_bias is not None else torch.empty(0, device=p.device))
    ctx.cfg = (sm_scale, column, trim, bias is not None, gate_bias is not None)
    return ops.packed_attention_fwd(p, bias, kmask, gate_bias, sm_scale, column=column, trim=trim)

  @staticmethod
  def backward(ctx, dout):
    p, bias, kmask, gate_bias = ctx.saved_tensors
    sm_scale, column, trim, has_bias, gated = ctx.cfg
    bias = bias if has_bias else None
    pp = p.transpose(0, 1) if column else p              # [batch, seq, G, H, D]
    do = dout.transpose(0, 1) if column else dout
    q, k, v = (pp[:, :, i].contiguous() for i in range(3))  # seq-major [b, s, h, d]
    o_att, lse = ops.attention_fwd(q, k, v, bias, kmask, sm_scale, seq_major=True, want_lse=True)
    do = do.contiguous()
    if trim:
      # the trimmed forward writes zeros for batch rows without a live key and for queries past the last live key of
      # any row (packed_attn.py:132-137): those outputs carry no gradient
      lim = ops.trim_limits(kmask)
      rows = (lim[:-1] > 0)[:, None] & (torch.arange(do.shape[1], device=do.device) < lim[-1])[None, :]
      do = do * rows[:, :, None, None].to(do.dtype)
    dg = None
    if gated:
      sig = torch.sigmoid(pp[:, :, 3].float() + gate_bias.float())
      dg = do.float() * o_att.float() * sig * (1 - sig)
      do = (do.float() * sig).to(p.dtype)
    dq, dk, dv, dbias = ops.attention_bwd(q, k, v, bias, kmask, o_att, do, lse, sm_scale, seq_major=True,
                                          want_dbias=has_bias)
    parts = [dq, dk, dv] + ([dg.to(p.dtype)] if gated else [])
    dp = torch.stack(parts, dim=2)
    dp = dp.transpose(0, 1) if column else dp
    return (dp.contiguous(), dbias.to(bias.dtype) if has_bias else None, None,
            dg.sum(dim=(0, 1)).to(gate_bias.dtype) if gated else None, None, None, None)


def packed_attention(p, bias, kmask, gate_bias=None, *, sm_scale, column=False, trim=False):
  return _PackedAttention.apply(p, bias, kmask, gate_bias, float(sm_scale), bool(column), bool(trim))

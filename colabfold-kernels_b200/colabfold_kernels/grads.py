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

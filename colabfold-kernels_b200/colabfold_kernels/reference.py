"""float32 reference math of the fused ops, in PyTorch, on whatever device the tensors live on.

The reference package defines the backward of its forward-only fused kernels as the VJP of these functions,
recomputed in the backward pass (src/colabfold_kernels/grads.py:106-143 `differentiable_via`): the forward
runs the kernel, the gradient is autograd through the reference math.  This module is that reference math for
the same purpose; the forward paths never call it.
"""
import torch

NEG = -0.7 * 3.4028234663852886e38  # tri_flash.py:19


def _f(x):
  return None if x is None else x.float()


def ref_ln(xf, scale, offset, eps):
  """transition.py:61-65."""
  mean = xf.mean(-1, keepdim=True)
  var = ((xf - mean) ** 2).mean(-1, keepdim=True)
  return (xf - mean) * torch.rsqrt(var + eps) * scale + offset


def ref_gdp(x, wp, bp, wg, bg, mask, activation=torch.sigmoid):
  """tri_mul.py:454-457."""
  return mask[:, None] * (x @ wp + bp) * activation(x @ wg + bg)


def ref_ln_gdp(x, ln_scale, ln_offset, wp, bp, wg, bg, mask, *, eps=1e-5, transpose=False, pad=1, **_):
  """tri_mul.py:286-300."""
  x, mask = _f(x), torch.clamp(_f(mask), min=0)
  pair = None
  if x.ndim == 3:
    if transpose:
      x, mask = x.transpose(0, 1), mask.T
    pair = x.shape[:2]
    x, mask = x.reshape(-1, x.shape[-1]), mask.reshape(-1)
  y = ref_gdp(ref_ln(x, _f(ln_scale), _f(ln_offset), eps), _f(wp), _f(bp), _f(wg), _f(bg), mask)
  ci = wp.shape[1] // 2
  left, right = y[:, :ci].T, y[:, ci:].T
  if pair is None:
    return left, right
  rows = -(-pair[1] // pad) * pad
  shape = lambda h: torch.nn.functional.pad(h.reshape(ci, *pair), (0, rows - pair[1]))
  return shape(left), shape(right)


def ref_trimul_epilogue(x_cm, act, ln_scale, ln_offset, wo, bo, wg, bg, residual=None, *, eps=1e-5):
  """tri_mul.py:446-451."""
  y = ref_ln(_f(x_cm).T, _f(ln_scale), _f(ln_offset), eps)
  out = (y @ _f(wo) + _f(bo)) * torch.sigmoid(_f(act) @ _f(wg) + _f(bg))
  return out if residual is None else out + _f(residual)


def ref_trimul_epilogue_ln(x_cm, x, in_scale, in_offset, ln_scale, ln_offset, wo, bo, wg, bg, keep=None, *, eps=1e-5,
                           add_input=False):
  """tri_mul.py:441-444."""
  act = ref_ln(_f(x), _f(in_scale), _f(in_offset), eps)
  return ref_trimul_epilogue(x_cm, act, ln_scale, ln_offset, wo, bo, wg, bg, x if add_input else None, eps=eps)


def ref_contract(a, b):
  """contract.py:56-57."""
  return torch.einsum("cik,cjk->cij", _f(a), _f(b))


def ref_ln_projection(x, ln_scale, ln_offset, w=None, wb=None, keep=None, *, eps=1e-5, f8_slots=(), f8_scales=None, **_):
  """packed_attn.py:308-318: with f8_slots the third output holds those slots times their static scales (fp32 here,
  before any rounding) and p the others."""
  y = ref_ln(_f(x), _f(ln_scale), _f(ln_offset), eps)
  b = None if wb is None else (y @ _f(wb)).T
  if w is None:
    return None, b
  p = torch.einsum("ma,gan->mgn", y, _f(w))
  if not f8_slots:
    return p.reshape(x.shape[0], -1), b
  rest = [g for g in range(w.shape[0]) if g not in f8_slots]
  scales = torch.tensor(list(f8_scales or (1.0,) * len(f8_slots)), dtype=p.dtype)
  flat = lambda t: t.reshape(x.shape[0], -1)
  return flat(p[:, rest]), b, flat(p[:, list(f8_slots)] * scales[None, :, None])


def ref_output_projection(o, w, b, residual=None, keep=None):
  """packed_attn.py:387-389."""
  out = _f(o) @ _f(w) + _f(b)
  return out if residual is None else out + _f(residual)


def ref_opm_projection(x, ln_scale, ln_offset, lw, lb, rw, rb, mask, *, eps=1e-5):
  """opm.py:62-66."""
  y = ref_ln(_f(x), _f(ln_scale), _f(ln_offset), eps)
  mv = _f(mask)[..., None]
  return mv * (y @ _f(lw) + _f(lb)), mv * (y @ _f(rw) + _f(rb))


def ref_opm_update(lhs, t, bias, norm, residual=None, *, eps=1e-3):
  """opm.py:116-119."""
  out = torch.einsum("bk,kdf->bdf", _f(lhs), _f(t)) + _f(bias)
  out = out / (eps + _f(norm))[..., None]
  return out if residual is None else out + _f(residual)


def ref_opm_outer(left, right, w):
  """opm.py:165-168."""
  act = torch.einsum("abc,ade->bced", _f(left), _f(right))
  act = act.reshape(act.shape[0], -1, act.shape[-1])
  return torch.einsum("bkd,kf->bdf", act, _f(w))


def ref_transition(x, ln_scale, ln_offset, w1, b1, w2, b2, keep=None, *, eps=1e-5, add_input=False):
  """transition.py:141-146."""
  xf = _f(x)
  y = ref_ln(xf, _f(ln_scale), _f(ln_offset), eps)
  h = torch.relu(y @ _f(w1) + _f(b1))
  out = h @ _f(w2) + _f(b2)
  return out + xf if add_input else out

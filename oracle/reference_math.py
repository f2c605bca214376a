"""PyTorch-CPU restatement of the reference's fp32 ``ref_*`` math (test infrastructure only).

Every function casts its inputs to ``dtype`` (float32 as the reference does, or float64 for a
tighter check) and returns tensors of that dtype; callers round to the storage dtype where
they compare stored outputs.  Citations are paths inside mirditalab/colabfold-kernels v0.9.0.
"""
import math

import numpy as np
import torch

# src/colabfold_kernels/tri_flash.py:19-25
NEG = -0.7 * float(np.finfo(np.float32).max)
LOG2E = math.log2(math.e)
E4M3_MAX = 448.0
P_SHIFT = 8.0

__all__ = [
    "NEG", "LOG2E", "E4M3_MAX", "P_SHIFT", "e4m3", "kmask_from_mask_bias", "ref_attn", "ref_attn_lse",
    "ref_attention", "ref_attn_bwd", "ref_packed_attention", "trim_limits", "ref_trimmed",
    "attention_via", "ref_layer_norm", "ref_ln", "layer_norm_bwd", "ref_gdp", "gdp_bwd", "ref_ln_gdp",
    "ref_trimul_epilogue", "ref_trimul_epilogue_ln", "ref_contract", "ref_fp8_contract",
    "ref_ln_projection", "ref_output_projection", "ref_opm_projection", "ref_opm_update",
    "ref_opm_outer", "ref_opm_deep", "ref_transition", "rel_err", "rms_err", "vjp",
]


def _f(x, dtype=torch.float32):
  return None if x is None else torch.as_tensor(x).to(dtype)


def e4m3(x):
  """Saturating cast to float8 e4m3: clip to +-448 first (tri_flash.py:28-30)."""
  return torch.clamp(torch.as_tensor(x).float(), -E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)


# ---------------------------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------------------------
def kmask_from_mask_bias(mask_bias, b, sk):
  """mask_bias [b|1, 1, 1, Sk] additive -> bool [b, Sk] (tri_flash.py:472)."""
  return (torch.as_tensor(mask_bias)[:, 0, 0, :].float() > -1e3).expand(b, sk)


def ref_attn(q, k, v, bias, kmask, sm_scale, dtype=torch.float32):
  """Heads-major [N,H,S,D] attention (tri_flash.py:481-485; tests/test_pallas_vjp.py:14-17).

  logits = scale*q.k + bias; masked keys are REPLACED by the finite floor NEG, so a row with no
  live key is the uniform mean of all Sk values."""
  q, k, v, bias = _f(q, dtype), _f(k, dtype), _f(v, dtype), _f(bias, dtype)
  logits = torch.einsum("nhqd,nhkd->nhqk", q, k) * sm_scale + bias[None]
  logits = torch.where(torch.as_tensor(kmask)[:, None, None, :], logits, torch.tensor(NEG, dtype=dtype))
  w = torch.softmax(logits, dim=-1)
  return torch.einsum("nhqk,nhkd->nhqd", w, v)


def ref_attn_lse(q, k, bias, kmask, sm_scale, dtype=torch.float32):
  """The forward's row statistic: lse = m + log2(l) in the log2 domain, [N,H,Sq] (tri_flash.py:221-223)."""
  q, k, bias = _f(q, dtype), _f(k, dtype), _f(bias, dtype)
  s = (torch.einsum("nhqd,nhkd->nhqk", q, k) * sm_scale + bias[None]) * LOG2E
  s = torch.where(torch.as_tensor(kmask)[:, None, None, :], s, torch.tensor(NEG, dtype=dtype))
  m = s.max(dim=-1).values
  return m + torch.log2(torch.exp2(s - m[..., None]).sum(-1))


def ref_attention(q, k, v, mask_bias, nonbatched_bias, scale, layout="heads", dtype=torch.float32):
  """The public entry's semantics (tri_flash.py:452-478): mask_bias [b,1,1,Sk] -> kmask, a missing
  bias is zeros, 'seq' layout is [b,S,h,c]; returns q's layout."""
  q, k, v = _f(q, dtype), _f(k, dtype), _f(v, dtype)
  if layout == "seq":
    q, k, v = (t.transpose(1, 2) for t in (q, k, v))
  b, h, sq, _ = q.shape
  sk = k.shape[2]
  kmask = kmask_from_mask_bias(mask_bias, b, sk)
  bias = torch.zeros(h, sq, sk, dtype=dtype) if nonbatched_bias is None else _f(nonbatched_bias, dtype)
  o = ref_attn(q, k, v, bias, kmask, scale, dtype)
  return o.transpose(1, 2) if layout == "seq" else o


def ref_attn_bwd(q, k, v, bias, kmask, out, dout, lse, sm_scale, dtype=torch.float32, round_to=None):
  """Explicit backward of the flash kernel (tri_flash.py:313-355,380,434-446), heads-major.

  delta = sum_d out*dout; p = 2^(s - lse) (1/Sk on rows whose lse <= NEG/2: fully masked);
  ds = live ? p*(dp - delta) : 0; dv = p^T do; dk = scale ds^T q; dq = scale ds k; dbias = sum_n ds.
  round_to: dtype p and ds are rounded to before the three output GEMMs (tri_flash.py:347-351)."""
  q, k, v, bias, out, dout, lse = (_f(t, dtype) for t in (q, k, v, bias, out, dout, lse))
  kmask = torch.as_tensor(kmask)
  sk = k.shape[2]
  delta = (out * dout).sum(-1)
  live = kmask[:, None, None, :].expand(q.shape[0], q.shape[1], q.shape[2], sk)
  s = torch.where(live, (torch.einsum("nhqd,nhkd->nhqk", q, k) * sm_scale + bias[None]) * LOG2E,
                  torch.tensor(NEG, dtype=dtype))
  p = torch.where(lse[..., None] <= NEG / 2, torch.full_like(s, 1.0 / sk), torch.exp2(s - lse[..., None]))
  dp = torch.einsum("nhqd,nhkd->nhqk", dout, v)
  ds = torch.where(live, p * (dp - delta[..., None]), torch.zeros_like(p))
  if round_to is not None:
    pr, dsr = p.to(round_to).to(dtype), ds.to(round_to).to(dtype)
  else:
    pr, dsr = p, ds
  dv = torch.einsum("nhqk,nhqd->nhkd", pr, dout)
  dk = torch.einsum("nhqk,nhqd->nhkd", dsr, q) * sm_scale
  dq = torch.einsum("nhqk,nhkd->nhqd", dsr, k) * sm_scale
  return dq, dk, dv, ds.sum(0)


def trim_limits(kmask, block_k=1):
  """(ends [batch], lim [1]) as packed_attn.py:123-129."""
  kmask = torch.as_tensor(kmask)
  s = kmask.shape[1]
  anyk = kmask.any(dim=1)
  last = torch.where(anyk, s - torch.argmax(kmask.flip(1).to(torch.int32), dim=1), torch.zeros_like(anyk, dtype=torch.long))
  return (-(-last // block_k)).to(torch.int32), last.max().reshape(1).to(torch.int32)


def ref_trimmed(o, kmask, column=False):
  """Zeros where trim gives them (packed_attn.py:132-137)."""
  kmask = torch.as_tensor(kmask)
  _, lim = trim_limits(kmask, 1)
  rows = kmask.any(dim=1)[:, None] & (torch.arange(kmask.shape[1]) < lim)[None, :]
  rows = rows.T if column else rows
  return torch.where(rows[:, :, None, None], o, torch.zeros_like(o))


def ref_packed_attention(p, bias, kmask, gate_bias=None, kv=None, *, sm_scale, column=False, trim=False,
                         dtype=torch.float32):
  """Packed [X,Y,G,H,D] attention, rows or columns, optional gate (packed_attn.py:145-160)."""
  p = _f(p, dtype)
  if kv is not None:  # unsplit_kv, packed_attn.py:140-142
    p = torch.cat([p[:, :, :1], _f(kv, dtype), p[:, :, 1:]], dim=2)
  if column:
    p = p.transpose(0, 1)
  q, k, v = p[:, :, 0], p[:, :, 1], p[:, :, 2]
  logits = torch.einsum("bqhd,bkhd->bhqk", q, k) * sm_scale
  if bias is not None:
    logits = logits + _f(bias, dtype)[None]
  logits = torch.where(torch.as_tensor(kmask)[:, None, None, :], logits, torch.tensor(NEG, dtype=dtype))
  o = torch.einsum("bhqk,bkhd->bqhd", torch.softmax(logits, dim=-1), v)
  if gate_bias is not None:
    o = o * torch.sigmoid(p[:, :, 3] + _f(gate_bias, dtype))
  o = o.transpose(0, 1) if column else o
  return ref_trimmed(o, kmask, column) if trim else o


def attention_via(p, bias, kmask, gate_bias=None, *, sm_scale, column=False, dtype=torch.float32):
  """packed attention through the heads-major attention: the definition of its VJP (packed_attn.py:163-177)."""
  pp = _f(p, dtype)
  pp = pp.transpose(0, 1) if column else pp
  q, k, v = (pp[:, :, i].transpose(1, 2) for i in range(3))
  h, s = q.shape[1], q.shape[2]
  b = torch.zeros(h, s, s, dtype=dtype) if bias is None else _f(bias, dtype)
  o = ref_attn(q, k, v, b, kmask, sm_scale, dtype).transpose(1, 2)
  if gate_bias is not None:
    o = o * torch.sigmoid(pp[:, :, 3] + _f(gate_bias, dtype))
  return o.transpose(0, 1) if column else o


# ---------------------------------------------------------------------------------------------
# LayerNorm / gated dual projection / triangle multiplication
# ---------------------------------------------------------------------------------------------
def ref_ln(xf, scale, offset, eps):
  """fp32 LayerNorm over the last axis, biased variance (transition.py:61-65)."""
  mean = xf.mean(-1, keepdim=True)
  var = ((xf - mean) ** 2).mean(-1, keepdim=True)
  return (xf - mean) * torch.rsqrt(var + eps) * scale + offset


def ref_layer_norm(x, scale, offset, eps=1e-5, dtype=torch.float32):
  """tri_mul.py:515-520 (the result there is cast to x's dtype; here it stays `dtype`)."""
  return ref_ln(_f(x, dtype), _f(scale, dtype), _f(offset, dtype), eps)


def layer_norm_bwd(x, scale, dy, eps=1e-5, dtype=torch.float32):
  """grads.py:25-39 -> (dx, dscale, doffset)."""
  xf, dyf, sc = _f(x, dtype), _f(dy, dtype), _f(scale, dtype)
  mean = xf.mean(-1, keepdim=True)
  d = xf - mean
  rstd = torch.rsqrt((d * d).mean(-1, keepdim=True) + eps)
  xhat = d * rstd
  axes = tuple(range(xf.ndim - 1))
  dscale = (dyf * xhat).sum(axes)
  doffset = dyf.sum(axes)
  dxhat = dyf * sc
  dx = rstd * (dxhat - dxhat.mean(-1, keepdim=True) - xhat * (dxhat * xhat).mean(-1, keepdim=True))
  return dx, dscale, doffset


def _act(name):
  return {"sigmoid": torch.sigmoid, "swish": torch.nn.functional.silu}[name]


def ref_gdp(x, wp, bp, wg, bg, mask, activation="sigmoid", dtype=torch.float32):
  """mask * (x wp + bp) * act(x wg + bg) (tri_mul.py:454-457)."""
  x, wp, bp, wg, bg, mask = (_f(t, dtype) for t in (x, wp, bp, wg, bg, mask))
  return mask[:, None] * (x @ wp + bp) * _act(activation)(x @ wg + bg)


def gdp_bwd(x, wp, bp, wg, bg, mask, dy, activation="sigmoid", dtype=torch.float32):
  """grads.py:68-91 -> (dx, dwp, dbp, dwg, dbg, dmask); dy is the [M,P] cotangent."""
  x, wp, bp, wg, bg, mask, dy = (_f(t, dtype) for t in (x, wp, bp, wg, bg, mask, dy))
  proj = x @ wp + bp
  gate = (x @ wg + bg).detach().requires_grad_(True)
  act = _act(activation)(gate)
  m = mask[:, None]
  dproj = dy * m * act.detach()
  dgate, = torch.autograd.grad(act, gate, dy * m * proj)
  dx = dproj @ wp.T + dgate @ wg.T
  dmask = (dy * proj * act.detach()).sum(-1)
  return dx, x.T @ dproj, dproj.sum(0), x.T @ dgate, dgate.sum(0), dmask


def ref_ln_gdp(x, ln_scale, ln_offset, wp, bp, wg, bg, mask, *, eps=1e-5, transpose=False, pad=1,
               dtype=torch.float32):
  """LN then split channel-major GDP; pair form [A,B,K] with transpose/pad (tri_mul.py:286-300).
  A negative mask counts as zero (tri_mul.py:80)."""
  x, mask = _f(x, dtype), torch.clamp(_f(mask, dtype), min=0)
  pair = None
  if x.ndim == 3:
    if transpose:
      x, mask = x.transpose(0, 1), mask.T
    pair = x.shape[:2]
    x, mask = x.reshape(-1, x.shape[-1]), mask.reshape(-1)
  y = ref_gdp(ref_ln(x, _f(ln_scale, dtype), _f(ln_offset, dtype), eps), wp, bp, wg, bg, mask, dtype=dtype)
  ci = wp.shape[1] // 2
  left, right = y[:, :ci].T, y[:, ci:].T
  if pair is None:
    return left, right
  rows = -(-pair[1] // pad) * pad
  shape = lambda h: torch.nn.functional.pad(h.reshape(ci, *pair), (0, rows - pair[1]))
  return shape(left), shape(right)


def ref_trimul_epilogue(x_cm, act, ln_scale, ln_offset, wo, bo, wg, bg, residual=None, *, eps=1e-5,
                        dtype=torch.float32):
  """(LN(x_cm^T) wo + bo) * sigmoid(act wg + bg) (+ residual) (tri_mul.py:446-451)."""
  y = ref_ln(_f(x_cm, dtype).T, _f(ln_scale, dtype), _f(ln_offset, dtype), eps)
  out = y @ _f(wo, dtype) + _f(bo, dtype)
  out = out * torch.sigmoid(_f(act, dtype) @ _f(wg, dtype) + _f(bg, dtype))
  return out if residual is None else out + _f(residual, dtype)


def ref_trimul_epilogue_ln(x_cm, x, in_scale, in_offset, ln_scale, ln_offset, wo, bo, wg, bg, keep=None, *,
                           eps=1e-5, add_input=False, dtype=torch.float32):
  """The gate input recomputed as LN(x) (tri_mul.py:441-444)."""
  act = ref_ln(_f(x, dtype), _f(in_scale, dtype), _f(in_offset, dtype), eps)
  return ref_trimul_epilogue(x_cm, act, ln_scale, ln_offset, wo, bo, wg, bg, x if add_input else None, eps=eps,
                             dtype=dtype)


def ref_contract(a, b, dtype=torch.float32):
  """out[c,i,j] = sum_k a[c,i,k] b[c,j,k] (contract.py:1-4,56-57; the bf16 form is XLA's batched GEMM)."""
  return torch.einsum("cik,cjk->cij", _f(a, dtype), _f(b, dtype))


ref_fp8_contract = ref_contract  # operands arrive already rounded to e4m3 (contract.py:56-57)


# ---------------------------------------------------------------------------------------------
# projections around attention, outer product mean, transition
# ---------------------------------------------------------------------------------------------
def ref_ln_projection(x, ln_scale, ln_offset, w=None, wb=None, keep=None, *, eps=1e-5, f8_slots=(),
                      f8_scales=None, dtype=torch.float32):
  """packed_attn.py:308-318 -> (p [M, G*n], bias [h, M]) (+ the e4m3 slots scaled, before rounding)."""
  y = ref_ln(_f(x, dtype), _f(ln_scale, dtype), _f(ln_offset, dtype), eps)
  b = None if wb is None else (y @ _f(wb, dtype)).T
  if w is None:
    return None, b
  p = torch.einsum("ma,gan->mgn", y, _f(w, dtype))
  half = [g for g in range(w.shape[0]) if g not in f8_slots]
  flat = lambda gs: p[:, list(gs)].reshape(x.shape[0], -1)
  if f8_slots:
    scale = torch.repeat_interleave(torch.tensor(f8_scales or (1.0,) * len(f8_slots), dtype=dtype), w.shape[2])
    return flat(half), b, flat(f8_slots) * scale
  return flat(half), b


def ref_output_projection(o, w, b, residual=None, keep=None, dtype=torch.float32):
  """packed_attn.py:387-389."""
  out = _f(o, dtype) @ _f(w, dtype) + _f(b, dtype)
  return out if residual is None else out + _f(residual, dtype)


def ref_opm_projection(x, ln_scale, ln_offset, lw, lb, rw, rb, mask, *, eps=1e-5, dtype=torch.float32):
  """opm.py:62-66."""
  y = ref_ln(_f(x, dtype), _f(ln_scale, dtype), _f(ln_offset, dtype), eps)
  mv = _f(mask, dtype)[..., None]
  return mv * (y @ _f(lw, dtype) + _f(lb, dtype)), mv * (y @ _f(rw, dtype) + _f(rb, dtype))


def ref_opm_update(lhs, t, bias, norm, residual=None, *, eps=1e-3, dtype=torch.float32):
  """opm.py:116-119."""
  out = torch.einsum("bk,kdf->bdf", _f(lhs, dtype), _f(t, dtype)) + _f(bias, dtype)
  out = out / (eps + _f(norm, dtype))[..., None]
  return out if residual is None else out + _f(residual, dtype)


def ref_opm_outer(left, right, w, dtype=torch.float32):
  """opm.py:165-168: act[b,(c,e),d] = sum_a left[a,b,c] right[a,d,e]; out[b,d,f] = sum_k act[b,k,d] w[k,f]."""
  act = torch.einsum("abc,ade->bced", _f(left, dtype), _f(right, dtype))
  act = act.reshape(act.shape[0], -1, act.shape[-1])
  return torch.einsum("bkd,kf->bdf", act, _f(w, dtype))


def ref_opm_deep(left, right, mask, w, bias, residual=None, *, eps=1e-3, dtype=torch.float32):
  """Deep-MSA outer product mean as ColabFold composes it from the pieces above (not a reference
  function: parity unpinned): left/right [s,r,c] already masked, out[i,j,:] = (outer . w + bias) /
  (eps + sum_s mask[s,i] mask[s,j]) (+ residual)."""
  out = ref_opm_outer(left, right, w, dtype) + _f(bias, dtype)
  m = _f(mask, dtype)
  out = out / (eps + m.T @ m)[..., None]
  return out if residual is None else out + _f(residual, dtype)


def ref_transition(x, ln_scale, ln_offset, w1, b1, w2, b2, keep=None, *, eps=1e-5, add_input=False,
                   dtype=torch.float32):
  """relu(LN(x) w1 + b1) w2 + b2 (+ x) (transition.py:141-146)."""
  xf = _f(x, dtype)
  y = ref_ln(xf, _f(ln_scale, dtype), _f(ln_offset, dtype), eps)
  h = torch.relu(y @ _f(w1, dtype) + _f(b1, dtype))
  out = h @ _f(w2, dtype) + _f(b2, dtype)
  return out + xf if add_input else out


# ---------------------------------------------------------------------------------------------
# error metrics and a generic VJP helper
# ---------------------------------------------------------------------------------------------
def rel_err(a, b):
  """max|a-b| / max(max|b|, 1e-3) (tests/test_pallas_vjp.py:19-22); inf when a is not finite."""
  a = torch.as_tensor(a).detach().double().cpu()
  b = torch.as_tensor(b).detach().double().cpu()
  if not torch.isfinite(a).all():
    return float("inf")
  if a.numel() == 0:
    return 0.0
  return float((a - b).abs().max() / max(float(b.abs().max()), 1e-3))


def rms_err(a, b):
  """Relative RMS error (tests/test_ln_fusions.py:141-143)."""
  a = torch.as_tensor(a).detach().double().cpu()
  b = torch.as_tensor(b).detach().double().cpu()
  return float(torch.sqrt(((a - b) ** 2).mean()) / torch.sqrt((b ** 2).mean()).clamp_min(1e-30))


def vjp(fn, args, diff, cotangent, dtype=torch.float32):
  """Gradients of <fn(*args), cotangent> w.r.t. args[i] for i in diff, by autograd through the
  reference math: what grads.py:106-143 `differentiable_via` defines as each fused op's backward."""
  leaves = {i: _f(args[i], dtype).detach().clone().requires_grad_(True) for i in diff}
  full = [leaves.get(i, a) for i, a in enumerate(args)]
  out = fn(*full)
  outs = out if isinstance(out, (tuple, list)) else (out,)
  cots = cotangent if isinstance(cotangent, (tuple, list)) else (cotangent,)
  loss = sum((o * _f(c, dtype)).sum() for o, c in zip(outs, cots) if o is not None)
  return torch.autograd.grad(loss, [leaves[i] for i in diff])

"""Gradients THROUGH THE SELECTORS on the GPU against the VJP of the CPU oracle: for every fused op the reference
checks forward and the gradient of <out, cotangent> (tests/test_af2_fused_kernels.py:22-37,
tests/test_ln_gdp_grad.py:55-80, tests/test_fused_ops_grad.py:18-49).  Shapes are the reference's own lists
restricted to the widths this build takes.  bf16 bound 2e-2 (max-abs error over max-abs reference)."""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu
TOL = 2e-2
bf = torch.bfloat16


def cfg(**kw):
  from colabfold_kernels import dispatch
  return {**dispatch(), **kw}


def rnd(rng, *shape, s=.5, dtype=bf):
  return torch.from_numpy((rng.standard_normal(shape) * s).astype(np.float32)).to(dtype)


def run_vjp(fn, ref, args, diff, tol=TOL, cot_scale=.5, seed=99):
  """fn on CUDA copies of args with requires_grad on args[diff]; forward and every gradient against the oracle."""
  dev = [a.cuda() if torch.is_tensor(a) else a for a in args]
  for i in diff:
    dev[i] = dev[i].detach().requires_grad_(True)
  out = fn(*dev)
  outs = out if isinstance(out, (tuple, list)) else (out,)
  rout = ref(*args)
  routs = rout if isinstance(rout, (tuple, list)) else (rout,)
  rng = np.random.default_rng(seed)
  cots = [rnd(rng, *o.shape, s=cot_scale, dtype=o.dtype) for o in outs]
  errs = {}
  for k, (o, r) in enumerate(zip(outs, routs)):
    errs[f"out{k}"] = O.rel_err(o.detach().cpu().float(), r)
  loss = sum((o.float() * c.cuda().float()).sum() for o, c in zip(outs, cots))
  grads = torch.autograd.grad(loss, [dev[i] for i in diff], allow_unused=True)
  rgrads = O.vjp(ref, list(args), list(diff), [c.float() for c in cots])
  for i, g, rg in zip(diff, grads, rgrads):
    assert g is not None, f"no gradient for argument {i}"
    assert g.dtype == dev[i].dtype and g.shape == dev[i].shape
    errs[f"d{i}"] = O.rel_err(g.cpu().float(), rg)
  bad = {k: v for k, v in errs.items() if not v <= tol}
  assert not bad, (bad, errs)
  from colabfold_kernels import ops
  assert ops.device_status() == 0
  return errs


# ---- gated dual projection: tests/test_ln_gdp_grad.py:55-80 -------------------------------------------------------
@pytest.mark.parametrize("m,k,p,split,cm", [(2048, 128, 256, False, False), (2048, 128, 256, True, False),
                                            (2048, 128, 256, True, True), (999, 64, 128, True, True)])
@pytest.mark.parametrize("act", ["sigmoid", "swish"])
def test_gated_dual_proj_vjp(m, k, p, split, cm, act):
  from colabfold_kernels import fused_ops
  gdp = fused_ops.gated_dual_proj(cfg(), bf, act)
  assert gdp is not None
  rng = np.random.default_rng(0)
  x, wp, bp, wg, bg = rnd(rng, m, k), rnd(rng, k, p, s=k ** -.5), rnd(rng, p, s=.1), rnd(rng, k, p, s=k ** -.5), rnd(rng, p, s=.1)
  mask = torch.from_numpy((rng.random(m) > .1).astype(np.float32)).to(bf)

  def fn(x, wp, bp, wg, bg):
    return gdp(x, wp, bp, wg, bg, mask.cuda(), split=split, channel_major=cm)

  def ref(x, wp, bp, wg, bg):
    y = O.ref_gdp(x, wp, bp, wg, bg, mask, activation=act)
    if not split:
      return y
    l, r = y[:, :p // 2], y[:, p // 2:]
    return (l.T, r.T) if cm else (l, r)

  run_vjp(fn, ref, (x, wp, bp, wg, bg), [0, 1, 2, 3, 4])


# ---- packed attention: tests/test_af2_fused_kernels.py:44-62 (head dim 32 runs the tensor-core kernels, the others
# the fp32-math kernels behind the same selector) ---------------------------------------------------------------------
PACKED = [(64, 96, 4, 32, True, False), (96, 64, 4, 32, True, True), (37, 53, 8, 8, True, False),
          (50, 50, 4, 32, False, True), (40, 24, 8, 8, True, True), (33, 48, 4, 16, True, True), (5, 1, 4, 32, True, False),
          (7, 136, 4, 32, True, False), (136, 5, 2, 64, False, True), (10, 40, 8, 16, True, False), (40, 6, 4, 16, True, True)]


@pytest.mark.parametrize("x,y,h,d,gated,column", PACKED)
@pytest.mark.parametrize("with_bias", [True, False])
def test_packed_attention_vjp(x, y, h, d, gated, column, with_bias):
  from colabfold_kernels import fused_ops
  if not with_bias and (x, y) not in ((96, 64), (50, 50)):
    pytest.skip("the reference runs the no-bias form on two shapes")
  pa = fused_ops.packed_attention(cfg(), bf, d, d)
  assert pa is not None
  rng = np.random.default_rng(1)
  g = 4 if gated else 3
  nb, s = (y, x) if column else (x, y)
  p, bias = rnd(rng, x, y, g, h, d), rnd(rng, h, s, s)
  kmask = torch.from_numpy(rng.random((nb, s)) > .1)
  kmask[nb // 2] = False  # a fully masked (padding) row
  gb = rnd(rng, h, d) if gated else None
  scale = d ** -.5
  if with_bias and gated:
    fn = lambda p, b, gb: pa(p, b, kmask.cuda(), gb, sm_scale=scale, column=column)
    ref = lambda p, b, gb: O.ref_packed_attention(p, b, kmask, gb, sm_scale=scale, column=column)
    args = (p, bias, gb)
  elif with_bias:
    fn = lambda p, b: pa(p, b, kmask.cuda(), None, sm_scale=scale, column=column)
    ref = lambda p, b: O.ref_packed_attention(p, b, kmask, None, sm_scale=scale, column=column)
    args = (p, bias)
  elif gated:
    fn = lambda p, gb: pa(p, None, kmask.cuda(), gb, sm_scale=scale, column=column)
    ref = lambda p, gb: O.ref_packed_attention(p, None, kmask, gb, sm_scale=scale, column=column)
    args = (p, gb)
  else:
    fn = lambda p: pa(p, None, kmask.cuda(), None, sm_scale=scale, column=column)
    ref = lambda p: O.ref_packed_attention(p, None, kmask, None, sm_scale=scale, column=column)
    args = (p,)
  run_vjp(fn, ref, args, list(range(len(args))))


@pytest.mark.parametrize("column", [False, True])
def test_packed_attention_trim_vjp(column):
  """trim_padding: rows without a live key and queries past the last live key give zeros and carry no gradient
  (packed_attn.py:132-137,163-177)."""
  from colabfold_kernels import fused_ops
  pa = fused_ops.packed_attention(cfg(trim_padding=True), bf, 32, 32)
  rng = np.random.default_rng(2)
  x, y, h, d = 48, 72, 4, 32
  nb, s = (y, x) if column else (x, y)
  p, bias, gb = rnd(rng, x, y, 4, h, d), rnd(rng, h, s, s), rnd(rng, h, d)
  kmask = torch.from_numpy(rng.random((nb, s)) > .1)
  kmask[:, s - 9:] = False   # trailing padding
  kmask[nb // 3] = False     # a padding row
  scale = d ** -.5
  fn = lambda p, b, gb: pa(p, b, kmask.cuda(), gb, sm_scale=scale, column=column)
  ref = lambda p, b, gb: O.ref_packed_attention(p, b, kmask, gb, sm_scale=scale, column=column, trim=True)
  run_vjp(fn, ref, (p, bias, gb), [0, 1, 2])


# ---- attention through its selector: tests/test_fused_ops_grad.py:18-49 -----------------------------------------
@pytest.mark.parametrize("layout", ["heads", "seq"])
def test_attention_selector_vjp(layout):
  from colabfold_kernels import fused_ops
  b, h, s, c = 2, 4, 96, 32
  kernel = fused_ops.attention(cfg(), bf, c, c, layout)
  rng = np.random.default_rng(3)
  shape = (b, h, s, c) if layout == "heads" else (b, s, h, c)
  q, k, v, bias = rnd(rng, *shape), rnd(rng, *shape), rnd(rng, *shape), rnd(rng, h, s, s)
  live = torch.from_numpy(rng.random((b, s)) > .15)
  mask_bias = ((~live).float() * -1e9).reshape(b, 1, 1, s)
  fn = lambda q, k, v, bias: kernel(q, k, v, mask_bias.cuda().to(bf), bias, c ** -.5)
  ref = lambda q, k, v, bias: O.ref_attention(q, k, v, mask_bias, bias, c ** -.5, layout=layout)
  run_vjp(fn, ref, (q, k, v, bias), [0, 1, 2, 3])


# ---- every differentiable_via selector ------------------------------------------------------------------------------
@pytest.mark.parametrize("m", [59, 4101])
def test_ln_gated_dual_proj_vjp(m):
  from colabfold_kernels import fused_ops
  k, p = 128, 256
  sel = fused_ops.ln_gated_dual_proj(cfg(), bf, k, p // 2)
  rng = np.random.default_rng(4)
  x, wp, bp, wg, bg = rnd(rng, m, k), rnd(rng, k, p, s=k ** -.5), rnd(rng, p, s=.1), rnd(rng, k, p, s=k ** -.5), rnd(rng, p, s=.1)
  sc, of = 1 + rnd(rng, k, s=.1, dtype=torch.float32), rnd(rng, k, s=.1, dtype=torch.float32)
  mask = torch.from_numpy((rng.random(m) > .1).astype(np.float32)).to(bf)
  fn = lambda x, sc, of, wp, bp, wg, bg: sel(x, sc, of, wp, bp, wg, bg, mask.cuda(), eps=1e-5)
  ref = lambda x, sc, of, wp, bp, wg, bg: O.ref_ln_gdp(x, sc, of, wp, bp, wg, bg, mask)
  run_vjp(fn, ref, (x, sc, of, wp, bp, wg, bg), list(range(7)))


@pytest.mark.parametrize("transpose", [False, True])
def test_ln_gated_dual_proj_pair_vjp(transpose):
  from colabfold_kernels import fused_ops
  a, b, k, p = 40, 72, 128, 256
  sel = fused_ops.ln_gated_dual_proj(cfg(), bf, k, p // 2)
  rng = np.random.default_rng(5)
  x, wp, bp, wg, bg = rnd(rng, a, b, k), rnd(rng, k, p, s=k ** -.5), rnd(rng, p, s=.1), rnd(rng, k, p, s=k ** -.5), rnd(rng, p, s=.1)
  sc, of = 1 + rnd(rng, k, s=.1, dtype=torch.float32), rnd(rng, k, s=.1, dtype=torch.float32)
  mask = torch.from_numpy((rng.random((a, b)) > .1).astype(np.float32)).to(bf)
  fn = lambda x, wp, wg: sel(x, sc.cuda(), of.cuda(), wp, bp.cuda(), wg, bg.cuda(), mask.cuda(), eps=1e-5, transpose=transpose)
  ref = lambda x, wp, wg: O.ref_ln_gdp(x, sc, of, wp, bp, wg, bg, mask, transpose=transpose)
  run_vjp(fn, ref, (x, wp, wg), [0, 1, 2])


@pytest.mark.parametrize("m,add_input", [(999, False), (4096, True)])
def test_trimul_epilogue_ln_vjp(m, add_input):
  from colabfold_kernels import fused_ops
  c = 128
  sel = fused_ops.trimul_epilogue_ln(cfg(), bf)
  rng = np.random.default_rng(6)
  x_cm, x = rnd(rng, c, m), rnd(rng, m, c)
  isc, iof = 1 + rnd(rng, c, s=.1, dtype=torch.float32), rnd(rng, c, s=.1, dtype=torch.float32)
  sc, of = 1 + rnd(rng, c, s=.1, dtype=torch.float32), rnd(rng, c, s=.1, dtype=torch.float32)
  wo, bo, wg, bg = rnd(rng, c, c, s=c ** -.5), rnd(rng, c, s=.1), rnd(rng, c, c, s=c ** -.5), rnd(rng, c, s=.1)
  fn = lambda *a: sel(*a, eps=1e-5, add_input=add_input)
  ref = lambda *a: O.ref_trimul_epilogue_ln(*a, add_input=add_input)
  run_vjp(fn, ref, (x_cm, x, isc, iof, sc, of, wo, bo, wg, bg), list(range(10)))


@pytest.mark.parametrize("m", [999])
def test_trimul_epilogue_vjp(m):
  from colabfold_kernels import fused_ops
  c = 128
  sel = fused_ops.trimul_epilogue(cfg(), bf)
  rng = np.random.default_rng(7)
  x_cm, act, res = rnd(rng, c, m), rnd(rng, m, c), rnd(rng, m, c)
  sc, of = 1 + rnd(rng, c, s=.1, dtype=torch.float32), rnd(rng, c, s=.1, dtype=torch.float32)
  wo, bo, wg, bg = rnd(rng, c, c, s=c ** -.5), rnd(rng, c, s=.1), rnd(rng, c, c, s=c ** -.5), rnd(rng, c, s=.1)
  run_vjp(lambda *a: sel(*a), O.ref_trimul_epilogue, (x_cm, act, sc, of, wo, bo, wg, bg, res), list(range(9)))


@pytest.mark.parametrize("m,a,g,n,h", [(4101, 128, 4, 128, 4), (59, 64, 4, 64, 4)])
def test_ln_projection_vjp(m, a, g, n, h):
  from colabfold_kernels import fused_ops
  sel = fused_ops.ln_projection(cfg(), bf, a, n)
  rng = np.random.default_rng(8)
  x, w, wb = rnd(rng, m, a), rnd(rng, g, a, n, s=a ** -.5), rnd(rng, a, h, s=a ** -.5)
  sc, of = 1 + rnd(rng, a, s=.1, dtype=torch.float32), rnd(rng, a, s=.1, dtype=torch.float32)
  run_vjp(lambda *t: sel(*t, eps=1e-5), lambda *t: O.ref_ln_projection(*t), (x, sc, of, w, wb), list(range(5)))


@pytest.mark.parametrize("m,k,c", [(4101, 128, 128), (59, 64, 64)])
def test_output_projection_vjp(m, k, c):
  from colabfold_kernels import fused_ops
  sel = fused_ops.output_projection(cfg(), bf, k, c)
  rng = np.random.default_rng(9)
  o, w, b, res = rnd(rng, m, k), rnd(rng, k, c, s=k ** -.5), rnd(rng, c, s=.1), rnd(rng, m, c)
  run_vjp(lambda *t: sel(*t), O.ref_output_projection, (o, w, b, res), [0, 1, 2, 3])


def test_opm_projection_vjp():
  from colabfold_kernels import fused_ops
  s, r, c, k = 24, 50, 256, 32
  sel = fused_ops.opm_projection(cfg(), bf, c, k)
  rng = np.random.default_rng(10)
  x = rnd(rng, s, r, c)
  sc, of = 1 + rnd(rng, c, s=.1, dtype=torch.float32), rnd(rng, c, s=.1, dtype=torch.float32)
  lw, lb, rw, rb = rnd(rng, c, k, s=c ** -.5), rnd(rng, k, s=.1), rnd(rng, c, k, s=c ** -.5), rnd(rng, k, s=.1)
  mask = torch.from_numpy((rng.random((s, r)) > .1).astype(np.float32)).to(bf)
  fn = lambda x, sc, of, lw, lb, rw, rb: sel(x, sc, of, lw, lb, rw, rb, mask.cuda(), eps=1e-5)
  ref = lambda x, sc, of, lw, lb, rw, rb: O.ref_opm_projection(x, sc, of, lw, lb, rw, rb, mask)
  run_vjp(fn, ref, (x, sc, of, lw, lb, rw, rb), list(range(7)))


def test_opm_update_vjp():
  from colabfold_kernels import fused_ops
  bdim, k, ddim, f = 40, 64, 24, 128
  sel = fused_ops.opm_update(cfg(), bf, k, f)
  rng = np.random.default_rng(11)
  lhs, t, bias, res = rnd(rng, bdim, k), rnd(rng, k, ddim, f, s=k ** -.5), rnd(rng, f, s=.1), rnd(rng, bdim, ddim, f)
  norm = torch.from_numpy(rng.integers(1, 9, (bdim, ddim)).astype(np.float32))
  fn = lambda lhs, t, bias, res: sel(lhs, t, bias, norm.cuda(), res, eps=1e-3)
  ref = lambda lhs, t, bias, res: O.ref_opm_update(lhs, t, bias, norm, res)
  run_vjp(fn, ref, (lhs, t, bias, res), [0, 1, 2, 3])


@pytest.mark.parametrize("m,c,hd,add_input", [(4096, 128, 512, True), (777, 64, 256, False), (1000, 256, 1024, True)])
def test_transition_vjp(m, c, hd, add_input):
  from colabfold_kernels import fused_ops
  sel = fused_ops.transition(cfg(), bf, c, hd)
  rng = np.random.default_rng(12)
  x, w1, b1, w2, b2 = rnd(rng, m, c), rnd(rng, c, hd, s=c ** -.5), rnd(rng, hd, s=.1), rnd(rng, hd, c, s=hd ** -.5), rnd(rng, c, s=.1)
  sc, of = 1 + rnd(rng, c, s=.1, dtype=torch.float32), rnd(rng, c, s=.1, dtype=torch.float32)
  fn = lambda *a: sel(*a, eps=1e-5, add_input=add_input)
  ref = lambda *a: O.ref_transition(*a, add_input=add_input)
  run_vjp(fn, ref, (x, sc, of, w1, b1, w2, b2), list(range(7)))


def test_layer_norm_selector_vjp():
  from colabfold_kernels import fused_ops
  sel = fused_ops.layer_norm(cfg(), bf)
  rng = np.random.default_rng(13)
  m, c = 777, 64
  x = rnd(rng, m, c)
  sc, of = 1 + rnd(rng, c, s=.1, dtype=torch.float32), rnd(rng, c, s=.1, dtype=torch.float32)
  run_vjp(lambda *a: sel(*a, eps=1e-5), lambda *a: O.ref_layer_norm(*a), (x, sc, of), [0, 1, 2])


def test_bounded_wait_reports_and_blocks_until_cleared():
  """A wait nobody answers gives up within its limit, leaves its code in the status word, and from then on every entry
  answers CFK_ERR_DEVICE_WAIT until the word has been read and cleared; nothing traps, nothing spins on."""
  from colabfold_kernels import _lib, ops
  lib = _lib.load()
  assert ops.device_status() == 0
  stream = torch.cuda.current_stream().cuda_stream
  rc = lib.cfk_debug_wait_timeout(1 << 16, 4242, stream)
  assert rc == 0
  torch.cuda.synchronize()
  x = torch.randn(64, 128, device="cuda", dtype=bf)
  one = torch.ones(128, device="cuda")
  with pytest.raises(_lib.CfkError) as e:
    ops.layer_norm(x, one, one)
  assert e.value.code == -9
  assert ops.device_status(reset=True) == 4242
  assert ops.device_status() == 0
  ops.layer_norm(x, one, one)  # clean again
  torch.cuda.synchronize()

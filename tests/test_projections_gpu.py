"""The projection family on the GPU (row-block tcgen05 GEMM engine) against the CPU oracle: shapes and
tolerances of tests/test_ln_gdp_grad.py:58-59,75, tests/test_ln_fusions.py:38,127-138 and
tests/test_af2_fused_kernels.py:90-91 restricted to the widths this build takes (K in {64,128,256})."""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu
TOL = 2e-2  # bf16 bound of this build (the reference's own bound for these ops is 3e-2, tests/test_af2_fused_kernels.py:22)
bf = torch.bfloat16


def rnd(rng, *shape, s=.5):
  return torch.from_numpy((rng.standard_normal(shape) * s).astype(np.float32)).to(bf)


def chk(got, ref, tol=TOL):
  err = O.rel_err(got.cpu().float(), ref)
  assert err <= tol, err


@pytest.mark.parametrize("m,k,p,split,cm", [(2048, 128, 256, False, False), (2048, 128, 256, True, False),
                                            (2048, 128, 256, True, True), (999, 64, 128, True, True), (1, 128, 256, False, False),
                                            (300, 256, 128, True, False)])
@pytest.mark.parametrize("act", [0, 1])
def test_gated_dual_proj(m, k, p, split, cm, act):
  from colabfold_kernels import ops
  rng = np.random.default_rng(0)
  x, wp, bp, wg, bg = rnd(rng, m, k), rnd(rng, k, p, s=k ** -.5), rnd(rng, p, s=.1), rnd(rng, k, p, s=k ** -.5), rnd(rng, p, s=.1)
  mask = torch.from_numpy((rng.random(m) > .1).astype(np.float32)).to(bf)
  ref = O.ref_gdp(x, wp, bp, wg, bg, mask, activation="swish" if act else "sigmoid")
  out = ops.gated_dual_proj(x.cuda(), wp.cuda(), bp.cuda(), wg.cuda(), bg.cuda(), mask.cuda(), split=split,
                            channel_major=cm, activation=act)
  assert ops.device_status() == 0
  if not split:
    chk(out, ref)
  else:
    l, r = ref[:, :p // 2], ref[:, p // 2:]
    chk(out[0], l.T if cm else l)
    chk(out[1], r.T if cm else r)


@pytest.mark.parametrize("m", [1, 59, 4101, 260 * 260])
def test_ln_gdp_2d_and_fused_equals_unfused(m):
  from colabfold_kernels import ops
  rng = np.random.default_rng(1)
  k, p = 128, 256
  x, wp, bp, wg, bg = rnd(rng, m, k), rnd(rng, k, p, s=k ** -.5), rnd(rng, p, s=.1), rnd(rng, k, p, s=k ** -.5), rnd(rng, p, s=.1)
  sc = 1 + rnd(rng, k, s=.1).float()
  of = rnd(rng, k, s=.1).float()
  mask = torch.from_numpy((rng.random(m) > .1).astype(np.float32)).to(bf)
  l, r = ops.ln_gated_dual_proj(x.cuda(), sc.cuda(), of.cuda(), wp.cuda(), bp.cuda(), wg.cuda(), bg.cuda(), mask.cuda())
  assert ops.device_status() == 0
  rl, rr = O.ref_ln_gdp(x, sc, of, wp, bp, wg, bg, mask)
  chk(l, rl); chk(r, rr)
  # fused == LayerNorm kernel followed by the gated dual projection kernel (tests/test_ln_fusions.py:127-138)
  y = ops.layer_norm(x.cuda(), sc.cuda(), of.cuda())
  ul, ur = ops.gated_dual_proj(y, wp.cuda(), bp.cuda(), wg.cuda(), bg.cuda(), mask.cuda(), split=True, channel_major=True)
  assert O.rel_err(l.cpu().float(), ul.cpu().float()) <= 1e-2


@pytest.mark.parametrize("transpose", [False, True])
@pytest.mark.parametrize("fp8", [False, True])
def test_ln_gdp_pair(transpose, fp8):
  from colabfold_kernels import ops
  rng = np.random.default_rng(2)
  a, b, k, p = 70, 150, 128, 256
  x, wp, bp, wg, bg = rnd(rng, a, b, k), rnd(rng, k, p, s=k ** -.5), rnd(rng, p, s=.1), rnd(rng, k, p, s=k ** -.5), rnd(rng, p, s=.1)
  sc, of = 1 + rnd(rng, k, s=.1).float(), rnd(rng, k, s=.1).float()
  mask = torch.from_numpy((rng.random((a, b)) > .1).astype(np.float32)).to(bf)
  mask[3, :100] = -1  # negative mask values count as zero (a 128-row tile that is negative throughout is left unwritten:
  # tests/test_padding_skip_gpu.py)
  l, r = ops.ln_gated_dual_proj(x.cuda(), sc.cuda(), of.cuda(), wp.cuda(), bp.cuda(), wg.cuda(), bg.cuda(), mask.cuda(),
                                transpose=transpose, pad=16, fp8=fp8)
  assert ops.device_status() == 0
  rl, rr = O.ref_ln_gdp(x, sc, of, wp, bp, wg, bg, mask, transpose=transpose, pad=16)
  assert tuple(l.shape) == tuple(rl.shape)
  if fp8:
    assert O.rms_err(l.cpu().float(), rl) <= 5e-2 and O.rms_err(r.cpu().float(), rr) <= 5e-2
  else:
    chk(l, rl); chk(r, rr)
  # the zero padding of the contracted axis is exact
  inner = a if transpose else b
  assert float(l.cpu().float()[..., inner:].abs().max()) == 0.0


def test_ln_gdp_rows_far_from_zero_mean():
  """The 128-channel kernel multiplies the raw rows and adds the LayerNorm correction (-mean s + std t) as one more K
  step (split bf16 heads and remainders): rows whose mean is many standard deviations from zero must come out as the
  reference's normalise-then-multiply (tri_mul.py:222-300)."""
  from colabfold_kernels import ops
  rng = np.random.default_rng(42)
  a, b, k, p = 40, 200, 128, 256
  x = (rnd(rng, a, b, k).float() + torch.linspace(-24, 24, a * b).reshape(a, b, 1)).to(bf)
  wp, bp, wg, bg = rnd(rng, k, p, s=k ** -.5), rnd(rng, p, s=.1), rnd(rng, k, p, s=k ** -.5), rnd(rng, p, s=.1)
  sc, of = 1 + rnd(rng, k, s=.1).float(), rnd(rng, k, s=.1).float()
  mask = torch.ones(a, b, dtype=bf)
  for transpose in (False, True):
    l, r = ops.ln_gated_dual_proj(x.cuda(), sc.cuda(), of.cuda(), wp.cuda(), bp.cuda(), wg.cuda(), bg.cuda(), mask.cuda(),
                                  transpose=transpose, pad=16)
    assert ops.device_status() == 0
    rl, rr = O.ref_ln_gdp(x, sc, of, wp, bp, wg, bg, mask, transpose=transpose, pad=16)
    chk(l, rl); chk(r, rr)


def test_ln_gdp_e4m3_per_tensor_scale():
  """A projection whose values sit below e4m3's normal range (weights scaled by 2^-7): unscaled, the cast flushes
  most of them (large error); with a per-tensor scale of 2^7 before rounding and alpha = 2^-14 on the contraction the
  product meets the e4m3 bound.  Through ops and through the fp8_contraction selector."""
  from colabfold_kernels import dispatch, fused_ops, ops
  rng = np.random.default_rng(21)
  n, k, p = 128, 128, 256
  x = rnd(rng, n, n, k)
  wp, bp = rnd(rng, k, p, s=k ** -.5) * 2 ** -7, torch.zeros(p, dtype=bf)
  wg, bg = rnd(rng, k, p, s=k ** -.5), rnd(rng, p, s=.1)
  sc, of = 1 + rnd(rng, k, s=.1).float(), rnd(rng, k, s=.1).float()
  mask = torch.ones(n, n, dtype=bf)
  rl, rr = O.ref_ln_gdp(x, sc, of, wp, bp, wg, bg, mask, pad=16)
  ref = O.ref_contract(rl, rr)
  dev = [t.cuda() for t in (x, sc, of, wp, bp, wg, bg, mask)]
  errs = {}
  for scale in (1.0, 128.0):
    l, r = ops.ln_gated_dual_proj(*dev, pad=16, fp8=True, fp8_scale=scale)
    assert l.dtype == torch.float8_e4m3fn
    errs[scale] = O.rel_err(ops.contract(l, r, alpha=1.0 / scale ** 2).cpu().float(), ref)
  assert errs[128.0] <= 6e-2 < errs[1.0], errs
  sel = fused_ops.fp8_contraction({**dispatch(), "fp8": True, "fp8_scale": 128.0}, bf, k, p // 2, n)
  assert sel is not None
  proj, contract = sel
  l, r = proj(*dev, eps=1e-5)
  assert O.rel_err(contract(l, r).cpu().float(), ref) <= 6e-2
  with pytest.raises(ValueError):
    ops.ln_gated_dual_proj(*dev, pad=16, fp8=True, fp8_scale=0.0)
  assert ops.device_status() == 0


@pytest.mark.parametrize("m,c,xdt", [(4096, 128, bf), (999, 128, bf), (500, 64, bf), (1, 128, bf), (127, 128, bf),
                                     (999, 128, torch.float32)])
def test_trimul_epilogue(m, c, xdt):
  from colabfold_kernels import ops
  rng = np.random.default_rng(3)
  x_cm, act = rnd(rng, c, m).to(xdt), rnd(rng, m, c)
  sc, of = 1 + rnd(rng, c, s=.1).float(), rnd(rng, c, s=.1).float()
  wo, bo, wg, bg = rnd(rng, c, c, s=c ** -.5), rnd(rng, c, s=.1), rnd(rng, c, c, s=c ** -.5), rnd(rng, c, s=.1)
  res = rnd(rng, m, c)
  args = (x_cm.cuda(), act.cuda(), sc.cuda(), of.cuda(), wo.cuda(), bo.cuda(), wg.cuda(), bg.cuda())
  chk(ops.trimul_epilogue(*args), O.ref_trimul_epilogue(x_cm, act, sc, of, wo, bo, wg, bg))
  chk(ops.trimul_epilogue(*args, residual=res.cuda()), O.ref_trimul_epilogue(x_cm, act, sc, of, wo, bo, wg, bg, res))
  isc, iof = 1 + rnd(rng, c, s=.1).float(), rnd(rng, c, s=.1).float()
  got = ops.trimul_epilogue(*args, in_scale=isc.cuda(), in_offset=iof.cuda(), add_input=True)
  chk(got, O.ref_trimul_epilogue_ln(x_cm, act, isc, iof, sc, of, wo, bo, wg, bg, add_input=True))
  assert ops.device_status() == 0


@pytest.mark.parametrize("m,a,g,n,h", [(4101, 128, 4, 128, 4), (59, 64, 4, 64, 4), (1000, 256, 4, 256, 8), (1, 128, 3, 128, 4),
                                       (40000, 256, 4, 256, 8), (300, 256, 1, 128, 8), (777, 256, 3, 64, 4),
                                       (30000, 128, 3, 128, 4), (257, 128, 2, 256, 4), (129, 128, 1, 128, 4)])
def test_ln_projection(m, a, g, n, h):
  from colabfold_kernels import ops
  rng = np.random.default_rng(4)
  x, w, wb = rnd(rng, m, a), rnd(rng, g, a, n, s=a ** -.5), rnd(rng, a, h, s=a ** -.5)
  sc, of = 1 + rnd(rng, a, s=.1).float(), rnd(rng, a, s=.1).float()
  p, b = ops.ln_projection(x.cuda(), sc.cuda(), of.cuda(), w.cuda(), wb.cuda())
  assert ops.device_status() == 0
  rp, rb = O.ref_ln_projection(x, sc, of, w, wb)
  chk(p, rp); chk(b, rb)
  p8, _ = ops.ln_projection(x.cuda(), sc.cuda(), of.cuda(), w.cuda(), None, f8=True, f8_scale=0.5)
  assert O.rms_err(p8.cpu().float(), rp * 0.5) <= 5e-2  # tests/test_ln_fusions.py:192
  if a in (128, 256):  # the shape kernels' own row-block skipping: block 1 unkept (zeros), block 2 negative (unwritten)
    keep = torch.ones(m)
    keep[128:256] = 0
    keep[256:384] = -1
    pk, _ = ops.ln_projection(x.cuda(), sc.cuda(), of.cuda(), w.cuda(), None, keep=keep.cuda())
    live = keep > 0
    assert torch.equal(pk[live.cuda()], p[live.cuda()])
    assert m <= 128 or float(pk[128:256].float().abs().max()) == 0.0
    assert ops.device_status() == 0


def test_ln_projection_rows_far_from_zero_mean():
  """The 128-channel kernel multiplies the raw rows and takes the mean's part out afterwards (LN(x) w = rstd (x w' - mean s)
  + t): rows whose mean is many standard deviations from zero must come out as the reference's normalise-then-multiply
  (packed_attn.py:215-231)."""
  from colabfold_kernels import ops
  rng = np.random.default_rng(41)
  m, a, g, n = 700, 128, 4, 128
  x = (rnd(rng, m, a).float() + torch.linspace(-24, 24, m)[:, None]).to(torch.bfloat16)
  w = rnd(rng, g, a, n, s=a ** -.5)
  sc, of = 1 + rnd(rng, a, s=.1).float(), rnd(rng, a, s=.1).float()
  p, _ = ops.ln_projection(x.cuda(), sc.cuda(), of.cuda(), w.cuda(), None)
  assert ops.device_status() == 0
  rp, _ = O.ref_ln_projection(x, sc, of, w, None)
  chk(p, rp)


@pytest.mark.parametrize("m,k,c", [(4101, 128, 128), (59, 64, 64), (1000, 256, 256), (1, 128, 256)])
def test_output_projection(m, k, c):
  from colabfold_kernels import ops
  rng = np.random.default_rng(5)
  o, w, b, res = rnd(rng, m, k), rnd(rng, k, c, s=k ** -.5), rnd(rng, c, s=.1), rnd(rng, m, c)
  chk(ops.output_projection(o.cuda(), w.cuda(), b.cuda()), O.ref_output_projection(o, w, b))
  chk(ops.output_projection(o.cuda(), w.cuda(), b.cuda(), res.cuda()), O.ref_output_projection(o, w, b, res))
  assert ops.device_status() == 0


@pytest.mark.parametrize("s,r,c,k", [(6, 10, 64, 16), (64, 100, 256, 32), (3, 300, 128, 32)])
def test_opm_projection(s, r, c, k):
  from colabfold_kernels import ops
  rng = np.random.default_rng(6)
  x = rnd(rng, s, r, c)
  sc, of = 1 + rnd(rng, c, s=.1).float(), rnd(rng, c, s=.1).float()
  lw, lb, rw, rb = rnd(rng, c, k, s=c ** -.5), rnd(rng, k, s=.1), rnd(rng, c, k, s=c ** -.5), rnd(rng, k, s=.1)
  mask = torch.from_numpy((rng.random((s, r)) > .1).astype(np.float32)).to(bf)
  l, rr = ops.opm_projection(x.cuda(), sc.cuda(), of.cuda(), lw.cuda(), lb.cuda(), rw.cuda(), rb.cuda(), mask.cuda())
  assert ops.device_status() == 0
  rl, rrr = O.ref_opm_projection(x, sc, of, lw, lb, rw, rb, mask)
  chk(l, rl); chk(rr, rrr)


@pytest.mark.parametrize("m,c,hd", [(59, 128, 512), (4101, 128, 512), (300, 256, 1024), (2000, 64, 256), (260 * 260, 128, 512)])
@pytest.mark.parametrize("add_input", [False, True])
def test_transition(m, c, hd, add_input):
  """relu(LN(x) w1 + b1) w2 + b2 (+ x) against the oracle (transition.py:141-146)."""
  from colabfold_kernels import ops
  rng = np.random.default_rng(5)
  x, w1, b1, w2, b2 = rnd(rng, m, c), rnd(rng, c, hd, s=c ** -.5), rnd(rng, hd, s=.1), rnd(rng, hd, c, s=hd ** -.5), rnd(rng, c, s=.1)
  sc, of = 1 + rnd(rng, c, s=.1).float(), rnd(rng, c, s=.1).float()
  out = ops.transition(x.cuda(), sc.cuda(), of.cuda(), w1.cuda(), b1.cuda(), w2.cuda(), b2.cuda(), add_input=add_input)
  assert ops.device_status() == 0
  chk(out, O.ref_transition(x, sc, of, w1, b1, w2, b2, add_input=add_input))


def test_transition_keep_leaves_padding_blocks_as_the_reference_does():
  """A 128-row block keep marks nowhere is zeros (x with add_input); marked rows are computed as without keep
  (transition.py:88-92,108-110)."""
  from colabfold_kernels import ops
  rng = np.random.default_rng(6)
  m, c, hd = 1000, 128, 512
  x, w1, b1, w2, b2 = rnd(rng, m, c), rnd(rng, c, hd, s=c ** -.5), rnd(rng, hd, s=.1), rnd(rng, hd, c, s=hd ** -.5), rnd(rng, c, s=.1)
  sc, of = 1 + rnd(rng, c, s=.1).float(), rnd(rng, c, s=.1).float()
  keep = torch.ones(m)
  keep[256:640] = 0  # blocks 2, 3 and 4 are padding throughout
  keep[700] = 0      # a hole in a live block changes nothing
  args = [t.cuda() for t in (x, sc, of, w1, b1, w2, b2)]
  for add_input in (False, True):
    out = ops.transition(*args, keep=keep.cuda(), add_input=add_input)
    full = ops.transition(*args, add_input=add_input)
    live = torch.ones(m, dtype=torch.bool)
    live[256:640] = False
    assert torch.equal(out[live.cuda()], full[live.cuda()])
    pad = out[256:640]
    assert torch.equal(pad, x[256:640].cuda()) if add_input else torch.count_nonzero(pad) == 0
  # a block that is negative throughout is not written at all (transition.py:29-38); at 256 channels too
  for c2, hd2 in ((128, 512), (256, 1024)):
    x2, w1b, b1b, w2b, b2b = rnd(rng, 700, c2), rnd(rng, c2, hd2, s=c2 ** -.5), rnd(rng, hd2, s=.1), rnd(rng, hd2, c2, s=hd2 ** -.5), rnd(rng, c2, s=.1)
    sc2, of2 = 1 + rnd(rng, c2, s=.1).float(), rnd(rng, c2, s=.1).float()
    keep2 = torch.ones(700)
    keep2[128:256] = -1
    keep2[384:512] = 0
    out = torch.full((700, c2), 7.0, dtype=bf, device="cuda")
    from colabfold_kernels import _lib
    dev = [t.cuda().contiguous() for t in (x2, sc2, of2, w1b, b1b, w2b, b2b, keep2)]
    _lib.call("cfk_transition", *[t.data_ptr() for t in dev[:7]], dev[7].data_ptr(), ops.tag(torch.float32), out.data_ptr(), 700, c2,
              hd2, 1e-5, 1, torch.cuda.current_stream().cuda_stream)
    full = ops.transition(*dev[:7], add_input=True)
    assert bool((out[128:256] == 7.0).all()) and torch.equal(out[384:512], dev[0][384:512])
    live = torch.ones(700, dtype=torch.bool)
    live[128:256] = False
    live[384:512] = False
    assert torch.equal(out[live.cuda()], full[live.cuda()])
  assert ops.device_status() == 0

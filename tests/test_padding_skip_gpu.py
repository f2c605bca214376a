"""Row-block skipping (`keep`) of the projection family, after the reference's tests/test_padding_skip.py:62-146: real
rows are bit-identical with and without `keep`; a padded row holds either what the call without `keep` gives or what a
skipped block writes (zeros, or the residual / input unchanged); blocks below zero are not written."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
bf = torch.bfloat16


def rnd(rng, *shape, s=.5):
  return torch.from_numpy((rng.standard_normal(shape) * s).astype(np.float32)).to(bf).cuda()


def check_keep(with_keep, without, keep, pad_value):
  real = keep > 0
  a, b = with_keep.float(), without.float()
  assert torch.isfinite(a).all()
  assert torch.equal(a[real], b[real])                       # real rows: bit-identical
  pad = ~real
  same = (a[pad] == b[pad]).all(dim=-1)
  skipped = (a[pad] == pad_value.float()[pad]).all(dim=-1)
  assert bool((same | skipped).all())                        # padded rows: as without keep, or the skipped block's value
  return int(skipped.sum())


def setup(S, live, rng):
  tok = torch.zeros(S, dtype=torch.bool)
  tok[:live] = True
  keep = (tok[:, None] & tok[None, :]).reshape(-1).to(bf).cuda()   # pair rows that matter, as the reference builds it
  return keep


@pytest.mark.parametrize("S,live", [(48, 20), (64, 3), (40, 40)])
def test_keep_projection_family(S, live):
  from colabfold_kernels import ops
  rng = np.random.default_rng(S)
  m, c, n, h = S * S, 128, 128, 4
  keep = setup(S, live, rng)
  x = rnd(rng, m, c)
  sc, of = (1 + 0.1 * rnd(rng, c)).float(), (0.1 * rnd(rng, c)).float()
  w, wb = rnd(rng, 4, c, n, s=c ** -.5), rnd(rng, c, h, s=c ** -.5)
  zero = lambda t: torch.zeros_like(t)
  skipped = 0
  p0, b0 = ops.ln_projection(x, sc, of, w, wb)
  p1, b1 = ops.ln_projection(x, sc, of, w, wb, keep=keep)
  skipped += check_keep(p1, p0, keep, zero(p0))
  skipped += check_keep(b1.t(), b0.t(), keep, zero(b0.t()))
  o, wo, bo = rnd(rng, m, c), rnd(rng, c, c, s=c ** -.5), rnd(rng, c, s=.1)
  skipped += check_keep(ops.output_projection(o, wo, bo, x, keep=keep), ops.output_projection(o, wo, bo, x), keep, x)
  skipped += check_keep(ops.output_projection(o, wo, bo, None, keep=keep), ops.output_projection(o, wo, bo), keep, zero(x))
  tri = rnd(rng, c, m)
  g = [sc, of, rnd(rng, c, c, s=c ** -.5), rnd(rng, c, s=.1), rnd(rng, c, c, s=c ** -.5), rnd(rng, c, s=.1)]
  for add_input in (False, True):
    a = ops.trimul_epilogue(tri, x, *g, in_scale=sc, in_offset=of, add_input=add_input, keep=keep)
    b = ops.trimul_epilogue(tri, x, *g, in_scale=sc, in_offset=of, add_input=add_input)
    skipped += check_keep(a, b, keep, x if add_input else zero(x))
  if live * 2 < S:
    assert skipped > 0  # with this much padding whole 128-row tiles must have been skipped
  assert ops.device_status() == 0


def test_blocks_below_zero_are_left_unwritten():
  from colabfold_kernels import ops
  rng = np.random.default_rng(5)
  m, c = 1024, 128
  x = rnd(rng, m, c)
  sc, of = torch.ones(c).cuda(), torch.zeros(c).cuda()
  wo, bo = rnd(rng, c, c, s=c ** -.5), rnd(rng, c, s=.1)
  keep = torch.ones(m, device="cuda")
  keep[256:512] = 0     # two tiles of padding
  keep[512:] = -1       # four tiles outside what any consumer reads
  out = torch.full((m, c), 7.0, dtype=bf, device="cuda")
  ops.output_projection(x, wo, bo, None, out=out, keep=keep)
  ref = ops.output_projection(x, wo, bo)
  assert torch.equal(out[:256], ref[:256])
  assert float(out[256:512].float().abs().max()) == 0.0
  assert bool((out[512:] == 7.0).all())
  # LN -> gated dual projection: the mask itself filters the tiles
  wp, bp = rnd(rng, c, 256, s=c ** -.5), rnd(rng, 256, s=.1)
  mask = keep.to(bf)
  l, r = ops.ln_gated_dual_proj(x, sc, of, wp, bp, wp, bp, torch.ones(m, device="cuda", dtype=bf))
  l2 = torch.full_like(l, 7.0)
  r2 = torch.full_like(r, 7.0)
  from colabfold_kernels import _lib
  _lib.call("cfk_ln_gated_dual_proj", x.data_ptr(), sc.data_ptr(), of.data_ptr(), wp.data_ptr(), bp.data_ptr(), wp.data_ptr(),
            bp.data_ptr(), mask.data_ptr(), l2.data_ptr(), r2.data_ptr(), m, 0, c, 256, 0, 1, 0, 1.0, 1e-5,
            torch.cuda.current_stream().cuda_stream)
  torch.cuda.synchronize()
  assert torch.equal(l2[:, :256], l[:, :256]) and torch.equal(r2[:, :256], r[:, :256])
  assert float(l2[:, 256:512].float().abs().max()) == 0.0
  assert bool((l2[:, 512:] == 7.0).all()) and bool((r2[:, 512:] == 7.0).all())
  assert ops.device_status() == 0

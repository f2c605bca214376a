"""Triangle-multiplication contraction on the GPU against the CPU oracle: bf16 and e4m3 operands,
ragged I/J/K, both einsum orders of tests/test_ln_fusions.py:216-222."""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [(4, 128, 256, 64), (3, 200, 264, 136), (2, 512, 512, 512), (5, 24, 16, 32),
                                   (1, 1000, 1000, 1000), (128, 128, 128, 128)])
def test_contract_bf16(shape):
  from colabfold_kernels import ops
  c, i, j, k = shape
  rng = np.random.default_rng(0)
  a = torch.from_numpy(rng.standard_normal((c, i, k)).astype(np.float32)).to(torch.bfloat16)
  b = torch.from_numpy(rng.standard_normal((c, j, k)).astype(np.float32)).to(torch.bfloat16)
  out = ops.contract(a.cuda(), b.cuda())
  assert ops.device_status() == 0
  ref = O.ref_contract(a, b)
  # fp32 accumulation, one rounding to bf16 on store
  assert O.rel_err(out.cpu().float(), ref) <= 8e-3


@pytest.mark.parametrize("shape", [(4, 128, 256, 128), (3, 200, 264, 144), (2, 24, 16, 32)])
def test_contract_e4m3(shape, golden):
  from colabfold_kernels import ops
  c, i, j, k = shape
  rng = np.random.default_rng(1)
  a = O.e4m3(torch.from_numpy(rng.standard_normal((c, i, k)).astype(np.float32) * 2))
  b = O.e4m3(torch.from_numpy(rng.standard_normal((c, j, k)).astype(np.float32) * 2))
  out = ops.contract(a.cuda(), b.cuda())
  assert ops.device_status() == 0
  ref = O.ref_fp8_contract(a.float(), b.float())
  assert O.rel_err(out.cpu().float(), ref) <= 1e-2   # the reference's own bound, tests/test_ln_fusions.py:211
  g = golden("fp8_contract")
  out = ops.contract(O.e4m3(torch.from_numpy(g["a"])).cuda(), O.e4m3(torch.from_numpy(g["b"])).cuda())
  assert O.rel_err(out.cpu().float(), torch.from_numpy(g["out"])) <= 1e-2


def test_triangle_einsum_orders():
  """outgoing 'ikc,jkc->ijc' and incoming 'kjc,kic->ijc' through channel-major operands."""
  from colabfold_kernels import ops
  rng = np.random.default_rng(2)
  n, c = 72, 16
  l = torch.from_numpy(rng.standard_normal((n, n, c)).astype(np.float32)).to(torch.bfloat16)
  r = torch.from_numpy(rng.standard_normal((n, n, c)).astype(np.float32)).to(torch.bfloat16)
  out = ops.contract(l.permute(2, 0, 1).contiguous().cuda(), r.permute(2, 0, 1).contiguous().cuda())
  ref = torch.einsum("ikc,jkc->cij", l.float(), r.float())
  assert O.rel_err(out.cpu().float(), ref) <= 8e-3
  out = ops.contract(r.permute(2, 1, 0).contiguous().cuda(), l.permute(2, 1, 0).contiguous().cuda())
  ref = torch.einsum("kjc,kic->cij", l.float(), r.float())
  assert O.rel_err(out.cpu().float(), ref) <= 8e-3


@pytest.mark.parametrize("s,r", [(24, 10), (64, 36), (16, 130)])
def test_outer_product_mean_matches_oracle(s, r):
  """Deep-MSA outer product mean through the [i, j, c, e] store of the contraction kernel (row counts that are not
  multiples of the 4 x 8 residues a tile holds exercise the clipping of the 4-D store)."""
  from colabfold_kernels import ops
  rng = np.random.default_rng(s + r)
  mk = lambda *sh, sc=.5: torch.from_numpy((rng.standard_normal(sh) * sc).astype(np.float32)).to(torch.bfloat16)
  mask = torch.from_numpy((rng.random((s, r)) > .1).astype(np.float32))
  left, right = mk(s, r, 32) * mask[..., None].to(torch.bfloat16), mk(s, r, 32) * mask[..., None].to(torch.bfloat16)
  w, bias, res = mk(32 * 32, 128, sc=1 / 32), mk(128, sc=.1), mk(r, r, 128)
  ref = O.ref_opm_deep(left, right, mask, w, bias, res)
  got = ops.outer_product_mean(left.cuda(), right.cuda(), mask.cuda(), mask.cuda(), w.cuda(), bias.cuda(), residual=res.cuda())
  assert ops.device_status() == 0
  assert O.rel_err(got.cpu().float(), ref) <= 2e-2
  # row-sharded use: a slice of the left rows against all of the right
  part = ops.outer_product_mean(left[:, 2:7].cuda(), right.cuda(), mask[:, 2:7].cuda(), mask.cuda(), w.cuda(), bias.cuda(),
                                residual=res[2:7].cuda())
  assert torch.equal(part, got[2:7])


def test_shallow_opm_forms_match_the_reference_fixtures(golden):
  """opm_outer and opm_update through the selectors against the reference's own ref_* outputs (tests/golden)."""
  from colabfold_kernels import dispatch, fused_ops, ops
  cfg = dispatch()
  bf16 = lambda a: torch.from_numpy(np.asarray(a, dtype=np.float32)).to(torch.bfloat16).cuda()
  g = golden("opm_outer")
  rows, b, c = g["left"].shape
  d, e = g["right"].shape[1:]
  f = g["w"].shape[1]
  sel = fused_ops.opm_outer(cfg, torch.bfloat16, rows, c, d, f)
  assert callable(sel)
  got = sel(bf16(g["left"]), bf16(g["right"]), bf16(g["w"]))
  ref = O.ref_opm_outer(bf16(g["left"]).cpu(), bf16(g["right"]).cpu(), bf16(g["w"]).cpu())
  assert O.rel_err(got.cpu().float(), ref) <= 2e-2
  assert O.rel_err(got.cpu().float(), torch.from_numpy(np.asarray(g["out"], dtype=np.float32))) <= 2e-2
  g = golden("opm_update")
  k = g["lhs"].shape[1]
  f = g["t"].shape[2]
  sel = fused_ops.opm_update(cfg, torch.bfloat16, k, f)
  assert callable(sel)
  got = sel(bf16(g["lhs"]), bf16(g["t"]), bf16(g["bias"]), torch.from_numpy(np.asarray(g["norm"], dtype=np.float32)).cuda(),
            bf16(g["residual"]))
  ref = O.ref_opm_update(bf16(g["lhs"]).cpu(), bf16(g["t"]).cpu(), bf16(g["bias"]).cpu(),
                         torch.from_numpy(np.asarray(g["norm"], dtype=np.float32)), bf16(g["residual"]).cpu())
  assert O.rel_err(got.cpu().float(), ref) <= 2e-2
  assert fused_ops.opm_outer(cfg, torch.bfloat16, 12, c, d, f) is None       # not 16 rows: the caller's own path
  assert fused_ops.opm_update(cfg, torch.bfloat16, 40, 128) is None           # K not a multiple of 32
  assert ops.device_status() == 0


@pytest.mark.parametrize("parts,jp,dtype", [(2, 128, "bf16"), (3, 128, "bf16"), (4, 256, "bf16"), (8, 128, "e4m3"),
                                            (3, 384, "e4m3")])
def test_contract_reads_an_all_gathered_operand_in_place(parts, jp, dtype):
  """b as [parts, c, j/parts, k] (what an all-gather of per-rank right operands leaves) gives bit for bit the
  product of the re-laid-out [c, j, k] operand; part counts that leave j off the 256-row tile included."""
  from colabfold_kernels import ops
  c, i, k = 5, 200, 264 if dtype == "bf16" else 272
  g = torch.Generator().manual_seed(parts * 1000 + jp)
  dt = torch.bfloat16 if dtype == "bf16" else torch.float8_e4m3fn
  a = torch.randn(c, i, k, generator=g).to(dt).cuda()
  b_parts = torch.randn(parts, c, jp, k, generator=g).to(dt).cuda()
  whole = torch.cat(list(b_parts.unbind(0)), dim=1).contiguous()
  out = ops.contract_gathered(a, b_parts)
  ref = ops.contract(a, whole)
  assert ops.device_status() == 0
  assert out.shape == (c, i, parts * jp)
  assert torch.equal(out, ref)
  # and the reference itself is right (oracle), so the pair cannot be wrong together
  assert O.rel_err(ref.cpu().float(), O.ref_contract(a.cpu().float(), whole.cpu().float())) <= (8e-3 if dtype == "bf16" else 6e-2)


def test_contract_gathered_rejects_parts_that_split_a_tile():
  from colabfold_kernels import ops
  a = torch.zeros(1, 128, 64, dtype=torch.bfloat16, device="cuda")
  b = torch.zeros(2, 1, 64, 64, dtype=torch.bfloat16, device="cuda")
  with pytest.raises(RuntimeError):
    ops.contract_gathered(a, b)


def test_outer_product_mean_e4m3_opt_in():
  """The FP8 variant casts the two projections to e4m3 (saturating) before the outer product: checked against the
  oracle on the rounded projections at the bf16 tolerance, and against the unrounded ones at the FP8 tolerance."""
  from colabfold_kernels import ops
  s, r = 64, 40
  rng = np.random.default_rng(9)
  mk = lambda *sh, sc=.5: torch.from_numpy((rng.standard_normal(sh) * sc).astype(np.float32)).to(torch.bfloat16)
  mask = torch.from_numpy((rng.random((s, r)) > .1).astype(np.float32))
  left, right = mk(s, r, 32) * mask[..., None].to(torch.bfloat16), mk(s, r, 32) * mask[..., None].to(torch.bfloat16)
  left[0, 0, 0] = 1000.0  # beyond e4m3's range: saturates at 448 instead of becoming NaN
  w, bias, res = mk(32 * 32, 128, sc=1 / 32), mk(128, sc=.1), mk(r, r, 128)
  got = ops.outer_product_mean(left.cuda(), right.cuda(), mask.cuda(), mask.cuda(), w.cuda(), bias.cuda(), residual=res.cuda(), fp8=True)
  assert ops.device_status() == 0 and torch.isfinite(got).all()
  l8, r8 = O.e4m3(left).float(), O.e4m3(right).float()
  assert float(l8[0, 0, 0]) == 448.0
  assert O.rel_err(got.cpu().float(), O.ref_opm_deep(l8, r8, mask, w, bias, res)) <= 2e-2
  left[0, 0, 0] = 0.5
  got = ops.outer_product_mean(left.cuda(), right.cuda(), mask.cuda(), mask.cuda(), w.cuda(), bias.cuda(), residual=res.cuda(), fp8=True)
  assert O.rel_err(got.cpu().float(), O.ref_opm_deep(left, right, mask, w, bias, res)) <= 6e-2


@pytest.mark.parametrize("split_k", [False, True])
@pytest.mark.parametrize("dtype", ["bf16", "e4m3"])
def test_contract_exchanged_reads_and_writes_the_all_to_all_layouts(split_k, dtype):
  """cfk_contract_exchanged on operands laid out as an all-to-all over the channel axis leaves them (split by rows, or
  along the contracted axis) must equal cfk_contract on the assembled operands, stored as the all-to-all back wants
  it ([parts, c, i/parts, j])."""
  from colabfold_kernels import ops
  g = torch.Generator().manual_seed(11)
  parts, c, i, j, k = 4, 3, 512, 1024, 512
  a = (torch.randn(c, i, k, generator=g) * .5).to(torch.bfloat16).cuda()
  b = (torch.randn(c, j, k, generator=g) * .5).to(torch.bfloat16).cuda()
  if dtype == "e4m3":
    a, b = a.to(torch.float8_e4m3fn), b.to(torch.float8_e4m3fn)
  whole = ops.contract(a, b)  # [c, i, j]
  if split_k:
    ap = torch.stack(a.view(torch.uint8 if dtype == "e4m3" else a.dtype).chunk(parts, dim=2), 0).contiguous()
    bp = torch.stack(b.view(torch.uint8 if dtype == "e4m3" else b.dtype).chunk(parts, dim=2), 0).contiguous()
  else:
    ap = torch.stack(a.view(torch.uint8 if dtype == "e4m3" else a.dtype).chunk(parts, dim=1), 0).contiguous()
    bp = torch.stack(b.view(torch.uint8 if dtype == "e4m3" else b.dtype).chunk(parts, dim=1), 0).contiguous()
  if dtype == "e4m3":
    ap, bp = ap.view(torch.float8_e4m3fn), bp.view(torch.float8_e4m3fn)
  got = ops.contract_exchanged(ap, bp, split_k=split_k)  # [parts, c, i/parts, j]
  assert ops.device_status() == 0
  want = torch.stack(whole.chunk(parts, dim=1), 0)
  assert torch.equal(got, want)


@pytest.mark.parametrize("s,ri,rj,cm", [(70, 40, 40, 256), (64, 16, 8, 128), (200, 37, 53, 256), (512, 128, 256, 256)])
def test_fused_outer_product_mean(s, ri, rj, cm):
  """The one-kernel deep outer product mean (channel-major projections with the depth contiguous, outer product kept on
  chip, mask overlap count from the library) against the oracle, and against the three-kernel composition it
  replaces; ragged depth (70: pitch 72, tail beyond the last 64-deep slice), residue counts off the 16 x 8 tile,
  ri != rj (a row shard of the pair)."""
  from colabfold_kernels import ops
  rng = np.random.default_rng(s + ri)
  mk = lambda *sh, sc=1.0: torch.from_numpy((rng.standard_normal(sh) * sc).astype(np.float32)).to(torch.bfloat16)
  r = max(ri, rj)
  m = mk(s, r, cm)
  gamma, beta = 1 + mk(cm, sc=.02).float(), mk(cm, sc=.02).float()
  lw, rw = mk(cm, 32, sc=cm ** -.5), mk(cm, 32, sc=cm ** -.5)
  lb, rb = mk(32, sc=.1), mk(32, sc=.1)
  w, bias, res = mk(32 * 32, 128, sc=1 / 32), mk(128, sc=.1), mk(ri, rj, 128)
  mask = torch.from_numpy((rng.random((s, r)) < .9).astype(np.float32)).to(torch.bfloat16)
  cu = lambda *t: [x.cuda() for x in t]
  lcm, rcm = ops.opm_projection_cm(*cu(m, gamma, beta, lw, lb, rw, rb, mask))
  assert lcm.shape == (32, r, -(-s // 8) * 8)
  rl, rr = O.ref_opm_projection(m.reshape(s * r, cm), gamma, beta, lw, lb, rw, rb, mask.reshape(-1))
  rl, rr = rl.reshape(s, r, 32), rr.reshape(s, r, 32)
  # the projections themselves, in their new layout (and an exactly zero tail)
  assert O.rel_err(lcm[:, :, :s].permute(2, 1, 0).cpu().float(), rl) <= 2e-2
  assert O.rel_err(rcm[:, :, :s].permute(2, 1, 0).cpu().float(), rr) <= 2e-2
  assert float(lcm[:, :, s:].float().abs().max() if lcm.shape[2] > s else 0.0) == 0.0
  lcm, rcm = lcm[:, :ri].contiguous(), rcm[:, :rj].contiguous()
  got = ops.outer_product_mean_cm(lcm, rcm, mask[:, :ri].cuda(), mask[:, :rj].cuda(), w.cuda(), bias.cuda(), residual=res.cuda())
  assert ops.device_status() == 0
  # oracle on the projections the kernel saw (bf16), so the bound is the GEMMs' alone
  lq, rq = lcm[:, :, :s].permute(2, 1, 0).cpu().float(), rcm[:, :, :s].permute(2, 1, 0).cpu().float()
  outer = torch.einsum("sia,sjb->ijab", lq, rq).reshape(ri, rj, 1024)
  ref = (outer @ w.float() + bias.float()) / (1e-3 + mask[:, :ri].float().T @ mask[:, :rj].float())[..., None] + res.float()
  assert O.rel_err(got.cpu().float(), ref) <= 2e-2
  # and the composition of the three kernels on the same projections (it needs a depth in whole 16-byte rows)
  if s % 8 == 0:
    comp = ops.outer_product_mean(lcm[:, :, :s].permute(2, 1, 0).contiguous(), rcm[:, :, :s].permute(2, 1, 0).contiguous(),
                                  mask[:, :ri].cuda(), mask[:, :rj].cuda(), w.cuda(), bias.cuda(), residual=res.cuda())
    assert O.rel_err(got.cpu().float(), comp.cpu().float()) <= 1e-2
  # without a residual, and the unsupported widths say so
  got0 = ops.outer_product_mean_cm(lcm, rcm, mask[:, :ri].cuda(), mask[:, :rj].cuda(), w.cuda(), bias.cuda())
  assert O.rel_err(got0.cpu().float(), ref - res.float()) <= 2e-2
  assert not ops.opm_fused_supported(16, 128, torch.bfloat16) and ops.opm_fused_supported(32, 128, torch.bfloat16)


def test_opm_outer_selector_takes_the_fused_kernel_and_the_composed_path():
  """opm_outer at AF2's widths (32 x 32 channels, 128 outputs) runs the one-kernel form (product never written); other
  widths compose the contraction kernels.  Both against the oracle on the same inputs, through the selector."""
  from colabfold_kernels import dispatch, fused_ops, ops
  rng = np.random.default_rng(31)
  mk = lambda *sh, sc=1.0: torch.from_numpy((rng.standard_normal(sh) * sc).astype(np.float32)).to(torch.bfloat16)
  for c, f, bdim, ddim in ((32, 128, 40, 24), (16, 64, 40, 24)):
    left, right, w = mk(16, bdim, c, sc=.5), mk(16, ddim, c, sc=.5), mk(c * c, f, sc=1 / c)
    sel = fused_ops.opm_outer(dispatch(), torch.bfloat16, 16, c, ddim, f)
    assert callable(sel)
    launches = ops._lib.load().cfk_launch_count(1)
    got = sel(left.cuda(), right.cuda(), w.cuda())
    launches = ops._lib.load().cfk_launch_count(0)
    assert launches == (1 if c == 32 else 2), launches      # one kernel of the library, or outer product + output weights
    assert O.rel_err(got.cpu().float(), O.ref_opm_outer(left, right, w)) <= 2e-2
  assert ops.device_status() == 0

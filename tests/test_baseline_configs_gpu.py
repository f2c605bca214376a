"""Parity at the exact shapes of the baseline configurations 2, 3 and 4 (distributions as the reference's
own tests draw them: N(0,1) activations, LayerNorm gamma ~ N(1, 0.02) and beta ~ N(0, 0.02), Xavier-normal weights,
Bernoulli masks), GPU kernels through the selectors against the CPU oracle.  bf16 bound 2e-2, e4m3 bound 6e-2."""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu
BF16_TOL, FP8_TOL = 2e-2, 6e-2
bf = torch.bfloat16


def cfg(**kw):
  from colabfold_kernels import dispatch
  return {**dispatch(), **kw}


def normal(rng, *shape, s=1.0, dtype=bf):
  return torch.from_numpy((rng.standard_normal(shape) * s).astype(np.float32)).to(dtype)


def xavier(rng, fan_in, fan_out, *lead):
  std = (2.0 / (fan_in + fan_out)) ** .5
  return normal(rng, *lead, fan_in, fan_out, s=std)


def test_config2_triangle_attention_starting_node_forward_and_vjp():
  """z [384, 384, 128] -> LayerNorm -> q/k/v/gate projections (4 heads x 32) + triangle bias [4, 384, 384] -> attention
  batched over the 384 rows with a Bernoulli(0.95) residue mask -> forward and the VJP of <out, cotangent> with
  respect to z, the projection weights, the bias weights and the gate bias."""
  from colabfold_kernels import fused_ops
  rng = np.random.default_rng(1)
  r, c, h, d = 384, 128, 4, 32
  z = normal(rng, r, r, c)
  gamma = 1 + normal(rng, c, s=.02, dtype=torch.float32)
  beta = normal(rng, c, s=.02, dtype=torch.float32)
  w, wb = xavier(rng, c, h * d, 4), xavier(rng, c, h)
  gate_bias = normal(rng, h, d, s=.1)
  res_mask = torch.from_numpy(rng.random(r) < 0.95)
  kmask = res_mask[None, :].expand(r, r).contiguous()
  cot = normal(rng, r, r, h, d, s=.5)
  proj = fused_ops.ln_projection(cfg(), bf, c, h * d)
  attn = fused_ops.packed_attention(cfg(), bf, d, d)
  assert proj is not None and attn is not None

  def forward(z, gamma, beta, w, wb, gate_bias, K):
    p, bias = K["proj"](z.reshape(r * r, c), gamma, beta, w, wb)
    return K["attn"](p.reshape(r, r, 4, h, d), bias.reshape(h, r, r), K["kmask"], gate_bias)

  cuda_k = {"proj": lambda *a: proj(*a, eps=1e-5), "attn": lambda p, b, km, gb: attn(p, b, km, gb, sm_scale=d ** -.5),
            "kmask": kmask.cuda()}
  ref_k = {"proj": lambda *a: O.ref_ln_projection(*a),
           "attn": lambda p, b, km, gb: O.ref_packed_attention(p, b, km, gb, sm_scale=d ** -.5), "kmask": kmask}
  args = (z, gamma, beta, w, wb, gate_bias)
  dev = [a.cuda().requires_grad_(True) for a in args]
  out = forward(*dev, cuda_k)
  grads = torch.autograd.grad((out.float() * cot.cuda().float()).sum(), dev)
  ref_out = forward(*[a.float() for a in args], ref_k)
  rgrads = O.vjp(lambda *a: forward(*a, ref_k), list(args), list(range(6)), cot.float())
  errs = {"out": O.rel_err(out.detach().cpu().float(), ref_out)}
  for name, g, rg in zip(("dz", "dgamma", "dbeta", "dw", "dwb", "dgate_bias"), grads, rgrads):
    errs[name] = O.rel_err(g.cpu().float(), rg)
  assert max(errs.values()) <= BF16_TOL, errs


def test_config3_triangle_multiplication_outgoing_chained():
  """z [512, 512, 128]: LN -> gated dual projection (a, b: 128 -> 128 each) with a Bernoulli(0.95) pair mask ->
  einsum('ikc,jkc->ijc') -> output LN, 128 -> 128 linear, sigmoid gate from LN(z), added to z; every stage feeds the
  next on the GPU, the oracle runs the same chain in float32."""
  from colabfold_kernels import fused_ops
  rng = np.random.default_rng(2)
  n, c = 512, 128
  z = normal(rng, n, n, c)
  g_in, b_in = 1 + normal(rng, c, s=.02, dtype=torch.float32), normal(rng, c, s=.02, dtype=torch.float32)
  g_c, b_c = 1 + normal(rng, c, s=.02, dtype=torch.float32), normal(rng, c, s=.02, dtype=torch.float32)
  wp, wg = xavier(rng, c, 2 * c), xavier(rng, c, 2 * c)
  bp, bg = torch.zeros(2 * c, dtype=bf), torch.zeros(2 * c, dtype=bf)
  wo, wgo = xavier(rng, c, c), xavier(rng, c, c)
  bo, bgo = torch.zeros(c, dtype=bf), torch.zeros(c, dtype=bf)
  mask = torch.from_numpy((rng.random((n, n)) < 0.95).astype(np.float32)).to(bf)
  proj = fused_ops.ln_gated_dual_proj(cfg(), bf, c, c)
  contract = fused_ops.contraction(cfg(), bf)
  epi = fused_ops.trimul_epilogue_ln(cfg(), bf)
  assert proj is not None and contract is not None and epi is not None
  cu = lambda *t: [x.cuda() for x in t]
  left, right = proj(*cu(z, g_in, b_in, wp, bp, wg, bg, mask), eps=1e-5)
  x_cm = contract(left, right)                               # [c, i, j]
  out = epi(x_cm.reshape(c, n * n), z.cuda().reshape(n * n, c), *cu(g_in, b_in, g_c, b_c, wo, bo, wgo, bgo), eps=1e-5,
            add_input=True)
  rl, rr = O.ref_ln_gdp(z, g_in, b_in, wp, bp, wg, bg, mask)
  rx = O.ref_contract(rl, rr)
  ref = O.ref_trimul_epilogue_ln(rx.reshape(c, n * n), z.reshape(n * n, c), g_in, b_in, g_c, b_c, wo, bo, wgo, bgo,
                                 add_input=True)
  errs = {"left": O.rel_err(left.cpu().float(), rl), "right": O.rel_err(right.cpu().float(), rr),
          "contraction": O.rel_err(x_cm.cpu().float(), rx), "out": O.rel_err(out.cpu().float(), ref)}
  assert max(errs.values()) <= BF16_TOL, errs


@pytest.mark.parametrize("fp8", [False, True])
def test_config4_outer_product_mean(fp8):
  """m [512, 256, 256]: LN -> two 256 -> 32 projections with a Bernoulli(0.9) MSA mask -> per-sequence outer product
  summed over the 512 sequences -> 1024 -> 128 linear -> divided by eps + the mask overlap count; bf16 and the e4m3
  opt-in (projections cast to e4m3 for the outer product)."""
  from colabfold_kernels import fused_ops, ops
  rng = np.random.default_rng(3)
  s, r, cm, k, f = 512, 256, 256, 32, 128
  m = normal(rng, s, r, cm)
  gamma, beta = 1 + normal(rng, cm, s=.02, dtype=torch.float32), normal(rng, cm, s=.02, dtype=torch.float32)
  lw, rw = xavier(rng, cm, k), xavier(rng, cm, k)
  lb, rb = torch.zeros(k, dtype=bf), torch.zeros(k, dtype=bf)
  w, bias = xavier(rng, k * k, f), torch.zeros(f, dtype=bf)
  mask = torch.from_numpy((rng.random((s, r)) < 0.9).astype(np.float32)).to(bf)
  proj = fused_ops.opm_projection(cfg(), bf, cm, k)
  assert proj is not None
  cu = lambda *t: [x.cuda() for x in t]
  left, right = proj(*cu(m, gamma, beta, lw, lb, rw, rb, mask), eps=1e-5)
  out = ops.outer_product_mean(left, right, mask.cuda(), mask.cuda(), w.cuda(), bias.cuda(), eps=1e-3, fp8=fp8)
  rl, rr = O.ref_opm_projection(m, gamma, beta, lw, lb, rw, rb, mask)
  ref = O.ref_opm_deep(rl, rr, mask, w, bias)
  assert O.rel_err(left.cpu().float(), rl) <= BF16_TOL and O.rel_err(right.cpu().float(), rr) <= BF16_TOL
  err = O.rel_err(out.cpu().float(), ref)
  assert err <= (FP8_TOL if fp8 else BF16_TOL), err

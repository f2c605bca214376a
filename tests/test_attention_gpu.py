"""Attention parity on the GPU through the C ABI: golden fixtures, seeded cases against the CPU
oracle, the reference's own shape list (tests/test_pallas_vjp.py:27-28) and its edge cases
(fully masked rows, ragged sizes, packed rows/columns, gate, trim)."""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

F32_TOL = 1e-4   # float32: max-abs
BF16_TOL = 2e-2  # bf16: max|a-b| / max|b|


def dev(a, dtype=None):
  t = torch.as_tensor(np.asarray(a)) if not torch.is_tensor(a) else a
  t = t.cuda()
  return t if dtype is None else t.to(dtype)


def make_case(seed, b, h, sq, sk, d, p_live=0.85, full_mask_row=None):
  rng = np.random.default_rng(seed)
  f = lambda *sh: torch.from_numpy((rng.standard_normal(sh) * .5).astype(np.float32))
  q, k, v, bias, do = f(b, h, sq, d), f(b, h, sk, d), f(b, h, sk, d), f(h, sq, sk), f(b, h, sq, d)
  kmask = torch.from_numpy(rng.random((b, sk)) < p_live)
  kmask[:, 0] |= ~kmask.any(1)  # keep at least one key live unless asked otherwise
  if full_mask_row is not None:
    kmask[full_mask_row] = False
  return q, k, v, bias, kmask, do


@pytest.mark.parametrize("idx", range(5))
def test_fp32_golden(golden, idx):
  from colabfold_kernels import ops
  g = golden(f"attn_{idx}")
  out = ops.attention_fwd(dev(g["q"]), dev(g["k"]), dev(g["v"]), dev(g["bias"]), dev(g["kmask"]), float(g["scale"]))
  assert float((out.cpu() - torch.from_numpy(g["out"])).abs().max()) <= F32_TOL


@pytest.mark.parametrize("shape", [(2, 4, 96, 96, 32), (2, 4, 70, 83, 16), (1, 8, 64, 64, 48), (2, 2, 128, 128, 8),
                                   (2, 2, 96, 96, 4), (1, 4, 96, 96, 96), (64, 8, 128, 128, 32)])
def test_fp32_forward_backward(shape):
  """float32 tensors take the fp32-math kernels: max-abs <= 1e-4 forward, rel <= 1e-4 backward."""
  from colabfold_kernels import ops
  b, h, sq, sk, d = shape
  q, k, v, bias, kmask, do = make_case(0, *shape, full_mask_row=b - 1 if b > 1 else None)
  scale = d ** -0.5
  ref = O.ref_attn(q, k, v, bias, kmask, scale, torch.float64)
  lse_ref = O.ref_attn_lse(q, k, bias, kmask, scale, torch.float64)
  out, lse = ops.attention_fwd(dev(q), dev(k), dev(v), dev(bias), dev(kmask), scale, want_lse=True)
  assert float((out.cpu().double() - ref).abs().max()) <= F32_TOL
  live_rows = kmask.any(1)
  assert float((lse.cpu().double() - lse_ref)[live_rows].abs().max()) <= 1e-3
  # asking for lse must not perturb the output (tests/test_pallas_vjp.py:43-46)
  out2 = ops.attention_fwd(dev(q), dev(k), dev(v), dev(bias), dev(kmask), scale)
  assert torch.equal(out, out2)
  rq, rk, rv, rb = O.ref_attn_bwd(q, k, v, bias, kmask, ref, do, lse_ref, scale, torch.float64)
  dq, dk, dv, db = ops.attention_bwd(dev(q), dev(k), dev(v), dev(bias), dev(kmask), out, dev(do), lse, scale)
  for name, a, r in (("dq", dq, rq), ("dk", dk, rk), ("dv", dv, rv), ("dbias", db, rb)):
    assert O.rel_err(a, r) <= 2e-4, name


def test_fp32_seq_layout_and_no_bias():
  from colabfold_kernels import ops
  q, k, v, bias, kmask, do = make_case(3, 3, 4, 50, 61, 32)
  scale = 32 ** -0.5
  ref = O.ref_attn(q, k, v, torch.zeros_like(bias), kmask, scale, torch.float64)
  out = ops.attention_fwd(dev(q.transpose(1, 2)), dev(k.transpose(1, 2)), dev(v.transpose(1, 2)), None, dev(kmask),
                          scale, seq_major=True)
  assert float((out.cpu().double().transpose(1, 2) - ref).abs().max()) <= F32_TOL


BF16_SHAPES = [(2, 4, 96, 96, 32), (5, 2, 128, 128, 32), (3, 4, 200, 264, 32), (8, 8, 384, 384, 32), (1, 1, 8, 8, 32),
               (9, 4, 130, 136, 32)]


@pytest.mark.parametrize("shape", BF16_SHAPES)
@pytest.mark.parametrize("seq_major", [False, True])
def test_bf16_forward(shape, seq_major):
  """bf16, head dim 32: the tcgen05 kernel. rel <= 2e-2 against the fp32 oracle on the bf16-rounded inputs;
  rows of a fully masked batch row are the uniform mean of V."""
  from colabfold_kernels import ops
  b, h, sq, sk, d = shape
  q, k, v, bias, kmask, _ = make_case(1, *shape, p_live=0.9, full_mask_row=b - 1 if b > 1 else None)
  bf = lambda t: t.to(torch.bfloat16)
  qb, kb, vb, bb = bf(q), bf(k), bf(v), bf(bias)
  scale = d ** -0.5
  ref = O.ref_attn(qb, kb, vb, bb, kmask, scale)
  lse_ref = O.ref_attn_lse(qb, kb, bb, kmask, scale)
  tr = (lambda t: t.transpose(1, 2).contiguous()) if seq_major else (lambda t: t)
  out, lse = ops.attention_fwd(dev(tr(qb)), dev(tr(kb)), dev(tr(vb)), dev(bb), dev(kmask), scale, seq_major=seq_major,
                               want_lse=True)
  assert ops.device_status() == 0
  out = tr(out.cpu().float()) if seq_major else out.cpu().float()
  assert O.rel_err(out, ref) <= BF16_TOL
  live = kmask.any(1)
  assert float((lse.cpu() - lse_ref)[live].abs().max()) <= 5e-2
  if b > 1:
    mean_v = vb.float()[b - 1].mean(dim=1, keepdim=True).expand(h, sq, d)
    assert O.rel_err(out[b - 1], mean_v) <= BF16_TOL
    assert bool((lse.cpu()[b - 1] <= O.NEG / 2).all())


@pytest.mark.parametrize("idx", range(5))
def test_packed_golden(golden, idx):
  """Packed rows/columns, gate, no-bias, a fully masked row, trim: float32 through the fp32-math kernels."""
  from colabfold_kernels import ops
  g = golden(f"packed_{idx}")
  bias = dev(g["bias"]) if "bias" in g else None
  gb = dev(g["gate_bias"]) if "gate_bias" in g else None
  out = ops.packed_attention_fwd(dev(g["p"]), bias, dev(g["kmask"]), gb, float(g["scale"]), column=bool(g["column"]),
                                 trim=bool(g["trim"]))
  assert float((out.cpu() - torch.from_numpy(g["out"])).abs().max()) <= F32_TOL


@pytest.mark.parametrize("case", [(64, 96, 4, 32, True, False), (96, 64, 4, 32, True, True), (50, 56, 4, 32, False, True),
                                  (5, 8, 4, 32, True, False), (7, 136, 4, 32, True, False), (136, 8, 2, 32, False, True),
                                  (1, 40, 4, 32, True, True)])
def test_packed_bf16(case):
  """The packed layouts of tests/test_af2_fused_kernels.py:44-49 with head dim 32 in bf16 (tcgen05 kernel reading
  q/k/v/gate in place; column attention over X == 1 must not read past the end of p)."""
  from colabfold_kernels import ops
  X, Y, H, D, gated, column = case
  rng = np.random.default_rng(5)
  f = lambda *sh: torch.from_numpy((rng.standard_normal(sh) * .5).astype(np.float32)).to(torch.bfloat16)
  G = 4 if gated else 3
  nb, s = (Y, X) if column else (X, Y)
  p, bias = f(X, Y, G, H, D), f(H, s, s)
  kmask = torch.from_numpy(rng.random((nb, s)) > .1)
  kmask[nb // 2] = False
  gb = f(H, D) if gated else None
  ref = O.ref_packed_attention(p, bias, kmask, gb, sm_scale=D ** -.5, column=column)
  out = ops.packed_attention_fwd(dev(p), dev(bias), dev(kmask), None if gb is None else dev(gb), D ** -.5, column=column)
  assert ops.device_status() == 0
  assert O.rel_err(out.cpu().float(), ref) <= BF16_TOL
  ref_t = O.ref_packed_attention(p, bias, kmask, gb, sm_scale=D ** -.5, column=column, trim=True)
  out_t = ops.packed_attention_fwd(dev(p), dev(bias), dev(kmask), None if gb is None else dev(gb), D ** -.5,
                                   column=column, trim=True)
  assert O.rel_err(out_t.cpu().float(), ref_t) <= BF16_TOL
  assert bool((out_t.cpu().float()[ref_t == 0] == 0).all())  # trimmed positions are exact zeros


@pytest.mark.parametrize("shape", BF16_SHAPES + [(7, 2, 256, 384, 32)])
@pytest.mark.parametrize("seq_major", [False, True])
def test_bf16_backward(shape, seq_major):
  """bf16 backward (tcgen05 kernel: dq, dk, dv in bf16, dbias in fp32): rel <= 2e-2 against the oracle's explicit
  flash backward on the bf16-rounded inputs; a fully masked batch row differentiates the uniform softmax."""
  from colabfold_kernels import ops
  b, h, sq, sk, d = shape
  q, k, v, bias, kmask, do = make_case(2, *shape, p_live=0.9, full_mask_row=b - 1 if b > 1 else None)
  bf = lambda t: t.to(torch.bfloat16)
  qb, kb, vb, bb, dob = bf(q), bf(k), bf(v), bf(bias), bf(do)
  scale = d ** -0.5
  tr = (lambda t: t.transpose(1, 2).contiguous()) if seq_major else (lambda t: t)
  out, lse = ops.attention_fwd(dev(tr(qb)), dev(tr(kb)), dev(tr(vb)), dev(bb), dev(kmask), scale, seq_major=seq_major,
                               want_lse=True)
  dq, dk, dv, db = ops.attention_bwd(dev(tr(qb)), dev(tr(kb)), dev(tr(vb)), dev(bb), dev(kmask), out, dev(tr(dob)), lse,
                                     scale, seq_major=seq_major)
  assert ops.device_status() == 0
  ref = O.ref_attn(qb, kb, vb, bb, kmask, scale)
  lse_ref = O.ref_attn_lse(qb, kb, bb, kmask, scale)
  rq, rk, rv, rb = O.ref_attn_bwd(qb, kb, vb, bb, kmask, ref, dob, lse_ref, scale)
  un = (lambda t: t.cpu().float().transpose(1, 2)) if seq_major else (lambda t: t.cpu().float())
  for name, a, r in (("dq", un(dq), rq), ("dk", un(dk), rk), ("dv", un(dv), rv), ("dbias", db.cpu(), rb)):
    assert O.rel_err(a, r) <= BF16_TOL, name
  # no dbias wanted: the other gradients are unchanged
  dq2, dk2, dv2, none = ops.attention_bwd(dev(tr(qb)), dev(tr(kb)), dev(tr(vb)), dev(bb), dev(kmask), out, dev(tr(dob)),
                                          lse, scale, seq_major=seq_major, want_dbias=False)
  assert none is None and torch.equal(dk, dk2) and torch.equal(dv, dv2)

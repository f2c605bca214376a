"""The opt-in FP8 packed attention (q and k in e4m3, scores on the 8-bit tensor-core path) against the CPU oracle,
following tests/test_ln_fusions.py:166-194 of the reference: q is rounded after its static scale sm_scale * log2(e), k
as it is; p keeps v and the gate."""
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu
LOG2E = 1.4426950408889634
bf = torch.bfloat16


def _case(n, h, d, seed):
  g = torch.Generator().manual_seed(seed)
  p = torch.randn(n, n, 4, h, d, generator=g).to(bf)
  bias = torch.randn(h, n, n, generator=g).to(bf)
  gb = torch.randn(h, d, generator=g).to(bf)
  kmask = torch.rand(n, n, generator=g) > 0.1
  scales = torch.tensor([d ** -0.5 * LOG2E, 1.0])
  qk8 = O.e4m3(p[:, :, :2].float() * scales[None, None, :, None, None])
  return p, bias, gb, kmask, qk8


@pytest.mark.parametrize("column", [False, True])
@pytest.mark.parametrize("n", [264, 136])
def test_qk8_attention(n, column):
  from colabfold_kernels import ops
  h, d = 4, 32
  p, bias, gb, kmask, qk8 = _case(n, h, d, seed=n)
  sm = d ** -0.5
  out = ops.packed_attention_fwd(p[:, :, 2:].contiguous().cuda(), bias.cuda(), kmask.cuda(), gb.cuda(), sm, column=column,
                                 p8=qk8.cuda())
  assert ops.device_status() == 0
  # (1) the kernel's own arithmetic: the oracle on the operands the kernel saw (e4m3 values are exact in fp32, and
  # so are their products), bf16 tolerance
  deq = torch.cat([qk8[:, :, :1].float() / (sm * LOG2E), qk8[:, :, 1:].float(), p[:, :, 2:].float()], dim=2)
  ref_same = O.ref_packed_attention(deq, bias, kmask, gb, sm_scale=sm, column=column)
  assert O.rel_err(out.cpu().float(), ref_same) <= 2e-2
  # (2) the reference's criterion against the unrounded operands (test_ln_fusions.py:179-181): e4m3 rounds q and k
  # by ~3 % each, so the logits and their softmax move by about that much
  ref_full = O.ref_packed_attention(p, bias, kmask, gb, sm_scale=sm, column=column)
  assert O.rms_err(out.cpu().float(), ref_full) < 0.08


def test_qk8_attention_without_gate_and_with_trim():
  from colabfold_kernels import ops
  n, h, d = 200, 4, 32
  p, bias, _, kmask, qk8 = _case(n, h, d, seed=7)
  kmask[:, 150:] = False  # padding: trimmed queries and keys
  kmask[5] = False        # a row with no live key
  sm = d ** -0.5
  v = p[:, :, 2:3].contiguous()
  out = ops.packed_attention_fwd(v.cuda(), bias.cuda(), kmask.cuda(), None, sm, trim=True, p8=qk8.cuda())
  assert ops.device_status() == 0
  deq = torch.cat([qk8[:, :, :1].float() / (sm * LOG2E), qk8[:, :, 1:].float(), v.float()], dim=2)
  ref = O.ref_packed_attention(deq, bias, kmask, None, sm_scale=sm, trim=True)
  assert O.rel_err(out.cpu().float(), ref) <= 2e-2
  assert torch.count_nonzero(out[5]) == 0 and torch.count_nonzero(out[:, 150:]) == 0  # trimmed positions exact zeros


def test_ln_projection_writes_the_e4m3_slots_the_selector_names():
  """ln_projection(..., f8_slots, f8_scales) -> (p, bias, p8) (packed_attn.py:234-305; test_ln_fusions.py:183-194),
  and the result drives the FP8 attention end to end."""
  from colabfold_kernels import dispatch, fused_ops, ops
  g = torch.Generator().manual_seed(11)
  n, a, h, d = 136, 128, 4, 32
  x = (2 * torch.randn(n * n, a, generator=g)).to(bf)
  sc, of = 1 + 0.1 * torch.randn(a, generator=g), 0.1 * torch.randn(a, generator=g)
  w4 = (0.1 * torch.randn(4, a, h * d, generator=g)).to(bf)
  wb = (0.1 * torch.randn(a, h, generator=g)).to(bf)
  slots, scales = fused_ops.fp8_attention_slots({"fp8": True}, bf, d, n)
  assert slots == (0, 1) and abs(scales[0] - d ** -0.5 * LOG2E) < 1e-12 and scales[1] == 1.0
  proj = fused_ops.ln_projection(dispatch(), bf, a, h * d)
  ph, b8, p8 = proj(x.cuda(), sc.cuda(), of.cuda(), w4.cuda(), wb.cuda(), f8_slots=slots, f8_scales=scales)
  rp, rb, r8 = O.ref_ln_projection(x, sc, of, w4, wb, f8_slots=slots, f8_scales=scales)
  assert ph.shape == (n * n, 2 * h * d) and p8.shape == (n * n, 2 * h * d) and p8.dtype == torch.float8_e4m3fn
  assert O.rel_err(ph.cpu().float(), rp) <= 2e-2 and O.rel_err(b8.cpu().float(), rb) <= 2e-2
  assert O.rms_err(p8.cpu().float(), r8) < 0.05
  # end to end: projection -> FP8 attention against the bf16 path of the same inputs
  kmask = (torch.rand(n, n, generator=g) > 0.1).cuda()
  gb = torch.randn(h, d, generator=g).to(bf).cuda()
  attn = fused_ops.packed_attention({**dispatch(), "fp8": True}, bf, d, d)
  o8 = attn(ph.reshape(n, n, 2, h, d), b8.reshape(h, n, n), kmask, gb, p8.reshape(n, n, 2, h, d), sm_scale=d ** -0.5)
  p16, _ = ops.ln_projection(x.cuda(), sc.cuda(), of.cuda(), w4.cuda(), None)
  o16 = ops.packed_attention_fwd(p16.reshape(n, n, 4, h, d), b8.reshape(h, n, n), kmask, gb, d ** -0.5)
  assert ops.device_status() == 0
  assert O.rms_err(o8.cpu().float(), o16.cpu().float()) < 0.08


def test_fp8_attention_is_refused_where_the_8_bit_mma_does_not_fit():
  """Head dims below the 8-bit MMA's K of 32 are never offered e4m3 (test_ln_fusions.py:162-165); without the fp8
  flag nothing is."""
  from colabfold_kernels import fused_ops
  for d in (8, 16):
    assert fused_ops.fp8_attention_slots({"fp8": True}, bf, d, 64) is None
    assert not fused_ops.fp8_attention({"fp8": True}, d)
  assert fused_ops.fp8_attention_slots({}, bf, 32, 64) is None
  assert not fused_ops.fp8_attention({"fp8": True}, 32)  # q and k, not k and v: as where the reference's Mosaic kernel runs

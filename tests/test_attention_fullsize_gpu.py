"""Size-independent properties of the attention kernels at the headline shape (b=512, h=8, s=1024, d=32), where the
CPU oracle is too slow to run: rows of the softmax sum to one, masked keys cannot influence the output, the backward
is linear in the cotangent, and dBias equals the sum over the batch of per-row score gradients on a slice."""
import pytest
import torch

from colabfold_kernels import ops
import oracle as O

pytestmark = pytest.mark.gpu
B, H, S, D = 512, 8, 1024, 32
bf = torch.bfloat16


@pytest.fixture(scope="module")
def data():
  g = torch.Generator(device="cuda").manual_seed(7)
  mk = lambda *s: torch.randn(*s, device="cuda", generator=g).to(bf)
  q, k, v, do = mk(B, S, H, D), mk(B, S, H, D), mk(B, S, H, D), mk(B, S, H, D)
  bias = mk(H, S, S)
  kmask = torch.rand(B, S, device="cuda", generator=g) < 0.95
  return q, k, v, do, bias, kmask


def test_rows_sum_to_one_and_masked_keys_are_inert(data):
  q, k, v, do, bias, kmask = data
  scale = D ** -0.5
  ones = torch.ones_like(v)
  out = ops.attention_fwd(q, k, ones, bias, kmask, scale, seq_major=True)
  assert float((out.float() - 1).abs().max()) <= 1e-2  # sum_k p = 1 (bf16 p, fp32 accumulate, bf16 out)
  base = ops.attention_fwd(q, k, v, bias, kmask, scale, seq_major=True)
  dead = ~kmask
  k2, v2 = k.clone(), v.clone()
  k2[dead] = 37.0   # garbage on masked keys only
  v2[dead] = -91.0
  again = ops.attention_fwd(q, k2, v2, bias, kmask, scale, seq_major=True)
  assert torch.equal(base, again)  # masked positions contribute exactly zero
  assert ops.device_status() == 0


def test_backward_is_linear_in_the_cotangent_and_matches_oracle_on_a_slice(data):
  q, k, v, do, bias, kmask = data
  scale = D ** -0.5
  out, lse = ops.attention_fwd(q, k, v, bias, kmask, scale, seq_major=True, want_lse=True)
  g1 = ops.attention_bwd(q, k, v, bias, kmask, out, do, lse, scale, seq_major=True, want_dbias=False)
  g2 = ops.attention_bwd(q, k, v, bias, kmask, out, do * 2, lse, scale, seq_major=True, want_dbias=False)
  for a, b in zip(g1[:3], g2[:3]):
    assert torch.equal(a.float() * 2, b.float())  # doubling is exact in bf16 and in fp32
  # two batch rows against the CPU oracle (forward outputs and all gradients)
  sl = slice(0, 2)
  qs, ks, vs, dos = (t[sl].transpose(1, 2).float().cpu() for t in (q, k, v, do))
  ref_out = O.ref_attn(qs, ks, vs, bias.float().cpu(), kmask[sl].cpu(), scale)
  assert O.rel_err(out[sl].transpose(1, 2).float().cpu(), ref_out) <= 2e-2
  ref_lse = O.ref_attn_lse(qs, ks, bias.float().cpu(), kmask[sl].cpu(), scale)
  rdq, rdk, rdv, _ = O.ref_attn_bwd(qs, ks, vs, bias.float().cpu(), kmask[sl].cpu(), ref_out, dos, ref_lse, scale)
  for got, want in ((g1[0], rdq), (g1[1], rdk), (g1[2], rdv)):
    assert O.rel_err(got[sl].transpose(1, 2).float().cpu(), want) <= 2e-2
  assert ops.device_status() == 0

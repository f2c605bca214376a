"""The CPU oracle against the fixtures produced by the reference's own ref_* functions
(tests/golden/make_golden.py), plus the self-consistency of its explicit backward formulas."""
import numpy as np
import pytest
import torch

import oracle as O

TOL = 2e-5  # float32 vs float32, different summation orders


def t(a):
  return torch.from_numpy(np.asarray(a))


def close(a, b, tol=TOL):
  err = O.rel_err(a, t(b))
  assert err < tol, err


@pytest.mark.parametrize("idx", range(5))
def test_attention_golden(golden, idx):
  g = golden(f"attn_{idx}")
  out = O.ref_attn(g["q"], g["k"], g["v"], g["bias"], g["kmask"], float(g["scale"]))
  close(out, g["out"])
  # the public entry's glue: additive mask -> kmask, seq layout
  mb = np.where(g["kmask"], 0.0, -1e9).astype(np.float32)[:, None, None, :]
  out2 = O.ref_attention(t(g["q"]).transpose(1, 2), t(g["k"]).transpose(1, 2), t(g["v"]).transpose(1, 2), mb,
                         g["bias"], float(g["scale"]), layout="seq")
  close(out2.transpose(1, 2), g["out"])


def test_fully_masked_row_is_uniform_mean(golden):
  g = golden("attn_0")
  out = O.ref_attn(g["q"], g["k"], g["v"], g["bias"], g["kmask"], float(g["scale"]))
  assert not g["kmask"][1].any()
  mean_v = t(g["v"])[1].mean(dim=1, keepdim=True).expand_as(out[1])
  close(out[1], mean_v.numpy(), 1e-5)


@pytest.mark.parametrize("idx", range(5))
def test_packed_attention_golden(golden, idx):
  g = golden(f"packed_{idx}")
  out = O.ref_packed_attention(g["p"], g.get("bias"), g["kmask"], g.get("gate_bias"), sm_scale=float(g["scale"]),
                               column=bool(g["column"]), trim=bool(g["trim"]))
  close(out, g["out"])
  if not bool(g["trim"]):
    via = O.attention_via(g["p"], g.get("bias"), g["kmask"], g.get("gate_bias"), sm_scale=float(g["scale"]),
                          column=bool(g["column"]))
    close(via, g["out"])


def test_layer_norm_gdp_golden(golden):
  g = golden("layer_norm")
  close(O.ref_layer_norm(g["x"], g["scale"], g["offset"], 1e-5), g["out"])
  close(O.ref_ln(t(g["x"]), t(g["scale"]), t(g["offset"]), 1e-5), g["out_ln"])
  g = golden("gdp")
  close(O.ref_gdp(g["x"], g["wp"], g["bp"], g["wg"], g["bg"], g["mask"]), g["out"])
  g = golden("ln_gdp_2d")
  l, r = O.ref_ln_gdp(g["x"], g["scale"], g["offset"], g["wp"], g["bp"], g["wg"], g["bg"], g["mask"])
  close(l, g["left"]); close(r, g["right"])
  for tr in (0, 1):
    g = golden(f"ln_gdp_pair_{tr}")
    l, r = O.ref_ln_gdp(g["x"], g["scale"], g["offset"], g["wp"], g["bp"], g["wg"], g["bg"], g["mask"],
                        transpose=bool(tr), pad=16)
    assert tuple(l.shape) == g["left"].shape
    close(l, g["left"]); close(r, g["right"])


def test_epilogue_contract_golden(golden):
  g = golden("trimul_epilogue")
  args = [g[k] for k in ("x_cm", "act", "scale", "offset", "wo", "bo", "wg", "bg")]
  close(O.ref_trimul_epilogue(*args), g["out"])
  close(O.ref_trimul_epilogue(*args, g["residual"]), g["out_res"])
  g = golden("trimul_epilogue_ln")
  close(O.ref_trimul_epilogue_ln(*[g[k] for k in ("x_cm", "x", "in_scale", "in_offset", "scale", "offset", "wo", "bo",
                                                 "wg", "bg")], add_input=True), g["out"])
  g = golden("fp8_contract")
  close(O.ref_fp8_contract(g["a"], g["b"]), g["out"])
  # the saturating cast: past 448 clips instead of NaN
  assert float(O.e4m3(torch.tensor([1e6, -1e6])).float().abs().max()) == 448.0


def test_projection_opm_transition_golden(golden):
  g = golden("ln_projection")
  p, b = O.ref_ln_projection(g["x"], g["scale"], g["offset"], g["w"], g["wb"])
  close(p, g["p"]); close(b, g["bias"])
  g = golden("output_projection")
  close(O.ref_output_projection(g["o"], g["w"], g["b"], g["residual"]), g["out"])
  g = golden("opm_projection")
  l, r = O.ref_opm_projection(*[g[k] for k in ("x", "scale", "offset", "lw", "lb", "rw", "rb", "mask")])
  close(l, g["left"]); close(r, g["right"])
  g = golden("opm_outer")
  close(O.ref_opm_outer(g["left"], g["right"], g["w"]), g["out"])
  g = golden("opm_update")
  close(O.ref_opm_update(g["lhs"], g["t"], g["bias"], g["norm"], g["residual"]), g["out"])
  g = golden("transition")
  close(O.ref_transition(*[g[k] for k in ("x", "scale", "offset", "w1", "b1", "w2", "b2")], add_input=True), g["out"])


@pytest.mark.parametrize("idx", [0, 1])
def test_explicit_attention_backward_matches_autograd(golden, idx):
  """The flash backward's formulas (incl. the uniform softmax of a fully masked row) equal the
  gradient of the reference forward."""
  g = golden(f"attn_{idx}")
  dt = torch.float64
  scale = float(g["scale"])
  rng = np.random.default_rng(1)
  do = t(rng.standard_normal(g["out"].shape))
  fn = lambda q, k, v, b: O.ref_attn(q, k, v, b, g["kmask"], scale, dt)
  gq, gk, gv, gb = O.vjp(fn, (g["q"], g["k"], g["v"], g["bias"]), (0, 1, 2, 3), do, dt)
  out = fn(*(t(g[k]) for k in ("q", "k", "v", "bias")))
  lse = O.ref_attn_lse(g["q"], g["k"], g["bias"], g["kmask"], scale, dt)
  dq, dk, dv, db = O.ref_attn_bwd(g["q"], g["k"], g["v"], g["bias"], g["kmask"], out, do, lse, scale, dt)
  for a, b in ((dq, gq), (dk, gk), (dv, gv)):
    assert O.rel_err(a, b) < 1e-9
  # masked logits are constants: the explicit form gives them zero gradient, autograd of where() too
  assert O.rel_err(db, gb) < 1e-9


def test_explicit_ln_gdp_backward_matches_autograd(golden):
  dt = torch.float64
  g = golden("layer_norm")
  rng = np.random.default_rng(2)
  dy = rng.standard_normal(g["x"].shape)
  ref = O.vjp(lambda x, s, o: O.ref_layer_norm(x, s, o, 1e-5, dt), (g["x"], g["scale"], g["offset"]), (0, 1, 2), dy, dt)
  got = O.layer_norm_bwd(g["x"], g["scale"], dy, 1e-5, dt)
  for a, b in zip(got, ref):
    assert O.rel_err(a, b) < 1e-9
  g = golden("gdp")
  dy = rng.standard_normal(g["out"].shape)
  for act in ("sigmoid", "swish"):
    args = tuple(g[k] for k in ("x", "wp", "bp", "wg", "bg", "mask"))
    ref = O.vjp(lambda *a: O.ref_gdp(*a, activation=act, dtype=dt), args, (0, 1, 2, 3, 4, 5), dy, dt)
    got = O.gdp_bwd(*args, dy, activation=act, dtype=dt)
    for a, b in zip(got, ref):
      assert O.rel_err(a, b) < 1e-9

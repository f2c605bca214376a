"""colabfold_kernels/reference.py is what `differentiable_via` differentiates (the role the ref_* functions play in
the reference's grads.py:106-143): it must reproduce the committed fixtures of the reference's own ref_* functions.
Runs on CPU."""
import importlib.util
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
spec = importlib.util.spec_from_file_location(
    "cfk_reference", os.path.join(HERE, "..", "colabfold-kernels_b200", "colabfold_kernels", "reference.py"))
R = importlib.util.module_from_spec(spec)
spec.loader.exec_module(R)


def t(a):
  return torch.from_numpy(np.asarray(a))


def close(got, want, tol=2e-5):
  got, want = got.double(), t(want).double()
  assert tuple(got.shape) == tuple(want.shape)
  assert float((got - want).abs().max()) <= tol * max(1.0, float(want.abs().max()))


def pick(g, *names):
  return [t(g[k]) for k in names]


def test_ln_gdp(golden):
  g = golden("ln_gdp_2d")
  l, r = R.ref_ln_gdp(*pick(g, "x", "scale", "offset", "wp", "bp", "wg", "bg", "mask"))
  close(l, g["left"]); close(r, g["right"])
  for i, transpose in enumerate((False, True)):
    g = golden(f"ln_gdp_pair_{i}")
    l, r = R.ref_ln_gdp(*pick(g, "x", "scale", "offset", "wp", "bp", "wg", "bg", "mask"), transpose=transpose, pad=16)
    close(l, g["left"]); close(r, g["right"])


def test_gdp(golden):
  g = golden("gdp")
  x, wp, bp, wg, bg, mask = (v.float() for v in pick(g, "x", "wp", "bp", "wg", "bg", "mask"))
  close(R.ref_gdp(x, wp, bp, wg, bg, mask), g["out"])


def test_trimul_epilogue(golden):
  g = golden("trimul_epilogue")
  args = pick(g, "x_cm", "act", "scale", "offset", "wo", "bo", "wg", "bg")
  close(R.ref_trimul_epilogue(*args), g["out"])
  close(R.ref_trimul_epilogue(*args, t(g["residual"])), g["out_res"])
  g = golden("trimul_epilogue_ln")
  close(R.ref_trimul_epilogue_ln(*pick(g, "x_cm", "x", "in_scale", "in_offset", "scale", "offset", "wo", "bo", "wg", "bg"),
                                 add_input=True), g["out"])


def test_contract(golden):
  g = golden("fp8_contract")
  close(R.ref_contract(t(g["a"]), t(g["b"])), g["out"])


def test_projections(golden):
  g = golden("ln_projection")
  p, b = R.ref_ln_projection(*pick(g, "x", "scale", "offset", "w", "wb"))
  close(p, g["p"]); close(b, g["bias"])
  g = golden("output_projection")
  close(R.ref_output_projection(*pick(g, "o", "w", "b", "residual")), g["out"])


def test_opm(golden):
  g = golden("opm_projection")
  l, r = R.ref_opm_projection(*pick(g, "x", "scale", "offset", "lw", "lb", "rw", "rb", "mask"))
  close(l, g["left"]); close(r, g["right"])
  g = golden("opm_update")
  close(R.ref_opm_update(*pick(g, "lhs", "t", "bias", "norm", "residual")), g["out"])
  g = golden("opm_outer")
  close(R.ref_opm_outer(*pick(g, "left", "right", "w")), g["out"])


def test_transition(golden):
  g = golden("transition")
  close(R.ref_transition(*pick(g, "x", "scale", "offset", "w1", "b1", "w2", "b2"), add_input=True), g["out"])

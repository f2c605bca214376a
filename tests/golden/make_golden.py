"""Generate the golden fixtures in this folder from the reference's OWN ``ref_*`` functions.

The reference (mirditalab/colabfold-kernels v0.9.0) is pure Python on JAX, and JAX is not
installed where this project is built.  Its float32 ``ref_*`` functions are plain ``jnp`` code, so
this script installs a small NumPy stand-in for the ``jax`` modules they touch, imports the
reference's source files unmodified from ``--src`` (default: the read-only mount), runs the
``ref_*`` functions on seeded inputs and stores inputs + outputs as ``.npz`` files.  The Pallas
kernels themselves are never executed (they need a GPU and real JAX).

  python tests/golden/make_golden.py [--src /path/to/colabfold-kernels/src]

The fixtures are committed; nothing at test time reads the reference tree.
"""
import argparse
import functools
import os
import sys
import types

import ml_dtypes
import numpy as np


def _install_numpy_jax():
  """Modules named jax, jax.numpy, jax.nn, jax.lax, jax.experimental.pallas(.triton) backed by NumPy."""
  jnp = types.ModuleType("jax.numpy")
  for name in dir(np):
    if not name.startswith("_"):
      setattr(jnp, name, getattr(np, name))
  jnp.bfloat16 = ml_dtypes.bfloat16
  jnp.float8_e4m3fn = ml_dtypes.float8_e4m3fn
  jnp.bool_ = np.bool_

  nn = types.ModuleType("jax.nn")
  def softmax(x, axis=-1):
    m = np.max(x, axis=axis, keepdims=True)
    e = np.exp(x - m)
    return e / np.sum(e, axis=axis, keepdims=True)
  nn.softmax = softmax
  nn.sigmoid = lambda x: 1.0 / (1.0 + np.exp(-x))
  nn.relu = lambda x: np.maximum(x, 0)
  nn.swish = nn.silu = lambda x: x / (1.0 + np.exp(-x))

  lax = types.ModuleType("jax.lax")
  lax.rsqrt = lambda x: (1.0 / np.sqrt(x)).astype(np.asarray(x).dtype)

  class _CustomVjp:
    def __init__(self, fn, nondiff_argnums=()):
      self.fn = fn
      functools.update_wrapper(self, fn)
    def defvjp(self, fwd, bwd):
      pass
    def __call__(self, *a, **k):
      return self.fn(*a, **k)

  jax = types.ModuleType("jax")
  jax.numpy, jax.nn, jax.lax = jnp, nn, lax
  jax.jit = lambda fn=None, **kw: fn if fn is not None else (lambda f: f)
  jax.custom_vjp = _CustomVjp
  jax.ShapeDtypeStruct = lambda shape, dtype: (shape, dtype)
  jax.dtypes = types.SimpleNamespace(float0=np.dtype([("float0", np.void, 0)]))
  exp = types.ModuleType("jax.experimental")
  pallas = types.ModuleType("jax.experimental.pallas")
  triton = types.ModuleType("jax.experimental.pallas.triton")
  exp.pallas, pallas.triton = pallas, triton
  jax.experimental = exp
  sys.modules.update({"jax": jax, "jax.numpy": jnp, "jax.nn": nn, "jax.lax": lax, "jax.experimental": exp,
                      "jax.experimental.pallas": pallas, "jax.experimental.pallas.triton": triton})


def main():
  ap = argparse.ArgumentParser()
  ap.add_argument("--src", required=True, help="the `src` directory of a checkout of the reference (holds colabfold_kernels/)")
  ap.add_argument("--out", default=os.path.dirname(os.path.abspath(__file__)))
  args = ap.parse_args()
  _install_numpy_jax()
  sys.path.insert(0, args.src)
  from colabfold_kernels import contract, opm, packed_attn, transition, tri_flash, tri_mul

  f32 = np.float32
  def save(name, **arrays):
    np.savez_compressed(os.path.join(args.out, name + ".npz"), **arrays)
    print(name, {k: getattr(v, "shape", v) for k, v in arrays.items()})

  # --- attention: the shapes of tests/test_pallas_vjp.py:27-28, its mask and scale ------------
  for idx, (b, h, sq, sk, c) in enumerate(((2, 4, 96, 96, 32), (2, 4, 70, 83, 16), (1, 8, 64, 64, 48),
                                           (2, 2, 128, 128, 8), (1, 4, 96, 96, 96))):
    rng = np.random.default_rng(0)
    f = lambda *sh: (rng.standard_normal(sh) * .5).astype(f32)
    q, k, v, nb = f(b, h, sq, c), f(b, h, sk, c), f(b, h, sk, c), f(h, sq, sk)
    mb = np.where(rng.random((b, 1, 1, sk)) > .15, 0.0, -1e9).astype(f32)
    kmask = mb[:, 0, 0, :] > -1e3
    if idx == 0:
      kmask[1, :] = False   # a fully masked batch row: the uniform mean over Sk keys
    out = tri_flash.ref_attn(q, k, v, nb, kmask, float(c) ** -0.5)
    save(f"attn_{idx}", q=q, k=k, v=v, bias=nb, kmask=kmask, scale=f32(float(c) ** -0.5), out=out.astype(f32))

  # --- packed attention: rows/columns, gated/ungated, no bias, fully masked row, trim ----------
  rng = np.random.default_rng(0)
  f = lambda *sh, s=.5: (rng.standard_normal(sh) * s).astype(f32)
  for idx, (X, Y, H, D, gated, column, biased, trim) in enumerate((
      (16, 24, 4, 32, True, False, True, False), (24, 16, 4, 32, True, True, True, False),
      (9, 13, 2, 8, False, True, False, False), (5, 1, 4, 32, True, False, True, False),
      (12, 20, 2, 16, True, False, True, True))):
    G = 4 if gated else 3
    nbatch, s = (Y, X) if column else (X, Y)
    p = f(X, Y, G, H, D)
    bias = f(H, s, s) if biased else None
    kmask = rng.random((nbatch, s)) > .1
    kmask[nbatch // 2] = False
    if trim:
      kmask[:, s - 3:] = False
    gb = f(H, D) if gated else None
    out = packed_attn.ref_packed_attention(p, bias, kmask, gb, sm_scale=D ** -.5, column=column, trim=trim)
    extra = {} if bias is None else {"bias": bias}
    if gated:
      extra["gate_bias"] = gb
    save(f"packed_{idx}", p=p, kmask=kmask, scale=f32(D ** -.5), column=np.bool_(column), trim=np.bool_(trim),
         out=np.asarray(out, f32), **extra)

  # --- LayerNorm, GDP, LN->GDP, epilogue --------------------------------------------------------
  M, C, P = 77, 64, 128
  x, sc, of = f(M, C), 1 + f(C, s=.1), f(C, s=.1)
  save("layer_norm", x=x, scale=sc, offset=of, out=np.asarray(tri_mul.ref_layer_norm(x, sc, of, 1e-5), f32),
       out_ln=np.asarray(transition.ref_ln(x, sc, of, 1e-5), f32))
  wp, bp, wg, bg = f(C, P, s=C ** -.5), f(P, s=.1), f(C, P, s=C ** -.5), f(P, s=.1)
  mask = (rng.random(M) > .1).astype(f32)
  save("gdp", x=x, wp=wp, bp=bp, wg=wg, bg=bg, mask=mask, out=np.asarray(tri_mul.ref_gdp(x, wp, bp, wg, bg, mask), f32))
  l, r = tri_mul.ref_ln_gdp(x, sc, of, wp, bp, wg, bg, mask, eps=1e-5)
  save("ln_gdp_2d", x=x, scale=sc, offset=of, wp=wp, bp=bp, wg=wg, bg=bg, mask=mask, left=np.asarray(l, f32),
       right=np.asarray(r, f32))
  A, B = 11, 13
  xp = f(A, B, C)
  mp = (rng.random((A, B)) > .1).astype(f32)
  for tr in (False, True):
    l, r = tri_mul.ref_ln_gdp(xp, sc, of, wp, bp, wg, bg, mp, eps=1e-5, transpose=tr, pad=16)
    save(f"ln_gdp_pair_{int(tr)}", x=xp, scale=sc, offset=of, wp=wp, bp=bp, wg=wg, bg=bg, mask=mp,
         left=np.asarray(l, f32), right=np.asarray(r, f32))
  x_cm, act = f(C, M), f(M, C)
  wo, bo, wg2, bg2 = f(C, C, s=C ** -.5), f(C, s=.1), f(C, C, s=C ** -.5), f(C, s=.1)
  res = f(M, C)
  save("trimul_epilogue", x_cm=x_cm, act=act, scale=sc, offset=of, wo=wo, bo=bo, wg=wg2, bg=bg2, residual=res,
       out=np.asarray(tri_mul.ref_trimul_epilogue(x_cm, act, sc, of, wo, bo, wg2, bg2, eps=1e-5), f32),
       out_res=np.asarray(tri_mul.ref_trimul_epilogue(x_cm, act, sc, of, wo, bo, wg2, bg2, res, eps=1e-5), f32))
  in_sc, in_of = 1 + f(C, s=.1), f(C, s=.1)
  save("trimul_epilogue_ln", x_cm=x_cm, x=act, in_scale=in_sc, in_offset=in_of, scale=sc, offset=of, wo=wo, bo=bo,
       wg=wg2, bg=bg2,
       out=np.asarray(tri_mul.ref_trimul_epilogue_ln(x_cm, act, in_sc, in_of, sc, of, wo, bo, wg2, bg2, eps=1e-5,
                                                     add_input=True), f32))

  # --- contraction (the e4m3 operands are exact in float32) ------------------------------------
  a8 = np.asarray(np.clip(f(4, 24, 32, s=2.), -448, 448).astype(ml_dtypes.float8_e4m3fn))
  b8 = np.asarray(np.clip(f(4, 16, 32, s=2.), -448, 448).astype(ml_dtypes.float8_e4m3fn))
  save("fp8_contract", a=a8.astype(f32), b=b8.astype(f32), out=np.asarray(contract.ref_fp8_contract(a8, b8), f32))

  # --- projections around attention --------------------------------------------------------------
  a, n, G, h = 64, 32, 4, 4
  xq, w, wb = f(M, a), f(G, a, n, s=a ** -.5), f(a, h, s=a ** -.5)
  pq, bq = packed_attn.ref_ln_projection(xq, sc, of, w, wb, eps=1e-5)
  save("ln_projection", x=xq, scale=sc, offset=of, w=w, wb=wb, p=np.asarray(pq, f32), bias=np.asarray(bq, f32))
  o, wo2, bo2, res2 = f(M, 128), f(128, C, s=128 ** -.5), f(C, s=.1), f(M, C)
  save("output_projection", o=o, w=wo2, b=bo2, residual=res2,
       out=np.asarray(packed_attn.ref_output_projection(o, wo2, bo2, res2), f32))

  # --- outer product mean pieces, transition ----------------------------------------------------
  S, R, cm, k = 6, 10, 64, 16
  xm = f(S, R, cm)
  lw, lb, rw, rb = f(cm, k, s=cm ** -.5), f(k, s=.1), f(cm, k, s=cm ** -.5), f(k, s=.1)
  mm = (rng.random((S, R)) > .1).astype(f32)
  la, ra = opm.ref_opm_projection(xm, sc, of, lw, lb, rw, rb, mm, eps=1e-5)
  save("opm_projection", x=xm, scale=sc, offset=of, lw=lw, lb=lb, rw=rw, rb=rb, mask=mm,
       left=np.asarray(la, f32), right=np.asarray(ra, f32))
  left, right, w3 = f(16, 12, 16), f(16, 8, 16), f(256, 32, s=1 / 16)
  save("opm_outer", left=left, right=right, w=w3, out=np.asarray(opm.ref_opm_outer(left, right, w3), f32))
  lhs, t, bias3, norm, res3 = f(12, 64), f(64, 8, 32, s=.125), f(32, s=.1), rng.integers(0, 6, (12, 8)).astype(f32), f(12, 8, 32)
  save("opm_update", lhs=lhs, t=t, bias=bias3, norm=norm, residual=res3,
       out=np.asarray(opm.ref_opm_update(lhs, t, bias3, norm, res3, eps=1e-3), f32))
  w1, b1, w2, b2 = f(C, 4 * C, s=C ** -.5), f(4 * C, s=.1), f(4 * C, C, s=(4 * C) ** -.5), f(C, s=.1)
  save("transition", x=x, scale=sc, offset=of, w1=w1, b1=b1, w2=w2, b2=b2,
       out=np.asarray(transition.ref_transition(x, sc, of, w1, b1, w2, b2, eps=1e-5, add_input=True), f32))


if __name__ == "__main__":
  main()

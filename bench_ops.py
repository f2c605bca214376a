#!/usr/bin/env python
"""Per-operator timings of the fused Evoformer ops at the pair / MSA sizes of the configs (one JSON line per op).

  python bench_ops.py [--ops all|name,name] [--rows M] [--n N] [--iters K]

HBM-bound ops report GB/s of ALGORITHMIC bytes (every activation read once and written once) and the fraction of
the measured copy bandwidth; contraction-bound ops report TFLOP/s against the measured dense bf16 peak.  Inputs of
the default sizes are larger than the 126 MB L2, the host runs ahead of the device (one long sleep kernel first) so
that the events time kernels only.  `--rows` shrinks the row count for profiler captures.
"""
import argparse
import json
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "colabfold-kernels_b200"))
from colabfold_kernels import ops  # noqa: E402

bf = torch.bfloat16


def peaks():
  path = os.path.join(HERE, "MEASURED_PEAKS.json")
  if os.path.exists(path):
    d = json.load(open(path))
    return float(d["bf16_tflops"]), float(d["hbm_gbs"]), "measured"
  return 1590.0, 6650.0, "fallback"


def timed(fn, iters):
  for _ in range(3):
    fn()
  torch.cuda.synchronize()
  e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
  torch.cuda._sleep(int(4e7))  # lets the host queue every launch before the first one runs
  e0.record()
  for _ in range(iters):
    fn()
  e1.record()
  torch.cuda.synchronize()
  return e0.elapsed_time(e1) / iters


def make_cases(m, n, c=128):
  """name -> (callable, algorithmic bytes, flops).  m rows of c channels; n = residues of the contraction."""
  dev = "cuda"
  g = torch.Generator(device=dev).manual_seed(3)
  rnd = lambda *s: torch.randn(*s, device=dev, generator=g)
  x = rnd(m, c).to(bf)
  x_cm = rnd(c, m).to(bf)
  ones, zeros = torch.ones(c, device=dev), torch.zeros(c, device=dev)
  w = (rnd(c, c) * c ** -0.5).to(bf)
  b = torch.zeros(c, device=dev, dtype=bf)
  wp = (rnd(c, 2 * c) * c ** -0.5).to(bf)
  bp = torch.zeros(2 * c, device=dev, dtype=bf)
  w4 = (rnd(4, c, c) * c ** -0.5).to(bf)
  wbias = (rnd(c, 8) * c ** -0.5).to(bf)
  mask = (torch.rand(m, device=dev, generator=g) < 0.95).to(bf)
  res = rnd(m, c).to(bf)
  lw = (rnd(c, 32) * c ** -0.5).to(bf)
  lb = torch.zeros(32, device=dev, dtype=bf)
  a = rnd(c, n, n).to(bf)
  a2 = rnd(c, n, n).to(bf)
  a8, b8 = a.to(torch.float8_e4m3fn), a2.to(torch.float8_e4m3fn)
  E = 2  # bytes per bf16
  # triangle attention of the block: 4 heads of 32 over an [n, n] pair, packed q/k/v/gate
  h, d = 4, 32
  pk = rnd(n, n, 4, h, d).to(bf)
  tri_bias = rnd(h, n, n).to(bf)
  kmask = torch.rand(n, n, device=dev, generator=g) < 0.95
  gb = rnd(h, d).to(bf)
  qscale = torch.tensor([d ** -0.5 * 1.4426950408889634, 1.0], device=dev)
  qk8 = (pk[:, :, :2].float() * qscale[None, None, :, None, None]).clamp(-448, 448).to(torch.float8_e4m3fn)
  vg = pk[:, :, 2:].contiguous()
  # the block's two transitions: pair [m, 128] with 512 hidden, MSA [m / 2, 256] with 1024 hidden
  tw1 = (rnd(c, 4 * c) * c ** -0.5).to(bf)
  tw2 = (rnd(4 * c, c) * (4 * c) ** -0.5).to(bf)
  tb1, tb2 = torch.zeros(4 * c, device=dev, dtype=bf), torch.zeros(c, device=dev, dtype=bf)
  c2, m2 = 2 * c, m // 2
  x2 = rnd(m2, c2).to(bf)
  ones2, zeros2 = torch.ones(c2, device=dev), torch.zeros(c2, device=dev)
  uw1 = (rnd(c2, 4 * c2) * c2 ** -0.5).to(bf)
  w4m = (rnd(4, c2, c2) * c2 ** -0.5).to(bf)
  uw2 = (rnd(4 * c2, c2) * (4 * c2) ** -0.5).to(bf)
  ub1, ub2 = torch.zeros(4 * c2, device=dev, dtype=bf), torch.zeros(c2, device=dev, dtype=bf)
  # outer product mean at N_seq 512: projections of the MSA [512, n, 256] and the fused product / mean / output linear
  depth, cm = 512, 256
  msa = rnd(depth, n, cm).to(bf)
  ones_m, zeros_m = torch.ones(cm, device=dev), torch.zeros(cm, device=dev)
  ow = (rnd(cm, 32) * cm ** -0.5).to(bf)
  ob = torch.zeros(32, device=dev, dtype=bf)
  omask = (torch.rand(depth, n, device=dev, generator=g) < 0.95).to(bf)
  opm_w = (rnd(1024, c) / 32).to(bf)
  pair_res = rnd(n, n, c).to(bf)
  lcm, rcm = ops.opm_projection_cm(msa, ones_m, zeros_m, ow, ob, ow, ob, omask)
  opm_flops = 2.0 * n * n * 1024 * (depth + c)
  attn_flops = 4.0 * n * h * n * n * d
  attn_bytes = 5 * n * n * h * d * E + h * n * n * E + n * n
  return {
      "packed_attention": (lambda: ops.packed_attention_fwd(pk, tri_bias, kmask, gb, d ** -0.5), attn_bytes, attn_flops),
      "packed_attention_qk_e4m3": (lambda: ops.packed_attention_fwd(vg, tri_bias, kmask, gb, d ** -0.5, p8=qk8),
                                   attn_bytes - 2 * n * n * h * d, attn_flops),
      "layer_norm": (lambda: ops.layer_norm(x, ones, zeros), 2 * m * c * E, 0),
      "ln_gated_dual_proj": (lambda: ops.ln_gated_dual_proj(x, ones, zeros, wp, bp, wp, bp, mask), m * c * E + 2 * m * c * E + m * E,
                             2.0 * m * c * 4 * c),
      "ln_gated_dual_proj_e4m3": (lambda: ops.ln_gated_dual_proj(x, ones, zeros, wp, bp, wp, bp, mask, fp8=True),
                                  m * c * E + 2 * m * c + m * E, 2.0 * m * c * 4 * c),
      "gated_dual_proj": (lambda: ops.gated_dual_proj(x, wp, bp, wp, bp, mask), m * c * E + 2 * m * c * E + m * E, 2.0 * m * c * 4 * c),
      "trimul_epilogue": (lambda: ops.trimul_epilogue(x_cm, x, ones, zeros, w, b, w, b, in_scale=ones, in_offset=zeros, add_input=True),
                          3 * m * c * E, 4.0 * m * c * c),
      "ln_projection": (lambda: ops.ln_projection(x, ones, zeros, w4, None), m * c * E + 4 * m * c * E, 2.0 * m * c * 4 * c),
      "ln_projection_msa": (lambda: ops.ln_projection(x2, ones2, zeros2, w4m, None), m2 * c2 * E + 4 * m2 * c2 * E,
                            2.0 * m2 * c2 * 4 * c2),
      "ln_head_bias": (lambda: ops.ln_projection(x, ones, zeros, None, wbias), m * c * E + 8 * m * E, 2.0 * m * c * 8),
      "output_projection": (lambda: ops.output_projection(x, w, b, res), 3 * m * c * E, 2.0 * m * c * c),
      "opm_projection": (lambda: ops.opm_projection(x, ones, zeros, lw, lb, lw, lb, mask), m * c * E + 2 * m * 32 * E + m * E,
                         2.0 * m * c * 64),
      "transition_pair": (lambda: ops.transition(x, ones, zeros, tw1, tb1, tw2, tb2, add_input=True), 2 * m * c * E,
                          16.0 * m * c * c),
      "transition_msa": (lambda: ops.transition(x2, ones2, zeros2, uw1, ub1, uw2, ub2, add_input=True), 2 * m2 * c2 * E,
                         16.0 * m2 * c2 * c2),
      "opm_projection_cm": (lambda: ops.opm_projection_cm(msa, ones_m, zeros_m, ow, ob, ow, ob, omask),
                            depth * n * cm * E + 2 * depth * n * 32 * E + depth * n * E, 2.0 * depth * n * cm * 64),
      "outer_product_mean_fused": (lambda: ops.outer_product_mean_cm(lcm, rcm, omask, omask, opm_w, b, residual=pair_res),
                                   2 * depth * n * 32 * E + 2 * n * n * c * E, opm_flops),
      "contract_bf16": (lambda: ops.contract(a, a2), 3 * c * n * n * E, 2.0 * c * n ** 3),
      "contract_e4m3": (lambda: ops.contract(a8, b8), 2 * c * n * n + c * n * n * E, 2.0 * c * n ** 3),
  }


def main():
  ap = argparse.ArgumentParser()
  ap.add_argument("--ops", default="all")
  ap.add_argument("--rows", type=int, default=1048576, help="rows M of the [M, 128] activations (1024 x 1024 pair)")
  ap.add_argument("--n", type=int, default=1024, help="residues of the triangle contraction")
  ap.add_argument("--iters", type=int, default=20)
  args = ap.parse_args()
  if not torch.cuda.is_available():
    raise SystemExit("bench_ops.py needs a CUDA device: the library has no CPU path")
  peak_tf, peak_gb, kind = peaks()
  cases = make_cases(args.rows, args.n)
  names = list(cases) if args.ops == "all" else args.ops.split(",")
  for name in names:
    fn, nbytes, flops = cases[name]
    ms = timed(fn, args.iters)
    gbs, tfs = nbytes / ms / 1e6, flops / ms / 1e9
    tensor_bound = name.startswith(("contract", "packed_attention", "transition", "outer_product_mean"))
    print(json.dumps({
        "op": name, "rows": args.rows if not tensor_bound else None, "n": args.n if tensor_bound else None, "ms": round(ms, 4),
        "gb_per_s": round(gbs, 1), "tflop_per_s": round(tfs, 1), "bound": "tensor" if tensor_bound else "hbm",
        "frac_of_peak": round(tfs / peak_tf if tensor_bound else gbs / peak_gb, 4), "peak_source": kind,
        "device_status": ops.device_status()}), flush=True)


if __name__ == "__main__":
  main()

"""An ops namespace for colabfold_kernels.evoformer built on the CPU oracle (test infrastructure only).

The block wiring is not in the reference (it lives in ColabFold/AlphaFold): parity of the composition is
unpinned; each op it calls is the pinned restatement from reference_math."""
import types

import torch

from oracle import reference_math as R


def oracle_kernels(dtype=torch.float32):
  def ln_projection(x, ln_scale, ln_offset, w=None, wb=None, eps=1e-5):
    return R.ref_ln_projection(x, ln_scale, ln_offset, w, wb, eps=eps, dtype=dtype)

  def packed_attention(p, bias, kmask, gate_bias, sm_scale, column=False):
    return R.ref_packed_attention(p, bias, kmask, gate_bias, sm_scale=sm_scale, column=column, dtype=dtype)

  def output_projection(o, w, b, residual=None):
    return R.ref_output_projection(o, w, b, residual, dtype=dtype)

  def opm_projection(x, s, o, lw, lb, rw, rb, mask, eps=1e-5):
    return R.ref_opm_projection(x, s, o, lw, lb, rw, rb, mask, eps=eps, dtype=dtype)

  def outer_product_mean(left, right, mask_left, mask_right, w, bias, residual=None, eps=1e-3):
    out = R.ref_opm_outer(left, right, w, dtype) + bias.to(dtype)
    out = out / (eps + mask_left.to(dtype).T @ mask_right.to(dtype))[..., None]
    return out if residual is None else out + residual.to(dtype)

  def opm_projection_cm(x, s, o, lw, lb, rw, rb, mask, eps=1e-5):
    # x [depth, r, c] -> left, right [k, r, depth]: the projections channel-major with the MSA depth contiguous
    depth, r, c = x.shape
    left, right = R.ref_opm_projection(x.reshape(depth * r, c), s, o, lw, lb, rw, rb, mask.reshape(-1), eps=eps, dtype=dtype)
    return tuple(t.reshape(depth, r, -1).permute(2, 1, 0).contiguous() for t in (left, right))

  def outer_product_mean_cm(left_cm, right_cm, mask_left, mask_right, w, bias, residual=None, eps=1e-3):
    return outer_product_mean(left_cm.permute(2, 1, 0), right_cm.permute(2, 1, 0), mask_left, mask_right, w, bias, residual, eps)

  def ln_gated_dual_proj(x, s, o, wp, bp, wg, bg, mask, eps=1e-5, transpose=False, pad=1):
    return R.ref_ln_gdp(x, s, o, wp, bp, wg, bg, mask, eps=eps, transpose=transpose, pad=pad, dtype=dtype)

  def contract(a, b):
    return R.ref_contract(a, b, dtype)

  def contract_gathered(a, b_parts):  # b_parts [parts, c, j/parts, k]: the right operand as an all-gather leaves it
    return R.ref_contract(a, torch.cat(list(b_parts.unbind(0)), dim=1), dtype)

  def contract_exchanged(a_parts, b_parts, split_k=False):
    # the operands as an all-to-all over the channel axis leaves them: [P, c, i/P, k] (rows split) or [P, c, i, k/P]
    # (contracted axis split); the product as the all-to-all back wants it: [P, c, i/P, j]
    cat = (lambda t: torch.cat(list(t.unbind(0)), dim=2)) if split_k else (lambda t: torch.cat(list(t.unbind(0)), dim=1))
    out = R.ref_contract(cat(a_parts), cat(b_parts), dtype)
    return torch.stack(out.chunk(a_parts.shape[0], dim=1), dim=0)

  def trimul_epilogue(x_cm, act, ln_scale, ln_offset, wo, bo, wg, bg, residual=None, in_scale=None, in_offset=None,
                      eps=1e-5, add_input=False):
    if in_scale is None:
      return R.ref_trimul_epilogue(x_cm, act, ln_scale, ln_offset, wo, bo, wg, bg, residual, eps=eps, dtype=dtype)
    return R.ref_trimul_epilogue_ln(x_cm, act, in_scale, in_offset, ln_scale, ln_offset, wo, bo, wg, bg, eps=eps,
                                    add_input=add_input, dtype=dtype)

  def transition(x, ln, w1, b1, w2, b2):
    return R.ref_transition(x, ln[0], ln[1], w1, b1, w2, b2, add_input=True, dtype=dtype)

  return types.SimpleNamespace(ln_projection=ln_projection, packed_attention=packed_attention,
                               output_projection=output_projection, opm_projection=opm_projection,
                               outer_product_mean=outer_product_mean, opm_projection_cm=opm_projection_cm,
                               outer_product_mean_cm=outer_product_mean_cm, ln_gated_dual_proj=ln_gated_dual_proj,
                               contract=contract, contract_gathered=contract_gathered, contract_exchanged=contract_exchanged,
                               trimul_epilogue=trimul_epilogue, transition=transition)

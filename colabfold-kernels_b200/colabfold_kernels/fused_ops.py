"""Pick the fused kernel for each op: the reference's selector surface (src/colabfold_kernels/fused_ops.py)
over one backend, the B200 C library.  Every selector returns a callable with the reference's signature, or
None when the caller should run its own path (unsupported dtype/width, kernels switched off)."""
import functools

import torch

_HALF = (torch.bfloat16,)


def _norm_dtype(dtype):
  """torch dtypes, their names, and numpy/ml_dtypes/jax dtype objects all name a dtype here."""
  if isinstance(dtype, torch.dtype):
    return dtype
  name = getattr(dtype, "name", None) or getattr(dtype, "__name__", None) or str(dtype)
  return {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32,
          "float8_e4m3fn": torch.float8_e4m3fn}.get(name.replace("torch.", ""))


def _enabled(global_config):
  """Everything is off unless global_config['use_pallas'] is true (fused_ops.py:49,378,397); the Volta/Turing
  backend of the reference has no counterpart here."""
  if not global_config.get("use_pallas", False):
    return False
  if global_config.get("kernel_backend", "b200") == "cuda_legacy":
    return False
  from colabfold_kernels import _lib
  return _lib.available()


def register_ffi_targets(global_config):
  """Load the library eagerly, as the reference registers its FFI targets for models compiled ahead of time
  (fused_ops.py:17-32)."""
  if _enabled(global_config):
    from colabfold_kernels import _lib
    _lib.load()


def attention(global_config, dtype, key_dim, value_dim, layout="heads"):
  """-> f(q, k, v, mask_bias, nonbatched_bias, scale) or None (fused_ops.py:43-64).

  layout 'heads' takes q/k/v as [b, h, S, c], 'seq' as [b, S, h, c].  bfloat16 runs the tcgen05 kernels (head dim
  32 with a key count that is a multiple of 8) or the fp32-math kernels; float32 - which the reference declines -
  runs the fp32-math kernels, because its 1e-4 parity bound rules the tensor cores out."""
  dtype = _norm_dtype(dtype)
  if not _enabled(global_config) or dtype not in (torch.bfloat16, torch.float32):
    return None
  if key_dim != value_dim or key_dim > 128:
    return None
  from colabfold_kernels import grads
  return functools.partial(grads.attention, seq_major=(layout == "seq"))


def layer_norm(global_config, dtype):
  """-> f(x, scale, offset, *, eps) or None: last-axis LayerNorm (fused_ops.py:375-390)."""
  dtype = _norm_dtype(dtype)
  if not _enabled(global_config) or dtype not in (torch.bfloat16, torch.float32):
    return None
  from colabfold_kernels import grads
  return grads.layer_norm


def _half_ok(global_config, dtype):
  """The forward-only fused kernels run in bfloat16 (fused_ops.py:67-72 `_pallas_half`; float16 has no kernels here)."""
  return _enabled(global_config) and _norm_dtype(dtype) == torch.bfloat16


def _k_ok(k):
  return k in (64, 128, 256)


def fp8_attention(global_config, key_dim):
  """The k/v form of the e4m3 packed attention (fused_ops.py:75-80) is not this backend's: its kernel takes q and k
  (fp8_attention_slots), as the reference's Mosaic kernel does, so this answers False like there."""
  return False


LOG2E = 1.4426950408889634


def fp8_attention_slots(global_config, dtype, key_dim, seq_len):
  """(f8_slots, f8_scales) for the projection to write in e4m3 for packed_attention, or None (fused_ops.py:83-97):
  asked for by global_config.fp8 at the head dim the tensor-core kernel serves (32: one K = 32 step of the 8-bit
  MMA).  q (slot 0) is rounded after its static scale sm_scale * log2(e), k (slot 1) as it is."""
  if not global_config.get("fp8", False) or key_dim != 32:
    return None
  if dtype is not None and _norm_dtype(dtype) != torch.bfloat16:
    return None
  return (0, 1), (key_dim ** -0.5 * LOG2E, 1.0)


def half_attention(global_config):
  """The f16 softmax is an Ampere/Hopper tuning (fused_ops.py:142-149): off."""
  return False


def packed_attention(global_config, dtype, key_dim, value_dim):
  """-> f(p, bias, kmask, gate_bias, *, sm_scale, column) or None; p is the packed [X, Y, G, H, D] projection
  (fused_ops.py:152-178).  global_config.trim_padding selects the trim semantics."""
  if attention(global_config, dtype, key_dim, value_dim) is None or key_dim != value_dim:
    return None
  from colabfold_kernels import grads, ops
  trim = bool(global_config.get("trim_padding", False))

  def call(p, bias, kmask, gate_bias=None, p8=None, *, sm_scale, column=False):
    if p8 is not None:  # the e4m3 q.k form is forward only, like the reference's (fused_ops.py:122-136)
      return ops.packed_attention_fwd(p, bias, kmask, gate_bias, sm_scale, column=column, trim=trim, p8=p8)
    return grads.packed_attention(p, bias, kmask, gate_bias, sm_scale=sm_scale, column=column, trim=trim)
  return call


def gated_dual_proj(global_config, dtype, activation=None):
  """-> f(x, wp, bp, wg, bg, mask, *, split, channel_major) or None; activation None/'sigmoid' or 'swish'
  (fused_ops.py:393-413)."""
  if not _half_ok(global_config, dtype):
    return None
  name = getattr(activation, "__name__", activation)
  act = {None: 0, "sigmoid": 0, "swish": 1, "silu": 1}.get(name)
  if act is None:
    return None
  from colabfold_kernels import grads

  def call(x, wp, bp, wg, bg, mask, *, split=False, channel_major=False):
    if not _k_ok(x.shape[-1]):
      raise ValueError("gated_dual_proj: contracted width must be 64, 128 or 256")
    return grads.gated_dual_proj(x, wp, bp, wg, bg, mask, split=split, channel_major=channel_major, activation=act)
  return call


def ln_gated_dual_proj(global_config, dtype, num_channel, num_intermediate):
  """-> f(x, ln_scale, ln_offset, wp, bp, wg, bg, mask, *, eps, transpose) -> (left, right) channel major, or None
  (fused_ops.py:238-259)."""
  if not _half_ok(global_config, dtype) or not _k_ok(num_channel) or num_intermediate % 64 != 0:
    return None
  from colabfold_kernels import grads, ops, reference
  return grads.differentiable_via(ops.ln_gated_dual_proj, reference.ref_ln_gdp, nondiff=("eps", "transpose", "pad"))


def fp8_contraction(global_config, dtype, num_channel, num_intermediate, num_res):
  """-> (projection, contract) or None: the projection writing e4m3 halves padded to 16 and their contraction
  (fused_ops.py:262-275).  global_config.fp8_scale (default 1.0) is a per-tensor scale applied before rounding and
  undone by the contraction."""
  if not global_config.get("fp8", False) or num_res % 8 != 0:
    return None
  if ln_gated_dual_proj(global_config, dtype, num_channel, num_intermediate) is None:
    return None
  from colabfold_kernels import grads, ops, reference
  # per-tensor scale of the e4m3 operands (global_config.fp8_scale, default 1.0 = the reference's unscaled cast,
  # tri_mul.py:228): the projection rounds value * scale, the contraction multiplies by 1 / scale^2
  scale = float(global_config.get("fp8_scale", 1.0))
  proj = grads.differentiable_via(functools.partial(ops.ln_gated_dual_proj, fp8=True, pad=16, fp8_scale=scale),
                                  functools.partial(reference.ref_ln_gdp, pad=16), nondiff=("eps", "transpose"))
  return proj, grads.differentiable_via(functools.partial(ops.contract, alpha=1.0 / (scale * scale)), reference.ref_contract)


def contraction(global_config, dtype):
  """-> f(a, b) -> [C, I, J] bf16 for a [C, I, K], b [C, J, K], or None.  The reference leaves the bf16 contraction
  to XLA's batched GEMM (tri_mul.py:6-7); here it is a kernel of the library."""
  if not _half_ok(global_config, dtype):
    return None
  from colabfold_kernels import grads, ops, reference
  return grads.differentiable_via(ops.contract, reference.ref_contract)


def trimul_epilogue(global_config, dtype):
  """-> f(x_cm, act, ln_scale, ln_offset, wo, bo, wg, bg, residual=None, *, eps) or None (fused_ops.py:212-218)."""
  if not _half_ok(global_config, dtype):
    return None
  from colabfold_kernels import grads, ops, reference
  return grads.differentiable_via(ops.trimul_epilogue, reference.ref_trimul_epilogue, nondiff=("eps",))


def trimul_epilogue_ln(global_config, dtype):
  """-> f(x_cm, x, in_scale, in_offset, ln_scale, ln_offset, wo, bo, wg, bg, *, eps, add_input) or None
  (fused_ops.py:221-235)."""
  if not _half_ok(global_config, dtype):
    return None
  from colabfold_kernels import grads, ops, reference

  def fwd(x_cm, x, in_scale, in_offset, ln_scale, ln_offset, wo, bo, wg, bg, keep=None, *, eps=1e-5, add_input=False):
    return ops.trimul_epilogue(x_cm, x, ln_scale, ln_offset, wo, bo, wg, bg, in_scale=in_scale, in_offset=in_offset,
                               eps=eps, add_input=add_input, keep=keep)
  return grads.differentiable_via(fwd, reference.ref_trimul_epilogue_ln, nondiff=("eps", "add_input"))


def ln_projection(global_config, dtype, num_channel, num_output=None):
  """-> f(x, ln_scale, ln_offset, w, wb, *, eps) -> (p, bias) or None (fused_ops.py:278-304)."""
  if not _half_ok(global_config, dtype) or not _k_ok(num_channel):
    return None
  if num_output is not None and num_output % 64 != 0:
    return None
  from colabfold_kernels import grads, ops, reference

  def fwd(x, ln_scale, ln_offset, w=None, wb=None, keep=None, *, eps=1e-5):
    return ops.ln_projection(x, ln_scale, ln_offset, w, wb, eps=eps, keep=keep)
  diff = grads.differentiable_via(fwd, reference.ref_ln_projection, nondiff=("eps",))

  def call(x, ln_scale, ln_offset, w=None, wb=None, keep=None, *, eps=1e-5, f8_slots=(), f8_scales=None):
    if f8_slots:  # -> (p, bias, p8): the e4m3 slots feed the forward-only FP8 attention
      return ops.ln_projection(x, ln_scale, ln_offset, w, wb, eps=eps, keep=keep, f8_slots=f8_slots, f8_scales=f8_scales)
    return diff(x, ln_scale, ln_offset, w, wb, keep, eps=eps)
  return call


def output_projection(global_config, dtype, num_input, num_output):
  """-> f(o, w, b, residual=None, keep=None) or None (fused_ops.py:307-323)."""
  if not _half_ok(global_config, dtype) or not _k_ok(num_input) or num_output % 8 != 0:
    return None
  from colabfold_kernels import grads, ops, reference

  def fwd(o, w, b, residual=None, keep=None):
    return ops.output_projection(o, w, b, residual, keep=keep)
  return grads.differentiable_via(fwd, reference.ref_output_projection)


def opm_projection(global_config, dtype, num_channel, num_outer):
  """-> f(x, ln_scale, ln_offset, lw, lb, rw, rb, mask, *, eps) -> (left_act, right_act) or None (fused_ops.py:364-372)."""
  if not _half_ok(global_config, dtype) or not _k_ok(num_channel) or num_outer % 8 != 0 or num_outer > 128:
    return None
  from colabfold_kernels import grads, ops, reference
  return grads.differentiable_via(ops.opm_projection, reference.ref_opm_projection, nondiff=("eps",))


def opm_update(global_config, dtype, num_inner, num_output):
  """-> f(lhs, t, bias, norm, residual=None, *, eps) or None: the shallow outer product mean's whole pair update
  (fused_ops.py:326-342): one tensor-core GEMM and the normalising tail.  Widths as the reference's `supported`
  (opm.py:88-90): K a multiple of 32, F a power of two from 16 to 128."""
  if not _half_ok(global_config, dtype):
    return None
  if num_inner % 32 != 0 or num_output & (num_output - 1) or not 16 <= num_output <= 128:
    return None
  from colabfold_kernels import grads, ops, reference
  return grads.differentiable_via(ops.opm_update, reference.ref_opm_update, nondiff=("eps",))


def opm_outer(global_config, dtype, rows, num_inner, d, num_output):
  """-> f(left, right, w) or None: the outer product mean in AF2's own order on 16 rows (fused_ops.py:345-361): the rows'
  outer product (stored by the contraction kernel in the layout the output weights read), then w.  Shapes as the
  reference's `outer_supported` (opm.py:142-144)."""
  if not _half_ok(global_config, dtype):
    return None
  if rows != 16 or num_inner % 16 != 0 or d % 4 != 0 or num_output & (num_output - 1) or not 16 <= num_output <= 128:
    return None
  from colabfold_kernels import grads, ops, reference
  return grads.differentiable_via(ops.opm_outer, reference.ref_opm_outer)


def transition(global_config, dtype, num_channel, num_intermediate):
  """-> f(x, ln_scale, ln_offset, w1, b1, w2, b2, keep=None, *, eps, add_input) or None: the LN-MLP transition
  (fused_ops.py:181-198).  LayerNorm -> first GEMM -> bias -> relu is one kernel of the library; the second GEMM with
  its bias and the residual is the library GEMM."""
  if not _half_ok(global_config, dtype) or not _k_ok(num_channel) or num_intermediate % 64 != 0:
    return None
  from colabfold_kernels import grads, ops, reference
  return grads.differentiable_via(ops.transition, reference.ref_transition, nondiff=("eps", "add_input"))


def glu_transition(global_config, dtype, num_channel, num_intermediate):
  """AF3's swish-GLU transition (fused_ops.py:201-209) is outside the Evoformer path: None."""
  return None

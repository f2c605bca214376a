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

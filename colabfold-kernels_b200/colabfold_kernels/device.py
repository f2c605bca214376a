"""What the GPU here can run (mirrors src/colabfold_kernels/device.py of the reference, NVIDIA B200 only)."""
import functools


def compute_capability():
  """The compute capability as an integer, e.g. 100 on a B200, or None without a CUDA device (device.py:5-13)."""
  try:
    import torch
    if not torch.cuda.is_available():
      return None
    major, minor = torch.cuda.get_device_capability()
    return major * 10 + minor
  except Exception:
    return None


def is_rocm():
  """Always False: this build targets sm_100a only (device.py:16-20)."""
  return False


@functools.lru_cache(maxsize=None)
def l2_cache_size():
  """The GPU's L2 in bytes, or None (device.py:23-32)."""
  try:
    import torch
    return int(torch.cuda.get_device_properties(torch.cuda.current_device()).L2_cache_size)
  except Exception:
    return None


def shared_memory_limit():
  """The opt-in shared memory per block in bytes, or None (device.py:35-41)."""
  try:
    import torch
    props = torch.cuda.get_device_properties(torch.cuda.current_device())
    return int(getattr(props, "shared_memory_per_block_optin", 0)) or None
  except Exception:
    return None


def dispatch(backend="auto"):
  """The mapping the fused_ops selectors read (device.py:44-50).  'auto' selects the B200 library when the
  device is compute capability 10.x and the library loads; the keys are the reference's."""
  cc = compute_capability()
  if backend == "auto":
    backend = "b200"
  return {"use_pallas": True, "kernel_backend": backend, "compute_capability": cc}

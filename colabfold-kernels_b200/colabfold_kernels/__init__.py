"""B200-native kernels for ColabFold's Evoformer hot path behind colabfold-kernels' selector API
(src/colabfold_kernels/__init__.py:3-9 of the reference)."""

from colabfold_kernels.device import compute_capability, dispatch, shared_memory_limit
from colabfold_kernels.fused_ops import attention, gated_dual_proj, layer_norm

__all__ = ["attention", "compute_capability", "dispatch", "gated_dual_proj", "layer_norm", "shared_memory_limit",
           "__version__"]

__version__ = "0.9.0+b200"

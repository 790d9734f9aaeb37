"""B200-native SMO / SMO8bit optimizer step (drop-in for mcarbonell/smo-optimizer).

``from smo_optimizer_b200 import SMO, SMO8bit`` gives torch.optim.Optimizer
classes with the reference's constructor arguments and state layout whose
step runs as hand-written sm_100a CUDA kernels (libsmo_b200.so).
"""

from ._host import MIN_SPATIAL_DIM, compression_view
from .optimizers import SMO, SMO8bit, protected_param_groups

# The reference exports Triton variants behind these flags; this build has no
# Triton path.
HAS_TRITON = False
HAS_TRITON_SPATIAL = False

__all__ = ["SMO", "SMO8bit", "MIN_SPATIAL_DIM", "compression_view", "protected_param_groups",
           "HAS_TRITON", "HAS_TRITON_SPATIAL"]

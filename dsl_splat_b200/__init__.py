"""dsl_splat_b200: a B200-native drop-in for dsl_splat's gs3d, RaDe-GS and
AAA-Gaussians rasterisers.

`dsl_splat_b200.gs3d.rasterize`, `dsl_splat_b200.rade.rasterize`,
`dsl_splat_b200.aaa.rasterize` and their `gsplat.rasterization` adapters keep
dsl_splat's signatures; the compute path
is libsplat200.so (hand-written CUDA for sm_100a) reached through the C ABI
in include/splat200.h.
"""

from .cameras import PinholeCamera
from .statistics import MaskedContributionCount, WeightedContributionSum
from . import aaa
from . import gs3d
from . import rade
from . import torch_ops  # registers torch.ops.splat200.*

__all__ = ["aaa", "gs3d", "rade", "torch_ops", "PinholeCamera", "MaskedContributionCount",
           "WeightedContributionSum"]

"""AAA-Gaussians on the sm_100a kernels (dsl_splat/aaa): adaptive 3D
antialiasing, 3D ray evaluation and StopThePop hierarchical (HIER 64/8/4)
per-tile sorting, forward and backward."""

from . import gsplat, ops, stages
from .api import RasterizationResult, rasterize
from .config import default_settings, validate_settings
from .settings import ExtendedSettings

__all__ = ["rasterize", "RasterizationResult", "default_settings", "validate_settings",
           "ExtendedSettings", "gsplat", "ops", "stages"]

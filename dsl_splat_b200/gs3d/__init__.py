"""Original 3D Gaussian Splatting on hand-written sm_100a kernels (gs3d/__init__.py)."""

from . import ops
from .api import RasterizationResult, rasterize

__all__ = ["rasterize", "RasterizationResult", "ops"]

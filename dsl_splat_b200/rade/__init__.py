"""RaDe-GS (rade/__init__.py) on the sm_100a kernels: ray-plane expected and
median depth, camera-space normals and radial sorting, behind the reference's
rasterize / ops / gsplat interfaces."""

from . import ops
from .api import RasterizationResult, rasterize
from .filtering import apply_3d_filter

__all__ = ["rasterize", "RasterizationResult", "apply_3d_filter", "ops"]

"""AAA's recommended configuration and its validation (aaa/config.py:41-65)."""

from __future__ import annotations

from .settings import (CullingSettings, ExtendedSettings, GlobalSortOrder, SortMode,
                       SortSettings)


def default_settings(*, antialiased: bool = True) -> ExtendedSettings:
    """eval_3D, HIER 64/8/4, PTD_MAX order, load balancing and every culling
    stage; antialiased selects the EWA opacity compensation."""
    return ExtendedSettings(
        sort_settings=SortSettings(sort_mode=SortMode.HIER, sort_order=GlobalSortOrder.PTD_MAX),
        culling_settings=CullingSettings(True, True, True, True),
        load_balancing=True, proper_ewa_scaling=antialiased, eval_3D=True, new_aabb=True)


def validate_settings(settings: ExtendedSettings) -> None:
    """The algorithm both differentiable entry points implement."""
    if not isinstance(settings, ExtendedSettings):
        raise ValueError("settings must be ExtendedSettings")
    if not settings.eval_3D or int(settings.sort_settings.sort_mode) != 3:
        raise ValueError("settings must use eval_3D=True and HIER sorting")
    queues = settings.sort_settings.queue_sizes
    if (queues.tile_4x4, queues.tile_2x2, queues.per_pixel) != (64, 8, 4):
        raise ValueError("settings require HIER queue sizes 64/8/4")


__all__ = ["default_settings", "validate_settings"]

"""ctypes binding of libsplat200.so (the C ABI declared in include/splat200.h).

The library is the only compute path: importing this module fails loudly when
the shared object is missing or lacks a symbol, and every call raises
RuntimeError on a non-zero status.  There is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsplat200.so")

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_Z = ctypes.c_size_t
_L = ctypes.c_longlong
_U = ctypes.c_uint

# name -> (restype, argtypes)
SIGNATURES: dict[str, tuple] = {
    "splat_abi_version": (_I, []),
    "splat_last_error": (ctypes.c_char_p, []),
    "splat_launch_count": (ctypes.c_ulonglong, []),
    "splat_device_error": (_I, [_P, _P]),
    "splat_device_error_read": (_I, [_P, _P]),
    "splat_test_lookback_expiry": (_I, [_P, _U, _P, _P]),
    "splat_test_trig": (_I, [_I, _P, _P, _P, _P, _P]),
    "splat_cameras_prepare": (_I, [_I, _P, _P, _I, _I, _I, _P, _P, _P, _P, _P]),
    "splat_cameras_backward": (_I, [_I, _P, _P, _I, _I, _P, _P, _P, _P]),
    "splat_project_forward": (_I, [_I, _P, _P, _P, _P, _P, _P, _P, _I, _I, _F, _F, _F,
                                   _P, _P, _P, _P, _P, _I, _P]),
    "splat_project_forward_fused": (_I, [_I, _P, _P, _I, _P, _P, _P, _P, _P, _I, _I, _F, _F, _F,
                                         _P, _P, _P, _P, _P, _I, _I, _P, _P, _P, _I, _P,
                                         _P, _P, _P, _I, _P]),
    "splat_project_forward_views": (_I, [_I, _I, _P, _P, _I, _P, _P, _P, _P, _P, _I, _I, _F,
                                         _F, _F, _P, _P, _P, _P, _P, _I, _I, _P, _P, _P, _I,
                                         _P, _P, _P, _P, _I, _P]),
    "splat_metadata": (_I, [_I, _P, _P, _P, _P, _P, _P, _P]),
    "splat_project_backward": (_I, [_I, _P, _P, _P, _P, _P, _P, _I, _I, _P, _P, _P, _P, _P,
                                    _P, _P, _P, _P]),
    "splat_project_backward_fused": (_I, [_I, _P, _P, _P, _P, _P, _P, _P, _I, _I, _P, _P, _P,
                                          _P, _P, _P, _P, _I, _P, _I, _I, _P, _P, _P, _P,
                                          _I, _P, _P]),
    "splat_project_backward_views": (_I, [_I, _I, _P, _P, _P, _P, _P, _P, _P, _I, _I, _P, _P,
                                          _P, _P, _P, _P, _P, _I, _I, _I, _P, _P, _P, _P, _I,
                                          _P, _P]),
    "splat_sh_forward": (_I, [_I, _I, _I, _P, _P, _P, _P, _P, _P]),
    "splat_sh_backward": (_I, [_I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P]),
    "splat_scan_workspace_bytes": (_Z, [_I]),
    "splat_scan_counts": (_I, [_I, _P, _P, _P, _P, _Z, _P]),
    "splat_scan_counts_static": (_I, [_I, _P, _P, _P, _P]),
    "splat_bin_workspace_bytes": (_Z, [_I, _I, _I, _I]),
    "splat_bin_pairs_workspace_bytes": (_Z, [_L, _I, _I, _I]),
    "splat_bin_prepare": (_I, [_I, _P, _P, _P, _P, _P, _I, _I, _I, _P, _Z, _P, _P, _P]),
    "splat_bin_emit": (_I, [_I, _L, _I, _I, _I, _P, _P, _P, _P, _Z, _P, _Z, _P, _P]),
    "splat_tile_order": (_I, [_P, _I, _P, _P]),
    "splat_render_forward": (_I, [_I, _I, _P, _P, _L, _I, _P, _P, _P, _I, _I, _P, _I, _I, _I,
                                  _P, _P, _I, _I, _P, _P, _P, _P, _P]),
    "splat_render_forward_statistics": (_I, [_I, _I, _P, _P, _L, _I, _P, _P, _P, _I, _I, _P,
                                             _I, _I, _I, _P, _P, _I, _I, _P, _P, _P, _I, _I,
                                             _P, _P, _P, _P, _P]),
    "splat_render_backward": (_I, [_I, _I, _P, _P, _L, _I, _P, _P, _P, _I, _I, _P, _I, _I, _I,
                                   _P, _P, _P, _P, _I, _I, _P, _I, _P, _P, _P, _P, _P, _I,
                                   _P, _P]),
    "splat_rade_project_forward": (_I, [_I, _P, _P, _I, _P, _P, _P, _P, _P, _I, _I, _F, _F, _F,
                                        _F, _P, _P, _P, _P, _P, _P, _P, _I, _I, _P, _P, _P,
                                        _P, _P, _P, _P, _P]),
    "splat_rade_project_backward": (_I, [_I, _P, _P, _I, _P, _P, _P, _P, _P, _I, _I, _F, _P,
                                         _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _P,
                                         _P, _P, _P, _P, _P, _P]),
    "splat_rade_render_forward": (_I, [_I, _I, _P, _P, _L, _I, _P, _P, _P, _P, _P, _I, _I, _P,
                                       _I, _I, _P, _P, _P, _I, _I, _P, _I, _P, _I, _P, _I,
                                       _P, _I, _I, _P, _P, _I, _I, _P, _P, _P, _P, _P]),
    "splat_rade_render_backward": (_I, [_I, _I, _P, _P, _L, _I, _P, _P, _P, _P, _P, _I, _I,
                                        _P, _I, _I, _P, _P, _P, _I, _P, _I, _I, _P, _P, _P,
                                        _I, _I, _P, _I, _I, _P, _I, _P, _I, _P, _I, _P, _I,
                                        _I, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "splat_debug_expf": (_I, [_I, _P, _P, _P, _P]),
    "splat_aaa_preprocess": (_I, [_P] + [_P] * 12 + [_P]),
    "splat_aaa_cull_remainder": (_I, [_I, _P, _P, _P, _P, _P, _P, _I, _I, _P, _P, _P, _P]),
    "splat_aaa_bin_workspace_bytes": (_Z, [_L]),
    "splat_aaa_bin": (_I, [_I, _L, _P, _P, _P, _P, _P, _P, _I, _I, _P, _Z, _P, _P, _P]),
    "splat_aaa_emit": (_I, [_I, _L, _P, _P, _P, _P, _P, _P, _I, _I, _P, _P, _P, _P]),
    "splat_aaa_render": (_I, [_I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                              _I, _P, _P, _P, _I, _I, _P, _P, _P, _P]),
    "splat_aaa_record_bytes": (_Z, [_I, _I, _I]),
    "splat_aaa_metadata": (_I, [_I, _P, _F, _F, _F, _F, _P, _P, _P, _P, _P, _P, _P, _P]),
    "splat_aaa_render_backward": (_I, [_I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                       _P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _P]),
    "splat_aaa_preprocess_backward": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "splat_aaa_camera_backward": (_I, [_P, _P, _P, _P, _P, _P, _P]),
}


class SplatAaaFrame(ctypes.Structure):
    """include/splat200.h SplatAaaFrame: one AAA view's inputs (device
    pointers) and switches."""

    _fields_ = [("n", _I), ("width", _I), ("height", _I),
                ("means", _P), ("scales", _P), ("quats", _P), ("opacities", _P),
                ("sh", _P), ("sh_k", _I), ("sh_degree", _I), ("filters", _P),
                ("campos", _P), ("view", _P), ("proj", _P),
                ("tanfov_x", _F), ("tanfov_y", _F), ("principal_x", _F), ("principal_y", _F),
                ("scale_modifier", _F), ("focal_x", _F), ("focal_max", _F),
                ("sort_order", _I), ("ewa", _I), ("new_aabb", _I), ("near_clipping", _I),
                ("tile_culling", _I), ("complete", _I), ("cooperative", _I),
                ("normalize_quats", _I)]


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"libsplat200.so not found at {LIB_PATH}; build it with "
            "`python dsl_splat_b200/build.py` (nvcc, sm_100a)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)  # AttributeError -> missing symbol: fail loudly
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


lib = _load()


class SplatError(RuntimeError):
    pass


def check(status: int, what: str) -> None:
    if status != 0:
        msg = lib.splat_last_error().decode(errors="replace")
        raise SplatError(f"{what} failed with status {status}: {msg}")


def ptr(t: torch.Tensor | None) -> int | None:
    """Device address of a tensor (None -> NULL)."""
    if t is None:
        return None
    return t.data_ptr()


def stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")


def device_error(device: torch.device) -> int:
    code = ctypes.c_int(0)
    with torch.cuda.device(device):
        check(lib.splat_device_error(ctypes.addressof(code), stream(device)), "splat_device_error")
    return code.value

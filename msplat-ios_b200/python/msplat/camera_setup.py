"""Camera setup through the library (Model::prepareCam in C++)."""
from __future__ import annotations

import ctypes as C

import numpy as np


def prepare_cam(B, cam_to_world, fx, fy, cx, cy, width, height):
    """MsplatCamera for an OpenGL camToWorld matrix (msplat_prepare_camera)."""
    L = B.load()
    if not getattr(L, "_prep_typed", False):
        L.msplat_prepare_camera.argtypes = [C.POINTER(C.c_float), C.c_float, C.c_float, C.c_float, C.c_float,
                                            C.c_int32, C.c_int32, C.POINTER(B.MsplatCamera)]
        L.msplat_prepare_camera.restype = C.c_int
        L._prep_typed = True
    m = np.ascontiguousarray(np.asarray(cam_to_world, np.float32).reshape(16))
    cam = B.MsplatCamera()
    code = L.msplat_prepare_camera(m.ctypes.data_as(C.POINTER(C.c_float)), fx, fy, cx, cy, width, height,
                                   C.byref(cam))
    B._check(code)
    return cam

"""The C-ABI library loads without a GPU and exports every entry point that
include/*.h declares (no compute calls)."""
import ctypes
import os
import re

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INCLUDE = os.path.join(REPO, "include")


def declared_functions():
    names = set()
    for f in os.listdir(INCLUDE):
        if not f.endswith(".h"):
            continue
        src = open(os.path.join(INCLUDE, f)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        src = re.sub(r"//[^\n]*", "", src)
        inline = set(re.findall(r"static\s+inline\s+\w+\s+(msplat_[A-Za-z0-9_]+)\s*\(", src))
        for m in re.finditer(r"\b(msplat_[A-Za-z0-9_]+)\s*\(", src):
            if m.group(1) not in inline:  # header-only helpers (msplat_default_config)
                names.add(m.group(1))
    return sorted(names)


def test_headers_declare_entry_points():
    names = declared_functions()
    for must in ("msplat_render", "msplat_train_step_2dgs", "msplat_fused_adam", "msplat_train_step_fused",
                 "msplat_last_tensor", "msplat_last_error", "msplat_prepare_camera", "msplat_trainer_step",
                 "msplat_trainer_create", "msplat_dataset_create", "msplat_trainer_render_pose_to_buffer"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from msplat import _backend as B
    if not os.path.exists(B.LIB_PATH):
        pytest.fail("libmsplat_b200.so is not built (run python msplat-ios_b200/build.py)")
    lib = ctypes.CDLL(B.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_host_only_entry_points_work_without_gpu():
    from msplat import _backend as B
    import numpy as np
    cam = B.prepare_camera(np.eye(4, dtype=np.float32), 100.0, 100.0, 32.0, 24.0, 64, 48)
    assert cam.width == 64 and cam.height == 48
    # identity camToWorld: the OpenGL->OpenCV flip makes the clip w = -z_world
    assert abs(cam.projmat[15]) < 1e-6 and cam.projmat[14] == -1.0
    with pytest.raises(B.MsplatError):
        B.prepare_camera(np.eye(4, dtype=np.float32), -1.0, 100.0, 32.0, 24.0, 64, 48)

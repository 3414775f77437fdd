"""The fixed tables of the path against values captured from the reference
itself (tests/golden/ref_constants.json, made by make_ref_constants.py): the SH
basis constants and the 11-tap SSIM window of core/metal/msplat_metal.metal,
and the 11x11 window that the reference's own C++ (core/src/ssim.cpp
createSSIMWindow, built from its sources) computes. The CUDA sources
(sh_math.cuh, ssim_loss.cu) and the CPU checker (oracle.cpp) must hold the
same float32 values bit for bit; the separable window's outer product must
equal the reference C++ window to float rounding."""
import json
import os
import re
import struct

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = json.load(open(os.path.join(REPO, "tests", "golden", "ref_constants.json")))


def f32(x: float) -> float:
    return struct.unpack("f", struct.pack("f", x))[0]


def table(src: str, name: str):
    m = re.search(r"\b%s\[\d*\]\s*=\s*\{([^}]*)\}" % name, src)
    assert m, name
    return [f32(float(v.strip().rstrip("f"))) for v in m.group(1).split(",") if v.strip()]


def scalar(src: str, name: str):
    m = re.search(r"\b%s\s*=\s*([-0-9.e]+)f;" % name, src)
    assert m, name
    return f32(float(m.group(1)))


def _src(*parts):
    return open(os.path.join(REPO, *parts)).read()


def test_sh_constants_match_the_reference():
    for src in (_src("msplat-ios_b200", "csrc", "sh_math.cuh"), _src("oracle", "oracle.cpp")):
        assert scalar(src, "SH_C0") == REF["SH_C0"]
        assert scalar(src, "SH_C1") == REF["SH_C1"]
        assert table(src, "SH_C2") == REF["SH_C2"]
        assert table(src, "SH_C3") == REF["SH_C3"]


def test_ssim_window_matches_the_reference():
    assert table(_src("msplat-ios_b200", "csrc", "ssim_loss.cu"), "kW") == REF["SSIM_GAUSS_KERNEL"]
    assert table(_src("oracle", "oracle.cpp"), "kSsimW") == REF["SSIM_GAUSS_KERNEL"]
    g = np.array(REF["SSIM_GAUSS_KERNEL"], np.float32)
    w2 = np.outer(g, g).astype(np.float32).ravel()
    cpp = np.array(REF["ssim_window_cpp"], np.float32)
    assert cpp.size == 121
    np.testing.assert_allclose(w2, cpp, rtol=2e-6, atol=0)
    assert abs(float(g.astype(np.float64).sum()) - 1.0) < 1e-6

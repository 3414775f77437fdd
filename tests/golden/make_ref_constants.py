"""Generates tests/golden/ref_constants.json from the reference itself (run in
the container that holds the reference sources; the committed fixture is what
the tests read):

* SH_C0, SH_C1, SH_C2[5], SH_C3[7] and SSIM_GAUSS_KERNEL[11], parsed from
  core/metal/msplat_metal.metal (:19-44, :2804-2816) as float32 values;
* the 11x11 SSIM window of core/src/ssim.cpp createSSIMWindow (:7-24),
  computed by the reference's own C++ built by `make -C oracle ref`
  (oracle/_ref/ssim_window).

    python tests/golden/make_ref_constants.py [/path/to/reference]
"""
import json
import os
import re
import struct
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def f32(x: float) -> float:
    return struct.unpack("f", struct.pack("f", x))[0]


def parse_metal(src: str):
    out = {}
    for name in ("SH_C0", "SH_C1"):
        m = re.search(r"constant float %s = ([-0-9.e]+)f?;" % name, src)
        out[name] = f32(float(m.group(1)))
    for name in ("SH_C2", "SH_C3", "SSIM_GAUSS_KERNEL"):
        m = re.search(r"constant float %s\[\d*\] = \{([^}]*)\}" % name, src)
        out[name] = [f32(float(v.strip().rstrip("f"))) for v in m.group(1).split(",") if v.strip()]
    return out


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else "/root/reference"
    src = open(os.path.join(ref, "core", "metal", "msplat_metal.metal")).read()
    consts = parse_metal(src)
    subprocess.run(["make", "-s", "-C", os.path.join(REPO, "oracle"), "ref", f"REF={ref}"], check=True)
    lines = subprocess.run([os.path.join(REPO, "oracle", "_ref", "ssim_window")], capture_output=True, text=True,
                           check=True).stdout.split()
    consts["ssim_window_cpp"] = [float.fromhex(v) for v in lines]
    consts["source"] = ("core/metal/msplat_metal.metal:19-44 (SH constants), :2804-2816 (SSIM_GAUSS_KERNEL); "
                        "core/src/ssim.cpp:7-24 createSSIMWindow(11, 1.5) run from the reference's C++")
    json.dump(consts, open(os.path.join(HERE, "ref_constants.json"), "w"), indent=1)
    print("wrote", os.path.join(HERE, "ref_constants.json"))


if __name__ == "__main__":
    main()

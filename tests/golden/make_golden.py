"""Generates tests/golden/golden_small.npz with the CPU oracle.

    python tests/golden/make_golden.py

Inputs are regenerated from a seed with msplat.synthetic (numpy's PCG64), so
the fixture only stores outputs: projection results, tile bins and the sorted
per-tile order, the rendered image and side outputs, loss, all per-group
gradients and the parameters after one Adam step. test_golden.py checks the
oracle (CPU) and the CUDA path (GPU) against it.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "msplat-ios_b200", "python"))

from msplat import synthetic as S  # noqa: E402
from oracle import oracle as O  # noqa: E402

CFG = S.small_config(1_000, 3, 80, 56, focal=70.0, num_cameras=2)
SEED = 0


def case():
    scene = S.make_scene(CFG, seed=SEED)
    fx, fy, cx, cy = scene.intrinsics
    cam = O.prepare_cam(scene.cam_to_world[1], fx, fy, cx, cy, CFG.width, CFG.height)
    gt = O.render(scene.jittered().params(), CFG.degree, CFG.degree, S.BACKGROUND, cam)
    return scene, cam, gt


def compute():
    scene, cam, gt = case()
    p = O.project_forward(*scene.params(), CFG.degree, CFG.degree, cam)
    bins = O.bin_and_sort(p, cam)
    fwd = O.rasterize_forward(bins, O.pack(bins, p), cam, S.BACKGROUND)
    tr = O.OracleTrainer(scene.params(), CFG.degree)
    out = tr.step(cam, gt, S.BACKGROUND, want_grads=True)
    res = dict(radii=p["radii"], xys=p["xys"], depths=p["depths"], transmats=p["transmats"],
               raw_counts=bins["raw_counts"], tile_bins=bins["tile_bins"], gaussian_ids=bins["gaussian_ids"],
               final_idx=fwd["final_idx"], loss=np.float64(out["loss"]), grads=out["grads"])
    for k in ("out_img", "final_Ts", "out_depth", "out_normal", "out_alpha", "out_median_depth", "out_distortion"):
        res[k] = fwd[k]
    for name, arr in zip(("means", "scales", "quats", "opacities", "f_dc", "f_rest"), tr.params()):
        res["after_" + name] = arr
    return res


if __name__ == "__main__":
    np.savez_compressed(os.path.join(HERE, "golden_small.npz"), **compute())
    print("wrote", os.path.join(HERE, "golden_small.npz"))

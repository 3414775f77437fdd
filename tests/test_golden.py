"""Golden fixture (tests/golden/golden_small.npz, made by make_golden.py).

CPU: the oracle reproduces the fixture (bit-exact for binning and the forward).
GPU: the CUDA path matches it through the C ABI within the path's tolerances.
"""
import os
import sys

import numpy as np
import pytest

from _cases import rel_l2

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_golden as MG  # noqa: E402

GOLD = np.load(os.path.join(HERE, "golden", "golden_small.npz"))


def test_oracle_reproduces_golden():
    res = MG.compute()
    for k in ("radii", "raw_counts", "tile_bins", "gaussian_ids", "final_idx"):
        assert np.array_equal(res[k], GOLD[k]), k
    for k in ("xys", "depths", "transmats", "out_img", "final_Ts", "out_depth", "out_normal", "out_alpha",
              "out_median_depth", "out_distortion"):
        assert np.array_equal(res[k].view(np.uint32), GOLD[k].view(np.uint32)), k
    assert abs(float(res["loss"]) - float(GOLD["loss"])) <= 1e-7 * abs(float(GOLD["loss"]))
    assert rel_l2(res["grads"], GOLD["grads"]) < 1e-6
    for k in GOLD.files:
        if k.startswith("after_"):
            assert np.allclose(res[k], GOLD[k], rtol=1e-6, atol=1e-7), k


@pytest.mark.gpu
def test_cuda_matches_golden():
    torch = pytest.importorskip("torch")
    from msplat import _backend as B
    B.load()
    scene, ocam, gt = MG.case()
    g = B.DeviceGaussians(*scene.params(), sh_degree=MG.CFG.degree)
    cam = B.camera_from_oracle(ocam)
    n = MG.CFG.n
    B.train_step_2dgs(g, cam, MG.CFG.degree, MG.S.BACKGROUND, torch.as_tensor(gt).cuda(), 0.8, 0.0, 0.2)
    torch.cuda.synchronize()
    t = lambda name: B.last_tensor(name).cpu().numpy()
    assert np.array_equal(t("radii"), GOLD["radii"])
    assert np.array_equal(t("tile_bins"), GOLD["tile_bins"])
    assert np.array_equal(t("gaussian_ids"), GOLD["gaussian_ids"])
    assert np.abs(t("out_img") - GOLD["out_img"]).max() <= 1e-4
    K = (MG.CFG.degree + 1) ** 2 - 1
    grads = np.concatenate([t("dL_dmean3D").ravel(), t("dL_dscale").ravel(), t("dL_dquat").ravel(),
                            t("dL_dfeatures_dc").ravel(), t("dL_dfeatures_rest").ravel(), t("dL_dopacity").ravel()])
    assert grads.size == 13 * n + 3 * K * n
    assert rel_l2(grads, GOLD["grads"]) <= 1e-3

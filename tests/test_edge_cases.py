"""Edge cases of the C ABI against the oracle: no Gaussians, every Gaussian
culled (camera looking away), a single partial tile, a training step on an
empty scene."""
import numpy as np
import pytest

from msplat import synthetic as S
from oracle import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _B():
    from msplat import _backend as B
    B.load()
    return B


def _scene(n, degree, width, height, seed=0, **kw):
    cfg = S.small_config(max(n, 1), degree, width, height, num_cameras=2, **kw)
    sc = S.make_scene(cfg, seed=seed)
    params = [np.ascontiguousarray(a[:n]) for a in sc.params()]
    return cfg, sc, params


def _render_both(params, degree, cam_to_world, intr, width, height):
    B = _B()
    fx, fy, cx, cy = intr
    ocam = O.prepare_cam(cam_to_world, fx, fy, cx, cy, width, height)
    want = O.render(params, degree, degree, S.BACKGROUND, ocam)
    g = B.DeviceGaussians(*params, sh_degree=degree)
    out = torch.zeros(height, width, 3, device="cuda")
    B.render(g, B.camera_from_oracle(ocam), degree, S.BACKGROUND, out_img=out)
    torch.cuda.synchronize()
    return out.cpu().numpy(), want


def test_no_gaussians_renders_the_background():
    cfg, sc, params = _scene(0, 1, 64, 48)
    got, want = _render_both(params, 1, sc.cam_to_world[0], sc.intrinsics, 64, 48)
    np.testing.assert_array_equal(got, want)
    np.testing.assert_array_equal(got, np.broadcast_to(np.float32(S.BACKGROUND), got.shape))


def test_every_gaussian_culled_renders_the_background():
    cfg, sc, params = _scene(2000, 1, 64, 48)
    c2w = np.array(sc.cam_to_world[0], np.float32).copy()
    c2w[:3, 2] *= -1.0  # look away from the scene (the camera's -z axis now points outwards)
    c2w[:3, 0] *= -1.0  # keep a right-handed frame
    got, want = _render_both(params, 1, c2w, sc.intrinsics, 64, 48)
    np.testing.assert_array_equal(got, want)
    B = _B()
    radii = B.last_tensor("radii").cpu().numpy()
    assert (radii == 0).all()
    np.testing.assert_array_equal(got, np.broadcast_to(np.float32(S.BACKGROUND), got.shape))


@pytest.mark.parametrize("width,height", [(16, 16), (13, 7), (1, 1)])
def test_single_partial_tile_matches_oracle(width, height):
    cfg, sc, params = _scene(3000, 2, width, height, focal=12.0)
    got, want = _render_both(params, 2, sc.cam_to_world[0], sc.intrinsics, width, height)
    np.testing.assert_array_equal(got, want)


def test_training_step_on_an_empty_scene():
    B = _B()
    cfg, sc, params = _scene(0, 0, 40, 24)
    fx, fy, cx, cy = sc.intrinsics
    ocam = O.prepare_cam(sc.cam_to_world[0], fx, fy, cx, cy, 40, 24)
    rng = np.random.default_rng(0)
    gt = rng.uniform(0, 1, (24, 40, 3)).astype(np.float32)
    g = B.DeviceGaussians(*params, sh_degree=0)
    adam = B.AdamState(g)
    loss = torch.zeros(1, device="cuda")
    B.train_step_fused(g, B.camera_from_oracle(ocam), 0, S.BACKGROUND, torch.from_numpy(gt).cuda(), 0.8, 0.0, 0.2,
                       adam, loss_dev=loss)
    torch.cuda.synchronize()
    img = np.broadcast_to(np.float32(S.BACKGROUND), gt.shape).copy()
    want = O.loss_ssim(img, gt, np.zeros(gt.shape[:2], np.float32), 0.8, 0.0, 0.2)["loss"]
    assert abs(float(loss.cpu()[0]) - want) <= 1e-5 * abs(want)


def test_overfull_tiles_with_more_than_2_24_gaussians():
    """Ids above 2^24 take part in the overfull-tile selection (the 2048 lowest
    ids of a tile): a third radix digit keeps them from aliasing lower ids."""
    B = _B()
    n = 16_900_000  # > 2^24 = 16,777,216
    cfg = S.small_config(n, 0, 32, 32, num_cameras=1)
    sc = S.make_scene(cfg, seed=3)
    fx, fy, cx, cy = sc.intrinsics
    ocam = O.prepare_cam(sc.cam_to_world[0], fx, fy, cx, cy, 32, 32)
    p = O.project_forward(*sc.params(), 0, 0, ocam)
    bins = O.bin_and_sort(p, ocam)
    assert bins["raw_counts"].min() > 2048 and (p["radii"][1 << 24:] > 0).any()
    g = B.DeviceGaussians(*sc.params(), sh_degree=0)
    B.render(g, B.camera_from_oracle(ocam), 0, S.BACKGROUND)
    torch.cuda.synchronize()
    assert B.last_num_intersections() == bins["kept"]
    np.testing.assert_array_equal(B.last_tensor("tile_bins").cpu().numpy(), bins["tile_bins"])
    np.testing.assert_array_equal(B.last_tensor("gaussian_ids").cpu().numpy(), bins["gaussian_ids"])

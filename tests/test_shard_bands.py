"""The sharded forward/backward (msplat_shard_forward_backward) on one GPU:
for every rank of a 2- and 3-way split the library picks a work-balanced band
of tile rows; the bands must tile the image exactly, and the ranks' raster
gradients and loss sums must add up to those of one whole-image call (the
same kernels over all rows; float atomics reorder the sums)."""
import numpy as np
import pytest

from _cases import Case

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _call(B, g, cam, case, gt, **kw):
    n = case.cfg.n
    rg = torch.zeros(n, 16, device="cuda")
    parts = torch.zeros(3, dtype=torch.float64, device="cuda")
    rows = B.shard_forward_backward(g, cam, case.degree, case.bg, gt, 0.8, 0.1, 0.2, rg, parts, **kw)
    torch.cuda.synchronize()
    return rows, rg.cpu().numpy().astype(np.float64), parts.cpu().numpy()


@pytest.mark.parametrize("name", ["sh3_small", "overflow"])
@pytest.mark.parametrize("world", [2, 3])
def test_bands_tile_the_image_and_sum_to_the_whole(name, world):
    from msplat import _backend as B
    B.load()
    case = Case(name)
    g = B.DeviceGaussians(*case.scene.params(), sh_degree=case.degree)
    cam = B.camera_from_oracle(case.ocam)
    gt = torch.as_tensor(case.gt).cuda()
    ty = (case.cfg.height + 15) // 16
    (r0, r1), want_rg, want_parts = _call(B, g, cam, case, gt, rows=(0, ty))
    assert (r0, r1) == (0, ty)
    got_rg = np.zeros_like(want_rg)
    got_parts = np.zeros(3)
    bands = []
    for rank in range(world):
        (b0, b1), rg, parts = _call(B, g, cam, case, gt, world=world, rank=rank)
        bands.append((b0, b1))
        got_rg += rg
        got_parts += parts
    assert bands[0][0] == 0 and bands[-1][1] == ty
    assert all(bands[k][1] == bands[k + 1][0] for k in range(world - 1))
    np.testing.assert_allclose(got_parts, want_parts, rtol=1e-9, atol=1e-12)
    err = np.linalg.norm(got_rg - want_rg) / np.linalg.norm(want_rg)
    assert err < 1e-5, err


def test_colour_exchange_path_matches_the_evaluated_colours():
    """msplat_shard_colors + msplat_shard_forward_backward_rgb give the same
    gradients and loss sums as the evaluated-colour path."""
    from msplat import _backend as B
    B.load()
    case = Case("sh3_small")
    n = case.cfg.n
    g = B.DeviceGaussians(*case.scene.params(), sh_degree=case.degree)
    cam = B.camera_from_oracle(case.ocam)
    gt = torch.as_tensor(case.gt).cuda()
    (r0, r1), want_rg, want_parts = _call(B, g, cam, case, gt, world=2, rank=1)
    rgb = torch.zeros(n, 3, device="cuda")
    B.shard_colors(g, cam, case.degree, 0, n, rgb)
    rg = torch.zeros(n, 16, device="cuda")
    parts = torch.zeros(3, dtype=torch.float64, device="cuda")
    rows = B.shard_forward_backward_rgb(g, cam, case.degree, case.bg, gt, 0.8, 0.1, 0.2, rg, parts, rgb,
                                        world=2, rank=1)
    torch.cuda.synchronize()
    assert rows == (r0, r1)
    np.testing.assert_array_equal(parts.cpu().numpy(), want_parts)
    err = np.linalg.norm(rg.cpu().numpy() - want_rg) / np.linalg.norm(want_rg)
    assert err < 1e-6, err

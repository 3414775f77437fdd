"""The identities the backward rasteriser's flush relies on (rasterize.cu,
colour-only k_raster_bwd): with k = px Tw - Tu and l = py Tw - Tv affine in
the pixel, the per-pixel terms dk = l x dp, dl = dp x k and px dk + py dl
(the reference's per-pixel dL/dT rows, core/metal/msplat_metal.metal:
1705-1979) summed over any set of pixels equal cross products of the three
moments sum dp, sum px dp and sum py dp with the rows of T. So a warp sums 9
values per (pixel, surfel) and the cross products are taken once per
surfel."""
import numpy as np


def test_summed_cross_products_equal_moment_cross_products():
    rng = np.random.default_rng(7)
    for _ in range(50):
        Tu, Tv, Tw = rng.normal(0, 100, (3, 3))
        n = int(rng.integers(1, 33))
        px = rng.integers(0, 5000, n).astype(np.float64)
        py = rng.integers(0, 3000, n).astype(np.float64)
        dp = rng.normal(0, 1e-3, (n, 3))
        k = px[:, None] * Tw - Tu
        l = py[:, None] * Tw - Tv
        dk = np.cross(l, dp)
        dl = np.cross(dp, k)
        row3 = px[:, None] * dk + py[:, None] * dl
        s, a, b = dp.sum(0), (px[:, None] * dp).sum(0), (py[:, None] * dp).sum(0)
        np.testing.assert_allclose(dk.sum(0), np.cross(Tw, b) - np.cross(Tv, s), rtol=1e-9, atol=1e-6)
        np.testing.assert_allclose(dl.sum(0), np.cross(a, Tw) - np.cross(s, Tu), rtol=1e-9, atol=1e-6)
        np.testing.assert_allclose(row3.sum(0), np.cross(Tu, b) - np.cross(Tv, a), rtol=1e-9, atol=1e-3)

"""The forward rasteriser skips (warp block, surfel) pairs with a conic test
built by the projection (cull records). The test must never skip a pair that
the exact per-pixel evaluation would blend: strongly anisotropic surfels in
every orientation (thin, grazing, partly behind the camera) are rendered
bit-exact against the oracle over several seeds and cameras."""
import numpy as np
import pytest

from _cases import Case

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.mark.parametrize("seed", [0, 1, 2])
@pytest.mark.parametrize("cam_index", [0, 1])
def test_thin_surfels_render_bit_exact(seed, cam_index):
    from msplat import _backend as B
    B.load()
    case = Case("thin", cam_index=cam_index, seed=seed)
    g = B.DeviceGaussians(*case.scene.params(), sh_degree=case.degree)
    B.render(g, B.camera_from_oracle(case.ocam), case.degree, case.bg)
    torch.cuda.synchronize()
    _, bins, _, fwd = case.oracle_forward()
    assert B.last_num_intersections() == bins["kept"]
    for k in ("out_img", "final_Ts", "out_depth", "out_alpha", "out_distortion"):
        got = B.last_tensor(k).cpu().numpy()
        assert np.array_equal(got, fwd[k]), f"{k}: max abs {np.abs(got - fwd[k]).max()}"
    assert np.array_equal(B.last_tensor("final_idx").cpu().numpy(), fwd["final_idx"])

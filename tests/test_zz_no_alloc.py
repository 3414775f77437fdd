"""The allocation-free loss entry point, msplat_loss_ssim_noalloc.

Some programs that embed this library must not let it allocate GPU memory
while they run: a host that gives out all device memory from its own pool
allocator, or a system whose memory budget is fixed when it starts. For them
the library has msplat_loss_ssim_noalloc, which keeps its working memory in a
fixed array inside the library itself and never calls cudaMalloc. This test
calls it through the C ABI and checks it against the loss and dL/dimage that
the regular entry point (msplat_train_step_2dgs) computes for the same image,
on two calls in a row with different image sizes, checks a tall image whose
regular loss grid would need more blocks than the fixed array holds, and
checks that an image too wide for the fixed array is refused. The file is
named so that pytest collects it last.
"""
import ctypes as C

import numpy as np
import pytest

from _cases import Case, rel_l2

pytestmark = pytest.mark.gpu

GRAD_TOL = 1e-3
LOSS_TOL = 1e-5


def _lib():
    from msplat import _backend as B
    L = B.load()
    f = L.msplat_loss_ssim_noalloc
    f.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_float, C.c_float, C.c_float,
                  C.c_void_p, C.c_void_p, C.c_void_p]
    f.restype = C.c_int
    L.msplat_last_error.restype = C.c_char_p
    return B, L


def test_noalloc_loss_matches_regular_entry_point_twice():
    torch = pytest.importorskip("torch")
    B, L = _lib()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for name in ("cfg0", "sh1_odd"):  # 256x256, then 203x117: the second call reuses the scratch
        case = Case(name)
        g = B.DeviceGaussians(*case.scene.params(), sh_degree=case.degree)
        cam = B.camera_from_oracle(case.ocam)
        gt = torch.as_tensor(case.gt).cuda()
        loss_ref = B.train_step_2dgs(g, cam, case.degree, case.bg, gt, 0.8, 0.0, 0.2)
        img = B.last_tensor("out_img").clone()
        dimg_ref = B.last_tensor("dL_dout_img").clone()
        dimg = torch.full_like(img, float("nan"))
        loss = torch.full((1,), float("nan"), device="cuda")
        H, W = img.shape[0], img.shape[1]
        rc = L.msplat_loss_ssim_noalloc(img.data_ptr(), gt.data_ptr(), None, W, H, 0.8, 0.0, 0.2,
                                        dimg.data_ptr(), loss.data_ptr(), stream)
        assert rc == 0, L.msplat_last_error().decode()
        torch.cuda.synchronize()
        assert rel_l2(dimg.cpu().numpy(), dimg_ref.cpu().numpy()) <= GRAD_TOL
        got = float(loss.cpu()[0])
        assert abs(got - loss_ref) <= LOSS_TOL * abs(loss_ref), (name, got, loss_ref)


def test_noalloc_loss_rejects_images_beyond_its_fixed_scratch():
    torch = pytest.importorskip("torch")
    B, L = _lib()
    # 500000 x 1 pixels need 9260 loss blocks (54-column strips), more than
    # the 8192 the fixed scratch holds. The buffers are full-sized anyway, so
    # a regression in the size check cannot make the kernel read or write
    # outside them.
    w, h = 500_000, 1
    img = torch.zeros(h, w, 3, device="cuda")
    gt = torch.zeros_like(img)
    dimg = torch.zeros_like(img)
    loss = torch.zeros(1, device="cuda")
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = L.msplat_loss_ssim_noalloc(img.data_ptr(), gt.data_ptr(), None, w, h, 0.8, 0.0, 0.2, dimg.data_ptr(),
                                    loss.data_ptr(), stream)
    torch.cuda.synchronize()
    assert rc == 1
    assert "too wide" in L.msplat_last_error().decode()


def test_noalloc_loss_caps_its_grid_for_tall_images():
    """112000 x 2000 pixels: the regular loss grid would use 2075 strips x 4
    row segments = 8300 blocks, more than the 8192 the fixed scratch holds;
    this entry point lays out fewer row segments instead of refusing. Image
    and target vary by row only, so every column at least 10 pixels from the
    left and right edges has the same loss terms and gradient as the middle
    column of a 64-column image with the same rows: the oracle on 64- and
    65-column images gives the expected SSIM sum by linearity in the width,
    and the expected dL/dimage (scaled by the ratio of the 1/(3HW) factors)."""
    torch = pytest.importorskip("torch")
    from oracle import oracle as O
    B, L = _lib()
    W, H = 112_000, 2_000
    y = np.arange(H, dtype=np.float64)[:, None]
    img_rows = (np.array([0.30, 0.60, 0.10]) + 0.2 * np.sin(0.05 * y)).astype(np.float32)        # [H, 3]
    gt_rows = (np.array([0.50, 0.20, 0.10]) + 0.1 * np.cos(0.031 * y)).astype(np.float32)
    lam_l1, lam_dssim = 0.8, 0.2

    def narrow(w):
        return (np.ascontiguousarray(np.broadcast_to(img_rows[:, None, :], (H, w, 3))),
                np.ascontiguousarray(np.broadcast_to(gt_rows[:, None, :], (H, w, 3))))

    r64 = O.loss_ssim(*narrow(64), None, lam_l1, 0.0, lam_dssim)
    r65 = O.loss_ssim(*narrow(65), None, lam_l1, 0.0, lam_dssim)
    ssim_sum = r64["ssim_sum"] + (W - 64) * (r65["ssim_sum"] - r64["ssim_sum"])
    l1_mean = float(np.abs(img_rows.astype(np.float64) - gt_rows).mean())
    loss_want = lam_l1 * l1_mean + lam_dssim * (1.0 - ssim_sum / (3.0 * H * W))
    col_want = torch.as_tensor(r64["dL_dout_img"][:, 32, :].astype(np.float64) * (64.0 / W)).cuda()

    img = torch.as_tensor(img_rows).cuda()[:, None, :].expand(H, W, 3).contiguous()
    gt = torch.as_tensor(gt_rows).cuda()[:, None, :].expand(H, W, 3).contiguous()
    dimg = torch.full_like(img, float("nan"))
    loss = torch.full((1,), float("nan"), device="cuda")
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = L.msplat_loss_ssim_noalloc(img.data_ptr(), gt.data_ptr(), None, W, H, lam_l1, 0.0, lam_dssim,
                                    dimg.data_ptr(), loss.data_ptr(), stream)
    assert rc == 0, L.msplat_last_error().decode()
    torch.cuda.synchronize()
    got = float(loss.cpu()[0])
    assert abs(got - loss_want) <= LOSS_TOL * abs(loss_want), (got, loss_want)
    assert not torch.isnan(dimg).any()  # every pixel written
    inner = dimg[:, 10:W - 10, :].double()
    err = (inner - col_want[:, None, :]).abs().max().item()
    assert err <= GRAD_TOL * col_want.abs().max().item(), err
    del img, gt, dimg, inner
    torch.cuda.empty_cache()

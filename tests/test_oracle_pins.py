"""Pins of the CPU oracle (CPU only).

The reference's own tests hold no golden vectors for this path and its Metal
kernels cannot run here, so the oracle is pinned independently:
  * its exp against numpy,
  * its SSIM+L1 loss and gradient against a torch-autograd restatement of the
    reference's definition (F.conv2d, zero padding, C1 = 1e-4, C2 = 9e-4),
  * its rasteriser / projection VJPs against central finite differences of its
    own forward (with the reference's documented gradient conventions),
  * an analytic single-surfel known-answer case,
  * its binning policy against a numpy restatement.
"""
import math

import numpy as np
import pytest

from _cases import rel_l2
from msplat import synthetic as S
from oracle import oracle as O


def test_det_exp_accuracy():
    xs = np.concatenate([np.linspace(-86, 88, 20001), np.array([-1e-8, 0.0, 1e-8, -0.5, -4.5])]).astype(np.float32)
    got = np.array([O.det_exp(float(x)) for x in xs], dtype=np.float64)
    ref = np.exp(xs.astype(np.float64))
    rel = np.abs(got - ref) / ref
    assert rel.max() < 5e-7
    assert O.det_exp(-87.0) == 0.0
    assert math.isinf(O.det_exp(89.0))


def _torch_loss(img, gt, lam_l1, lam_dssim):
    torch = pytest.importorskip("torch")
    F = torch.nn.functional
    x = torch.tensor(img, dtype=torch.float64, requires_grad=True)
    y = torch.tensor(gt, dtype=torch.float64)
    w1 = torch.exp(-(torch.arange(11, dtype=torch.float64) - 5) ** 2 / (2 * 1.5 ** 2))
    w1 = w1 / w1.sum()
    win = (w1[:, None] * w1[None, :]).expand(3, 1, 11, 11).contiguous()
    a = x.permute(2, 0, 1)[None]
    b = y.permute(2, 0, 1)[None]
    conv = lambda t: F.conv2d(t, win, padding=5, groups=3)
    mu1, mu2 = conv(a), conv(b)
    s1 = conv(a * a) - mu1 ** 2
    s2 = conv(b * b) - mu2 ** 2
    s12 = conv(a * b) - mu1 * mu2
    C1, C2 = 1e-4, 9e-4
    ssim = ((2 * mu1 * mu2 + C1) * (2 * s12 + C2)) / ((mu1 ** 2 + mu2 ** 2 + C1) * (s1 + s2 + C2))
    loss = lam_l1 * (a - b).abs().mean() + lam_dssim * (1 - ssim.mean())
    loss.backward()
    return float(loss), x.grad.numpy(), float(ssim.sum())


@pytest.mark.parametrize("shape", [(48, 64), (37, 53)])
def test_ssim_loss_matches_torch_autograd(shape):
    rng = np.random.default_rng(7)
    H, W = shape
    gt = rng.random((H, W, 3)).astype(np.float32)
    img = np.clip(gt + rng.normal(0, 0.1, gt.shape), 0, 1).astype(np.float32)
    out = O.loss_ssim(img, gt, np.zeros((H, W), np.float32), 0.8, 0.0, 0.2)
    loss, grad, ssum = _torch_loss(img, gt, 0.8, 0.2)
    assert abs(out["loss"] - loss) < 1e-6 * max(1, abs(loss))
    assert abs(out["ssim_sum"] - ssum) < 1e-5 * abs(ssum)
    assert rel_l2(out["dL_dout_img"], grad) < 1e-4


def _fd_scene(n=30, seed=5, degree=2):
    rng = np.random.default_rng(seed)
    means = np.concatenate([rng.uniform(-0.6, 0.6, (n, 2)), rng.uniform(-0.5, 0.5, (n, 1))], 1).astype(np.float32)
    scales = (np.log(0.12) + rng.normal(0, 0.2, (n, 2))).astype(np.float32)
    # surfels roughly facing the camera at (0, 0, 4): normal close to +z
    ang = rng.normal(0, 0.25, (n, 3))
    quats = np.concatenate([np.ones((n, 1)), 0.5 * ang], 1)
    quats = (quats / np.linalg.norm(quats, axis=1, keepdims=True)).astype(np.float32)
    opac = rng.uniform(-3.0, -1.2, (n, 1)).astype(np.float32)  # o < 0.24: alpha < 1/255 before the 3-sigma cut
    f_dc = rng.uniform(-0.5, 0.5, (n, 3)).astype(np.float32)
    K = (degree + 1) ** 2 - 1
    f_rest = rng.normal(0, 0.2, (n, K, 3)).astype(np.float32)
    W, H = 72, 56
    cam = O.prepare_cam(S.look_at_gl((0.3, 0.2, 4.0)), 70.0, 70.0, W / 2, H / 2, W, H)
    return [means, scales, quats, opac, f_dc, f_rest], degree, cam


def _threshold_mask(p, cam, lo=0.3 / 255, hi=3.0 / 255):
    """1 where no surfel's alpha at the pixel lies near the reference's 1/255
    cut-off (metal:662-663): the image is piecewise smooth there only."""
    H, W = cam.height, cam.width
    ys, xs = np.mgrid[0:H, 0:W].astype(np.float64)
    mask = np.ones((H, W), bool)
    for i in np.nonzero(p["radii"] > 0)[0]:
        T = p["transmats"][i].astype(np.float64)
        Tu, Tv, Tw = T[0:3], T[3:6], T[6:9]
        k = xs[..., None] * Tw - Tu
        l = ys[..., None] * Tw - Tv
        pc = np.cross(k, l)
        u, v = pc[..., 0] / pc[..., 2], pc[..., 1] / pc[..., 2]
        d2 = (p["xys"][i, 0] - xs) ** 2 + (p["xys"][i, 1] - ys) ** 2
        rho = np.minimum(u * u + v * v, 2.0 * d2)
        o = 1.0 / (1.0 + np.exp(-float(p["normal_opacity"][i, 3])))
        a = o * np.exp(-0.5 * rho)
        mask &= ~((a > lo) & (a < hi))
    return mask


def _render_linear(params, degree, cam, wgt, bg):
    img = O.render(params, degree, degree, bg, cam)
    return float(np.sum(img.astype(np.float64) * wgt))


def test_vjps_match_finite_differences():
    params, degree, cam = _fd_scene()
    bg = S.BACKGROUND
    rng = np.random.default_rng(11)
    p = O.project_forward(*params, degree, degree, cam)
    # the loss is a random linear functional of the image, restricted to
    # pixels away from the alpha cut-off so that it is differentiable
    wgt = rng.normal(0, 1, (cam.height, cam.width, 3)).astype(np.float32)
    wgt *= _threshold_mask(p, cam)[..., None]
    bins = O.bin_and_sort(p, cam)
    packed = O.pack(bins, p)
    fwd = O.rasterize_forward(bins, packed, cam, bg)
    n = params[0].shape[0]
    rb = O.rasterize_backward(n, bins, packed, fwd, cam, bg, wgt)
    pb = O.project_backward(params[0], params[1], params[2], cam, p["radii"], rb["dL_dtransMat"], rb["dL_dnormal3D"],
                            rb["dL_dcolors"], degree, degree, params[5])
    q = params[2].astype(np.float64)
    gq = pb["dL_dquat"].astype(np.float64)
    gq_tan = gq - np.sum(gq * q, 1, keepdims=True) * q  # the reference VJP ignores the normalisation
    analytic = [pb["dL_dmean3D"], pb["dL_dscale"], gq_tan, rb["dL_dopacity"], pb["dL_dfeatures_dc"],
                pb["dL_dfeatures_rest"]]
    steps = [5e-4, 5e-4, 5e-4, 5e-4, 5e-4, 5e-4]
    visible = np.nonzero(p["radii"] > 0)[0]
    assert len(visible) > 10
    for gi, (ana, h) in enumerate(zip(analytic, steps)):
        fd_vals, an_vals = [], []
        for i in visible[:12]:
            for j in range(min(params[gi][i].size, 4)):
                idx = np.unravel_index(j, params[gi][i].shape)
                pp = [a.copy() for a in params]
                pm = [a.copy() for a in params]
                pp[gi][i][idx] += h
                pm[gi][i][idx] -= h
                fd = (_render_linear(pp, degree, cam, wgt, bg) - _render_linear(pm, degree, cam, wgt, bg)) / (2 * h)
                fd_vals.append(fd)
                an_vals.append(float(np.asarray(ana[i])[idx]))
        fd_vals, an_vals = np.array(fd_vals), np.array(an_vals)
        cos = np.dot(fd_vals, an_vals) / (np.linalg.norm(fd_vals) * np.linalg.norm(an_vals) + 1e-30)
        assert cos > 0.999, (gi, cos)
        assert rel_l2(an_vals, fd_vals) < 0.02, (gi, rel_l2(an_vals, fd_vals))


def test_single_surfel_known_answer():
    """One surfel at the origin facing the camera at (0, 0, 4): closed-form
    centre, depth, footprint radius and per-pixel alpha."""
    W = H = 256
    f = 205.0
    cam = O.prepare_cam(S.look_at_gl((0.0, 0.0, 4.0)), f, f, 128.0, 128.0, W, H)
    s = 0.1
    means = np.zeros((1, 3), np.float32)
    scales = np.full((1, 2), np.log(s), np.float32)
    quats = np.array([[1, 0, 0, 0]], np.float32)
    opac = np.zeros((1, 1), np.float32)  # sigmoid -> 0.5
    f_dc = np.array([[0.3, -0.2, 0.1]], np.float32)
    f_rest = np.zeros((1, 3, 3), np.float32)
    f_rest[0, 1] = [0.2, 0.4, -0.6]  # band-1 "z" coefficient
    p = O.project_forward(means, scales, quats, opac, f_dc, f_rest, 1, 1, cam)
    assert p["depths"][0] == pytest.approx(4.0, abs=1e-6)
    assert np.allclose(p["xys"][0], [127.5, 127.5], atol=1e-4)
    sigma_px = s * f / 4.0
    assert p["radii"][0] == math.ceil(3 * sigma_px)
    # SH: viewdir = (0, 0, -1): colour = C0 dc + C1 * z * rest[1] = C0 dc - C1 rest[1]
    C0, C1 = 0.28209479177387814, 0.4886025119029199
    assert np.allclose(p["colors"][0], C0 * f_dc[0] - C1 * f_rest[0, 1], atol=1e-6)
    bins = O.bin_and_sort(p, cam)
    fwd = O.rasterize_forward(bins, O.pack(bins, p), cam, S.BACKGROUND)
    for (py, px) in [(127, 127), (120, 131), (127, 140)]:
        d2 = (px - 127.5) ** 2 + (py - 127.5) ** 2
        alpha = 0.5 * math.exp(-0.5 * d2 / sigma_px ** 2)
        assert fwd["out_alpha"][py, px] == pytest.approx(alpha, rel=2e-5)
        assert fwd["out_depth"][py, px] == pytest.approx(4.0 * alpha, rel=2e-5)
        col = np.maximum(p["colors"][0] + 0.5, 0) * alpha + S.BACKGROUND * (1 - alpha)
        assert np.allclose(fwd["out_img"][py, px], col, rtol=2e-5)
        assert np.allclose(fwd["out_normal"][py, px], [0, 0, alpha], atol=1e-6)
    # outside the 3-sigma footprint nothing is drawn
    assert fwd["out_alpha"][127, 127 + 40] == 0.0


@pytest.mark.parametrize("name", ["cfg0", "overflow"])
def test_binning_policy_restated_in_numpy(name):
    from _cases import Case
    case = Case(name)
    p = O.project_forward(*case.scene.params(), case.degree, case.degree, case.ocam)
    bins = O.bin_and_sort(p, case.ocam)
    tx, ty = O.tiles(case.ocam)
    lists = [[] for _ in range(tx * ty)]
    f16 = np.float32(16.0)
    for i in np.nonzero(p["radii"] > 0)[0]:
        cx, cy = p["xys"][i]
        r = p["aabb"][i, 0]
        tcx, tcy, tr = cx / f16, cy / f16, r / f16
        x0 = min(max(0, int(np.float32(tcx - tr))), tx)
        x1 = min(max(0, int(np.float32(np.float32(tcx + tr) + np.float32(1)))), tx)
        y0 = min(max(0, int(np.float32(tcy - tr))), ty)
        y1 = min(max(0, int(np.float32(np.float32(tcy + tr) + np.float32(1)))), ty)
        for y in range(y0, y1):
            for x in range(x0, x1):
                lists[y * tx + x].append(i)
    start = 0
    for t, L in enumerate(lists):
        assert bins["raw_counts"][t] == len(L)
        kept = sorted(L)[:2048]  # lowest ids survive an overfull tile
        kept.sort(key=lambda i: (int(p["depths"][i].view(np.uint32)), i))
        assert tuple(bins["tile_bins"][t]) == (start, start + len(kept))
        assert list(bins["gaussian_ids"][start:start + len(kept)]) == kept
        start += len(kept)
    if name == "overflow":
        assert max(len(L) for L in lists) > 2048

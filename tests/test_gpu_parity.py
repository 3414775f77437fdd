"""CUDA path vs the CPU oracle, through the C ABI (libmsplat_b200.so).

Tolerances (from the spec of this path): tile counts, offsets and per-tile
order bit-exact; rendered images within 1e-4 max abs; gradients within 1e-3
relative L2; Adam-updated parameters within 1e-5 relative (on identical
gradients).
"""
import numpy as np
import pytest

from _cases import Case, rel_l2

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

IMG_TOL = 1e-4
GRAD_TOL = 1e-3
ADAM_TOL = 1e-5


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")


def _B():
    from msplat import _backend as B
    B.load()
    return B


def _np(t):
    return t.detach().cpu().numpy()


def _device_scene(case):
    B = _B()
    return B.DeviceGaussians(*case.scene.params(), sh_degree=case.degree)


CASES = ["cfg0", "sh3_small", "sh1_odd", "overflow", "thin"]


@pytest.mark.parametrize("name", CASES)
def test_forward_and_binning_bit_exact(name):
    case = Case(name)
    B = _B()
    g = _device_scene(case)
    cam = B.camera_from_oracle(case.ocam)
    B.render(g, cam, case.degree, case.bg)
    torch.cuda.synchronize()
    p, bins, packed, fwd = case.oracle_forward()
    # projection outputs
    assert np.array_equal(_np(B.last_tensor("radii")), p["radii"])
    assert np.array_equal(_np(B.last_tensor("num_tiles_hit")), p["num_tiles_hit"])
    for k, name_ in (("depths", "depths"), ("xys", "xys"), ("transmats", "transMats"),
                     ("normal_opacity", "normal_opacity"), ("colors", "colors")):
        got = _np(B.last_tensor(name_))
        assert np.array_equal(got.view(np.uint32), p[k].view(np.uint32)), f"{k} differs (max abs " \
            f"{np.abs(got - p[k]).max()})"
    # binning: counts, offsets, per-tile order
    assert np.array_equal(_np(B.last_tensor("raw_tile_counts")).astype(np.int64), bins["raw_counts"])
    assert np.array_equal(_np(B.last_tensor("tile_bins")), bins["tile_bins"])
    assert B.last_num_intersections() == bins["kept"]
    assert np.array_equal(_np(B.last_tensor("gaussian_ids")), bins["gaussian_ids"])
    if name == "overflow":
        assert bins["raw_counts"].max() > 2048
        assert B.last_status_flags() & 1
    # rasteriser outputs
    for k in ("out_img", "final_Ts", "out_depth", "out_normal", "out_alpha", "out_median_depth", "out_distortion"):
        d = np.abs(_np(B.last_tensor(k)) - fwd[k]).max()
        assert d <= IMG_TOL, f"{k}: max abs {d}"
    assert np.array_equal(_np(B.last_tensor("final_idx")), fwd["final_idx"])


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("lambda_dist", [0.0, 0.3])
def test_train_step_gradients(name, lambda_dist):
    from oracle import oracle as O
    case = Case(name)
    B = _B()
    g = _device_scene(case)
    cam = B.camera_from_oracle(case.ocam)
    gt = torch.as_tensor(case.gt).cuda()
    n = case.cfg.n
    stats = [torch.zeros(n, device="cuda") for _ in range(3)]
    lam_l1, lam_dssim = 0.8, 0.2
    loss = B.train_step_2dgs(g, cam, case.degree, case.bg, gt, lam_l1, lambda_dist, lam_dssim, stats=stats)
    torch.cuda.synchronize()
    p, bins, packed, fwd = case.oracle_forward()
    ls = O.loss_ssim(fwd["out_img"], case.gt, fwd["out_distortion"], lam_l1, lambda_dist, lam_dssim)
    assert abs(loss - ls["loss"]) <= 1e-5 * max(1.0, abs(ls["loss"])), (loss, ls["loss"])
    assert rel_l2(_np(B.last_tensor("dL_dout_img")), ls["dL_dout_img"]) <= GRAD_TOL
    rb = O.rasterize_backward(n, bins, packed, fwd, case.ocam, case.bg, ls["dL_dout_img"],
                              dL_dout_distortion=ls["dL_dout_distortion"])
    for k in ("dL_dtransMat", "dL_dopacity", "dL_dcolors", "dL_dnormal3D"):
        e = rel_l2(_np(B.last_tensor(k)), rb[k])
        assert e <= GRAD_TOL, f"{k}: rel L2 {e}"
    ostats = [np.zeros(n, np.float32) for _ in range(3)]
    pb = O.project_backward(case.scene.means, case.scene.scales, case.scene.quats, case.ocam, p["radii"],
                            rb["dL_dtransMat"], rb["dL_dnormal3D"], rb["dL_dcolors"], case.degree, case.degree,
                            case.scene.f_rest, stats=ostats)
    for k in ("dL_dmean3D", "dL_dscale", "dL_dquat", "dL_dmean2D", "dL_dfeatures_dc"):
        e = rel_l2(_np(B.last_tensor(k)), pb[k])
        assert e <= GRAD_TOL, f"{k}: rel L2 {e}"
    if case.degree > 0:
        e = rel_l2(_np(B.last_tensor("dL_dfeatures_rest")), pb["dL_dfeatures_rest"])
        assert e <= GRAD_TOL, f"dL_dfeatures_rest: rel L2 {e}"
    assert np.array_equal(_np(stats[1]), ostats[1])          # vis_counts
    assert np.allclose(_np(stats[2]), ostats[2], rtol=0, atol=0)  # max_2d_size
    assert rel_l2(_np(stats[0]), ostats[0]) <= GRAD_TOL       # xys_grad_norm


def test_fused_adam_identical_inputs():
    from oracle import oracle as O
    B = _B()
    rng = np.random.default_rng(3)
    n = 1_000_003
    p = rng.standard_normal(n).astype(np.float32)
    gr = (rng.standard_normal(n) * 1e-3).astype(np.float32)
    m = (rng.standard_normal(n) * 1e-4).astype(np.float32)
    v = np.abs(rng.standard_normal(n) * 1e-7).astype(np.float32)
    args = (0.0025 / (1 - 0.9 ** 7), 0.9, 0.999, float(np.sqrt(1 - 0.999 ** 7)), 1e-8)
    tp, tg, tm, tv = (torch.as_tensor(a).cuda() for a in (p, gr, m, v))
    B.fused_adam(tp, tg, tm, tv, *args)
    # unaligned start exercises the scalar tail path
    tp2, tg2, tm2, tv2 = (torch.as_tensor(a).cuda() for a in (p, gr, m, v))
    B.fused_adam(tp2[1:], tg2[1:], tm2[1:], tv2[1:], *args)
    torch.cuda.synchronize()
    O.fused_adam(p, gr, m, v, *args)
    for got, ref in ((tp, p), (tm, m), (tv, v)):
        g_ = _np(got)
        assert np.max(np.abs(g_ - ref) / np.maximum(np.abs(ref), 1e-30)) <= ADAM_TOL
    assert np.max(np.abs(_np(tp2)[1:] - p[1:]) / np.maximum(np.abs(p[1:]), 1e-30)) <= ADAM_TOL


@pytest.mark.parametrize("name", ["cfg0", "sh3_small"])
def test_fused_step_adam_matches_oracle_on_its_gradients(name):
    """msplat_train_step_fused applies Adam inside the projection VJP; its
    updated parameters must equal the reference Adam applied to the gradients
    the same call materialises (write_grads=1)."""
    from oracle import oracle as O
    case = Case(name)
    B = _B()
    g = _device_scene(case)
    cam = B.camera_from_oracle(case.ocam)
    gt = torch.as_tensor(case.gt).cuda()
    adam = B.AdamState(g)
    # one warm step so that the moments are non-zero
    B.train_step_fused(g, cam, case.degree, case.bg, gt, 0.8, 0.0, 0.2, adam)
    before = [_np(t).copy() for t in g.groups()]
    m_before = [_np(t).copy() for t in adam.m]
    v_before = [_np(t).copy() for t in adam.v]
    loss_dev = torch.zeros(1, device="cuda")
    B.train_step_fused(g, cam, case.degree, case.bg, gt, 0.8, 0.0, 0.2, adam, loss_dev=loss_dev, write_grads=True)
    torch.cuda.synchronize()
    names = ["dL_dmean3D", "dL_dscale", "dL_dquat", "dL_dfeatures_dc", "dL_dfeatures_rest", "dL_dopacity"]
    # Model keeps beta1/beta2 as float and calls std::pow(float, int) (double)
    bc1 = np.float32(1.0 - float(np.float32(0.9)) ** adam.step)
    bc2 = np.float32(1.0 - float(np.float32(0.999)) ** adam.step)
    for k in range(6):
        if before[k].size == 0:
            continue
        grads = _np(B.last_tensor(names[k])).reshape(before[k].shape)
        p, m, v = before[k].copy(), m_before[k].copy(), v_before[k].copy()
        O.fused_adam(p, grads, m, v, np.float32(adam.lr[k]) / bc1, 0.9, 0.999, float(np.sqrt(bc2)), 1e-8)
        got = _np(g.groups()[k])
        # the fused update computes its step with approximate sqrt/division
        # (a few ulp); p_new = p_old - step, so its error is bounded relative
        # to the operands, max(|p_old|, |p_new|), not to p_new alone, which
        # can be ~0 where the step cancels the old value
        scale = np.maximum(np.maximum(np.abs(p), np.abs(before[k])), 1e-6)
        err = np.max(np.abs(got - p) / scale)
        assert err <= ADAM_TOL, f"group {k}: {err}"
        # the moments are computed with fused multiply-adds only
        for got_m, want_m in ((adam.m[k], m), (adam.v[k], v)):
            gm = _np(got_m).reshape(want_m.shape)
            assert np.max(np.abs(gm - want_m) / np.maximum(np.abs(want_m), 1e-30)) <= ADAM_TOL
    assert np.isfinite(_np(loss_dev)).all()


def test_fused_step_loss_and_descent():
    """Ten fused steps on cfg0 lower the loss, matching the oracle's trajectory."""
    from oracle import oracle as O
    case = Case("cfg0")
    B = _B()
    g = _device_scene(case)
    cam = B.camera_from_oracle(case.ocam)
    gt = torch.as_tensor(case.gt).cuda()
    adam = B.AdamState(g)
    tr = O.OracleTrainer(case.scene.params(), case.degree)
    loss_dev = torch.zeros(1, device="cuda")
    gl, ol = [], []
    for _ in range(10):
        B.train_step_fused(g, cam, case.degree, case.bg, gt, 0.8, 0.0, 0.2, adam, loss_dev=loss_dev)
        gl.append(float(_np(loss_dev)[0]))
        ol.append(tr.step(case.ocam, case.gt, case.bg)["loss"])
    assert gl[-1] < gl[0]
    assert abs(gl[0] - ol[0]) <= 1e-5 * abs(ol[0])
    # trajectories stay within 1% over ten steps (Adam sign flips on noise-level
    # gradients make later steps differ slightly)
    assert max(abs(a - b) / abs(b) for a, b in zip(gl, ol)) < 1e-2


def test_render_matches_oracle_render():
    from oracle import oracle as O
    case = Case("sh3_small", cam_index=1)
    B = _B()
    g = _device_scene(case)
    cam = B.camera_from_oracle(case.ocam)
    out = torch.zeros(case.cfg.height, case.cfg.width, 3, device="cuda")
    B.render(g, cam, case.degree, case.bg, out_img=out)
    torch.cuda.synchronize()
    ref = O.render(case.scene.params(), case.degree, case.degree, case.bg, case.ocam)
    assert np.abs(_np(out) - ref).max() <= IMG_TOL


def test_errors_are_reported_not_raised_through_the_abi():
    B = _B()
    case = Case("cfg0")
    g = _device_scene(case)
    cam = B.camera_from_oracle(case.ocam)
    with pytest.raises(B.MsplatError) as ei:
        B.render(g, cam, 2, case.bg)  # degrees_to_use > sh_degree
    assert ei.value.code == 1
    assert "degrees_to_use" in str(ei.value)
    with pytest.raises(B.MsplatError):
        B.last_tensor("no_such_tensor")


def test_fused_step_light_forward_matches_full_forward():
    """A colour-only fused step that returns no gradients computes only the
    forward outputs it reads (image, T, last contributor). Its loss, image and
    updated parameters equal the same step with every forward output
    (write_grads=True), and the skipped outputs are reported as not produced."""
    case = Case("sh3_small")
    B = _B()
    cam = B.camera_from_oracle(case.ocam)
    gt = torch.as_tensor(case.gt).cuda()
    res = []
    for write in (True, False):
        g = _device_scene(case)
        adam = B.AdamState(g)
        loss_dev = torch.zeros(1, device="cuda")
        B.train_step_fused(g, cam, case.degree, case.bg, gt, 0.8, 0.0, 0.2, adam, loss_dev=loss_dev,
                           write_grads=write)
        torch.cuda.synchronize()
        res.append((float(_np(loss_dev)[0]), _np(B.last_tensor("out_img")).copy(), [_np(t).copy() for t in g.groups()]))
    (l_full, img_full, p_full), (l_light, img_light, p_light) = res
    assert l_full == l_light
    assert np.array_equal(img_full, img_light)
    for a, b in zip(p_full, p_light):
        # float atomics in the backward may reorder sums between two runs
        assert np.allclose(a, b, rtol=1e-5, atol=1e-6)
    for k in ("out_depth", "out_distortion", "final_Ts", "final_idx"):
        with pytest.raises(B.MsplatError):
            B.last_tensor(k)


def test_raster_counters_switch():
    """msplat_set_raster_counters: off (the default) leaves the counters at
    zero; on, a step counts forward visits and blended pairs (at most 32 per
    visit), and the backward visits at most the forward's visits and replays
    about the same blended pairs (its replay uses the hardware exponential)."""
    case = Case("sh3_small")
    B = _B()
    g = _device_scene(case)
    cam = B.camera_from_oracle(case.ocam)
    gt = torch.as_tensor(case.gt).cuda()
    adam = B.AdamState(g)
    B.train_step_fused(g, cam, case.degree, case.bg, gt, 0.8, 0.0, 0.2, adam)
    torch.cuda.synchronize()
    assert not _np(B.last_tensor("raster_counters")).any()
    B.set_raster_counters(True)
    try:
        B.train_step_fused(g, cam, case.degree, case.bg, gt, 0.8, 0.0, 0.2, adam)
        torch.cuda.synchronize()
        fb, fv, bv, bb = (int(x) for x in _np(B.last_tensor("raster_counters")))
    finally:
        B.set_raster_counters(False)
    assert fv > 0 and 0 < fb <= 32 * fv
    assert 0 < bv <= fv and 0 < bb <= 32 * bv
    assert abs(bb - fb) <= 1e-3 * fb

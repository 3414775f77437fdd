"""Trainer-level I/O and the step-end schedule of the reference's C API:
"MSPL" v1 checkpoints (core/src/model.cpp:341-498), PLY and .splat export
(core/src/loaders/save_gaussians.cpp:11-111), densification and the opacity
reset inside Trainer::step (Model::afterTrain, model.cpp:240-306)."""
import struct

import numpy as np
import pytest

import msplat
from msplat import synthetic as S

pytestmark = pytest.mark.gpu


def _dataset(n=3000, cams=1, width=96, height=64, seed=0):
    from oracle import oracle as O
    cfg = S.small_config(n, 1, width, height, num_cameras=max(cams, 2))
    scene = S.make_scene(cfg, seed=seed)
    fx, fy, cx, cy = scene.intrinsics
    target = scene.jittered()
    imgs = []
    for k in range(cams):
        ocam = O.prepare_cam(scene.cam_to_world[k], fx, fy, cx, cy, width, height)
        imgs.append(O.render(target.params(), cfg.degree, cfg.degree, S.BACKGROUND, ocam))
    ds = msplat.Dataset.from_memory(scene.cam_to_world[:cams], np.tile([fx, fy, cx, cy], (cams, 1)), width, height,
                                    np.stack(imgs))
    return ds, scene, cfg


def _trainer(ds, scene, **kw):
    base = dict(iterations=1000, sh_degree=1, num_downscales=0, sh_degree_interval=1, refine_every=10 ** 6)
    base.update(kw)
    return msplat.GaussianTrainer(ds, msplat.TrainingConfig(**base), params=scene.params())


def _read_checkpoint(path):
    buf = open(path, "rb").read()
    magic, version, step, n, sh, adam_steps = struct.unpack_from("<6I", buf, 0)
    off = 24
    lrs = struct.unpack_from("<6f", buf, off)
    off += 24
    lr_init, lr_final = struct.unpack_from("<2f", buf, off)
    off += 8
    tensors = []
    for _ in range(18):
        (ndim,) = struct.unpack_from("<I", buf, off)
        off += 4
        shape = struct.unpack_from("<%dq" % ndim, buf, off)
        off += 8 * ndim
        (nbytes,) = struct.unpack_from("<Q", buf, off)
        off += 8
        tensors.append(np.frombuffer(buf, np.float32, nbytes // 4, off).reshape(shape))
        off += nbytes
    assert off == len(buf)
    return dict(magic=magic, version=version, step=step, n=n, sh=sh, adam_steps=adam_steps, lrs=lrs,
                lr_init=lr_init, lr_final=lr_final, tensors=tensors)


def test_checkpoint_layout_and_resume(tmp_path):
    ds, scene, cfg = _dataset()
    tr = _trainer(ds, scene)
    for _ in range(3):
        tr.step()
    path = tmp_path / "a.ckpt"
    tr.save_checkpoint(path)
    ck = _read_checkpoint(path)
    assert (ck["magic"], ck["version"], ck["step"], ck["n"], ck["sh"], ck["adam_steps"]) == \
        (0x4C50534D, 1, 3, cfg.n, 1, 3)
    assert ck["lr_init"] == pytest.approx(0.00016) and ck["lr_final"] == pytest.approx(0.0000016)
    assert ck["lrs"][1:] == pytest.approx((0.005, 0.001, 0.0025, 0.000125, 0.05))
    shapes = [t.shape for t in ck["tensors"][:6]]
    assert shapes == [(cfg.n, 3), (cfg.n, 2), (cfg.n, 4), (cfg.n, 3), (cfg.n, 3, 3), (cfg.n, 1)]
    got = tr.get_params()  # means, scales, quats, opacities, f_dc, f_rest
    mine = [got[0], got[1], got[2], got[4], got[5], got[3]]
    for a, b in zip(ck["tensors"][:6], mine):
        np.testing.assert_array_equal(a, b.reshape(a.shape))
    assert all(np.abs(t).sum() > 0 for t in ck["tensors"][6:12]), "first moments are non-zero after 3 steps"

    # a fresh trainer resumes from the file: same parameters, step and next loss
    tr2 = _trainer(ds, scene)
    assert tr2.load_checkpoint(path) == 3 and tr2.iteration == 3
    for a, b in zip(tr2.get_params(), got):
        np.testing.assert_array_equal(a, b)
    s1, s2 = tr.step(), tr2.step()
    assert s1.loss == s2.loss  # the forward is deterministic; one training camera
    for a, b in zip(tr.get_params(), tr2.get_params()):
        assert np.isclose(a, b, rtol=1e-5, atol=1e-7).mean() > 0.98


def test_checkpoint_errors(tmp_path):
    ds, scene, cfg = _dataset(n=500)
    tr = _trainer(ds, scene)
    bad = tmp_path / "bad.ckpt"
    bad.write_bytes(b"NOPE" + b"\0" * 64)
    with pytest.raises(RuntimeError, match="Not a valid msplat checkpoint file"):
        tr.load_checkpoint(bad)
    with pytest.raises(RuntimeError, match="Cannot open checkpoint file"):
        tr.load_checkpoint(tmp_path / "missing.ckpt")
    tr.step()
    good = tmp_path / "good.ckpt"
    tr.save_checkpoint(good)
    other = _trainer(ds, scene, sh_degree=0)
    with pytest.raises(RuntimeError, match="SH degree"):
        other.load_checkpoint(good)


def test_ply_export_layout(tmp_path):
    ds, scene, cfg = _dataset(n=800)
    tr = _trainer(ds, scene)
    tr.step()
    path = tmp_path / "g.ply"
    tr.export_ply(path)
    raw = open(path, "rb").read()
    end = raw.index(b"end_header\n") + len(b"end_header\n")
    header = raw[:end].decode().splitlines()
    assert header[:4] == ["ply", "format binary_little_endian 1.0", "comment msplat v1", "element vertex %d" % cfg.n]
    props = [h.split()[-1] for h in header if h.startswith("property float")]
    assert props == (["x", "y", "z", "nx", "ny", "nz", "f_dc_0", "f_dc_1", "f_dc_2"] +
                     ["f_rest_%d" % i for i in range(9)] + ["opacity", "scale_0", "scale_1"] +
                     ["rot_0", "rot_1", "rot_2", "rot_3"])
    body = np.frombuffer(raw[end:], np.float32).reshape(cfg.n, len(props))
    means, scales, quats, opac, f_dc, f_rest = tr.get_params()
    np.testing.assert_array_equal(body[:, 0:3], means)
    assert not body[:, 3:6].any()
    np.testing.assert_array_equal(body[:, 6:9], f_dc)
    np.testing.assert_array_equal(body[:, 9:18], f_rest.transpose(0, 2, 1).reshape(cfg.n, 9))  # [3, bases]
    np.testing.assert_array_equal(body[:, 18], opac[:, 0])
    np.testing.assert_array_equal(body[:, 19:21], scales)
    np.testing.assert_array_equal(body[:, 21:25], quats)


def test_splat_export_layout(tmp_path):
    ds, scene, cfg = _dataset(n=800)
    tr = _trainer(ds, scene)
    path = tmp_path / "g.splat"
    tr.export_splat(path)
    raw = open(path, "rb").read()
    assert len(raw) == 32 * cfg.n
    rec = np.dtype([("pos", "<f4", 3), ("scale", "<f4", 3), ("rgba", "u1", 4), ("rot", "u1", 4)])
    body = np.frombuffer(raw, rec)
    means, scales, quats, opac, f_dc, f_rest = tr.get_params()
    size = np.exp(scales).sum(1) / (1 + np.exp(-opac[:, 0]))
    assert np.all(np.diff(size[_match_rows(body["pos"], means)]) <= 1e-6)  # largest first
    idx = _match_rows(body["pos"], means)
    np.testing.assert_allclose(body["scale"][:, :2], np.exp(scales[idx]), rtol=1e-6)
    assert np.all(body["scale"][:, 2] == np.float32(1e-5))
    rgb = np.clip((f_dc[idx].astype(np.float64) * 0.28209479177387814 + 0.5) * 255.0, 0, 255).astype(np.uint8)
    np.testing.assert_array_equal(body["rgba"][:, :3], rgb)
    q = np.clip(quats[idx] * 128.0 + 128.0, 0, 255).astype(np.uint8)
    np.testing.assert_array_equal(body["rot"], q)


def _match_rows(pos, means):
    order = {tuple(m.tolist()): i for i, m in enumerate(means)}
    return np.array([order[tuple(p.tolist())] for p in pos])


def test_densification_and_opacity_reset_in_the_step_schedule():
    """refineEvery 5, warm-up 5, resetAlphaEvery 4 (reset interval 20), one
    training camera: densify at steps 10 and 15 (step % 20 > 1 + 5), opacity
    reset at step 25 (step % 20 == 5)."""
    ds, scene, cfg = _dataset(n=3000)
    tr = _trainer(ds, scene, refine_every=5, warmup_length=5, reset_alpha_every=4, densify_grad_thresh=1e-7)
    counts = []
    for _ in range(25):
        st = tr.step()
        assert np.isfinite(st.loss)
        counts.append(st.splat_count)
    assert counts[:9] == [cfg.n] * 9              # steps 1..9: no refinement
    assert counts[9] != cfg.n                     # step 10 densified
    assert counts[9] == counts[13]                # unchanged until step 15
    opac = tr.get_params()[3]
    assert opac.shape[0] == tr.splat_count
    assert float(opac.max()) <= -1.3862943611198906 + 1e-6  # step 25 reset every logit above logit(0.2)
    means = tr.get_params()[0]
    assert np.isfinite(means).all()
    st = tr.step()
    assert np.isfinite(st.loss)

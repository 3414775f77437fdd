"""The reference's Python/C surface (tests/test_msplat.py of the reference is
the model): config defaults, training steps, rendering, evaluation, and
equivalence of the trainer-level API with the oracle's training step."""
import numpy as np
import pytest

import msplat
from msplat import synthetic as S


def test_import():
    for name in ("GaussianTrainer", "TrainingConfig", "Dataset", "load_dataset", "sync", "cleanup"):
        assert hasattr(msplat, name)


def test_training_config_defaults():
    cfg = msplat.TrainingConfig()
    assert cfg.iterations == 30000
    assert cfg.sh_degree == 3
    assert cfg.ssim_weight == pytest.approx(0.2)
    assert cfg.refine_every == 100
    assert cfg.warmup_length == 500
    assert cfg.bg_color == pytest.approx([0.6130, 0.0101, 0.3984])


def test_training_config_custom_and_mutable():
    cfg = msplat.TrainingConfig(iterations=100, sh_degree=1, ssim_weight=0.0)
    assert (cfg.iterations, cfg.sh_degree, cfg.ssim_weight) == (100, 1, 0.0)
    cfg.iterations = 500
    assert cfg.iterations == 500
    c = cfg.to_c()
    assert c.iterations == 500 and c.shDegree == 1


def test_file_loaders_are_reported_missing():
    with pytest.raises(NotImplementedError, match="not part of this build"):
        msplat.load_dataset("datasets/mipnerf360/garden")


def _synthetic_dataset(n=8000, width=128, height=96, cams=6, eval_mode=False):
    """Ring cameras around a seeded scene; targets rendered by the CPU oracle."""
    from oracle import oracle as O
    cfg = S.small_config(n, 1, width, height, num_cameras=cams)
    scene = S.make_scene(cfg, seed=0)
    fx, fy, cx, cy = scene.intrinsics
    target = scene.jittered()
    imgs = []
    for k in range(cams):
        ocam = O.prepare_cam(scene.cam_to_world[k], fx, fy, cx, cy, width, height)
        imgs.append(O.render(target.params(), cfg.degree, cfg.degree, S.BACKGROUND, ocam))
    rgb = np.clip((scene.f_dc * 0.28209479177387814 + 0.5) * 255, 0, 255).astype(np.uint8)
    ds = msplat.Dataset.from_memory(scene.cam_to_world, np.tile([fx, fy, cx, cy], (cams, 1)), width, height,
                                    np.stack(imgs), scene.means, rgb, eval_mode=eval_mode, test_every=3)
    return ds, scene, cfg, imgs


@pytest.mark.gpu
def test_train_steps_render_and_evaluate():
    ds, scene, cfg, imgs = _synthetic_dataset(eval_mode=True)
    assert ds.num_train == 4 and ds.num_test == 2
    tcfg = msplat.TrainingConfig(iterations=20, sh_degree=1, num_downscales=0, sh_degree_interval=5)
    trainer = msplat.GaussianTrainer(ds, tcfg)  # point-cloud initialisation (KNN scales, random quats)
    seen = []
    trainer.train(lambda s: seen.append(s.iteration), callback_every=5)
    assert trainer.iteration == 20 and seen == [5, 10, 15, 20]
    assert trainer.splat_count == cfg.n
    st = trainer.step()
    assert st.iteration == 21 and st.splat_count == cfg.n and st.ms_per_step > 0 and np.isfinite(st.loss)
    img = trainer.render(0)
    assert img.dtype == np.float32 and img.shape == (cfg.height, cfg.width, 3)
    assert img.min() >= -0.1 and img.max() <= 1.5
    pose = ds.camera_pose(1)
    assert np.allclose(trainer.render_from_pose(pose, 1), trainer.render(1))
    rgba = trainer.render_rgba(pose, 1)
    assert rgba.shape == (cfg.height, cfg.width, 4) and (rgba[..., 3] == 255).all()
    m = trainer.evaluate()
    assert m["num_test"] == 2 and m["psnr"] > 10 and 0 < m["ssim"] < 1 and m["l1"] > 0


@pytest.mark.gpu
def test_resolution_schedule_downscales_targets():
    ds, scene, cfg, imgs = _synthetic_dataset(width=128, height=96)
    tcfg = msplat.TrainingConfig(iterations=10, sh_degree=1, num_downscales=1, resolution_schedule=5)
    trainer = msplat.GaussianTrainer(ds, tcfg, params=scene.params())
    assert trainer.render(0).shape == (48, 64, 3)  # step 0: factor 2
    for _ in range(5):
        assert np.isfinite(trainer.step().loss)
    assert trainer.render(0).shape == (96, 128, 3)  # step 5: factor 1


@pytest.mark.gpu
def test_trainer_step_matches_oracle_step():
    """Single training camera: the C API trainer (its own camera setup, target
    upload and fused step) and the oracle give the same loss, and the
    trainer's updated parameters equal the reference Adam
    (fused_adam_kernel, core/metal/msplat_metal.metal:1383-1406, first step:
    zero moments, bias corrections of t = 1) applied to the gradients the
    trainer's own step materialised, within 1e-5."""
    from msplat import _backend as B
    from oracle import oracle as O
    ds, scene, cfg, imgs = _synthetic_dataset(cams=1)
    tcfg = msplat.TrainingConfig(iterations=1000, sh_degree=1, num_downscales=0, sh_degree_interval=1)
    trainer = msplat.GaussianTrainer(ds, tcfg, params=scene.params())
    trainer.set_write_gradients(True)
    fx, fy, cx, cy = scene.intrinsics
    ocam = O.prepare_cam(scene.cam_to_world[0], fx, fy, cx, cy, cfg.width, cfg.height)
    otr = O.OracleTrainer(scene.params(), cfg.degree)
    before = [np.array(a, np.float32).copy() for a in scene.params()]  # means, scales, quats, opac, f_dc, f_rest
    st = trainer.step()
    ref = otr.step(ocam, imgs[0], S.BACKGROUND, degrees_to_use=1)
    assert abs(st.loss - ref["loss"]) <= 1e-5 * abs(ref["loss"])
    got = trainer.get_params()  # means, scales, quats, opacities, f_dc, f_rest
    names = ["dL_dmean3D", "dL_dscale", "dL_dquat", "dL_dopacity", "dL_dfeatures_dc", "dL_dfeatures_rest"]
    lrs = [O.LR_INIT[0], O.LR_INIT[1], O.LR_INIT[2], O.LR_INIT[5], O.LR_INIT[3], O.LR_INIT[4]]
    bc1 = np.float32(1.0 - float(np.float32(0.9)))
    bc2 = np.float32(1.0 - float(np.float32(0.999)))
    for a, p0, name, lr in zip(got, before, names, lrs):
        grads = B.last_tensor(name).cpu().numpy().reshape(p0.shape)
        assert np.isfinite(grads).all() and np.abs(grads).max() > 0
        p = p0.reshape(a.shape).copy()
        m = np.zeros_like(p)
        v = np.zeros_like(p)
        O.fused_adam(p, grads.reshape(p.shape), m, v, np.float32(lr) / bc1, 0.9, 0.999, float(np.sqrt(bc2)), 1e-8)
        # approximate sqrt/division in the fused update: bound the error by
        # the operands, max(|p_old|, |p_new|)
        scale = np.maximum(np.maximum(np.abs(p), np.abs(p0.reshape(a.shape))), 1e-6)
        err = np.max(np.abs(a - p) / scale)
        assert err <= 1e-5, (name, err)

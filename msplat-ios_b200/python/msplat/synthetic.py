"""Seeded synthetic scenes standing in for the reference's datasets.

The reference trains on real captures (Mip-NeRF 360 garden, loaded by
core/src/loaders/*). No dataset is available here, so the five workload
configurations of this build are generated from seeded distributions with the
shapes and value ranges of those captures:

  cfg 0  10k Gaussians, SH0, 256x256, one camera at (0,0,4)
  cfg 1  200k, SH3, 1297x840, fx=fy=1040, 16 ring cameras
  cfg 2  1M, SH3, 1920x1080, fx=fy=1500, core+shell positions
  cfg 3  3M, SH3, 4946x3286, fx=fy=3900, 32 ring cameras
  cfg 4  6M, SH3, 4946x3286, 20% of means in a clump in front of camera 0

Parameters follow the reference's storage layout (core/include/model.hpp:
means [N,3], scales [N,2] log-space, quats [N,4], opacities [N,1] logit,
featuresDc [N,3], featuresRest [N,K,3]). Cameras are OpenGL camToWorld 4x4
row-major matrices on a radius-4 ring around the origin, as Model::prepareCam
(core/src/model.cpp:500-544) expects. The target image of a camera is the
render of a jittered copy of the scene (means + N(0, 0.005), DC + N(0, 0.05)),
which the caller renders with whichever renderer it is testing.
"""
from __future__ import annotations

import dataclasses
import math

import numpy as np

BACKGROUND = np.array([0.6130, 0.0101, 0.3984], dtype=np.float32)  # model.cpp:117-118


@dataclasses.dataclass(frozen=True)
class SceneConfig:
    name: str
    n: int
    degree: int
    width: int
    height: int
    focal: float
    num_cameras: int
    layout: str            # "ball" | "core_shell" | "clump"
    log_scale_mean: float
    log_scale_std: float

    @property
    def rest_bases(self) -> int:
        return (self.degree + 1) ** 2 - 1


CONFIGS = {
    0: SceneConfig("cfg0", 10_000, 0, 256, 256, 205.0, 1, "ball", math.log(0.01), 0.5),
    1: SceneConfig("cfg1", 200_000, 3, 1297, 840, 1040.0, 16, "ball", math.log(0.01), 0.5),
    2: SceneConfig("cfg2", 1_000_000, 3, 1920, 1080, 1500.0, 16, "core_shell", math.log(0.005), 0.7),
    3: SceneConfig("cfg3", 3_000_000, 3, 4946, 3286, 3900.0, 32, "core_shell", math.log(0.005), 0.7),
    4: SceneConfig("cfg4", 6_000_000, 3, 4946, 3286, 3900.0, 32, "clump", math.log(0.02), 1.0),
}


def small_config(n: int, degree: int, width: int, height: int, focal: float | None = None,
                 num_cameras: int = 4, layout: str = "ball",
                 log_scale_mean: float = math.log(0.01), log_scale_std: float = 0.5) -> SceneConfig:
    """A reduced-size configuration for parity tests the CPU oracle finishes in seconds."""
    if focal is None:
        focal = 0.8 * width
    return SceneConfig(f"small_{n}_{degree}_{width}x{height}", n, degree, width, height, focal,
                       num_cameras, layout, log_scale_mean, log_scale_std)


def _uniform_ball(rng: np.random.Generator, n: int, radius: float) -> np.ndarray:
    d = rng.standard_normal((n, 3))
    d /= np.linalg.norm(d, axis=1, keepdims=True) + 1e-12
    r = radius * rng.random(n) ** (1.0 / 3.0)
    return d * r[:, None]


def look_at_gl(pos: np.ndarray, target=(0.0, 0.0, 0.0), up=(0.0, 1.0, 0.0)) -> np.ndarray:
    """OpenGL camToWorld (columns right, up, back, position), row-major float32."""
    pos = np.asarray(pos, dtype=np.float64)
    back = pos - np.asarray(target, dtype=np.float64)
    back /= np.linalg.norm(back)
    right = np.cross(np.asarray(up, dtype=np.float64), back)
    right /= np.linalg.norm(right)
    upv = np.cross(back, right)
    m = np.eye(4)
    m[:3, 0], m[:3, 1], m[:3, 2], m[:3, 3] = right, upv, back, pos
    return m.astype(np.float32)


def ring_cameras(num: int, radius: float = 4.0) -> np.ndarray:
    """num camToWorld matrices on a ring in the x-z plane; camera 0 sits at (0, 0, radius)."""
    mats = []
    for k in range(num):
        th = 2.0 * math.pi * k / num
        mats.append(look_at_gl((radius * math.sin(th), 0.0, radius * math.cos(th))))
    return np.stack(mats)


@dataclasses.dataclass
class Scene:
    cfg: SceneConfig
    means: np.ndarray
    scales: np.ndarray
    quats: np.ndarray
    opacities: np.ndarray
    f_dc: np.ndarray
    f_rest: np.ndarray
    cam_to_world: np.ndarray  # [C, 4, 4]

    def params(self):
        return (self.means, self.scales, self.quats, self.opacities, self.f_dc, self.f_rest)

    @property
    def intrinsics(self):
        c = self.cfg
        return (c.focal, c.focal, c.width / 2.0, c.height / 2.0)

    def jittered(self, seed: int = 1) -> "Scene":
        """The target scene: means + N(0, 0.005), DC + N(0, 0.05)."""
        rng = np.random.default_rng(seed)
        means = self.means + rng.normal(0.0, 0.005, self.means.shape).astype(np.float32)
        f_dc = self.f_dc + rng.normal(0.0, 0.05, self.f_dc.shape).astype(np.float32)
        return dataclasses.replace(self, means=means.astype(np.float32), f_dc=f_dc.astype(np.float32))


def make_scene(cfg: SceneConfig, seed: int = 0) -> Scene:
    rng = np.random.default_rng(seed)
    n = cfg.n
    if cfg.layout == "ball":
        means = _uniform_ball(rng, n, 1.0)
    elif cfg.layout == "core_shell":
        n_core = int(round(0.7 * n))
        core = rng.normal(0.0, 0.3, (n_core, 3))
        shell = _uniform_ball(rng, n - n_core, 3.0)
        means = np.concatenate([core, shell])
    elif cfg.layout == "clump":
        n_clump = int(round(0.2 * n))
        # camera 0 sits at (0, 0, 4) looking at the origin: the clump centre is
        # 2.5 in front of it on its optical axis.
        clump = rng.normal(0.0, 0.02, (n_clump, 3)) + np.array([0.0, 0.0, 1.5])
        rest = _uniform_ball(rng, n - n_clump, 3.0)
        means = np.concatenate([clump, rest])
    else:
        raise ValueError(cfg.layout)
    means = means.astype(np.float32)
    scales = rng.normal(cfg.log_scale_mean, cfg.log_scale_std, (n, 2)).astype(np.float32)
    q = rng.standard_normal((n, 4))
    q /= np.linalg.norm(q, axis=1, keepdims=True) + 1e-12
    quats = q.astype(np.float32)
    opac = rng.standard_normal((n, 1)).astype(np.float32)
    f_dc = rng.uniform(-0.5, 0.5, (n, 3)).astype(np.float32)
    k = cfg.rest_bases
    f_rest = (rng.normal(0.0, 0.05, (n, k, 3)) if k > 0 else np.zeros((n, 0, 3))).astype(np.float32)
    return Scene(cfg, means, scales, quats, opac, f_dc, f_rest, ring_cameras(cfg.num_cameras))

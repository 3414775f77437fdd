"""Shared scene cases for the parity tests (seeded, small enough for the CPU oracle)."""
from __future__ import annotations

import math

import numpy as np

from msplat import synthetic as S
from oracle import oracle as O


def case_config(name: str) -> S.SceneConfig:
    if name == "cfg0":
        return S.CONFIGS[0]
    if name == "sh3_small":
        return S.small_config(20_000, 3, 320, 240, num_cameras=3)
    if name == "sh1_odd":
        # image size not a multiple of the 16-pixel tile
        return S.small_config(8_000, 1, 203, 117, focal=170.0, num_cameras=2)
    if name == "overflow":
        # big surfels on a small image: most tiles exceed the 2048 cap
        return S.small_config(24_000, 2, 96, 80, focal=90.0, num_cameras=1,
                              log_scale_mean=math.log(0.08), log_scale_std=0.3)
    if name == "thin":
        # strongly anisotropic surfels in every orientation: thin, grazing
        # ellipses exercise the rasteriser's conic cull at its boundary
        return S.small_config(12_000, 1, 256, 192, focal=230.0, num_cameras=2,
                              log_scale_mean=math.log(0.02), log_scale_std=1.6)
    if name == "dense":
        # large surfels on a small image: the middle tile rows hold 50,000 to
        # 126,000 Gaussians per tile, far over the 2048 cap (route summaries,
        # bands and payloads under heavy tiles)
        return S.small_config(150_000, 1, 48, 96, focal=60.0, num_cameras=1,
                              log_scale_mean=math.log(0.15), log_scale_std=0.2)
    if name in ("cfg1", "cfg2", "cfg3", "cfg4"):
        return S.CONFIGS[int(name[3:])]
    raise KeyError(name)


class Case:
    """Scene, first camera, oracle camera and the oracle-rendered target."""

    def __init__(self, name: str, cam_index: int = 0, seed: int = 0):
        self.name = name
        self.cam_index = cam_index
        self.cfg = case_config(name)
        self.scene = S.make_scene(self.cfg, seed=seed)
        fx, fy, cx, cy = self.scene.intrinsics
        self.ocam = O.prepare_cam(self.scene.cam_to_world[cam_index], fx, fy, cx, cy, self.cfg.width,
                                  self.cfg.height)
        self.degree = self.cfg.degree
        self.bg = S.BACKGROUND
        self._gt = None

    @property
    def gt(self) -> np.ndarray:
        if self._gt is None:
            self._gt = O.render(self.scene.jittered().params(), self.degree, self.degree, self.bg, self.ocam)
        return self._gt

    def product_camera(self, B):
        """The camera as the product builds it (msplat_prepare_camera)."""
        fx, fy, cx, cy = self.scene.intrinsics
        return B.prepare_camera(self.scene.cam_to_world[self.cam_index], fx, fy, cx, cy, self.cfg.width,
                                self.cfg.height)

    def oracle_forward(self):
        p = O.project_forward(*self.scene.params(), self.degree, self.degree, self.ocam)
        bins = O.bin_and_sort(p, self.ocam)
        packed = O.pack(bins, p)
        fwd = O.rasterize_forward(bins, packed, self.ocam, self.bg)
        return p, bins, packed, fwd


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    den = np.linalg.norm(b)
    if den == 0:
        return float(np.linalg.norm(a))
    return float(np.linalg.norm(a - b) / den)

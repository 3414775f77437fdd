"""Python surface mirroring the reference's python/msplat package
(python/bindings.cpp:25-280, python/msplat/__init__.py), implemented over the
trainer-level C API (include/msplat_c_api.h) of libmsplat_b200.so."""
from __future__ import annotations

import ctypes as C
import os
import dataclasses
from typing import Callable, List, Optional

import numpy as np

from . import _backend


class MsplatConfig(C.Structure):
    _fields_ = [("iterations", C.c_int), ("shDegree", C.c_int), ("shDegreeInterval", C.c_int),
                ("ssimWeight", C.c_float), ("numDownscales", C.c_int), ("resolutionSchedule", C.c_int),
                ("refineEvery", C.c_int), ("warmupLength", C.c_int), ("resetAlphaEvery", C.c_int),
                ("densifyGradThresh", C.c_float), ("densifySizeThresh", C.c_float), ("stopScreenSizeAt", C.c_int),
                ("splitScreenSize", C.c_float), ("keepCrs", C.c_bool), ("downscaleFactor", C.c_float),
                ("bgColor", C.c_float * 3)]


class MsplatStats(C.Structure):
    _fields_ = [("iteration", C.c_int), ("splatCount", C.c_int), ("msPerStep", C.c_float), ("loss", C.c_float)]


class MsplatEvalMetrics(C.Structure):
    _fields_ = [("psnr", C.c_float), ("ssim", C.c_float), ("l1", C.c_float), ("numTest", C.c_int),
                ("numGaussians", C.c_int)]


class MsplatPixelBuffer(C.Structure):
    _fields_ = [("data", C.POINTER(C.c_float)), ("width", C.c_int), ("height", C.c_int)]


@dataclasses.dataclass
class TrainingConfig:
    """Defaults of python/bindings.cpp:25-46 (and MsplatConfig, msplat_c_api.h:35-53)."""
    iterations: int = 30000
    sh_degree: int = 3
    sh_degree_interval: int = 1000
    ssim_weight: float = 0.2
    num_downscales: int = 2
    resolution_schedule: int = 3000
    refine_every: int = 100
    warmup_length: int = 500
    reset_alpha_every: int = 30
    densify_grad_thresh: float = 0.0002
    densify_size_thresh: float = 0.01
    stop_screen_size_at: int = 4000
    split_screen_size: float = 0.05
    keep_crs: bool = False
    downscale_factor: float = 1.0
    output: str = "splat.ply"
    save_every: int = -1
    bg_color: List[float] = dataclasses.field(default_factory=lambda: [0.6130, 0.0101, 0.3984])

    def to_c(self) -> MsplatConfig:
        c = MsplatConfig()
        c.iterations, c.shDegree, c.shDegreeInterval = self.iterations, self.sh_degree, self.sh_degree_interval
        c.ssimWeight, c.numDownscales, c.resolutionSchedule = self.ssim_weight, self.num_downscales, \
            self.resolution_schedule
        c.refineEvery, c.warmupLength, c.resetAlphaEvery = self.refine_every, self.warmup_length, \
            self.reset_alpha_every
        c.densifyGradThresh, c.densifySizeThresh = self.densify_grad_thresh, self.densify_size_thresh
        c.stopScreenSizeAt, c.splitScreenSize = self.stop_screen_size_at, self.split_screen_size
        c.keepCrs, c.downscaleFactor = self.keep_crs, self.downscale_factor
        c.bgColor[:] = [float(x) for x in self.bg_color]
        return c


@dataclasses.dataclass
class TrainingStats:
    """python/bindings.cpp:50-54, plus the step's loss."""
    iteration: int
    splat_count: int
    ms_per_step: float
    loss: float = 0.0


def _lib():
    L = _backend.load()
    if getattr(L, "_api_typed", False):
        return L
    vp, i, f, b = C.c_void_p, C.c_int, C.c_float, C.c_bool
    fp = C.POINTER(C.c_float)
    L.msplat_dataset_create.argtypes = [C.c_char_p, f, b, i]
    L.msplat_dataset_create.restype = vp
    L.msplat_dataset_create_from_memory.argtypes = [i, fp, fp, i, i, fp, i, fp, C.POINTER(C.c_uint8), b, i]
    L.msplat_dataset_create_from_memory.restype = vp
    L.msplat_dataset_destroy.argtypes = [vp]
    for nm in ("msplat_dataset_num_train", "msplat_dataset_num_test"):
        getattr(L, nm).argtypes = [vp]
        getattr(L, nm).restype = i
    L.msplat_dataset_camera_pose.argtypes = [vp, i, fp]
    L.msplat_trainer_create.argtypes = [vp, MsplatConfig]
    L.msplat_trainer_create.restype = vp
    L.msplat_trainer_create_from_params.argtypes = [vp, MsplatConfig, i, fp, fp, fp, fp, fp, fp]
    L.msplat_trainer_create_from_params.restype = vp
    L.msplat_trainer_destroy.argtypes = [vp]
    L.msplat_trainer_step.argtypes = [vp]
    L.msplat_trainer_step.restype = MsplatStats
    L.msplat_trainer_train.argtypes = [vp]
    L.msplat_trainer_evaluate.argtypes = [vp]
    L.msplat_trainer_evaluate.restype = MsplatEvalMetrics
    L.msplat_trainer_render.argtypes = [vp, i, b]
    L.msplat_trainer_render.restype = MsplatPixelBuffer
    L.msplat_trainer_render_pose.argtypes = [vp, fp, i]
    L.msplat_trainer_render_pose.restype = MsplatPixelBuffer
    L.msplat_trainer_render_pose_to_buffer.argtypes = [vp, fp, i, C.POINTER(C.c_uint8), C.POINTER(i), C.POINTER(i)]
    for nm in ("msplat_trainer_splat_count", "msplat_trainer_iteration"):
        getattr(L, nm).argtypes = [vp]
        getattr(L, nm).restype = i
    L.msplat_trainer_get_params.argtypes = [vp, fp, fp, fp, fp, fp, fp]
    L.msplat_trainer_get_params.restype = i
    L.msplat_trainer_set_write_gradients.argtypes = [vp, i]
    L.msplat_trainer_set_write_gradients.restype = i
    for nm in ("msplat_trainer_export_ply", "msplat_trainer_export_splat", "msplat_trainer_save_checkpoint"):
        getattr(L, nm).argtypes = [vp, C.c_char_p]
        getattr(L, nm).restype = None
    L.msplat_trainer_load_checkpoint.argtypes = [vp, C.c_char_p]
    L.msplat_trainer_load_checkpoint.restype = i
    L.msplat_sync.argtypes = []
    L.msplat_cleanup.argtypes = []
    L._libc = C.CDLL(None)
    L._libc.free.argtypes = [vp]
    L._api_typed = True
    return L


def _err(L) -> str:
    return L.msplat_last_error().decode()


def _fptr(a):
    return None if a is None else a.ctypes.data_as(C.POINTER(C.c_float))


class Dataset:
    """A set of posed cameras with target images and an initial point cloud.

    The reference's loaders (COLMAP, Nerfstudio, Polycam; python/bindings.cpp:
    59-97) are not part of this build: construct datasets from memory with
    Dataset.from_memory."""

    def __init__(self, path: str, downscale_factor: float = 1.0, eval_mode: bool = False, test_every: int = 8):
        L = _lib()
        h = L.msplat_dataset_create(str(path).encode(), downscale_factor, eval_mode, test_every)
        if not h:
            raise NotImplementedError(_err(L))
        self._h = h

    @classmethod
    def from_memory(cls, cam_to_world, intrinsics, width: int, height: int, images=None, xyz=None, rgb=None,
                    eval_mode: bool = False, test_every: int = 8) -> "Dataset":
        L = _lib()
        c2w = np.ascontiguousarray(cam_to_world, np.float32).reshape(-1, 16)
        intr = np.ascontiguousarray(intrinsics, np.float32).reshape(-1, 4)
        imgs = None if images is None else np.ascontiguousarray(images, np.float32)
        xyz = np.zeros((0, 3), np.float32) if xyz is None else np.ascontiguousarray(xyz, np.float32)
        rgb = np.zeros((0, 3), np.uint8) if rgb is None else np.ascontiguousarray(rgb, np.uint8)
        h = L.msplat_dataset_create_from_memory(len(c2w), _fptr(c2w), _fptr(intr), width, height, _fptr(imgs),
                                                len(xyz), _fptr(xyz), rgb.ctypes.data_as(C.POINTER(C.c_uint8)),
                                                eval_mode, test_every)
        if not h:
            raise RuntimeError(_err(L))
        self = cls.__new__(cls)
        self._h = h
        return self

    @property
    def num_train(self) -> int:
        return _lib().msplat_dataset_num_train(self._h)

    @property
    def num_test(self) -> int:
        return _lib().msplat_dataset_num_test(self._h)

    def camera_pose(self, index: int) -> np.ndarray:
        if index < 0 or index >= self.num_train:
            raise RuntimeError("Camera index out of range")
        out = np.zeros(16, np.float32)
        _lib().msplat_dataset_camera_pose(self._h, index, _fptr(out))
        return out.reshape(4, 4)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            _lib().msplat_dataset_destroy(h)
            self._h = None


class GaussianTrainer:
    """python/bindings.cpp:101-280 over msplat_trainer_*."""

    def __init__(self, dataset: Dataset, config: Optional[TrainingConfig] = None, params=None):
        L = _lib()
        self.dataset = dataset  # keeps the dataset alive
        self.config = config or TrainingConfig()
        c = self.config.to_c()
        if params is None:
            h = L.msplat_trainer_create(dataset._h, c)
        else:
            means, scales, quats, opac, f_dc, f_rest = [np.ascontiguousarray(p, np.float32) for p in params]
            h = L.msplat_trainer_create_from_params(dataset._h, c, len(means), _fptr(means), _fptr(scales),
                                                    _fptr(quats), _fptr(opac.reshape(-1)), _fptr(f_dc),
                                                    _fptr(f_rest) if f_rest.size else None)
        if not h:
            raise RuntimeError(_err(L))
        self._h = h

    def step(self) -> TrainingStats:
        L = _lib()
        s = L.msplat_trainer_step(self._h)
        msg = _err(L)
        if msg:
            raise RuntimeError(msg)
        return TrainingStats(s.iteration, s.splatCount, s.msPerStep, s.loss)

    def train(self, callback: Optional[Callable[[TrainingStats], None]] = None, callback_every: int = 0):
        while self.iteration < self.config.iterations:
            st = self.step()
            if callback is not None and callback_every > 0 and st.iteration % callback_every == 0:
                callback(st)

    def _pixels(self, buf: MsplatPixelBuffer) -> np.ndarray:
        L = _lib()
        if not buf.data:
            raise RuntimeError(_err(L) or "render failed")
        arr = np.ctypeslib.as_array(buf.data, shape=(buf.height, buf.width, 3)).copy()
        L._libc.free(C.cast(buf.data, C.c_void_p))
        return arr

    def render(self, camera_index: int, use_test: bool = False) -> np.ndarray:
        return self._pixels(_lib().msplat_trainer_render(self._h, camera_index, use_test))

    def render_from_pose(self, cam_to_world, ref_camera_index: int = 0) -> np.ndarray:
        m = np.ascontiguousarray(cam_to_world, np.float32).reshape(16)
        return self._pixels(_lib().msplat_trainer_render_pose(self._h, _fptr(m), ref_camera_index))

    def render_rgba(self, cam_to_world, ref_camera_index: int = 0) -> np.ndarray:
        L = _lib()
        m = np.ascontiguousarray(cam_to_world, np.float32).reshape(16)
        w, h = C.c_int(), C.c_int()
        L.msplat_trainer_render_pose_to_buffer(self._h, _fptr(m), ref_camera_index, None, C.byref(w), C.byref(h))
        out = np.zeros((h.value, w.value, 4), np.uint8)
        L.msplat_trainer_render_pose_to_buffer(self._h, _fptr(m), ref_camera_index,
                                               out.ctypes.data_as(C.POINTER(C.c_uint8)), C.byref(w), C.byref(h))
        return out

    def evaluate(self) -> dict:
        if self.dataset.num_test == 0:
            raise RuntimeError("No test cameras. Load dataset with eval_mode=True.")
        m = _lib().msplat_trainer_evaluate(self._h)
        return {"psnr": m.psnr, "ssim": m.ssim, "l1": m.l1, "num_test": m.numTest, "num_gaussians": m.numGaussians}

    def set_write_gradients(self, enable: bool = True):
        """Make every later step also write its per-group gradients to the
        backend workspace (msplat_backend last tensors dL_dmean3D, ...)."""
        if _lib().msplat_trainer_set_write_gradients(self._h, 1 if enable else 0):
            raise RuntimeError(_err(_lib()))

    def get_params(self):
        n = self.splat_count
        k = (self.config.sh_degree + 1) ** 2 - 1
        out = [np.zeros((n, 3), np.float32), np.zeros((n, 2), np.float32), np.zeros((n, 4), np.float32),
               np.zeros((n, 1), np.float32), np.zeros((n, 3), np.float32), np.zeros((n, k, 3), np.float32)]
        rc = _lib().msplat_trainer_get_params(self._h, *[_fptr(a) for a in out])
        if rc:
            raise RuntimeError(_err(_lib()))
        return out

    def _path_call(self, name: str, path: str):
        L = _lib()
        r = getattr(L, name)(self._h, os.fspath(path).encode())
        msg = _err(L)
        if msg:
            raise RuntimeError(msg)
        return r

    def export_ply(self, path: str):
        """Export the current Gaussians as a PLY file (saveGaussianPly)."""
        self._path_call("msplat_trainer_export_ply", path)

    def export_splat(self, path: str):
        """Export the current Gaussians as a .splat file (saveGaussianSplat)."""
        self._path_call("msplat_trainer_export_splat", path)

    def save_checkpoint(self, path: str):
        """Save a training checkpoint ("MSPL" version 1)."""
        self._path_call("msplat_trainer_save_checkpoint", path)

    def load_checkpoint(self, path: str) -> int:
        """Load a training checkpoint and resume from the saved iteration."""
        return self._path_call("msplat_trainer_load_checkpoint", path)

    @property
    def splat_count(self) -> int:
        return _lib().msplat_trainer_splat_count(self._h)

    @property
    def iteration(self) -> int:
        return _lib().msplat_trainer_iteration(self._h)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            _lib().msplat_trainer_destroy(h)
            self._h = None


def sync():
    _lib().msplat_sync()


def cleanup():
    _lib().msplat_cleanup()


def load_dataset(path: str, downscale_factor: float = 1.0, eval_mode: bool = False, test_every: int = 8) -> Dataset:
    """Load a dataset from disk (raises NotImplementedError: loaders are not part of this build)."""
    return Dataset(path, downscale_factor, eval_mode, test_every)

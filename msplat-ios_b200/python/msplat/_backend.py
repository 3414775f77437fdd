"""ctypes binding of include/msplat_backend.h (libmsplat_b200.so).

Torch is used here only for device memory and streams: tensors are passed to
the C ABI as raw device pointers. There is no CPU or PyTorch fallback: if the
CUDA library is missing or a call fails, an exception is raised.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_PKG = os.path.dirname(os.path.abspath(__file__))
_ROOT = os.path.dirname(os.path.dirname(_PKG))  # msplat-ios_b200/
LIB_PATH = os.path.join(_ROOT, "lib", "libmsplat_b200.so")

MSPLAT_OK = 0


class MsplatError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"msplat error {code}: {msg}")
        self.code = code


class MsplatCamera(C.Structure):
    _fields_ = [("viewmat", C.c_float * 16), ("projmat", C.c_float * 16), ("fx", C.c_float), ("fy", C.c_float),
                ("cx", C.c_float), ("cy", C.c_float), ("width", C.c_int32), ("height", C.c_int32),
                ("cam_pos", C.c_float * 3)]


class MsplatGaussians(C.Structure):
    _fields_ = [("num_points", C.c_int32), ("sh_degree", C.c_int32), ("means", C.c_void_p), ("scales", C.c_void_p),
                ("quats", C.c_void_p), ("opacities", C.c_void_p), ("features_dc", C.c_void_p),
                ("features_rest", C.c_void_p)]


class MsplatAdamState(C.Structure):
    _fields_ = [("exp_avg", C.c_void_p * 6), ("exp_avg_sq", C.c_void_p * 6), ("lr", C.c_float * 6),
                ("step", C.c_int32), ("beta1", C.c_float), ("beta2", C.c_float), ("eps", C.c_float)]


class MsplatDensifyArgs(C.Structure):
    _fields_ = [("grad_thresh", C.c_float), ("size_thresh", C.c_float), ("screen_thresh", C.c_float),
                ("check_screen", C.c_int32), ("cull_alpha_thresh", C.c_float), ("cull_scale_thresh", C.c_float),
                ("cull_screen_size", C.c_float), ("check_huge", C.c_int32), ("half_max_dim", C.c_float),
                ("log_size_fac", C.c_float), ("xys_grad_norm", C.c_void_p), ("vis_counts", C.c_void_p),
                ("max_2d_size", C.c_void_p)]


class MsplatDensifyPlan(C.Structure):
    _fields_ = [("num_splits", C.c_int32), ("num_dups", C.c_int32), ("new_count", C.c_int32)]


MAX_PEER_RANKS = 16


class MsplatPeerParams(C.Structure):
    _fields_ = [("world", C.c_int32), ("chunk", C.c_int32), ("base", (C.c_void_p * MAX_PEER_RANKS) * 6)]


class MsplatRoutePeers(C.Structure):
    _fields_ = [("world", C.c_int32), ("rank", C.c_int32), ("inbox_items", C.c_int64),
                ("returnbox_items", C.c_int64), ("inbox", C.c_void_p * MAX_PEER_RANKS),
                ("returnbox", C.c_void_p * MAX_PEER_RANKS)]


class MsplatTensorRef(C.Structure):
    _fields_ = [("data", C.c_void_p), ("shape", C.c_int64 * 4), ("ndim", C.c_int32), ("dtype", C.c_int32)]


_lib = None


def lib_path() -> str:
    return LIB_PATH


def load():
    """Load libmsplat_b200.so (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `python msplat-ios_b200/build.py`")
    L = C.CDLL(LIB_PATH)
    vp, f, i32, i64, u32 = C.c_void_p, C.c_float, C.c_int32, C.c_int64, C.c_uint32
    fp3 = C.POINTER(C.c_float)
    L.msplat_render.argtypes = [C.POINTER(MsplatGaussians), C.POINTER(MsplatCamera), f, f, i32, fp3, vp, vp]
    L.msplat_train_step_2dgs.argtypes = [C.POINTER(MsplatGaussians), C.POINTER(MsplatCamera), f, f, i32, fp3, vp,
                                         f, f, f, vp, vp, vp, f, C.POINTER(C.c_float), vp]
    L.msplat_fused_adam.argtypes = [vp, vp, vp, vp, u32, f, f, f, f, f, vp]
    L.msplat_train_step_fused.argtypes = [C.POINTER(MsplatGaussians), C.POINTER(MsplatCamera), i32, fp3, vp, f, f,
                                          f, C.POINTER(MsplatAdamState), vp, vp, vp, vp, i32, vp]
    L.msplat_shard_forward_backward.argtypes = [C.POINTER(MsplatGaussians), C.POINTER(MsplatCamera), i32, fp3, vp,
                                                f, f, f, i32, i32, C.POINTER(C.c_int32), vp, vp, vp]
    L.msplat_shard_forward_backward_after.argtypes = [C.POINTER(MsplatGaussians), C.POINTER(MsplatCamera), i32, fp3,
                                                      vp, f, f, f, i32, i32, C.POINTER(C.c_int32), vp, vp, vp, i32,
                                                      vp]
    L.msplat_shard_forward_backward_peers.argtypes = [C.POINTER(MsplatGaussians), C.POINTER(MsplatPeerParams),
                                                      C.POINTER(MsplatCamera), i32, fp3, vp, f, f, f, i32, i32,
                                                      C.POINTER(C.c_int32), vp, vp, vp]
    L.msplat_shard_forward_backward_rgb.argtypes = [C.POINTER(MsplatGaussians), C.POINTER(MsplatCamera), i32, fp3,
                                                    vp, f, f, f, i32, i32, C.POINTER(C.c_int32), vp, vp, vp, vp,
                                                    vp]
    L.msplat_shard_colors.argtypes = [C.POINTER(MsplatGaussians), C.POINTER(MsplatCamera), i32, i32, i32, vp, vp]
    L.msplat_device_alloc.argtypes = [C.c_uint64, C.POINTER(C.c_void_p)]
    L.msplat_device_free.argtypes = [vp]
    L.msplat_ipc_handle.argtypes = [vp, C.c_char * 64]
    L.msplat_ipc_open.argtypes = [C.c_char * 64, C.POINTER(C.c_void_p)]
    L.msplat_ipc_close.argtypes = [vp]
    L.msplat_shard_project_backward_adam.argtypes = [C.POINTER(MsplatGaussians), C.POINTER(MsplatCamera), i32, vp,
                                                     i32, i32, C.POINTER(MsplatAdamState), vp, vp, vp, vp]
    L.msplat_last_tensor.argtypes = [C.c_char_p, C.POINTER(MsplatTensorRef)]
    L.msplat_route_project.argtypes = [C.POINTER(MsplatGaussians), C.POINTER(MsplatCamera), i32, i32, i32, vp, vp]
    L.msplat_route_summary_len.argtypes = [C.POINTER(MsplatCamera), C.POINTER(C.c_int64)]
    L.msplat_route_plan.argtypes = [vp, C.POINTER(MsplatCamera), i32, i32, C.POINTER(C.c_int32), C.POINTER(C.c_int64),
                                    C.POINTER(C.c_int64), vp]
    L.msplat_route_pack.argtypes = [vp, vp]
    L.msplat_route_pack_peers.argtypes = [C.POINTER(MsplatRoutePeers), vp]
    L.msplat_route_push_peers.argtypes = [C.POINTER(MsplatRoutePeers), vp, vp]
    L.msplat_route_band.argtypes = [C.POINTER(MsplatCamera), i32, vp, i64, i32, i32, fp3, vp, f, f, f, vp, vp, vp]
    L.msplat_route_return.argtypes = [vp, i64, vp, vp]
    L.msplat_route_project_backward_adam.argtypes = [C.POINTER(MsplatGaussians), C.POINTER(MsplatCamera), i32, vp,
                                                     C.POINTER(MsplatAdamState), vp, vp, vp, vp]
    L.msplat_prepare_camera.argtypes = [C.POINTER(C.c_float), f, f, f, f, i32, i32, C.POINTER(MsplatCamera)]
    L.msplat_densify_plan.argtypes = [C.POINTER(MsplatGaussians), C.POINTER(MsplatDensifyArgs),
                                      C.POINTER(MsplatDensifyPlan), vp]
    L.msplat_densify_apply.argtypes = [C.POINTER(MsplatGaussians), C.POINTER(MsplatAdamState),
                                       C.POINTER(MsplatDensifyArgs), vp, C.POINTER(MsplatGaussians),
                                       C.POINTER(MsplatAdamState), vp]
    L.msplat_reset_opacity.argtypes = [vp, vp, vp, i32, f, vp]
    L.msplat_normal_samples.argtypes = [u32, i64, vp]
    L.msplat_normal_samples.restype = C.c_int
    L.msplat_last_num_intersections.restype = i64
    L.msplat_last_status_flags.restype = u32
    L.msplat_launch_count.restype = i64
    L.msplat_set_stage_timing.argtypes = [i32]
    L.msplat_set_stage_timing.restype = C.c_int
    L.msplat_set_raster_counters.argtypes = [i32]
    L.msplat_set_raster_counters.restype = C.c_int
    L.msplat_stage_times.argtypes = [C.POINTER(C.c_double), C.POINTER(C.c_int64), i32]
    L.msplat_stage_times.restype = i32
    L.msplat_stage_name.argtypes = [i32]
    L.msplat_stage_name.restype = C.c_char_p
    L.msplat_last_error.restype = C.c_char_p
    for name in ("msplat_render", "msplat_train_step_2dgs", "msplat_fused_adam", "msplat_train_step_fused",
                 "msplat_shard_forward_backward", "msplat_shard_forward_backward_after",
                 "msplat_shard_forward_backward_peers", "msplat_shard_forward_backward_rgb", "msplat_shard_colors",
                 "msplat_device_alloc", "msplat_device_free",
                 "msplat_ipc_handle", "msplat_ipc_open", "msplat_ipc_close",
                 "msplat_shard_project_backward_adam", "msplat_last_tensor", "msplat_prepare_camera",
                 "msplat_route_summary_len", "msplat_route_project", "msplat_route_plan", "msplat_route_pack", "msplat_route_pack_peers",
                 "msplat_route_push_peers", "msplat_route_band",
                 "msplat_route_return", "msplat_route_project_backward_adam",
                 "msplat_densify_plan", "msplat_densify_apply", "msplat_reset_opacity"):
        getattr(L, name).restype = C.c_int
    _lib = L
    return L


def _check(code: int):
    if code != MSPLAT_OK:
        raise MsplatError(code, load().msplat_last_error().decode())


def _ptr(t):
    if t is None:
        return None
    if isinstance(t, int):
        return t
    import torch
    assert isinstance(t, torch.Tensor) and t.is_cuda and t.is_contiguous() and t.dtype in (
        torch.float32, torch.int32, torch.float64), (t.dtype, t.device)
    return t.data_ptr()


def _stream(stream=None):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def camera(viewmat, projmat, fx, fy, cx, cy, width, height, cam_pos) -> MsplatCamera:
    c = MsplatCamera()
    c.viewmat[:] = [float(x) for x in np.asarray(viewmat, np.float32).reshape(16)]
    c.projmat[:] = [float(x) for x in np.asarray(projmat, np.float32).reshape(16)]
    c.fx, c.fy, c.cx, c.cy = float(fx), float(fy), float(cx), float(cy)
    c.width, c.height = int(width), int(height)
    c.cam_pos[:] = [float(x) for x in np.asarray(cam_pos, np.float32).reshape(3)]
    return c


def prepare_camera(cam_to_world, fx, fy, cx, cy, width, height) -> MsplatCamera:
    """Model::prepareCam (core/src/model.cpp:500-544) in the library
    (msplat_prepare_camera): view and projection matrices of an OpenGL
    camToWorld matrix, host code, no GPU needed."""
    m = np.ascontiguousarray(np.asarray(cam_to_world, np.float32).reshape(16))
    cam = MsplatCamera()
    _check(load().msplat_prepare_camera(m.ctypes.data_as(C.POINTER(C.c_float)), fx, fy, cx, cy, width, height,
                                        C.byref(cam)))
    return cam


def camera_from_oracle(ocam) -> MsplatCamera:
    """Copy of a camera struct with the same field layout (e.g. the checker's)."""
    return camera(ocam.viewmat[:], ocam.projmat[:], ocam.fx, ocam.fy, ocam.cx, ocam.cy, ocam.width, ocam.height,
                  ocam.cam_pos[:])


class DeviceGaussians:
    """Parameters as torch CUDA tensors in the reference layout."""

    def __init__(self, means, scales, quats, opacities, f_dc, f_rest, sh_degree: int, device="cuda"):
        import torch
        t = lambda a: torch.as_tensor(np.ascontiguousarray(a, np.float32)).to(device).contiguous()
        self.means, self.scales, self.quats = t(means), t(scales), t(quats)
        self.opacities = t(np.asarray(opacities).reshape(-1, 1))
        self.f_dc = t(f_dc)
        self.f_rest = t(f_rest)
        self.sh_degree = sh_degree

    @property
    def n(self):
        return self.means.shape[0]

    def groups(self):
        return [self.means, self.scales, self.quats, self.f_dc, self.f_rest, self.opacities]

    def struct(self) -> MsplatGaussians:
        g = MsplatGaussians()
        g.num_points, g.sh_degree = self.n, self.sh_degree
        g.means, g.scales, g.quats = _ptr(self.means), _ptr(self.scales), _ptr(self.quats)
        g.opacities, g.features_dc = _ptr(self.opacities), _ptr(self.f_dc)
        g.features_rest = _ptr(self.f_rest) if self.f_rest.numel() else None
        return g


def _bg(background):
    return (C.c_float * 3)(*[float(x) for x in np.asarray(background, np.float32).reshape(3)])


def render(g: DeviceGaussians, cam: MsplatCamera, degrees_to_use: int, background, out_img=None, glob_scale=1.0,
           clip_thresh=0.01, stream=None):
    gs = g.struct()
    _check(load().msplat_render(C.byref(gs), C.byref(cam), glob_scale, clip_thresh, degrees_to_use, _bg(background),
                                _ptr(out_img), _stream(stream)))


def train_step_2dgs(g: DeviceGaussians, cam: MsplatCamera, degrees_to_use: int, background, gt, lambda_l1,
                    lambda_dist, lambda_dssim, stats=None, glob_scale=1.0, clip_thresh=0.01, stream=None) -> float:
    gs = g.struct()
    loss = C.c_float()
    sp = [None, None, None] if stats is None else [_ptr(s) for s in stats]
    inv_max_dim = 1.0 / max(cam.width, cam.height)
    _check(load().msplat_train_step_2dgs(C.byref(gs), C.byref(cam), glob_scale, clip_thresh, degrees_to_use,
                                         _bg(background), _ptr(gt), lambda_l1, lambda_dist, lambda_dssim, sp[0], sp[1],
                                         sp[2], inv_max_dim, C.byref(loss), _stream(stream)))
    return loss.value


def fused_adam(params, grads, m, v, step_size, beta1, beta2, bc2_sqrt, eps, stream=None):
    _check(load().msplat_fused_adam(_ptr(params), _ptr(grads), _ptr(m), _ptr(v), params.numel(), step_size, beta1,
                                    beta2, bc2_sqrt, eps, _stream(stream)))


class AdamState:
    LR_INIT = (0.00016, 0.005, 0.001, 0.0025, 0.000125, 0.05)  # model.cpp:142

    def __init__(self, g: DeviceGaussians):
        import torch
        self.m = [torch.zeros_like(p) for p in g.groups()]
        self.v = [torch.zeros_like(p) for p in g.groups()]
        self.lr = list(self.LR_INIT)
        self.step = 0
        self.beta1, self.beta2, self.eps = 0.9, 0.999, 1e-8

    def struct(self) -> MsplatAdamState:
        a = MsplatAdamState()
        for k in range(6):
            a.exp_avg[k] = _ptr(self.m[k]) if self.m[k].numel() else None
            a.exp_avg_sq[k] = _ptr(self.v[k]) if self.v[k].numel() else None
            a.lr[k] = self.lr[k]
        a.step, a.beta1, a.beta2, a.eps = self.step, self.beta1, self.beta2, self.eps
        return a


def train_step_fused(g: DeviceGaussians, cam: MsplatCamera, degrees_to_use: int, background, gt, lambda_l1,
                     lambda_dist, lambda_dssim, adam: AdamState, stats=None, loss_dev=None, write_grads=False,
                     stream=None):
    gs = g.struct()
    adam.step += 1
    st = adam.struct()
    sp = [None, None, None] if stats is None else [_ptr(s) for s in stats]
    _check(load().msplat_train_step_fused(C.byref(gs), C.byref(cam), degrees_to_use, _bg(background), _ptr(gt),
                                          lambda_l1, lambda_dist, lambda_dssim, C.byref(st), sp[0], sp[1], sp[2],
                                          _ptr(loss_dev), 1 if write_grads else 0, _stream(stream)))


def shard_forward_backward(g, cam, degrees_to_use, background, gt, lambda_l1, lambda_dist, lambda_dssim, raster_grads,
                           loss_parts, world=0, rank=0, rows=(0, 0), stream=None, features_ready=None,
                           split_color=False):
    """Part 1 of the sharded step. With world > 0 the library picks a
    work-balanced band for `rank`; returns the (begin, end) tile rows used.
    With split_color the SH colour is projected after binning, once the
    stream has waited for features_ready (a torch.cuda.Event, may be None)."""
    gs = g.struct()
    tr = (C.c_int32 * 2)(int(rows[0]), int(rows[1]))
    ev = None if features_ready is None else C.c_void_p(features_ready.cuda_event)
    _check(load().msplat_shard_forward_backward_after(C.byref(gs), C.byref(cam), degrees_to_use, _bg(background),
                                                      _ptr(gt), lambda_l1, lambda_dist, lambda_dssim, world, rank,
                                                      tr, _ptr(raster_grads), _ptr(loss_parts), ev,
                                                      1 if split_color else 0, _stream(stream)))
    return tr[0], tr[1]


def shard_forward_backward_rgb(g, cam, degrees_to_use, background, gt, lambda_l1, lambda_dist, lambda_dssim,
                               raster_grads, loss_parts, rgb, world=0, rank=0, rows=(0, 0), stream=None,
                               rgb_ready=None):
    """shard_forward_backward with the colours copied from rgb ([N, 3], the
    clamped colours for this camera that the owners computed with
    shard_colors and the ranks all-gathered), after rgb_ready (a
    torch.cuda.Event, may be None)."""
    gs = g.struct()
    tr = (C.c_int32 * 2)(int(rows[0]), int(rows[1]))
    ev = None if rgb_ready is None else C.c_void_p(rgb_ready.cuda_event)
    _check(load().msplat_shard_forward_backward_rgb(C.byref(gs), C.byref(cam), degrees_to_use, _bg(background),
                                                    _ptr(gt), lambda_l1, lambda_dist, lambda_dssim, world, rank,
                                                    tr, _ptr(raster_grads), _ptr(loss_parts), _ptr(rgb), ev,
                                                    _stream(stream)))
    return tr[0], tr[1]


def shard_colors(g, cam, degrees_to_use, g0, g1, rgb, stream=None):
    """Clamped SH colours of Gaussians [g0, g1) for camera cam into rows g0..g1
    of rgb (an [>= g1, 3] float tensor): msplat_shard_colors."""
    gs = g.struct()
    _check(load().msplat_shard_colors(C.byref(gs), C.byref(cam), degrees_to_use, g0, g1, _ptr(rgb), _stream(stream)))


def shard_project_backward_adam(g, cam, degrees_to_use, raster_grads, g0, g1, adam: AdamState, stats=None,
                                stream=None, count_step=True):
    """raster_grads: a [N, 16] tensor, or an int device address such that row i
    of the gradient record is at address + 64 * i for i in [g0, g1)."""
    if count_step:
        adam.step += 1
    gs = g.struct()
    st = adam.struct()
    sp = [None, None, None] if stats is None else [_ptr(s) for s in stats]
    _check(load().msplat_shard_project_backward_adam(C.byref(gs), C.byref(cam), degrees_to_use, _ptr(raster_grads),
                                                     g0, g1, C.byref(st), sp[0], sp[1], sp[2], _stream(stream)))


# ---- routed multi-GPU exchange (msplat_route_*) --------------------------------

ROUTE_PAYLOAD_FLOATS = 32  # 128 bytes per routed Gaussian


def route_summary_len(cam) -> int:
    """Length (int32 entries) of a slice's route summary for this camera."""
    n = C.c_int64()
    _check(load().msplat_route_summary_len(C.byref(cam), C.byref(n)))
    return int(n.value)


def route_project(g, cam, degrees_to_use, g0, g1, summary, stream=None):
    """Projects Gaussians [g0, g1) of g; summary (int32 [route_summary_len])
    receives the slice's per-tile intersection counts and the histograms of
    its tile rectangles' first and last rows."""
    gs = g.struct()
    _check(load().msplat_route_project(C.byref(gs), C.byref(cam), degrees_to_use, g0, g1, _ptr(summary),
                                       _stream(stream)))


def route_plan(summaries, cam, world, rank, stream=None):
    """(bands [world + 1], items sent to each rank [world], items received
    from each rank [world]) as host lists, from all ranks' summaries
    (int32 [world, route_summary_len])."""
    bands = (C.c_int32 * (world + 1))()
    send = (C.c_int64 * world)()
    recv = (C.c_int64 * world)()
    _check(load().msplat_route_plan(_ptr(summaries), C.byref(cam), world, rank, bands, send, recv, _stream(stream)))
    return list(bands), list(send), list(recv)


def route_pack(send_payload, stream=None):
    _check(load().msplat_route_pack(_ptr(send_payload) if send_payload.numel() else None, _stream(stream)))


def route_pack_peers(peers: MsplatRoutePeers, stream=None):
    """Packs into every destination's inbox (peer stores)."""
    _check(load().msplat_route_pack_peers(C.byref(peers), _stream(stream)))


def route_push_peers(peers: MsplatRoutePeers, raster_grads, stream=None):
    """The band's records back into their owners' return boxes (peer stores)."""
    _check(load().msplat_route_push_peers(C.byref(peers), _ptr(raster_grads) if raster_grads.numel() else None,
                                          _stream(stream)))


def route_band(cam, sh_degree, recv_payload, num_recv, band, background, gt, lambda_l1, lambda_dist, lambda_dssim,
               raster_grads, loss_parts, stream=None):
    _check(load().msplat_route_band(C.byref(cam), sh_degree, _ptr(recv_payload) if num_recv else None, num_recv,
                                    int(band[0]), int(band[1]), _bg(background), _ptr(gt), lambda_l1, lambda_dist,
                                    lambda_dssim, _ptr(raster_grads) if num_recv else None, _ptr(loss_parts),
                                    _stream(stream)))


def route_return(recv_grads, num_items, slice_grads, stream=None):
    _check(load().msplat_route_return(_ptr(recv_grads) if num_items else None, num_items, _ptr(slice_grads),
                                      _stream(stream)))


def route_project_backward_adam(g, cam, degrees_to_use, slice_grads, adam: "AdamState", stats=None, stream=None):
    gs = g.struct()
    st = adam.struct()
    sp = [None, None, None] if stats is None else [_ptr(s) for s in stats]
    _check(load().msplat_route_project_backward_adam(C.byref(gs), C.byref(cam), degrees_to_use, _ptr(slice_grads),
                                                     C.byref(st), sp[0], sp[1], sp[2], _stream(stream)))


_DT = {0: "float32", 1: "int32", 2: "int64"}


def last_tensor(name: str):
    """A torch view of a workspace tensor of the last call (aliases device memory)."""
    import torch
    ref = MsplatTensorRef()
    _check(load().msplat_last_tensor(name.encode(), C.byref(ref)))
    shape = tuple(ref.shape[k] for k in range(ref.ndim))
    dtype = {0: torch.float32, 1: torch.int32, 2: torch.int64, 3: torch.float64}[ref.dtype]
    numel = int(np.prod(shape)) if shape else 1
    if numel == 0:
        return torch.empty(shape, dtype=dtype, device="cuda")
    # Wrap the raw pointer without copying via the CUDA array interface.
    itemsize = torch.empty((), dtype=dtype).element_size()

    class _Holder:
        __cuda_array_interface__ = {"shape": shape, "typestr": {torch.float32: "<f4", torch.int32: "<i4",
                                                                 torch.int64: "<i8", torch.float64: "<f8"}[dtype],
                                    "data": (ref.data, False), "version": 2,
                                    "strides": None}

    t = torch.as_tensor(_Holder(), device="cuda")
    assert t.element_size() == itemsize
    return t


def last_num_intersections() -> int:
    return load().msplat_last_num_intersections()


def last_status_flags() -> int:
    return load().msplat_last_status_flags()


def launch_count() -> int:
    return load().msplat_launch_count()


def set_stage_timing(enable: bool):
    _check(load().msplat_set_stage_timing(1 if enable else 0))


def set_raster_counters(enable: bool):
    """Rasteriser work counters (last_tensor("raster_counters")); off by default."""
    _check(load().msplat_set_raster_counters(1 if enable else 0))


def stage_times() -> dict:
    """{stage name: (total ms, samples)} accumulated since set_stage_timing(True)."""
    L = load()
    ms = (C.c_double * 16)()
    cnt = (C.c_int64 * 16)()
    k = L.msplat_stage_times(ms, cnt, 16)
    if k < 0:
        raise MsplatError(2, L.msplat_last_error().decode())
    return {L.msplat_stage_name(i).decode(): (ms[i], cnt[i]) for i in range(k)}


def densify(g: "DeviceGaussians", adam: "AdamState", stats, args: dict, seed: int, stream=None):
    """Densification through msplat_densify_plan / msplat_densify_apply.
    stats = (xys_grad_norm, vis_counts, max_2d_size) device tensors; args holds
    the MsplatDensifyArgs thresholds; split samples are std::mt19937(seed)
    normals (as the reference draws them). Returns (new DeviceGaussians, new
    AdamState, plan dict)."""
    import torch
    a = MsplatDensifyArgs(**args)
    a.xys_grad_norm, a.vis_counts, a.max_2d_size = (_ptr(s) for s in stats)
    gs = g.struct()
    plan = MsplatDensifyPlan()
    L = load()
    _check(L.msplat_densify_plan(C.byref(gs), C.byref(a), C.byref(plan), _stream(stream)))
    n_new = plan.new_count
    dev = g.means.device
    samples = torch.from_numpy(normal_samples(seed, 6 * plan.num_splits)).to(dev) if plan.num_splits else None
    outs = [torch.zeros((n_new,) + tuple(t.shape[1:]), dtype=torch.float32, device=dev) for t in g.groups()]
    new_g = DeviceGaussians.__new__(DeviceGaussians)
    new_g.means, new_g.scales, new_g.quats, new_g.f_dc, new_g.f_rest, new_g.opacities = outs
    new_g.sh_degree = g.sh_degree
    new_adam = AdamState(new_g)
    new_adam.lr, new_adam.step = list(adam.lr), adam.step
    new_adam.beta1, new_adam.beta2, new_adam.eps = adam.beta1, adam.beta2, adam.eps
    ogs = new_g.struct()
    _check(L.msplat_densify_apply(C.byref(gs), C.byref(adam.struct()), C.byref(a), _ptr(samples), C.byref(ogs),
                                  C.byref(new_adam.struct()), _stream(stream)))
    return new_g, new_adam, {"num_splits": plan.num_splits, "num_dups": plan.num_dups, "new_count": n_new}


def normal_samples(seed: int, count: int):
    """std::mt19937(seed) / std::normal_distribution<float>(0, 1) draws from
    the library's host code (the draws the trainer makes for its splits)."""
    out = np.zeros(max(count, 1), np.float32)
    load().msplat_normal_samples(seed, count, out.ctypes.data)
    return out[:count]


def reset_opacity(opacities, exp_avg, exp_avg_sq, max_logit: float, stream=None):
    _check(load().msplat_reset_opacity(_ptr(opacities), _ptr(exp_avg), _ptr(exp_avg_sq), opacities.numel(),
                                       max_logit, _stream(stream)))


def shard_forward_backward_peers(g, peers: MsplatPeerParams, cam, degrees_to_use, background, gt, lambda_l1,
                                 lambda_dist, lambda_dssim, raster_grads, loss_parts, world=0, rank=0, rows=(0, 0),
                                 stream=None):
    """shard_forward_backward with the parameters read from their owner ranks
    through the peer view (msplat_shard_forward_backward_peers)."""
    gs = g.struct()
    tr = (C.c_int32 * 2)(int(rows[0]), int(rows[1]))
    _check(load().msplat_shard_forward_backward_peers(C.byref(gs), C.byref(peers), C.byref(cam), degrees_to_use,
                                                      _bg(background), _ptr(gt), lambda_l1, lambda_dist,
                                                      lambda_dssim, world, rank, tr, _ptr(raster_grads),
                                                      _ptr(loss_parts), _stream(stream)))
    return tr[0], tr[1]


def device_alloc(nbytes: int) -> int:
    p = C.c_void_p()
    _check(load().msplat_device_alloc(nbytes, C.byref(p)))
    return p.value


def device_free(ptr: int):
    _check(load().msplat_device_free(ptr))


def ipc_handle(ptr: int) -> bytes:
    h = (C.c_char * 64)()
    _check(load().msplat_ipc_handle(ptr, h))
    return bytes(h.raw)


def ipc_open(handle: bytes) -> int:
    h = (C.c_char * 64).from_buffer_copy(handle)
    p = C.c_void_p()
    _check(load().msplat_ipc_open(h, C.byref(p)))
    return p.value


def ipc_close(ptr: int):
    _check(load().msplat_ipc_close(ptr))


class DeviceArray:
    """A raw float32 device allocation seen by torch (zero copy) through the
    CUDA array interface; the owner frees the memory."""

    def __init__(self, ptr: int, shape):
        self.__cuda_array_interface__ = {"shape": tuple(int(x) for x in shape), "typestr": "<f4",
                                         "data": (int(ptr), False), "version": 3, "strides": None}

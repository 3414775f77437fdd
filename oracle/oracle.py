"""ctypes bindings of the CPU oracle — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
arm import this module, as the checker or the timed CPU baseline. It restates
the reference's Metal kernels (core/metal/msplat_metal.metal) on the host; see
oracle.h for the per-function citations and the parity-pin statement.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")


class OrcCamera(C.Structure):
    _fields_ = [("viewmat", C.c_float * 16), ("projmat", C.c_float * 16), ("fx", C.c_float),
                ("fy", C.c_float), ("cx", C.c_float), ("cy", C.c_float), ("width", C.c_int),
                ("height", C.c_int), ("cam_pos", C.c_float * 3)]

    def as_dict(self):
        return {"viewmat": np.array(self.viewmat[:], np.float32), "projmat": np.array(self.projmat[:], np.float32),
                "fx": self.fx, "fy": self.fy, "cx": self.cx, "cy": self.cy, "width": self.width,
                "height": self.height, "cam_pos": np.array(self.cam_pos[:], np.float32)}


class OrcStepArgs(C.Structure):
    _fields_ = [("n", C.c_int), ("degree", C.c_int), ("degrees_to_use", C.c_int),
                ("means", C.c_void_p), ("scales", C.c_void_p), ("quats", C.c_void_p),
                ("f_dc", C.c_void_p), ("f_rest", C.c_void_p), ("opacities", C.c_void_p),
                ("exp_avg", C.c_void_p * 6), ("exp_avg_sq", C.c_void_p * 6),
                ("xys_grad_norm", C.c_void_p), ("vis_counts", C.c_void_p), ("max_2d_size", C.c_void_p),
                ("background", C.c_void_p), ("gt", C.c_void_p), ("lr", C.c_float * 6),
                ("adam_step", C.c_int), ("lambda_l1", C.c_float), ("lambda_dist", C.c_float),
                ("lambda_dssim", C.c_float)]


class OrcDensifyArgs(C.Structure):
    _fields_ = [("grad_thresh", C.c_float), ("size_thresh", C.c_float), ("screen_thresh", C.c_float),
                ("check_screen", C.c_int), ("cull_alpha_thresh", C.c_float), ("cull_scale_thresh", C.c_float),
                ("cull_screen_size", C.c_float), ("check_huge", C.c_int), ("half_max_dim", C.c_float),
                ("log_size_fac", C.c_float)]


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        L.orc_exp.restype = C.c_float
        L.orc_exp.argtypes = [C.c_float]
        L.orc_set_threads.restype = C.c_int
        L.orc_set_threads.argtypes = [C.c_int]
        L.orc_prepare_cam.argtypes = [f32p, C.c_float, C.c_float, C.c_float, C.c_float, C.c_int, C.c_int,
                                      C.POINTER(OrcCamera)]
        L.orc_project_forward.argtypes = [C.c_int, f32p, f32p, C.c_float, f32p, f32p, f32p, f32p, C.c_int,
                                          C.c_int, C.POINTER(OrcCamera), C.c_float, f32p, f32p, i32p, f32p,
                                          i32p, f32p, f32p, f32p]
        L.orc_bin_and_sort.restype = C.c_int64
        L.orc_bin_and_sort.argtypes = [C.c_int, f32p, f32p, i32p, f32p, C.c_int, C.c_int, i64p, i32p, i32p,
                                       C.c_int64]
        L.orc_tile_counts.argtypes = [C.c_int, f32p, i32p, f32p, C.c_int, C.c_int, i64p]
        L.orc_tile_kept_ids.argtypes = [C.c_int, f32p, f32p, i32p, f32p, C.c_int, C.c_int, C.c_int, i32p, i32p,
                                        i32p]
        L.orc_pack.argtypes = [C.c_int64, i32p, f32p, f32p, f32p, f32p, f32p, f32p, f32p, f32p]
        L.orc_rasterize_forward.argtypes = [C.c_int, C.c_int, C.c_int, i32p, f32p, f32p, f32p, f32p, f32p,
                                            f32p, i32p, f32p, f32p, f32p, f32p, f32p, f32p]
        L.orc_loss_ssim.argtypes = [C.c_int, C.c_int, f32p, f32p, f32p, C.c_float, C.c_float, C.c_float, f32p,
                                    f32p, C.POINTER(C.c_double), C.POINTER(C.c_double)]
        L.orc_rasterize_backward.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, i32p, i32p, f32p, f32p, f32p,
                                             f32p, f32p, i32p, f32p, f32p] + [C.c_void_p] * 5 + [f32p] * 5
        L.orc_project_backward.argtypes = [C.c_int, f32p, f32p, C.c_float, f32p, C.POINTER(OrcCamera), i32p,
                                           f32p, f32p, f32p, C.c_int, C.c_int, f32p, f32p, f32p, f32p, f32p,
                                           f32p, f32p, f32p, f32p, f32p, C.c_float]
        L.orc_fused_adam.argtypes = [f32p, f32p, f32p, f32p, C.c_int64, C.c_float, C.c_float, C.c_float,
                                     C.c_float, C.c_float]
        L.orc_train_step.restype = C.c_float
        L.orc_train_step.argtypes = [C.POINTER(OrcStepArgs), C.POINTER(OrcCamera), C.c_void_p, C.c_void_p,
                                     C.POINTER(C.c_int64)]
        L.orc_render.argtypes = [C.c_int, f32p, f32p, f32p, f32p, f32p, f32p, C.c_int, C.c_int, f32p,
                                 C.POINTER(OrcCamera), f32p]
        L.orc_render_rows.argtypes = [C.c_int, f32p, f32p, f32p, f32p, f32p, f32p, C.c_int, C.c_int, f32p,
                                      C.POINTER(OrcCamera), C.c_int, f32p]
        L.orc_time_step_sample.restype = C.c_double
        L.orc_time_step_sample.argtypes = [C.POINTER(OrcStepArgs), C.POINTER(OrcCamera), C.c_int,
                                           C.POINTER(C.c_double)]
        L.orc_densify.restype = C.c_int
        L.orc_densify.argtypes = [C.c_int, C.c_int, C.c_int, C.POINTER(OrcDensifyArgs), f32p, f32p, f32p,
                                  C.c_void_p * 6, C.c_void_p * 6, C.c_void_p * 6, f32p, C.POINTER(C.c_int),
                                  C.POINTER(C.c_int)]
        L.orc_normal_samples.argtypes = [C.c_uint32, C.c_int64, f32p]
        _lib = L
    return _lib


def _c(a, dt=np.float32):
    return np.ascontiguousarray(a, dtype=dt)


def set_threads(n: int) -> int:
    return lib().orc_set_threads(n)


def det_exp(x: float) -> float:
    return lib().orc_exp(x)


def prepare_cam(cam_to_world, fx, fy, cx, cy, width, height) -> OrcCamera:
    cam = OrcCamera()
    lib().orc_prepare_cam(_c(np.asarray(cam_to_world).reshape(16)), fx, fy, cx, cy, width, height, C.byref(cam))
    return cam


def tiles(cam: OrcCamera):
    return (cam.width + 15) // 16, (cam.height + 15) // 16


def project_forward(means, scales, quats, opac, f_dc, f_rest, degree, degrees_to_use, cam, glob_scale=1.0,
                    clip=0.01):
    n = means.shape[0]
    out = dict(xys=np.zeros((n, 2), np.float32), depths=np.zeros(n, np.float32), radii=np.zeros(n, np.int32),
               transmats=np.zeros((n, 9), np.float32), num_tiles_hit=np.zeros(n, np.int32),
               normal_opacity=np.zeros((n, 4), np.float32), colors=np.zeros((n, 3), np.float32),
               aabb=np.zeros((n, 2), np.float32))
    lib().orc_project_forward(n, _c(means), _c(scales), glob_scale, _c(quats), _c(opac).reshape(-1), _c(f_dc),
                              _c(f_rest).reshape(-1) if f_rest.size else np.zeros(1, np.float32), degree,
                              degrees_to_use, C.byref(cam), clip, out["xys"], out["depths"], out["radii"],
                              out["transmats"], out["num_tiles_hit"], out["normal_opacity"], out["colors"],
                              out["aabb"])
    return out


def bin_and_sort(proj, cam):
    tx, ty = tiles(cam)
    T = tx * ty
    n = proj["xys"].shape[0]
    cap = int(min(int(proj["num_tiles_hit"].astype(np.int64).sum()), T * 2048))
    raw = np.zeros(T, np.int64)
    tile_bins = np.zeros((T, 2), np.int32)
    ids = np.zeros(max(cap, 1), np.int32)
    kept = lib().orc_bin_and_sort(n, proj["xys"], proj["depths"], proj["radii"], proj["aabb"], tx, ty, raw,
                                  tile_bins, ids, cap)
    assert kept >= 0
    return dict(raw_counts=raw, tile_bins=tile_bins, gaussian_ids=ids[:kept].copy(), kept=kept)


def tile_counts(proj, cam):
    """Raw per-tile intersection counts (no key lists)."""
    tx, ty = tiles(cam)
    raw = np.zeros(tx * ty, np.int64)
    lib().orc_tile_counts(proj["xys"].shape[0], proj["xys"], proj["radii"], proj["aabb"], tx, ty, raw)
    return raw


def tile_kept_ids(proj, cam, tile_list):
    """{tile: sorted kept ids} for the listed tiles (orc_bin_and_sort's policy)."""
    tx, ty = tiles(cam)
    tl = np.ascontiguousarray(np.asarray(tile_list, np.int32))
    ids = np.zeros((len(tl), 2048), np.int32)
    cnt = np.zeros(len(tl), np.int32)
    lib().orc_tile_kept_ids(proj["xys"].shape[0], proj["xys"], proj["depths"], proj["radii"], proj["aabb"], tx, ty,
                            len(tl), tl, ids, cnt)
    return {int(t): ids[k, :cnt[k]].copy() for k, t in enumerate(tl)}


def pack(bins, proj):
    k = max(bins["kept"], 1)
    out = dict(packed_xy=np.zeros((k, 2), np.float32), packed_transmat=np.zeros((k, 9), np.float32),
               packed_normal_opac=np.zeros((k, 4), np.float32), packed_rgb=np.zeros((k, 3), np.float32))
    ids = bins["gaussian_ids"] if bins["kept"] else np.zeros(1, np.int32)
    lib().orc_pack(bins["kept"], _c(ids, np.int32), proj["xys"], proj["transmats"], proj["normal_opacity"],
                   proj["colors"], out["packed_xy"], out["packed_transmat"], out["packed_normal_opac"],
                   out["packed_rgb"])
    return out


def rasterize_forward(bins, packed, cam, background):
    W, H = cam.width, cam.height
    tx, _ = tiles(cam)
    out = dict(final_Ts=np.zeros((H, W, 3), np.float32), final_idx=np.zeros((H, W, 2), np.int32),
               out_img=np.zeros((H, W, 3), np.float32), out_depth=np.zeros((H, W), np.float32),
               out_normal=np.zeros((H, W, 3), np.float32), out_alpha=np.zeros((H, W), np.float32),
               out_median_depth=np.zeros((H, W), np.float32), out_distortion=np.zeros((H, W), np.float32))
    lib().orc_rasterize_forward(W, H, tx, bins["tile_bins"], packed["packed_xy"], packed["packed_normal_opac"],
                                packed["packed_transmat"], packed["packed_rgb"], _c(background),
                                out["final_Ts"], out["final_idx"], out["out_img"], out["out_depth"],
                                out["out_normal"], out["out_alpha"], out["out_median_depth"],
                                out["out_distortion"])
    return out


def loss_ssim(out_img, gt, out_distortion, lambda_l1, lambda_dist, lambda_dssim):
    H, W, _ = out_img.shape
    dimg = np.zeros((H, W, 3), np.float32)
    ddist = np.zeros((H, W), np.float32)
    loss, ssum = C.c_double(), C.c_double()
    lib().orc_loss_ssim(W, H, _c(out_img), _c(gt), _c(out_distortion), lambda_l1, lambda_dist, lambda_dssim, dimg,
                        ddist, C.byref(loss), C.byref(ssum))
    return dict(dL_dout_img=dimg, dL_dout_distortion=ddist, loss=loss.value, ssim_sum=ssum.value)


def _ptr(a):
    return None if a is None else _c(a).ctypes.data


def rasterize_backward(n, bins, packed, fwd, cam, background, dL_dout_img, dL_dout_depth=None,
                       dL_dout_alpha=None, dL_dout_normal=None, dL_dout_median_depth=None,
                       dL_dout_distortion=None):
    W, H = cam.width, cam.height
    tx, _ = tiles(cam)
    out = dict(dL_dtransMat=np.zeros((n, 9), np.float32), dL_dmean2D=np.zeros((n, 2), np.float32),
               dL_dnormal3D=np.zeros((n, 3), np.float32), dL_dopacity=np.zeros((n, 1), np.float32),
               dL_dcolors=np.zeros((n, 3), np.float32))
    keep = [None if a is None else _c(a) for a in (dL_dout_depth, dL_dout_alpha, dL_dout_normal,
                                                    dL_dout_median_depth, dL_dout_distortion)]
    ids = bins["gaussian_ids"] if bins["kept"] else np.zeros(1, np.int32)
    lib().orc_rasterize_backward(n, W, H, tx, bins["tile_bins"], _c(ids, np.int32), packed["packed_xy"],
                                 packed["packed_normal_opac"], packed["packed_transmat"], packed["packed_rgb"],
                                 fwd["final_Ts"], fwd["final_idx"], _c(background), _c(dL_dout_img),
                                 *[None if a is None else a.ctypes.data for a in keep],
                                 out["dL_dtransMat"], out["dL_dmean2D"], out["dL_dnormal3D"], out["dL_dopacity"],
                                 out["dL_dcolors"])
    return out


def project_backward(means, scales, quats, cam, radii, dL_dtransMat, dL_dnormal3D, dL_dcolors, degree,
                     degrees_to_use, f_rest, stats=None, glob_scale=1.0):
    n = means.shape[0]
    K = (degree + 1) ** 2 - 1
    out = dict(dL_dmean3D=np.zeros((n, 3), np.float32), dL_dscale=np.zeros((n, 2), np.float32),
               dL_dquat=np.zeros((n, 4), np.float32), dL_dmean2D=np.zeros((n, 2), np.float32),
               dL_dfeatures_dc=np.zeros((n, 3), np.float32), dL_dfeatures_rest=np.zeros((n, K, 3), np.float32))
    if stats is None:
        stats = [np.zeros(n, np.float32) for _ in range(3)]
    W, H = cam.width, cam.height
    rest = _c(f_rest).reshape(-1) if K else np.zeros(1, np.float32)
    drest = out["dL_dfeatures_rest"].reshape(-1) if K else np.zeros(1, np.float32)
    lib().orc_project_backward(n, _c(means), _c(scales), glob_scale, _c(quats), C.byref(cam), _c(radii, np.int32),
                               _c(dL_dtransMat), _c(dL_dnormal3D), _c(dL_dcolors), degree, degrees_to_use, rest,
                               out["dL_dmean3D"], out["dL_dscale"], out["dL_dquat"], out["dL_dmean2D"],
                               out["dL_dfeatures_dc"], drest, stats[0], stats[1], stats[2],
                               1.0 / max(W, H))
    out["stats"] = stats
    return out


def fused_adam(params, grads, m, v, step_size, beta1, beta2, bc2_sqrt, eps):
    """In-place Adam on float32 arrays (fused_adam_kernel, metal:1383-1406)."""
    lib().orc_fused_adam(params.reshape(-1), _c(grads).reshape(-1), m.reshape(-1), v.reshape(-1), params.size,
                         step_size, beta1, beta2, bc2_sqrt, eps)


def render(scene_params, degree, degrees_to_use, background, cam):
    means, scales, quats, opac, f_dc, f_rest = scene_params
    n = means.shape[0]
    out = np.zeros((cam.height, cam.width, 3), np.float32)
    lib().orc_render(n, _c(means), _c(scales), _c(quats), _c(opac).reshape(-1), _c(f_dc),
                     _c(f_rest).reshape(-1) if f_rest.size else np.zeros(1, np.float32), degree, degrees_to_use,
                     _c(background), C.byref(cam), out)
    return out


def render_rows(scene_params, degree, degrees_to_use, background, cam, pixel_rows):
    """render() of pixel rows [0, pixel_rows) only (other rows zero)."""
    means, scales, quats, opac, f_dc, f_rest = scene_params
    n = means.shape[0]
    out = np.zeros((cam.height, cam.width, 3), np.float32)
    lib().orc_render_rows(n, _c(means), _c(scales), _c(quats), _c(opac).reshape(-1), _c(f_dc),
                          _c(f_rest).reshape(-1) if f_rest.size else np.zeros(1, np.float32), degree, degrees_to_use,
                          _c(background), C.byref(cam), int(pixel_rows), out)
    return out


LR_INIT = (0.00016, 0.005, 0.001, 0.0025, 0.000125, 0.05)  # model.cpp:142


class OracleTrainer:
    """Holds parameters + Adam state and runs orc_train_step (model.cpp:762-829)."""

    def __init__(self, params, degree):
        self.means, self.scales, self.quats, self.opac, self.f_dc, self.f_rest = [
            np.array(p, dtype=np.float32, copy=True) for p in params]
        self.opac = self.opac.reshape(-1, 1)
        self.degree = degree
        self.n = self.means.shape[0]
        groups = [self.means, self.scales, self.quats, self.f_dc, self.f_rest, self.opac]
        self.m = [np.zeros(g.shape, np.float32) for g in groups]
        self.v = [np.zeros(g.shape, np.float32) for g in groups]
        self.stats = [np.zeros(self.n, np.float32) for _ in range(3)]
        self.adam_step = 0
        self.lr = list(LR_INIT)

    def params(self):
        return (self.means, self.scales, self.quats, self.opac, self.f_dc, self.f_rest)

    def _args(self, cam, gt, background, degrees_to_use, ssim_weight, lambda_dist, lr):
        a = OrcStepArgs()
        a.n, a.degree = self.n, self.degree
        a.degrees_to_use = self.degree if degrees_to_use is None else degrees_to_use
        bufs = [self.means, self.scales, self.quats, self.f_dc, self.f_rest, self.opac]
        dummy = np.zeros(1, np.float32)
        a.means, a.scales, a.quats = self.means.ctypes.data, self.scales.ctypes.data, self.quats.ctypes.data
        a.f_dc = self.f_dc.ctypes.data
        a.f_rest = self.f_rest.ctypes.data if self.f_rest.size else dummy.ctypes.data
        a.opacities = self.opac.ctypes.data
        for g in range(6):
            a.exp_avg[g] = self.m[g].ctypes.data if self.m[g].size else dummy.ctypes.data
            a.exp_avg_sq[g] = self.v[g].ctypes.data if self.v[g].size else dummy.ctypes.data
        a.xys_grad_norm, a.vis_counts, a.max_2d_size = [s.ctypes.data for s in self.stats]
        bg = _c(background)
        gt_c = _c(gt)
        a.background, a.gt = bg.ctypes.data, gt_c.ctypes.data
        for g in range(6):
            a.lr[g] = (lr or self.lr)[g]
        a.adam_step = self.adam_step
        a.lambda_l1, a.lambda_dist, a.lambda_dssim = 1.0 - ssim_weight, lambda_dist, ssim_weight
        return a, (bufs, dummy, bg, gt_c)

    def time_sample(self, cam, gt, background, row_stride, degrees_to_use=None):
        """orc_time_step_sample: (estimated seconds per full step, per-stage seconds)."""
        self.adam_step += 1
        a, keep = self._args(cam, gt, background, degrees_to_use, 0.2, 0.0, None)
        st = (C.c_double * 7)()
        est = lib().orc_time_step_sample(C.byref(a), C.byref(cam), row_stride, st)
        del keep
        return est, list(st)

    def step(self, cam, gt, background, degrees_to_use=None, ssim_weight=0.2, lambda_dist=0.0,
             want_grads=False, lr=None):
        self.adam_step += 1
        a, keep = self._args(cam, gt, background, degrees_to_use, ssim_weight, lambda_dist, lr)
        K = (self.degree + 1) ** 2 - 1
        grads = np.zeros(13 * self.n + 3 * K * self.n, np.float32) if want_grads else None
        img = np.zeros((cam.height, cam.width, 3), np.float32)
        kept = C.c_int64()
        loss = lib().orc_train_step(C.byref(a), C.byref(cam), None if grads is None else grads.ctypes.data,
                                    img.ctypes.data, C.byref(kept))
        del keep
        return dict(loss=loss, grads=grads, out_img=img, kept=kept.value)


def normal_samples(seed: int, count: int):
    """std::mt19937(seed) / std::normal_distribution<float>(0, 1) draws (model.cpp:254-259)."""
    out = np.zeros(max(count, 1), np.float32)
    lib().orc_normal_samples(seed, count, out)
    return out[:count]


def densify(groups, m, v, degree, stats, args: dict, random_samples):
    """Staged reference densification (orc_densify). groups/m/v: six arrays each
    in Model order (means, scales, quats, f_dc, f_rest, opacities) with N rows;
    stats: (xys_grad_norm, vis_counts, max_2d_size). Returns (groups, m, v,
    num_splits, num_dups) with the new row count."""
    n = groups[0].shape[0]
    cap = 3 * n
    K = (degree + 1) ** 2 - 1
    widths = [3, 2, 4, 3, 3 * K, 1]
    bufs = []
    for arrs in (groups, m, v):
        row = []
        for a, w in zip(arrs, widths):
            b = np.zeros((cap, w) if w else (cap, 0), np.float32)
            b[:n] = np.asarray(a, np.float32).reshape(n, w)
            row.append(b)
        bufs.append(row)
    ptrs = [(C.c_void_p * 6)(*[b.ctypes.data if b.size else None for b in row]) for row in bufs]
    rs = _c(random_samples).reshape(-1)
    need = 6 * n
    if rs.size < need:
        rs = np.concatenate([rs, np.zeros(need - rs.size, np.float32)])
    a = OrcDensifyArgs(**args)
    ns, nd = C.c_int(0), C.c_int(0)
    new_n = lib().orc_densify(n, cap, K, C.byref(a), _c(stats[0]).reshape(-1), _c(stats[1]).reshape(-1),
                              _c(stats[2]).reshape(-1), ptrs[0], ptrs[1], ptrs[2], rs, C.byref(ns), C.byref(nd))
    if new_n < 0:
        raise RuntimeError("densify capacity exceeded")
    out = [[b[:new_n].copy() for b in row] for row in bufs]
    return out[0], out[1], out[2], ns.value, nd.value

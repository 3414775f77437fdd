"""Benchmark of the 2DGS training step (BASELINE.json metric: train iters/s and
fwd+bwd Mpix/s at 3M Gaussians, 4946x3286, SH degree 3 = config 3).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl ours|reference]

One step = one full training iteration (projection, binning, sort, rasterise,
SSIM+L1 loss, backward, Adam on all six groups) for one ring camera, cycling
through the cameras. Inputs are seeded synthetic scenes with the shapes and
distributions of the configuration (no dataset is available here).

value: iters/s with parameters, Adam state and target images resident in HBM
       (inputs are larger than L2), timed with CUDA events on the launch stream,
       max over ranks.
e2e:   the same metric through the C ABI with the step's target image copied
       host->device from pinned memory and the loss read back every step.
roofline: the dominant kernel against the measured HBM copy peak;
       roofline_all: every kernel of the step against its byte model;
       compute_roofline: the rasterisers' (warp, surfel) visits, blended pairs
       and issue rate against the SM issue peak.
config4: the load-skewed stress workload (6M Gaussians, every tile over the
       2048 cap) timed after the main run, with its tile-count imbalance.

N > 1 (torchrun, one process per GPU): image tile rows are sharded across
ranks (strong scaling: the image and the Gaussian set are fixed), per-Gaussian
raster gradients are reduce-scattered with NCCL, each rank runs the
projection VJP + Adam on its slice of Gaussians, and the updated parameters
are all-gathered. Before timing, a small scene is stepped twice both sharded
and on one GPU and the results are compared (`parity`); `ranks` breaks each
rank's step into its phases.

--impl reference: the CPU oracle (a restatement of the reference's Metal
kernels; the Metal code cannot run here) timed on the host cores on a bounded
sample of every step (see oracle.h: orc_time_step_sample), the value
extrapolated to the full step and labelled so.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "msplat-ios_b200", "python"))

import numpy as np  # noqa: E402

METRIC = "train iters/sec (3M Gaussians, 4946x3286, SH3)"
SSIM_WEIGHT = 0.2
SMS = 148  # B200


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--exchange", default="route-peer", choices=["peers", "nccl", "rgb", "route", "route-peer"],
                    help="multi-GPU parameter exchange: geometry all-gathered and the owners' colours for the "
                         "next camera all-gathered instead of the colour coefficients (rgb); NCCL "
                         "all-gathers of all groups with the colour groups overlapped with binning (nccl); "
                         "geometry all-gathered and colour read from its owner over NVLink (CUDA IPC, peers); "
                         "or each owner projects its slice and sends the projected Gaussians to the bands they "
                         "touch, gradients come back to the owner, nothing is gathered (route: NCCL "
                         "all-to-alls; route-peer, default: the pack and return kernels store straight into "
                         "the other GPUs' inboxes over NVLink)")
    ap.add_argument("--render-frames", type=int, default=20,
                    help="render-only frames timed after the training steps (single GPU); 0 = skip")
    ap.add_argument("--cameras", type=int, default=0,
                    help="use only the first C ring cameras (fewer target images on the device); 0 = all")
    ap.add_argument("--config4-steps", type=int, default=5,
                    help="timed steps of the config-4 stress run after the main run; 0 = skip")
    ap.add_argument("--no-parity", action="store_true", help="skip the multi-GPU parity check")
    return ap.parse_args()


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# ---------------------------------------------------------------- clocks
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = os.path.join("/tmp", f"msplat_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9:
                rows.append(f)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for r in rows for k in range(4) if r[5 + k].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------- scene
def build_scene(cfg_id: int):
    from msplat import synthetic as S
    cfg = S.CONFIGS[cfg_id]
    scene = S.make_scene(cfg, seed=0)
    return S, cfg, scene


def cameras(B, S, cfg, scene):
    fx, fy, cx, cy = scene.intrinsics
    return [B.prepare_camera(scene.cam_to_world[k], fx, fy, cx, cy, cfg.width, cfg.height)
            for k in range(len(scene.cam_to_world))]


# ---------------------------------------------------------------- byte models
# Algorithmic HBM bytes of one launch of each kernel of the step (every tensor
# it must touch, touched once), from the work units of the launch:
# n Gaussians, vis visible Gaussians, K SH-rest bases, T tiles, P pixels,
# emitted keys and kept intersections.
def param_bytes(K: int) -> int:
    return 4 * (3 + 2 + 4 + 1 + 3 + 3 * K)


def raster_bwd_bytes(kept: int, n_vis: int, pixels: int, aux: bool = False) -> int:
    """5 B per kept intersection (sorted id + the forward's per-warp blend
    byte), 80 B per visible Gaussian (raster record, read once), per pixel
    the final T, last index and dL/dimg (20 B; with the auxiliary outputs
    also M1/M2 and the median index, 32 B), 64 B read + 64 B written per
    visible Gaussian (gradient record)."""
    return 5 * kept + 80 * n_vis + (32 if aux else 20) * pixels + 128 * n_vis


def raster_fwd_bytes(kept: int, n_vis: int, pixels: int, aux: bool = False) -> int:
    """5 B per kept intersection (sorted id read, blend byte written), 112 B
    per visible Gaussian (80 B raster record + 32 B cull record), per pixel
    the outputs: image, final T and last index (20 B) for the colour-only
    training step; with the auxiliary outputs also M1/M2, median index,
    depth, normal, alpha, median and distortion (60 B)."""
    return 5 * kept + 112 * n_vis + (60 if aux else 20) * pixels


def byte_models(n, n_vis, K, T, P, emitted, kept, P_fwd=None, P_bwd=None):
    """{stage: algorithmic bytes per launch} for the kernels of one step
    (the colour-only training step: light forward and backward). n: the
    Gaussians projected (and updated by Adam); P: the loss's pixels; P_fwd,
    P_bwd: the rasterisers' pixels (default P)."""
    P_fwd = P if P_fwd is None else P_fwd
    P_bwd = P if P_bwd is None else P_bwd
    return {
        # parameters read; raster record 80 B, cull record 32 B, tile rect 8 B,
        # depth 4 B, radius 4 B written
        "project_forward": n * (param_bytes(K) + 128),
        # 32 per-id-chunk difference arrays of (tx+1)(ty+1) counts read; per
        # tile: raw, emitted and kept counts, id bound, key start, range
        "tile_counts": 4 * 32 * T + 40 * T,
        # tile rect + depth per Gaussian read, one 8 B key per emitted key
        "emit_keys": 12 * n + 8 * emitted,
        # keys read, sorted ids written, tile ranges read
        "tile_sort": 8 * emitted + 4 * kept + 8 * T,
        "rasterize_forward": raster_fwd_bytes(kept, n_vis, P_fwd),
        # image and target read, dL/dimg written
        "loss_ssim": 36 * P,
        "rasterize_backward": raster_bwd_bytes(kept, n_vis, P_bwd),
        # parameters, both Adam moments, gradient record and radius read;
        # parameters and both moments written; three densify statistics
        # read and written
        "project_backward_adam": n * (6 * param_bytes(K) + 64 + 4 + 24),
    }


def roofline_all(per_stage_ms, models, peak):
    out = {}
    for k, b in models.items():
        ms = per_stage_ms.get(k)
        if not ms:
            continue
        gbs = b / (ms * 1e-3) / 1e9
        out[k] = {"ms": round(ms, 4), "bytes": int(b), "gb_s": round(gbs, 1), "frac": round(gbs / peak, 4)}
    return out


def compute_roofline(per_stage_ms, counters, sm_mhz):
    """The rasterisers against the SM issue peak (4 warp instructions per
    clock per SM). counters: msplat raster_counters [forward blended pairs,
    forward visits, backward visits, backward blended pairs]; each (warp,
    surfel) visit evaluates 32 pixels; the counts come from one untimed step
    right after the timed region (the timed steps run without counting).
    Instructions per visit come from the committed ncu capture
    (profiles/raster_issue.json) when present."""
    ipv = {}
    try:
        ipv = json.load(open(os.path.join(REPO, "profiles", "raster_issue.json"))).get("instructions_per_visit", {})
    except (OSError, ValueError):
        pass
    clock = (sm_mhz or 1965.0) * 1e6
    peak = SMS * 4 * clock
    out = {"bound": "issue", "unit": "warp instructions/s", "peak": round(peak, 0),
           "peak_note": f"{SMS} SMs x 4 warp instructions per clock at the median SM clock"}
    for name, vi, ui in (("rasterize_forward", 1, 0), ("rasterize_backward", 2, 3)):
        ms = per_stage_ms.get(name)
        if not ms:
            continue
        t = ms * 1e-3
        v, u = int(counters[vi]), int(counters[ui])
        d = {"ms": round(ms, 4), "visits": v, "blended_pairs": u, "visits_per_s": round(v / t, 1),
             "pair_evals_per_s": round(32 * v / t, 1), "blended_pairs_per_s": round(u / t, 1),
             "useful_lane_frac": round(u / max(32 * v, 1), 4)}
        if name in ipv:
            ach = ipv[name] * v / t
            d.update({"instructions_per_visit": ipv[name], "achieved": round(ach, 1), "frac": round(ach / peak, 4)})
        out[name] = d
    return out


# ---------------------------------------------------------------- steppers
class Stepper:
    """One training step of a scene on this rank: the single-GPU fused step
    (msplat_train_step_fused) or, with ws > 1, the tile-row sharded step
    (msplat/sharding.py) with the chosen parameter exchange. step(k) trains
    on camera k % C; marks collect per-phase CUDA-event times of the sharded
    step while `timing` is set."""

    def __init__(self, B, dist, cfg, scene, cams, gts, ws, rank, dev, exchange, stats=True):
        import torch
        self.B, self.dist, self.cfg, self.cams, self.gts = B, dist, cfg, cams, gts
        self.ws, self.rank, self.dev = ws, rank, dev
        self.C = len(cams)
        n = cfg.n
        self.g = B.DeviceGaussians(*scene.params(), sh_degree=cfg.degree, device=dev)
        self.adam = B.AdamState(self.g)
        self.stats = [torch.zeros(n, device=dev) for _ in range(3)] if stats else None
        self.loss_dev = torch.zeros(1, device=dev)
        self.stream = torch.cuda.current_stream()
        self.exchange = None
        self.peers = None
        self.pending = [None]
        self.timing = False
        self.phase_ms = {}
        self._evlist = []
        self.rgb_full = None
        self.have_rgb = False
        self.use_peers = False
        self.route = None
        if ws == 1:
            return
        from msplat import sharding
        self.sharding = sharding
        self.plan = sharding.ShardPlan(n, (cfg.height + 15) // 16, ws, rank)
        self.exchange = "NCCL all-gather (colour groups overlapped with binning)"
        if exchange in ("route", "route-peer"):
            # the owner's slice is all a rank reads; the parameter groups stay
            # [padded, ...] only so that gathered_params can collect them
            sharding.pad_gaussians(self.g, self.plan.padded)
            self.route_peers = None
            how = "NCCL all-to-all"
            if exchange == "route-peer":
                self.route_peers = sharding.RoutePeers(B, dist, self.plan, n, dev)
                how = ("stored by the pack kernel straight into the destination GPU's inbox over NVLink "
                       "(CUDA IPC); records pushed back the same way")
                if not self.route_peers.ok:
                    how = "NCCL all-to-all (peer mapping failed: " + self.route_peers.error[:120] + ")"
            self.route = sharding.gpu_route_calls(B, self.g, cams[0], cfg.degree, _bg(), gts[0], 1.0 - SSIM_WEIGHT,
                                                  0.0, SSIM_WEIGHT, self.adam, self.stats, self.plan,
                                                  peers=self.route_peers)
            self.parts = torch.zeros(3, dtype=torch.float64, device=dev)
            self.exchange = ("routed: each owner projects its slice and sends the projected Gaussians (128 B) "
                             "to the tile-row bands they touch (" + how + "); gradient records (64 B) return "
                             "to the owner for the VJP and Adam; no parameter is gathered")
            return
        if exchange == "peers":
            self.peers = sharding.PeerParams(B, dist, self.plan, self.g)
            if self.peers.ok:
                self.exchange = ("geometry all-gathered; colour read from its owner over NVLink (CUDA IPC) for "
                                 "the rank's band only")
            else:
                self.exchange += "; peer mapping failed: " + self.peers.error[:120]
            self.adam = B.AdamState(self.g)
        else:
            sharding.pad_gaussians(self.g, self.plan.padded)
        self.use_peers = self.peers is not None and self.peers.ok
        self.rg = torch.zeros(self.plan.padded, 16, device=dev)
        self.rg_shard = torch.zeros(self.plan.chunk, 16, device=dev)
        self.parts = torch.zeros(3, dtype=torch.float64, device=dev)
        self.side = torch.cuda.Stream(device=dev)
        self.rgb_full = None
        if exchange == "rgb":
            self.rgb_full = torch.zeros(self.plan.padded, 3, device=dev)
            self.exchange = ("geometry all-gathered; each owner's clamped colours for the next camera all-gathered "
                             "(12 B per Gaussian) instead of the colour coefficients")
        self.have_rgb = False

    def _marks(self):
        import torch
        if not self.timing:
            return None
        ev = [("start", torch.cuda.Event(enable_timing=True))]
        ev[0][1].record(self.stream)
        self._ev = ev

        def mark(name):
            e = torch.cuda.Event(enable_timing=True)
            e.record(self.stream)
            ev.append((name, e))
        return mark

    def _collect(self):
        if not self.timing or not getattr(self, "_ev", None):
            return
        self._evlist.append(self._ev)
        self._ev = None

    def phase_summary(self):
        """Mean ms per phase over the timed steps (call after synchronize)."""
        for ev in self._evlist:
            for (_, a), (name, b) in zip(ev[:-1], ev[1:]):
                self.phase_ms.setdefault(name, []).append(a.elapsed_time(b))
        self._evlist = []
        return {k: sum(v) / len(v) for k, v in self.phase_ms.items() if v}

    def step(self, k, gt=None, cam_next_index=None, between=None):
        """between(): enqueued mid-step by the routed exchange (after the
        payload exchange, before the band); after the step otherwise."""
        B, C = self.B, self.C
        cam = self.cams[k % C]
        gt = self.gts[k % C] if gt is None else gt
        if self.ws == 1:
            B.train_step_fused(self.g, cam, self.cfg.degree, _bg(), gt, 1.0 - SSIM_WEIGHT, 0.0, SSIM_WEIGHT,
                               self.adam, stats=self.stats, loss_dev=self.loss_dev)
            return
        sh = self.sharding
        self.adam.step += 1
        if self.route is not None:
            self.route.cam, self.route.gt = cam, gt
            sh.routed_step(self.dist, self.plan, self.route, self.parts, marks=self._marks(), between=between)
            self._collect()
            return
        cam_next = self.cams[(k + 1) % C if cam_next_index is None else cam_next_index]
        fb, pa = sh.gpu_step_fns(B, self.g, cam, self.cfg.degree, _bg(), gt, 1.0 - SSIM_WEIGHT, 0.0, SSIM_WEIGHT,
                                 self.adam, self.stats, features_ready=self.pending[0],
                                 split_color=not self.use_peers, peers=self.peers if self.use_peers else None,
                                 rgb=self.rgb_full if self.have_rgb else None)
        colors_next = None if self.rgb_full is None else sh.colors_fn(B, self.g, cam_next, self.cfg.degree,
                                                                      self.rgb_full)
        self.pending[0] = sh.sharded_step(self.dist, self.plan, fb, pa, self.rg, self.rg_shard, self.g.full,
                                          self.parts, side_stream=None if self.use_peers else self.side,
                                          skip_color=self.use_peers or self.rgb_full is not None,
                                          colors_next=colors_next, rgb_full=self.rgb_full, marks=self._marks())
        self.have_rgb = self.rgb_full is not None
        self._collect()
        if between is not None:
            between()

    def prime_rgb(self, cam):
        """Colours for `cam` from the owners' current coefficients (the state
        a colour-exchange step expects before its first step on `cam`)."""
        import torch
        if self.rgb_full is None:
            return
        torch.cuda.synchronize()
        self.sharding.colors_fn(self.B, self.g, cam, self.cfg.degree, self.rgb_full)(self.plan.g_begin,
                                                                                    self.plan.g_end)
        rows = self.plan.slice_rows()
        self.dist.all_gather_into_tensor(self.rgb_full, self.rgb_full[rows])
        self.pending[0] = None
        self.have_rgb = True

    def finish(self):
        """Makes the stream wait for the last step's side-stream gather."""
        if self.ws > 1 and self.pending[0] is not None:
            self.stream.wait_event(self.pending[0])

    def gathered_params(self):
        """The whole parameter set on this rank (the colour groups are
        current only in the owner's rows under the peer and colour
        exchanges: gather them)."""
        import torch
        if self.ws == 1:
            return [t.detach().cpu().numpy() for t in self.g.groups()]
        self.finish()
        torch.cuda.synchronize()
        n = self.cfg.n
        rows = self.plan.slice_rows()
        out = []
        for full in self.g.full:
            o = torch.empty_like(full)
            if full.numel():
                self.dist.all_gather_into_tensor(o, full[rows].contiguous())
            out.append(o[:n].cpu().numpy())
        return out

    def close(self):
        import torch
        torch.cuda.synchronize()
        if self.peers is not None:
            self.peers.close()
        if getattr(self, "route_peers", None) is not None:
            self.route = None
            self.route_peers.close()
            self.route_peers = None


_BG = None


def _bg():
    global _BG
    if _BG is None:
        from msplat import synthetic as S
        _BG = S.BACKGROUND
    return _BG


def render_targets(B, cfg, scene, cams, dev):
    """Target of each camera: the render of the jittered scene (setup, untimed)."""
    import torch
    tgt = B.DeviceGaussians(*scene.jittered().params(), sh_degree=cfg.degree, device=dev)
    gts = []
    for c in cams:
        img = torch.empty(cfg.height, cfg.width, 3, device=dev)
        B.render(tgt, c, cfg.degree, _bg(), out_img=img)
        gts.append(img)
    torch.cuda.synchronize()
    del tgt
    return gts


# ---------------------------------------------------------------- multi-GPU parity
def parity_check(B, dist, ws, rank, dev, exchange):
    """Two sharded steps of a small scene (20k Gaussians, SH3, 320x240) with
    the benchmark's exchange against two single-GPU fused steps on rank 0
    (msplat_train_step_fused on a private copy): per parameter group the
    fraction of elements within 1e-5 relative and the largest error relative
    to max(|p_old|, |p_new|, 1e-6); the loss of the second step."""
    import torch
    from msplat import synthetic as S
    from msplat import sharding
    cfg = S.small_config(20_000, 3, 320, 240, num_cameras=1)
    scene = S.make_scene(cfg, seed=0)
    cams = cameras(B, S, cfg, scene)
    gts = render_targets(B, cfg, scene, cams, dev)
    st = Stepper(B, dist, cfg, scene, cams, gts, ws, rank, dev, exchange, stats=False)
    st.prime_rgb(cams[0])
    for k in range(2):
        st.step(k, cam_next_index=0)
    got = st.gathered_params()
    loss_sh = sharding.loss_from_parts(st.parts.cpu().numpy(), SSIM_WEIGHT, cfg.width, cfg.height)
    st.close()
    res = None
    if rank == 0:
        ref = Stepper(B, None, cfg, scene, cams, gts, 1, 0, dev, exchange, stats=False)
        before = [t.detach().cpu().numpy() for t in ref.g.groups()]
        losses = []
        for k in range(2):
            ref.step(k)
            losses.append(float(ref.loss_dev.cpu()[0]))
        want = [t.detach().cpu().numpy() for t in ref.g.groups()]
        names = ["means", "scales", "quats", "features_dc", "features_rest", "opacities"]
        groups = {}
        ok = True
        for k in range(6):
            if want[k].size == 0:
                continue
            a, b, p0 = got[k].reshape(want[k].shape), want[k], before[k].reshape(want[k].shape)
            frac = float(np.isclose(a, b, rtol=1e-5, atol=1e-7).mean())
            scale = np.maximum(np.maximum(np.abs(b), np.abs(p0)), 1e-6)
            groups[names[k]] = {"frac_within_1e-5": round(frac, 6), "max_rel_err": float(np.max(np.abs(a - b) / scale))}
            ok &= frac > 0.999
        lrel = abs(loss_sh - losses[-1]) / abs(losses[-1])
        ok &= lrel <= 1e-4
        res = {"case": "20k Gaussians SH3 320x240, 2 steps, sharded vs one GPU (msplat_train_step_fused)",
               "groups": groups, "loss_sharded": loss_sh, "loss_single": losses[-1], "loss_rel_err": lrel,
               "ok": bool(ok)}
        del ref
    torch.cuda.synchronize()
    dist.barrier()
    return res


# ---------------------------------------------------------------- our arm
def timed_run(B, dist, st, steps, warmup, ws, dev, local, collect_phases):
    """W untimed steps, then exactly `steps` steps bracketed by barrier +
    synchronize; returns (ms per step max over ranks, stage ms, launches,
    clocks)."""
    import torch
    for k in range(warmup):
        st.step(k)
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    launches0 = B.launch_count()
    B.set_stage_timing(True)
    st.timing = collect_phases
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0.record(st.stream)
    for k in range(steps):
        st.step(warmup + k)
    st.finish()  # the last step's side-stream gather belongs to the timed work
    e1.record(st.stream)
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    st.timing = False
    launches = B.launch_count() - launches0
    stage = B.stage_times()
    B.set_stage_timing(False)
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / steps
    if ws > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    per_stage = {k: (v[0] / max(v[1], 1)) for k, v in stage.items()}
    # the rasteriser work counters are compiled out of the timed steps; one
    # more (untimed) step counts the visits and blended pairs for the compute
    # roofline (last_tensor("raster_counters"))
    B.set_raster_counters(True)
    st.step(warmup + steps)
    st.finish()
    torch.cuda.synchronize()
    B.set_raster_counters(False)
    return ms, per_stage, launches, clk


def rank_breakdown(st, per_stage, kept, ws, rank, dist):
    """Per-rank phases of the sharded step (ms per step): replicated work
    (projection of every Gaussian, tile counts with the one host read),
    band-local binning, colour pass (includes the wait for the gathered
    colours), rasteriser + loss, and the phases between the library calls
    timed with CUDA events: reduce-scatter (includes waiting for the slowest
    rank), projection VJP + Adam (+ next camera's colours), geometry
    all-gather, loss all-reduce."""
    ph = st.phase_summary()
    g = lambda k: round(per_stage.get(k, 0.0), 4)
    mine = {"rank": rank, "tile_rows": [st.plan.row0, st.plan.row1], "intersections": kept,
            "replicated_project_counts_ms": round(per_stage.get("project_forward", 0.0) +
                                                  per_stage.get("tile_counts", 0.0), 4),
            "bin_sort_ms": round(per_stage.get("emit_keys", 0.0) + per_stage.get("tile_sort", 0.0), 4),
            "colour_pass_ms": g("project_color"),
            "raster_loss_ms": round(per_stage.get("rasterize_forward", 0.0) + per_stage.get("loss_ssim", 0.0) +
                                    per_stage.get("rasterize_backward", 0.0), 4),
            "rasterize_forward_ms": g("rasterize_forward"), "loss_ssim_ms": g("loss_ssim"),
            "rasterize_backward_ms": g("rasterize_backward"),
            "forward_backward_call_ms": round(ph.get("forward_backward", 0.0), 4),
            "reduce_scatter_ms": round(ph.get("reduce_scatter", 0.0), 4),
            "project_adam_ms": round(ph.get("project_adam", 0.0), 4),
            "all_gather_ms": round(ph.get("all_gather", 0.0), 4),
            "all_reduce_ms": round(ph.get("all_reduce", 0.0), 4)}
    if st.route is not None:
        # routed exchange: nothing is replicated; the phases between the
        # library calls (CUDA events): project + plan, payload dispatch,
        # band forward/loss/backward, gradient return, VJP + Adam, loss
        # all-reduce; and the kernel stages of the slice projection, the
        # exchange (summary, plan, pack and the waits for the other ranks)
        # and the band's unpack
        mine = {"rank": rank, "tile_rows": [st.plan.row0, st.plan.row1], "intersections": kept,
                "slice": [st.plan.g_begin, st.plan.g_end],
                "slice_project_ms": g("project_forward"), "route_exchange_ms": g("route_exchange"),
                "route_unpack_ms": g("route_unpack"),
                "bin_sort_ms": round(per_stage.get("tile_counts", 0.0) + per_stage.get("emit_keys", 0.0) +
                                     per_stage.get("tile_sort", 0.0), 4),
                "rasterize_forward_ms": g("rasterize_forward"), "loss_ssim_ms": g("loss_ssim"),
                "rasterize_backward_ms": g("rasterize_backward"),
                "project_adam_stage_ms": g("project_backward_adam"),
                "route_phases_ms": {k: round(v, 4) for k, v in ph.items()}}
    ranks = [None] * ws
    dist.all_gather_object(ranks, mine)
    return ranks


def run_ours(args, ws, rank, local):
    import torch
    import torch.distributed as dist
    from msplat import _backend as B

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    B.load()
    S, cfg, scene = build_scene(args.config)
    if ws > 1:
        # NCCL prints its version banner on stdout at communicator creation;
        # keep rank 0's stdout to the one JSON line
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
            dist.barrier()
        finally:
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)
    parity = None
    if ws > 1 and not args.no_parity:
        parity = parity_check(B, dist, ws, rank, dev, args.exchange)
    cams = cameras(B, S, cfg, scene)
    if args.cameras > 0:
        cams = cams[:args.cameras]
    C = len(cams)
    n = cfg.n
    gts = render_targets(B, cfg, scene, cams, dev)
    st = Stepper(B, dist if ws > 1 else None, cfg, scene, cams, gts, ws, rank, dev, args.exchange)
    st.prime_rgb(cams[0])
    ms, per_stage, launches, clk = timed_run(B, dist, st, args.steps, args.warmup, ws, dev, local, ws > 1)
    value = 1000.0 / ms
    pixels = cfg.width * cfg.height
    kept = B.last_num_intersections()
    n_vis = int((B.last_tensor("radii") > 0).sum().item())
    totals = B.last_tensor("intersection_totals").cpu().numpy()
    counters = B.last_tensor("raster_counters").cpu().numpy()
    T = ((cfg.width + 15) // 16) * ((cfg.height + 15) // 16)

    # roofline of the dominant kernel over the timed region
    kernel_stages = {k: v for k, v in per_stage.items() if k != "between_shard_calls"}
    dom = max(kernel_stages, key=kernel_stages.get)
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    if ws == 1:
        models = byte_models(n, n_vis, cfg.rest_bases, T, pixels, int(totals[0]), kept)
    else:
        # per rank: its band's pixels (the forward also renders the one-row
        # halo) and, under the routed exchange, its own slice's projection
        # and Adam; n_vis is the band's visible (received) set
        W_, H_ = cfg.width, cfg.height
        r0, r1 = st.plan.row0, st.plan.row1
        px_rows = lambda a, b: max(0, min(H_, b * 16) - min(H_, a * 16)) * W_
        band_px = px_rows(r0, r1)
        fwd_px = px_rows(max(0, r0 - 1), min((H_ + 15) // 16, r1 + 1)) if r1 > r0 else 0
        n_proj = (st.plan.g_end - st.plan.g_begin) if st.route is not None else n
        models = byte_models(n_proj, n_vis, cfg.rest_bases, T, band_px, int(totals[0]), kept, P_fwd=fwd_px,
                             P_bwd=band_px)

    traffic = None
    try:
        tr = json.load(open(os.path.join(REPO, "profiles", "traffic.json")))
        # the capture is of a single-GPU launch over the whole image
        if tr.get("kernel") == dom and tr.get("config") == args.config and ws == 1 and args.cameras == 0:
            traffic = tr.get("bytes_per_launch")
    except (OSError, ValueError):
        pass
    alg = models.get(dom)
    roof = None
    if alg is not None:
        ach = alg / (per_stage[dom] * 1e-3) / 1e9
        roof = {"kernel": dom, "bound": "hbm", "achieved": round(ach, 2), "peak": hbm_peak, "peak_source": peak_src,
                "unit": "GB/s", "frac": round(ach / hbm_peak, 5), "traffic": traffic,
                "algorithmic_bytes": alg, "ms_per_launch": round(per_stage[dom], 4)}
    roof_all = roofline_all(per_stage, models, hbm_peak)
    croof = compute_roofline(per_stage, counters, clk.get("sm_mhz"))

    render = None
    if ws == 1 and args.render_frames > 0:
        render = time_render(B, st.g, cams, cfg, st.stream, args.render_frames, dev)
    e2e = None
    e2e_steps = args.e2e_steps if args.e2e_steps is not None else min(args.steps, 10)
    if e2e_steps > 0 and ws == 1:
        e2e = e2e_trainer(B, S, cfg, scene, gts, C, args, e2e_steps, render)
    elif e2e_steps > 0:
        e2e = e2e_sharded(B, dist, st, gts, cams, e2e_steps, dev)
    ranks = rank_breakdown(st, per_stage, kept, ws, rank, dist) if ws > 1 else None
    exchange = st.exchange
    st.close()
    del st, gts
    torch.cuda.synchronize()
    torch.cuda.empty_cache()

    config4 = None
    if args.config4_steps > 0 and args.config != 4:
        config4 = run_config4(B, dist, args, ws, rank, local, dev)

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(S, cfg, scene, render_targets_np(B, cfg, scene, cams[:1], dev)[0], steps=1)

    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 3), "unit": "iters/s", "n_gpus": ws, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
                "scaling": "strong" if ws > 1 else "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded; shapes/distributions of BASELINE config %d)" % args.config,
                "config": {"workload": f"config {args.config}: {cfg.n} Gaussians SH{cfg.degree}, "
                                       f"{cfg.width}x{cfg.height}, {C} ring cameras",
                           "gaussians": cfg.n, "image": [cfg.width, cfg.height], "sh_degree": cfg.degree,
                           "parallelism": f"tile-row sharding x{ws}" if ws > 1 else "single GPU",
                           "exchange": exchange if ws > 1 else None,
                           "l2": "inputs larger than L2 (params+Adam state %.1f GB)" % (n * 58 * 12 / 1e9)},
                "mpix_per_s": round(pixels * value / 1e6, 2),
                "e2e": e2e, "render": render, "gpu_launches": int(launches), "clocks": clk, "roofline": roof,
                "roofline_all": roof_all, "compute_roofline": croof,
                "stage_ms": {k: round(v, 4) for k, v in per_stage.items()},
                "intersections": kept, "emitted_keys": int(totals[0]), "visible_gaussians": n_vis,
                "cpu_baseline": cpu, "config4": config4}
        if ranks is not None:
            line["ranks"] = ranks
            line["parity"] = parity
        print(json.dumps(line), flush=True)
    if ws > 1:
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()


def render_targets_np(B, cfg, scene, cams, dev):
    return [t.cpu().numpy() for t in render_targets(B, cfg, scene, cams, dev)]


def time_render(B, g, cams, cfg, stream, frames, dev):
    """Render-only forward (msplat_render, msplat_metal.mm:545-772):
    projection, binning, sort and the forward rasteriser per frame, image
    left on the device."""
    import torch
    C = len(cams)
    frame = torch.empty(cfg.height, cfg.width, 3, device=dev)
    for k in range(3):
        B.render(g, cams[k % C], cfg.degree, _bg(), out_img=frame)
    torch.cuda.synchronize()
    r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    r0.record(stream)
    for k in range(frames):
        B.render(g, cams[k % C], cfg.degree, _bg(), out_img=frame)
    r1.record(stream)
    torch.cuda.synchronize()
    rms = r0.elapsed_time(r1) / frames
    return {"value": round(1000.0 / rms, 2), "unit": "frames/s", "ms_per_frame": round(rms, 3), "frames": frames,
            "path": "msplat_render, image kept on the device"}


def h2d_gbs(host, dev_view, reps=3):
    """Host->device bandwidth of one pinned copy of `host` into `dev_view`
    (GB/s, best of `reps`, CUDA events on a private stream): what an e2e step
    that copies its target image is bounded by."""
    import torch
    s = torch.cuda.Stream()
    best = 0.0
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s):
            e0.record(s)
            dev_view.copy_(host, non_blocking=True)
            e1.record(s)
        e1.synchronize()
        ms = e0.elapsed_time(e1)
        if ms > 0:
            best = max(best, host.numel() * host.element_size() / (ms * 1e-3) / 1e9)
    return round(best, 2)


def e2e_trainer(B, S, cfg, scene, gts, C, args, e2e_steps, render):
    """The metric through the public trainer API (msplat_trainer_step): every
    step copies its target image host->device from pinned memory and reads
    the loss back, as a user of msplat_c_api.h does."""
    import msplat
    E = min(C, 4)
    host_imgs = np.stack([gts[k].cpu().numpy() for k in range(E)])
    fx, fy, cx, cy = scene.intrinsics
    ds = msplat.Dataset.from_memory(scene.cam_to_world[:E], np.tile([fx, fy, cx, cy], (E, 1)), cfg.width,
                                    cfg.height, host_imgs)
    tcfg = msplat.TrainingConfig(iterations=10 ** 9, sh_degree=cfg.degree, sh_degree_interval=1,
                                 num_downscales=0, ssim_weight=SSIM_WEIGHT)
    trainer = msplat.GaussianTrainer(ds, tcfg, params=scene.params())
    for _ in range(max(args.warmup, cfg.degree)):  # degrees_to_use ramps to sh_degree by step 3
        trainer.step()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        trainer.step()
    e2e_s = (time.perf_counter() - t0) / e2e_steps
    import torch
    probe_host = torch.from_numpy(host_imgs[0]).pin_memory()
    probe_dev = torch.empty_like(probe_host, device="cuda")
    bw = h2d_gbs(probe_host, probe_dev)
    del probe_host, probe_dev
    e2e = {"value": round(1.0 / e2e_s, 3), "unit": "iters/s", "h2d_bytes_per_step": int(host_imgs[0].nbytes),
           "d2h_bytes_per_step": 4, "steps": e2e_steps, "h2d_gbs_measured": bw,
           "path": ("msplat_trainer_step (public C API): each step's target image H2D from pinned memory "
                    "(the trainer copies the next camera's image on a copy stream during the current step), "
                    "loss D2H, sync")}
    if render is not None:
        # viewer path: msplat_trainer_render_pose_to_buffer, RGBA8 into a host buffer
        pose = ds.camera_pose(0)
        for _ in range(2):
            trainer.render_rgba(pose, 0)
        t0 = time.perf_counter()
        nv = min(10, args.render_frames)
        for _ in range(nv):
            trainer.render_rgba(pose, 0)
        render["e2e_rgba8"] = {"value": round(nv / (time.perf_counter() - t0), 2), "unit": "frames/s",
                               "d2h_bytes_per_frame": cfg.width * cfg.height * 4,
                               "path": "msplat_trainer_render_pose_to_buffer (public C API), RGBA8 to host"}
    del trainer, ds
    return e2e


def e2e_sharded(B, dist, st, gts, cams, e2e_steps, dev):
    """Each step's target image reaches every rank as 1/N of its rows copied
    host->device per rank (pinned memory, a copy stream) and an NCCL
    all-gather of the row blocks over NVLink, both for the next step while
    the current one computes (two device buffers; under the routed exchange
    the gather is enqueued after the payload exchange, so it runs under the
    band's compute); the loss sums are read back every step."""
    import torch
    ws, rank = st.ws, st.rank
    stream = st.stream
    H, W = gts[0].shape[0], gts[0].shape[1]
    rows = -(-H // ws)
    r0, r1 = min(H, rank * rows), min(H, (rank + 1) * rows)
    host_gt = [gts[k].cpu().pin_memory() for k in range(min(len(gts), 4))]
    dev_gt = [torch.empty((rows * ws,) + tuple(gts[0].shape[1:]), dtype=gts[0].dtype, device=dev) for _ in range(2)]
    copy_stream = torch.cuda.Stream(device=dev)
    copied = [torch.cuda.Event(), torch.cuda.Event()]
    ready = [torch.cuda.Event(), torch.cuda.Event()]
    free = [torch.cuda.Event(), torch.cuda.Event()]
    parts_host = torch.zeros(3, dtype=torch.float64).pin_memory()
    for b in range(2):
        free[b].record(stream)
    H_ = len(host_gt)

    def copy(k):
        b = k % 2
        copy_stream.wait_event(free[b])
        with torch.cuda.stream(copy_stream):
            if r1 > r0:
                dev_gt[b][r0:r1].copy_(host_gt[k % H_][r0:r1], non_blocking=True)
            copied[b].record(copy_stream)

    def gather(k):
        b = k % 2
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(copied[b])
            dist.all_gather_into_tensor(dev_gt[b], dev_gt[b][rank * rows:(rank + 1) * rows])
            ready[b].record(copy_stream)

    bw = h2d_gbs(host_gt[0][r0:r1], dev_gt[0][r0:r1]) if r1 > r0 else 0.0
    st.prime_rgb(cams[0])
    dist.barrier()
    t0 = time.perf_counter()
    copy(0)
    gather(0)
    for k in range(e2e_steps):
        b = k % 2
        stream.wait_event(ready[b])
        nxt = k + 1 < e2e_steps
        if nxt:
            copy(k + 1)
        st.step(k % H_, gt=dev_gt[b][:H], cam_next_index=(k + 1) % H_,
                between=(lambda: gather(k + 1)) if nxt else None)
        free[b].record(stream)
        parts_host.copy_(st.parts, non_blocking=True)
        stream.synchronize()
    if st.pending[0] is not None:
        st.pending[0].synchronize()
    torch.cuda.synchronize()
    e2e_s = torch.tensor([(time.perf_counter() - t0) / e2e_steps], device=dev, dtype=torch.float64)
    dist.all_reduce(e2e_s, op=dist.ReduceOp.MAX)
    return {"value": round(1.0 / float(e2e_s.item()), 3), "unit": "iters/s",
            "h2d_bytes_per_step": int(gts[0].numel() * 4), "d2h_bytes_per_step": 24 * ws, "steps": e2e_steps,
            "h2d_per_rank_bytes": int((r1 - r0) * gts[0][0].numel() * 4), "h2d_gbs_measured": bw,
            "path": (("msplat_route_*" if st.route is not None else "msplat_shard_*") +
                     " C ABI + NCCL per rank: each rank copies 1/N of the target's rows host->device "
                     "from pinned memory and the row blocks are all-gathered over NVLink, for the next "
                     "step while the current one computes; loss sums D2H")}


# ---------------------------------------------------------------- config 4
def run_config4(B, dist, args, ws, rank, local, dev):
    """The load-skewed stress workload (6M Gaussians, SH3,
    4946x3286, 20 % of the means in a clump in front of camera 0, heavy-tailed
    radii; every tile over the 2048 cap) on 4 ring cameras, timed like the
    main run, with its tile-count imbalance and the cost of the overfull-tile
    path (key emission + tile sort)."""
    import torch
    S, cfg, scene = build_scene(4)
    cams = cameras(B, S, cfg, scene)[:4]
    gts = render_targets(B, cfg, scene, cams, dev)
    st = Stepper(B, dist if ws > 1 else None, cfg, scene, cams, gts, ws, rank, dev, args.exchange)
    st.prime_rgb(cams[0])
    ms, per_stage, launches, clk = timed_run(B, dist, st, args.config4_steps, 2, ws, dev, local, ws > 1)
    raw = B.last_tensor("raw_tile_counts").double()
    tb = B.last_tensor("tile_bins")
    kept_t = (tb[:, 1] - tb[:, 0]).double()
    tx = (cfg.width + 15) // 16
    rows = (0, (cfg.height + 15) // 16) if ws == 1 else (st.plan.row0, st.plan.row1)
    band = kept_t.view(-1, tx)[rows[0]:rows[1]].reshape(-1)
    totals = B.last_tensor("intersection_totals").cpu().numpy()
    kept = B.last_num_intersections()
    ranks = rank_breakdown(st, per_stage, kept, ws, rank, dist) if ws > 1 else None
    st.close()
    del st, gts
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    stat = lambda t: {"mean": round(float(t.mean()), 1), "max": int(t.max()),
                      "max_over_mean": round(float(t.max() / max(t.mean(), 1e-9)), 2)}
    out = {"workload": f"config 4: {cfg.n} Gaussians SH{cfg.degree}, {cfg.width}x{cfg.height}, 4 ring cameras",
           "value": round(1000.0 / ms, 3), "unit": "iters/s", "ms_per_step": round(ms, 3),
           "steps": args.config4_steps, "warmup": 2, "gpu_launches": int(launches), "clocks": clk,
           "stage_ms": {k: round(v, 4) for k, v in per_stage.items()},
           "overfull_path_ms": round(per_stage.get("emit_keys", 0.0) + per_stage.get("tile_sort", 0.0), 4),
           "raw_intersections": int(raw.sum().item()), "emitted_keys": int(totals[0]),
           "kept_intersections_rank0": int(kept),
           "tiles_over_cap_frac": round(float((raw > 2048).double().mean().item()), 4),
           "raw_per_tile": stat(raw), "kept_per_tile_rank0_band": stat(band) if band.numel() else None}
    if ranks is not None:
        out["ranks"] = ranks
    return out


# ---------------------------------------------------------------- CPU baseline
def cpu_baseline(S, cfg, scene, gt_np, steps=1, warmup=0):
    """The CPU oracle (restatement of the reference kernels, OpenMP over
    pixels and Gaussians) on the host cores: (1) a bounded sample of one step
    of the benchmark's workload, extrapolated to the full step; (2) the full,
    unsampled config-0 step (10k Gaussians, SH0, 256x256), single-threaded
    and with all threads."""
    from oracle import oracle as O
    threads = O.set_threads(os.cpu_count() or 1)
    stride = {0: 1, 1: 1, 2: 4}.get(cfg_id(cfg), 16)
    fx, fy, cx, cy = scene.intrinsics
    ocam = O.prepare_cam(scene.cam_to_world[0], fx, fy, cx, cy, cfg.width, cfg.height)
    tr = O.OracleTrainer(scene.params(), cfg.degree)
    for _ in range(warmup):
        tr.time_sample(ocam, gt_np, S.BACKGROUND, stride)
    ests, walls = [], []
    stages = None
    for _ in range(steps):
        t0 = time.perf_counter()
        est, stages = tr.time_sample(ocam, gt_np, S.BACKGROUND, stride)
        walls.append(time.perf_counter() - t0)
        ests.append(est)
    est = sum(ests) / len(ests)
    out = {"value": round(1.0 / est, 5), "unit": "iters/s", "cores": threads, "kind": "port",
           "estimate": f"extrapolated: rasteriser rows sampled 1 in {stride}, scaled x{stride}" if stride > 1
           else "full step",
           "sample": (f"oracle step on config workload: per-Gaussian stages on all {cfg.n} Gaussians, binning "
                      f"of all tiles, rasteriser fwd/bwd on every {stride}th tile row and SSIM on "
                      f"{cfg.height // stride} pixel rows, both scaled x{stride}"),
           "stage_s": [round(x, 3) for x in stages], "est_s_per_step": round(est, 3),
           "sample_wall_s_per_step": round(sum(walls) / len(walls), 3), "nproc": os.cpu_count()}
    out["config0_full_step"] = config0_cpu(O, S)
    return out


def config0_cpu(O, S, steps=5):
    """Full config-0 training steps (orc_train_step: forward, loss, backward,
    Adam on six groups) timed with 1 thread and with all threads."""
    cfg = S.CONFIGS[0]
    scene = S.make_scene(cfg, seed=0)
    fx, fy, cx, cy = scene.intrinsics
    ocam = O.prepare_cam(scene.cam_to_world[0], fx, fy, cx, cy, cfg.width, cfg.height)
    gt = O.render(scene.jittered().params(), cfg.degree, cfg.degree, S.BACKGROUND, ocam)
    res = {"workload": "config 0: 10000 Gaussians SH0, 256x256, full step (no sampling)", "nproc": os.cpu_count()}
    for label, nt in (("threads_1", 1), ("threads_all", os.cpu_count() or 1)):
        used = O.set_threads(nt)
        tr = O.OracleTrainer(scene.params(), cfg.degree)
        tr.step(ocam, gt, S.BACKGROUND)  # warm-up
        t0 = time.perf_counter()
        for _ in range(steps):
            tr.step(ocam, gt, S.BACKGROUND)
        s = (time.perf_counter() - t0) / steps
        res[label] = {"threads": used, "ms_per_step": round(1000 * s, 3), "iters_per_s": round(1.0 / s, 3)}
    O.set_threads(os.cpu_count() or 1)
    return res


def cfg_id(cfg):
    from msplat import synthetic as S
    for k, v in S.CONFIGS.items():
        if v == cfg:
            return k
    return -1


def run_reference(args, ws, rank):
    """The reference arm: the oracle port of the reference's kernels on the
    host cores (all threads), each step a bounded sample of the config's
    step (sampled tile rows, see cpu_baseline), the target the oracle's render
    of the jittered scene on the pixel rows the sampled loss reads. value is
    the full step's iters/s extrapolated from the samples; ms_per_step is the
    measured wall time of one sampled step."""
    if rank != 0:
        return
    S, cfg, scene = build_scene(args.config)
    from oracle import oracle as O
    threads = O.set_threads(os.cpu_count() or 1)
    stride = {0: 1, 1: 1, 2: 4}.get(args.config, 16)
    fx, fy, cx, cy = scene.intrinsics
    ocam = O.prepare_cam(scene.cam_to_world[0], fx, fy, cx, cy, cfg.width, cfg.height)
    band = max(1, cfg.height // stride)
    gt = O.render_rows(scene.jittered().params(), cfg.degree, cfg.degree, S.BACKGROUND, ocam, band)
    tr = O.OracleTrainer(scene.params(), cfg.degree)
    for _ in range(args.warmup):
        tr.time_sample(ocam, gt, S.BACKGROUND, stride)
    ests, walls, stages = [], [], None
    for _ in range(args.steps):
        t0 = time.perf_counter()
        est, stages = tr.time_sample(ocam, gt, S.BACKGROUND, stride)
        walls.append(time.perf_counter() - t0)
        ests.append(est)
    est = sum(ests) / len(ests)
    wall = sum(walls) / len(walls)
    v = round(1.0 / est, 5)
    cb = {"value": v, "unit": "iters/s", "cores": threads, "kind": "port",
          "estimate": (f"extrapolated: rasteriser rows sampled 1 in {stride}, scaled x{stride}" if stride > 1
                       else "full step"),
          "sample": (f"oracle step: per-Gaussian stages on all {cfg.n} Gaussians, binning of all tiles, rasteriser "
                     f"fwd/bwd on every {stride}th tile row and the loss on pixel rows [0, {band}) (target rendered "
                     f"by the oracle on those rows), scaled x{stride}"),
          "stage_s": [round(x, 3) for x in stages], "est_s_per_step": round(est, 3),
          "sample_wall_s_per_step": round(wall, 3), "nproc": os.cpu_count()}
    line = {"metric": METRIC, "value": v, "unit": "iters/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(1000.0 * wall, 3), "higher_is_better": True,
            "scaling": "strong" if ws > 1 else "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded; shapes/distributions of BASELINE config %d)" % args.config,
            "config": {"workload": f"config {args.config}: {cfg.n} Gaussians SH{cfg.degree}, "
                                   f"{cfg.width}x{cfg.height}", "parallelism": "CPU host cores"},
            "value_note": (("value: iters/s of the full step extrapolated from the timed samples "
                            f"({round(est, 2)} s per full step); ms_per_step: measured wall time of one sampled "
                            "step") if stride > 1 else "full, unsampled step"),
            "impl": "reference", "cpu_baseline": cb,
            "e2e": {"value": v, "unit": "iters/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    ws, rank, local = dist_env()
    if args.impl == "reference":
        run_reference(args, ws, rank)
        return
    run_ours(args, ws, rank, local)


if __name__ == "__main__":
    main()

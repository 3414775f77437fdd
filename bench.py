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

N > 1 (torchrun, one process per GPU): image tile rows are sharded across
ranks (strong scaling: the image and the Gaussian set are fixed), per-Gaussian
raster gradients are reduce-scattered with NCCL, each rank runs the
projection VJP + Adam on its slice of Gaussians, and the updated parameters
are all-gathered.

--impl reference: the CPU oracle (a restatement of the reference's Metal
kernels; the Metal code cannot run here) timed on the host cores on a bounded
sample of every step (see oracle.h: orc_time_step_sample).
"""
from __future__ import annotations

import argparse
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


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--exchange", default="rgb", choices=["peers", "nccl", "rgb"],
                    help="multi-GPU parameter exchange: geometry all-gathered and the owners' colours for the "
                         "next camera all-gathered instead of the colour coefficients (rgb, default); NCCL "
                         "all-gathers of all groups with the colour groups overlapped with binning (nccl); or "
                         "geometry all-gathered and colour read from its owner over NVLink (CUDA IPC, peers)")
    ap.add_argument("--render-frames", type=int, default=20,
                    help="render-only frames timed after the training steps (single GPU); 0 = skip")
    ap.add_argument("--cameras", type=int, default=0,
                    help="use only the first C ring cameras (fewer target images on the device); 0 = all")
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


# ---------------------------------------------------------------- byte model
def raster_bwd_bytes(kept: int, n_vis: int, pixels: int) -> int:
    """Algorithmic HBM bytes of one rasterize_backward launch in this design:
    5 B per kept intersection (sorted id + the forward's per-warp blend byte),
    80 B per visible Gaussian (raster record, read once), 32 B per pixel
    (final T/M1/M2, last/median index, dL/dimg), 64 B read + 64 B written per
    visible Gaussian (gradient record)."""
    return 5 * kept + 80 * n_vis + 32 * pixels + 128 * n_vis


def raster_fwd_bytes(kept: int, n_vis: int, pixels: int) -> int:
    """5 B per kept intersection (sorted id read, blend byte written), 80 B per
    visible Gaussian, 60 B per pixel of outputs (image, T/M1/M2, indices,
    depth, normal, alpha, median, distortion)."""
    return 5 * kept + 80 * n_vis + 60 * pixels


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
            dist.init_process_group("nccl", device_id=dev, timeout=__import__("datetime").timedelta(seconds=300))
            dist.barrier()
        finally:
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)
    cams = cameras(B, S, cfg, scene)
    if args.cameras > 0:
        cams = cams[:args.cameras]
    C = len(cams)
    n = cfg.n
    bg = S.BACKGROUND
    # targets: render of the jittered scene for every camera (setup, untimed)
    tgt = B.DeviceGaussians(*scene.jittered().params(), sh_degree=cfg.degree)
    gts = []
    for c in cams:
        img = torch.empty(cfg.height, cfg.width, 3, device=dev)
        B.render(tgt, c, cfg.degree, bg, out_img=img)
        gts.append(img)
    torch.cuda.synchronize()
    del tgt
    g = B.DeviceGaussians(*scene.params(), sh_degree=cfg.degree)
    adam = B.AdamState(g)
    stats = [torch.zeros(n, device=dev) for _ in range(3)]
    loss_dev = torch.zeros(1, device=dev)
    l1, ld = 1.0 - SSIM_WEIGHT, 0.0
    stream = torch.cuda.current_stream()

    if ws == 1:
        def step(k):
            B.train_step_fused(g, cams[k % C], cfg.degree, bg, gts[k % C], l1, ld, SSIM_WEIGHT, adam, stats=stats,
                               loss_dev=loss_dev)
    else:
        from msplat import sharding
        plan = sharding.ShardPlan(n, (cfg.height + 15) // 16, ws, rank)
        peers = None
        exchange = "NCCL all-gather (colour groups overlapped with binning)"
        if args.exchange == "peers":
            peers = sharding.PeerParams(B, dist, plan, g)
            if peers.ok:
                exchange = ("geometry all-gathered; colour read from its owner over NVLink (CUDA IPC) for the "
                            "rank's band only")
            else:
                exchange += "; peer mapping failed: " + peers.error[:120]
            adam = B.AdamState(g)
        else:
            sharding.pad_gaussians(g, plan.padded)
        use_peers = peers is not None and peers.ok
        rg = torch.zeros(plan.padded, 16, device=dev)
        rg_shard = torch.zeros(plan.chunk, 16, device=dev)
        parts = torch.zeros(3, dtype=torch.float64, device=dev)

        side = torch.cuda.Stream(device=dev)
        pending = [None]  # event: colour groups (or colours) of the last step gathered
        rgb_full = None
        if args.exchange == "rgb":
            rgb_full = torch.zeros(plan.padded, 3, device=dev)
            exchange = ("geometry all-gathered; each owner's clamped colours for the next camera all-gathered "
                        "(12 B per Gaussian) instead of the colour coefficients")
        have_rgb = [False]

        def mstep(cam, gt, cam_next):
            adam.step += 1
            fb, pa = sharding.gpu_step_fns(B, g, cam, cfg.degree, bg, gt, l1, ld, SSIM_WEIGHT, adam, stats,
                                           features_ready=pending[0], split_color=not use_peers,
                                           peers=peers if use_peers else None,
                                           rgb=rgb_full if have_rgb[0] else None)
            colors_next = None if rgb_full is None else sharding.colors_fn(B, g, cam_next, cfg.degree, rgb_full)
            pending[0] = sharding.sharded_step(dist, plan, fb, pa, rg, rg_shard, g.full, parts,
                                               side_stream=None if use_peers else side,
                                               skip_color=use_peers or rgb_full is not None,
                                               colors_next=colors_next, rgb_full=rgb_full)
            have_rgb[0] = rgb_full is not None

        def prime_rgb(cam):
            # colours for `cam` from the owners' current coefficients
            torch.cuda.synchronize()
            sharding.colors_fn(B, g, cam, cfg.degree, rgb_full)(plan.g_begin, plan.g_end)
            rows = plan.slice_rows()
            dist.all_gather_into_tensor(rgb_full, rgb_full[rows])
            pending[0] = None
            have_rgb[0] = True

        def step(k):
            mstep(cams[k % C], gts[k % C], cams[(k + 1) % C])

    for k in range(args.warmup):
        step(k)
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    launches0 = B.launch_count()
    B.set_stage_timing(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for k in range(args.steps):
        step(args.warmup + k)
    if ws > 1 and pending[0] is not None:
        stream.wait_event(pending[0])  # the last step's gather belongs to the timed work
    e1.record(stream)
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    launches = B.launch_count() - launches0
    stage = B.stage_times()
    B.set_stage_timing(False)
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    if ws > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = 1000.0 / ms
    pixels = cfg.width * cfg.height

    # roofline of the dominant kernel over the timed region
    kept = B.last_num_intersections()
    n_vis = int((B.last_tensor("radii") > 0).sum().item())
    per_stage = {k: (v[0] / max(v[1], 1)) for k, v in stage.items()}
    kernel_stages = {k: v for k, v in per_stage.items() if k != "between_shard_calls"}
    dom = max(kernel_stages, key=kernel_stages.get)
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    byte_models = {"rasterize_backward": raster_bwd_bytes(kept, n_vis, pixels),
                   "rasterize_forward": raster_fwd_bytes(kept, n_vis, pixels)}
    traffic = None
    try:
        tr = json.load(open(os.path.join(REPO, "profiles", "traffic.json")))
        # the capture is of a single-GPU launch over the whole image
        if tr.get("kernel") == dom and tr.get("config") == args.config and ws == 1 and args.cameras == 0:
            traffic = tr.get("bytes_per_launch")
    except (OSError, ValueError):
        pass
    alg = byte_models.get(dom)
    roof = None
    if alg is not None:
        ach = alg / (per_stage[dom] * 1e-3) / 1e9
        roof = {"kernel": dom, "bound": "hbm", "achieved": round(ach, 2), "peak": hbm_peak, "peak_source": peak_src,
                "unit": "GB/s", "frac": round(ach / hbm_peak, 5), "traffic": traffic,
                "algorithmic_bytes": alg, "ms_per_launch": round(per_stage[dom], 4),
                "pairs_upper_bound_per_s": round(kept * 256 / (per_stage[dom] * 1e-3), 1)}

    # render-only forward (msplat_render, msplat_metal.mm:545-772): projection,
    # binning, sort and the forward rasteriser per frame, image left on the device
    render = None
    if ws == 1 and args.render_frames > 0:
        frame = torch.empty(cfg.height, cfg.width, 3, device=dev)
        for k in range(3):
            B.render(g, cams[k % C], cfg.degree, bg, out_img=frame)
        torch.cuda.synchronize()
        r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        r0.record(stream)
        for k in range(args.render_frames):
            B.render(g, cams[k % C], cfg.degree, bg, out_img=frame)
        r1.record(stream)
        torch.cuda.synchronize()
        rms = r0.elapsed_time(r1) / args.render_frames
        render = {"value": round(1000.0 / rms, 2), "unit": "frames/s", "ms_per_frame": round(rms, 3),
                  "frames": args.render_frames, "path": "msplat_render, image kept on the device"}
        del frame

    # e2e through the public trainer API (msplat_trainer_step): every step
    # copies its target image host->device from pinned memory and reads the
    # loss back, as a user of msplat_c_api.h does.
    e2e = None
    e2e_steps = args.e2e_steps if args.e2e_steps is not None else min(args.steps, 10)
    if e2e_steps > 0 and ws == 1:
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
        e2e = {"value": round(1.0 / e2e_s, 3), "unit": "iters/s", "h2d_bytes_per_step": int(host_imgs[0].nbytes),
               "d2h_bytes_per_step": 4, "steps": e2e_steps,
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
    elif e2e_steps > 0:
        # each step's target is copied host->device on a copy stream while the
        # previous step computes (two device buffers)
        host_gt = [gts[k].cpu().pin_memory() for k in range(min(C, 4))]
        dev_gt = [torch.empty_like(gts[0]), torch.empty_like(gts[0])]
        copy_stream = torch.cuda.Stream(device=dev)
        ready = [torch.cuda.Event(), torch.cuda.Event()]
        free = [torch.cuda.Event(), torch.cuda.Event()]
        parts_host = torch.zeros(3, dtype=torch.float64).pin_memory()
        for b in range(2):
            free[b].record(stream)

        def prefetch(k):
            b = k % 2
            copy_stream.wait_event(free[b])
            with torch.cuda.stream(copy_stream):
                dev_gt[b].copy_(host_gt[k % len(host_gt)], non_blocking=True)
                ready[b].record(copy_stream)

        H = len(host_gt)
        if rgb_full is not None:
            prime_rgb(cams[0])
        dist.barrier()
        t0 = time.perf_counter()
        prefetch(0)
        for k in range(e2e_steps):
            b = k % 2
            stream.wait_event(ready[b])
            mstep(cams[k % H], dev_gt[b], cams[(k + 1) % H])
            free[b].record(stream)
            if k + 1 < e2e_steps:
                prefetch(k + 1)
            parts_host.copy_(parts, non_blocking=True)
            stream.synchronize()
        if pending[0] is not None:
            pending[0].synchronize()
        e2e_s = torch.tensor([(time.perf_counter() - t0) / e2e_steps], device=dev, dtype=torch.float64)
        dist.all_reduce(e2e_s, op=dist.ReduceOp.MAX)
        e2e = {"value": round(1.0 / float(e2e_s.item()), 3), "unit": "iters/s",
               "h2d_bytes_per_step": int(gts[0].numel() * 4), "d2h_bytes_per_step": 24, "steps": e2e_steps,
               "path": ("msplat_shard_* C ABI + NCCL per rank: target image H2D from pinned memory on a copy "
                        "stream overlapping the previous step, loss sums D2H")}

    ranks = None
    if ws > 1:
        mine = {"rank": rank, "tile_rows": [plan.row0, plan.row1], "intersections": kept,
                "rasterize_forward_ms": round(per_stage.get("rasterize_forward", 0.0), 4),
                "rasterize_backward_ms": round(per_stage.get("rasterize_backward", 0.0), 4),
                "loss_ssim_ms": round(per_stage.get("loss_ssim", 0.0), 4),
                "between_shard_calls_ms": round(per_stage.get("between_shard_calls", 0.0), 4),
                "kernel_stage_sum_ms": round(sum(kernel_stages.values()), 4)}
        ranks = [None] * ws
        dist.all_gather_object(ranks, mine)

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(S, cfg, scene, gts[0].cpu().numpy(), steps=1)

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
                "stage_ms": {k: round(v, 4) for k, v in per_stage.items()},
                "intersections": kept, "visible_gaussians": n_vis, "cpu_baseline": cpu}
        if ranks is not None:
            line["ranks"] = ranks
        print(json.dumps(line), flush=True)
    if ws > 1:
        torch.cuda.synchronize()
        if peers is not None:
            peers.close()
        dist.barrier()
        dist.destroy_process_group()


def cpu_baseline(S, cfg, scene, gt_np, steps=1, warmup=0):
    """Times the CPU oracle (restatement of the reference kernels) on a bounded
    sample of one step of the same workload; returns the cpu_baseline dict."""
    from oracle import oracle as O
    threads = O.set_threads(0)
    stride = {0: 1, 1: 1, 2: 4}.get(cfg_id(cfg), 16)
    fx, fy, cx, cy = scene.intrinsics
    ocam = O.prepare_cam(scene.cam_to_world[0], fx, fy, cx, cy, cfg.width, cfg.height)
    tr = O.OracleTrainer(scene.params(), cfg.degree)
    for _ in range(warmup):
        tr.time_sample(ocam, gt_np, S.BACKGROUND, stride)
    ests = []
    stages = None
    for _ in range(steps):
        est, stages = tr.time_sample(ocam, gt_np, S.BACKGROUND, stride)
        ests.append(est)
    est = sum(ests) / len(ests)
    return {"value": round(1.0 / est, 5), "unit": "iters/s", "cores": threads, "kind": "port",
            "sample": (f"oracle step on config workload: per-Gaussian stages on all {cfg.n} Gaussians, binning "
                       f"of all tiles, rasteriser fwd/bwd on every {stride}th tile row and SSIM on "
                       f"{cfg.height // stride} pixel rows, both scaled x{stride}"),
            "stage_s": [round(x, 3) for x in stages], "est_s_per_step": round(est, 3)}


def cfg_id(cfg):
    from msplat import synthetic as S
    for k, v in S.CONFIGS.items():
        if v == cfg:
            return k
    return -1


def run_reference(args, ws, rank):
    if rank != 0:
        return
    import torch  # noqa: F401  (only for parity of the environment)
    S, cfg, scene = build_scene(args.config)
    from oracle import oracle as O
    fx, fy, cx, cy = scene.intrinsics
    ocam = O.prepare_cam(scene.cam_to_world[0], fx, fy, cx, cy, cfg.width, cfg.height)
    gt = O.render(scene.jittered().params(), cfg.degree, cfg.degree, S.BACKGROUND, ocam) if cfg.n <= 200_000 \
        else np.zeros((cfg.height, cfg.width, 3), np.float32) + 0.5
    cb = cpu_baseline(S, cfg, scene, gt, steps=args.steps, warmup=args.warmup)
    v = cb["value"]
    line = {"metric": METRIC, "value": v, "unit": "iters/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(1000.0 / v, 3), "higher_is_better": True,
            "scaling": "strong" if ws > 1 else "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded; shapes/distributions of BASELINE config %d)" % args.config,
            "config": {"workload": f"config {args.config}: {cfg.n} Gaussians SH{cfg.degree}, "
                                   f"{cfg.width}x{cfg.height}", "parallelism": "CPU host cores"},
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

"""Launched by tests/test_multigpu.py under torchrun (one process per GPU).

Each rank runs two sharded training steps (msplat/sharding.py) on a small
scene, exchanging parameters either with NCCL all-gathers (colour groups on a
side stream while the next step bins; MSPLAT_EXCHANGE=nccl), with the
geometry all-gathered and the colour read from its owner rank through CUDA
IPC (MSPLAT_EXCHANGE=peers), or with the geometry all-gathered and the
owners' clamped colours for the next camera all-gathered instead of the
colour coefficients (MSPLAT_EXCHANGE=rgb), or with the routed exchange
(MSPLAT_EXCHANGE=route: each owner projects its slice, the projected
Gaussians go to the bands they touch and the gradients come back to the
owner, by NCCL all-to-alls; MSPLAT_EXCHANGE=route-peer: by stores into the
other GPU's inbox and return box over NVLink; nothing is gathered); rank 0
also runs the same two
steps with the single-GPU fused
step on a private copy and compares the parameters. Prints "MULTIGPU OK" on
success (rank 0) and exits non-zero otherwise.
"""
import datetime
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
for p in (REPO, os.path.join(REPO, "msplat-ios_b200", "python"), HERE):
    sys.path.insert(0, p)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from _cases import Case  # noqa: E402
from msplat import _backend as B  # noqa: E402
from msplat import sharding  # noqa: E402


def main():
    rank, ws, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    B.load()
    case = Case("sh3_small")
    cfg, n = case.cfg, case.cfg.n
    cam = B.camera_from_oracle(case.ocam)
    gt = torch.as_tensor(case.gt).to(dev)
    g = B.DeviceGaussians(*case.scene.params(), sh_degree=case.degree, device=dev)
    adam = B.AdamState(g)
    plan = sharding.ShardPlan(n, (cfg.height + 15) // 16, ws, rank)
    exchange = os.environ.get("MSPLAT_EXCHANGE", "nccl")
    peers = None
    if exchange == "peers":
        # every rank reads each Gaussian from its owner's buffers (CUDA IPC)
        peers = sharding.PeerParams(B, dist, plan, g)
        adam = B.AdamState(g)
    else:
        sharding.pad_gaussians(g, plan.padded)
    route = route_peers = None
    if exchange in ("route", "route-peer"):
        if exchange == "route-peer":
            route_peers = sharding.RoutePeers(B, dist, plan, n, dev)
            if not route_peers.ok:
                print("peer mapping failed: " + route_peers.error, flush=True)
                sys.exit(1)
        route = sharding.gpu_route_calls(B, g, cam, case.degree, case.bg, gt, 0.8, 0.0, 0.2, adam, None, plan,
                                         peers=route_peers)
    rgb_full = torch.zeros(plan.padded, 3, device=dev) if exchange == "rgb" else None
    rg = torch.zeros(plan.padded, 16, device=dev)
    rg_shard = torch.zeros(plan.chunk, 16, device=dev)
    parts = torch.zeros(3, dtype=torch.float64, device=dev)
    # the overlapped schedule the benchmark runs with NCCL: colour groups
    # gathered on a side stream while the next step bins its geometry
    side = torch.cuda.Stream(device=dev)
    ready = None
    for step in range(2 if route is None else 0):
        adam.step += 1
        fb, pa = sharding.gpu_step_fns(B, g, cam, case.degree, case.bg, gt, 0.8, 0.0, 0.2, adam, None,
                                       features_ready=ready, split_color=peers is None, peers=peers,
                                       rgb=rgb_full if (rgb_full is not None and step > 0) else None)
        colors_next = None if rgb_full is None else sharding.colors_fn(B, g, cam, case.degree, rgb_full)
        ready = sharding.sharded_step(dist, plan, fb, pa, rg, rg_shard, g.full, parts,
                                      side_stream=None if peers else side,
                                      skip_color=peers is not None or rgb_full is not None,
                                      colors_next=colors_next, rgb_full=rgb_full)
    bands = None
    for step in range(2 if route is not None else 0):
        adam.step += 1
        bands = sharding.routed_step(dist, plan, route, parts)
    if bands is not None and rank == 0:
        print(f"bands {bands}", flush=True)
    torch.cuda.synchronize()
    loss_sh = sharding.loss_from_parts(parts.cpu().numpy(), 0.2, cfg.width, cfg.height)
    if peers is not None or rgb_full is not None or route is not None:
        # each rank's colour buffers are current only in the rows it owns:
        # gather them once to compare the whole parameter set
        rows = plan.slice_rows()
        gathered = []
        for full in g.full:
            out = torch.empty_like(full)
            if full.numel():
                dist.all_gather_into_tensor(out, full[rows].contiguous())
            gathered.append(out[:n])
        got = [t.cpu().numpy() for t in gathered]
        torch.cuda.synchronize()
        if peers is not None:
            peers.close()
        if route_peers is not None:
            route_peers.close()
    else:
        got = [t.cpu().numpy() for t in g.groups()]
    ok = True
    if rank == 0:
        g1 = B.DeviceGaussians(*case.scene.params(), sh_degree=case.degree, device=dev)
        a1 = B.AdamState(g1)
        loss_dev = torch.zeros(1, device=dev)
        losses = []
        for _ in range(2):
            B.train_step_fused(g1, cam, case.degree, case.bg, gt, 0.8, 0.0, 0.2, a1, loss_dev=loss_dev)
            losses.append(float(loss_dev.cpu()[0]))
        ref = [t.cpu().numpy() for t in g1.groups()]
        for k in range(6):
            if ref[k].size == 0:
                continue
            frac = np.isclose(got[k], ref[k], rtol=1e-5, atol=1e-7).mean()
            print(f"group {k}: {frac:.6f} of elements within 1e-5", flush=True)
            ok &= frac > 0.999
        print(f"loss sharded {loss_sh:.7f} single {losses[-1]:.7f}", flush=True)
        ok &= abs(loss_sh - losses[-1]) <= 1e-4 * abs(losses[-1])
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dist.destroy_process_group()
    if rank == 0:
        print("MULTIGPU OK" if flag.item() == 1 else "MULTIGPU FAIL", flush=True)
    sys.exit(0 if flag.item() == 1 else 1)


if __name__ == "__main__":
    main()

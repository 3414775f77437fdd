"""Multi-rank tile sharding on CPU ranks (gloo), with the oracle as the compute.

sharded_step (msplat/sharding.py) is the collective sequence the GPU ranks run
with NCCL. Here two gloo ranks run it with the CPU oracle standing in for the
CUDA kernels: each rank back-propagates only its own tile rows, the raster
gradients are reduce-scattered, each rank applies the projection VJP and Adam
to its slice, and the parameters are all-gathered. The result must equal one
single-process oracle step. The colour exchange (mode "rgb") gathers each
owner's clamped colours for the next camera instead of the colour
coefficients; those must equal the oracle's colours of the updated scene.
"""
import os
import socket

import numpy as np
import pytest

from msplat import sharding


def test_shard_plan_partitions_rows_and_gaussians():
    for n, ty, ws in [(10_000, 16, 2), (3_000_000, 206, 8), (1_000, 3, 4), (257, 1, 2)]:
        plans = [sharding.ShardPlan(n, ty, ws, r) for r in range(ws)]
        rows = [r for p in plans for r in range(p.row0, p.row1)]
        assert rows == list(range(ty))
        gs = [i for p in plans for i in range(p.g_begin, p.g_end)]
        assert gs == list(range(n))
        assert all(p.chunk % 256 == 0 and p.padded == p.chunk * ws and p.padded >= n for p in plans)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, ws, port, out_path, mode="coeffs"):
    import torch
    import torch.distributed as dist

    from _cases import Case
    from oracle import oracle as O
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    O.set_threads(2)
    case = Case("sh3_small")
    n, deg, cam, bg = case.cfg.n, case.degree, case.ocam, case.bg
    plan = sharding.ShardPlan(n, (cam.height + 15) // 16, ws, rank)
    p, bins, packed, fwd = case.oracle_forward()
    ls = O.loss_ssim(fwd["out_img"], case.gt, fwd["out_distortion"], 0.8, 0.0, 0.2)
    params = [np.array(a, np.float32) for a in (case.scene.means, case.scene.scales, case.scene.quats,
                                                 case.scene.f_dc, case.scene.f_rest,
                                                 case.scene.opacities.reshape(-1, 1))]
    fulls = []
    for a in params:
        f = torch.zeros((plan.padded,) + a.shape[1:], dtype=torch.float32)
        f[:n] = torch.from_numpy(a)
        fulls.append(f)
    m = [np.zeros_like(a) for a in params]
    v = [np.zeros_like(a) for a in params]

    def forward_backward(plan_, rg, parts):
        row0, row1 = plan_.row0, plan_.row1
        dimg = ls["dL_dout_img"].copy()
        dimg[: row0 * 16] = 0.0
        dimg[row1 * 16:] = 0.0
        rb = O.rasterize_backward(n, bins, packed, fwd, cam, bg, dimg)
        rec = np.concatenate([rb["dL_dtransMat"], rb["dL_dopacity"], rb["dL_dcolors"], rb["dL_dnormal3D"]], 1)
        rg.zero_()
        rg[:n] = torch.from_numpy(rec)
        own = slice(row0 * 16, min(row1 * 16, cam.height))
        parts[:] = torch.tensor([0.8 * np.abs(fwd["out_img"][own] - case.gt[own]).astype(np.float64).sum()
                                 / (3 * cam.width * cam.height), 0.0, 0.0], dtype=torch.float64)

    def project_adam(g0, g1, rg_shard):
        rec = rg_shard[: g1 - g0].numpy()
        sl = slice(g0, g1)
        pb = O.project_backward(params[0][sl], params[1][sl], params[2][sl], cam, p["radii"][sl],
                                np.ascontiguousarray(rec[:, 0:9]), np.ascontiguousarray(rec[:, 13:16]),
                                np.ascontiguousarray(rec[:, 10:13]), deg, deg, params[4][sl])
        grads = [pb["dL_dmean3D"], pb["dL_dscale"], pb["dL_dquat"], pb["dL_dfeatures_dc"], pb["dL_dfeatures_rest"],
                 np.ascontiguousarray(rec[:, 9:10])]
        bc1 = np.float32(1.0 - float(np.float32(0.9)))
        bc2 = np.float32(1.0 - float(np.float32(0.999)))
        for k in range(6):
            if params[k].size == 0:
                continue
            pk = np.ascontiguousarray(params[k][sl])
            mk, vk = np.ascontiguousarray(m[k][sl]), np.ascontiguousarray(v[k][sl])
            O.fused_adam(pk, grads[k], mk, vk, np.float32(O.LR_INIT[k]) / bc1, 0.9, 0.999,
                         float(np.sqrt(bc2)), 1e-8)
            fulls[k][sl] = torch.from_numpy(pk)

    rg = torch.zeros(plan.padded, sharding.GRAD_STRIDE)
    rg_shard = torch.zeros(plan.chunk, sharding.GRAD_STRIDE)
    parts = torch.zeros(3, dtype=torch.float64)
    colors_next, rgb_full = None, None
    if mode == "rgb":
        rgb_full = torch.zeros(plan.padded, 3)
        cam_next = Case("sh3_small", cam_index=1).ocam

        def colors_next(g0, g1):
            sl = slice(g0, g1)
            pn = O.project_forward(params[0][sl], params[1][sl], params[2][sl], params[5][sl], params[3][sl],
                                   params[4][sl], deg, deg, cam_next)
            rgb_full[sl] = torch.from_numpy(np.maximum(pn["colors"] + np.float32(0.5), np.float32(0.0)))
    sharding.sharded_step(dist, plan, forward_backward, project_adam, rg, rg_shard, fulls, parts,
                          skip_color=mode == "rgb", colors_next=colors_next, rgb_full=rgb_full)
    extra = {} if rgb_full is None else {"rgb": rgb_full[:n].numpy(), "g_begin": plan.g_begin, "g_end": plan.g_end}
    np.savez(out_path + f".{rank}.npz", *[f[:n].numpy() for f in fulls], parts=parts.numpy(), **extra)
    dist.destroy_process_group()


def test_two_gloo_ranks_equal_one_oracle_step(tmp_path):
    import torch.multiprocessing as mp

    from _cases import Case
    from oracle import oracle as O
    ws = 2
    out = str(tmp_path / "shard")
    mp.start_processes(_rank_main, args=(ws, _free_port(), out), nprocs=ws, start_method="spawn")
    res = [np.load(out + f".{r}.npz") for r in range(ws)]
    case = Case("sh3_small")
    tr = O.OracleTrainer(case.scene.params(), case.degree)
    ref = tr.step(case.ocam, case.gt, case.bg)
    ref_params = [tr.means, tr.scales, tr.quats, tr.f_dc, tr.f_rest, tr.opac]
    for k in range(6):
        a0, a1 = res[0][f"arr_{k}"], res[1][f"arr_{k}"]
        assert np.array_equal(a0, a1), "all-gathered parameters differ between ranks"
        ok = np.isclose(a0, ref_params[k], rtol=1e-5, atol=1e-7)
        # Adam's first step moves a parameter by about +-lr whatever the gradient
        # size, so a gradient that is zero up to rounding (summed in a different
        # order across ranks) may flip sign; allow a handful of such elements
        assert ok.mean() > 0.9995, (k, ok.mean())
    l1_total = 0.8 * np.abs(ref["out_img"] - case.gt).astype(np.float64).sum() / ref["out_img"].size
    assert abs(res[0]["parts"][0] - l1_total) < 1e-9


def test_two_gloo_ranks_exchange_next_camera_colours(tmp_path):
    """Mode rgb: the colour coefficients stay with their owners and every rank
    ends the step holding the clamped colours of all Gaussians for the next
    camera, equal to the oracle's colours of the updated scene."""
    import torch.multiprocessing as mp

    from _cases import Case
    from oracle import oracle as O
    ws = 2
    out = str(tmp_path / "shard_rgb")
    mp.start_processes(_rank_main, args=(ws, _free_port(), out, "rgb"), nprocs=ws, start_method="spawn")
    res = [np.load(out + f".{r}.npz") for r in range(ws)]
    case = Case("sh3_small")
    tr = O.OracleTrainer(case.scene.params(), case.degree)
    tr.step(case.ocam, case.gt, case.bg)
    nxt = Case("sh3_small", cam_index=1).ocam
    pn = O.project_forward(tr.means, tr.scales, tr.quats, tr.opac, tr.f_dc, tr.f_rest, case.degree, case.degree, nxt)
    want = np.maximum(pn["colors"] + np.float32(0.5), np.float32(0.0))
    assert np.array_equal(res[0]["rgb"], res[1]["rgb"]), "gathered colours differ between ranks"
    ok = np.isclose(res[0]["rgb"], want, rtol=1e-5, atol=1e-6)
    assert ok.mean() > 0.999, ok.mean()
    init = [case.scene.f_dc, case.scene.f_rest]
    for r in range(ws):
        g0, g1 = int(res[r]["g_begin"]), int(res[r]["g_end"])
        for k, a0 in ((3, init[0]), (4, init[1])):
            got = res[r][f"arr_{k}"]
            others = np.ones(got.shape[0], bool)
            others[g0:g1] = False
            assert np.array_equal(got[others], np.asarray(a0, np.float32)[others]), "colour groups were gathered"
            assert not np.array_equal(got[g0:g1], np.asarray(a0, np.float32)[g0:g1]), "owner slice not updated"


def test_three_gloo_ranks_equal_one_oracle_step(tmp_path):
    """Three ranks: uneven tile-row bands and Gaussian slices padded to a
    multiple of 256 per rank; the all-gathered parameters must still equal one
    oracle step on every rank."""
    import torch.multiprocessing as mp

    from _cases import Case
    from oracle import oracle as O
    ws = 3
    out = str(tmp_path / "shard3")
    mp.start_processes(_rank_main, args=(ws, _free_port(), out), nprocs=ws, start_method="spawn")
    res = [np.load(out + f".{r}.npz") for r in range(ws)]
    case = Case("sh3_small")
    tr = O.OracleTrainer(case.scene.params(), case.degree)
    tr.step(case.ocam, case.gt, case.bg)
    ref_params = [tr.means, tr.scales, tr.quats, tr.f_dc, tr.f_rest, tr.opac]
    for k in range(6):
        for r in range(1, ws):
            assert np.array_equal(res[0][f"arr_{k}"], res[r][f"arr_{k}"]), "ranks disagree"
        ok = np.isclose(res[0][f"arr_{k}"], ref_params[k], rtol=1e-5, atol=1e-7)
        assert ok.mean() > 0.9995, (k, ok.mean())

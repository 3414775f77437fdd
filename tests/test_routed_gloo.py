"""The routed exchange (sharding.routed_step) on CPU ranks (gloo), with the
oracle as the compute.

Each rank owns a slice of the Gaussians and a band of tile rows. routed_step
gathers every slice's summary (per-tile counts and the histograms of its
tile rectangles' first and last rows), cuts the bands, derives how many
Gaussians every rank sends to every rank, sends every projected
Gaussian to the ranks whose band (with a one-tile-row halo) its rectangle
meets, rasterises each band over what it received, and returns the gradient
records to the owners, which apply the projection VJP and Adam to their
slice. The stand-in calls restate the device side (route.cu): row work =
sum over the row's tiles of min(count, 2048) + 430 (route_row_work), bands
as the least-maximum-cost cover with the halo rows costed
(route_band_cuts), the count matrix from the histograms (checked against
each slice's own destinations), destinations by the halo rule, packing
grouped by destination in increasing id. The slices put together must
equal one single-process oracle step, every Gaussian that has a gradient in
a band must have reached that band, and nothing may reach a band it does
not touch.
"""
import os
import socket

import numpy as np

from msplat import sharding

CAP = 2048
ROW_WORK_PER_TILE = 430


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


ROW_TENTHS, HALO_TENTHS = 10, 4


def route_row_work(counts):
    """Restates k_route_row_work (route.cu): per tile min(raw, 2048) + 430,
    summed per tile row. counts: int64 [ty, tx]."""
    c = np.asarray(counts, np.int64)
    return (np.minimum(c, CAP) + ROW_WORK_PER_TILE).sum(1)


def route_band_cuts(work, world):
    """Restates k_route_cuts (route.cu): band cost in tenths of a row-work
    unit = 10 x the band's rows + 4 x each halo row it renders but does not
    own; the least L (to within one) for which the greedy cover (each band
    as long as possible, at most `world` bands) succeeds, found by 256-way
    search rounds, then the greedy cover at that L. Integer arithmetic."""
    w = [int(x) for x in work]
    ty = len(w)
    P = [0]
    for x in w:
        P.append(P[-1] + x)

    def cost(b0, b1):
        return ROW_TENTHS * (P[b1] - P[b0]) + (HALO_TENTHS * w[b0 - 1] if b0 > 0 else 0) + \
            (HALO_TENTHS * w[b1] if b1 < ty else 0)

    def greedy(L):
        cuts, b0 = [0], 0
        for _ in range(world):
            if b0 < ty:
                best, b1 = -1, b0 + 1
                while b1 <= ty and ROW_TENTHS * (P[b1] - P[b0]) <= L:
                    if cost(b0, b1) <= L:
                        best = b1
                    b1 += 1
                if best < 0:
                    return None
                b0 = best
            cuts.append(b0)
        return cuts if b0 == ty else None

    lo, hi = 0, ROW_TENTHS * P[ty] + 2 * HALO_TENTHS * max(w)
    for _ in range(12):
        if hi - lo <= 1:
            break
        cand = [lo + ((hi - lo) * (k + 1)) // 256 for k in range(256)]
        k = next(k for k in range(256) if greedy(cand[k]) is not None)
        lo, hi = (cand[k - 1] if k > 0 else lo), cand[k]
    cuts = greedy(hi)
    cuts[world] = ty
    return cuts


def route_matrix(starts, ends, bands, ty):
    """Items from rank r to rank q (restates k_route_cuts): r's Gaussians
    whose rectangle rows [y0, y1) meet q's band with its one-row halo
    [lo, hi), counted from the histograms of y0 (starts[r]) and y1 (ends[r]):
    all of them but those with y0 >= hi and those with y1 <= lo."""
    world = len(bands) - 1
    m = np.zeros((starts.shape[0], world), np.int64)
    for q in range(world):
        b0, b1 = bands[q], bands[q + 1]
        if b1 <= b0:
            continue
        lo, hi = max(0, b0 - 1), min(ty, b1 + 1)
        m[:, q] = starts.sum(1) - starts[:, hi:].sum(1) - ends[:, :lo + 1].sum(1)
    return m


class _OracleRouteCalls:
    """CPU stand-in for gpu_route_calls: projection, planning, packing and
    return on the owner's slice; the band's rasterisation backward from the
    oracle over the full scene with the image gradient masked to the band."""

    def __init__(self, case, plan, params, m, v):
        import torch

        from oracle import oracle as O
        from test_binning_chunks import _tile_rects
        self.O, self.case, self.shard_plan, self.params, self.m, self.v = O, case, plan, params, m, v
        self.cam = case.ocam
        self.tx, self.ty = O.tiles(self.cam)
        self.p, self.bins, self.packed, self.fwd = case.oracle_forward()
        self.ls = O.loss_ssim(self.fwd["out_img"], case.gt, self.fwd["out_distortion"], 0.8, 0.0, 0.2)
        self.x0, self.x1, self.y0, self.y1, self.vis = _tile_rects(self.p, self.tx, self.ty)
        self.g0, self.g1 = plan.g_begin, plan.g_end
        self.slice_grads = torch.zeros((self.g1 - self.g0, sharding.GRAD_STRIDE))
        self.received = None

    def project(self):
        import torch
        counts = np.zeros((self.ty, self.tx), np.int64)
        starts = np.zeros(self.ty + 1, np.int64)
        ends = np.zeros(self.ty + 1, np.int64)
        for i in range(self.g0, self.g1):
            if self.vis[i]:
                counts[self.y0[i]:self.y1[i], self.x0[i]:self.x1[i]] += 1
                starts[self.y0[i]] += 1
                ends[self.y1[i]] += 1
        return torch.from_numpy(np.concatenate([counts.reshape(-1), starts, ends]).astype(np.int32))

    def plan(self, summaries):
        world, rank, tiles = self.shard_plan.world, self.shard_plan.rank, self.tx * self.ty
        sm = summaries.numpy().astype(np.int64)
        assert sm.shape == (world, tiles + 2 * (self.ty + 1))
        c = sm[:, :tiles].sum(0).reshape(self.ty, self.tx)
        work = route_row_work(c)
        self.bands = route_band_cuts(work, world)
        matrix = route_matrix(sm[:, tiles:tiles + self.ty + 1], sm[:, tiles + self.ty + 1:], self.bands, self.ty)
        self.dest = []
        for q in range(world):
            b0, b1 = self.bands[q], self.bands[q + 1]
            if b1 <= b0:
                self.dest.append(np.zeros(0, np.int64))
                continue
            lo, hi = max(0, b0 - 1), min(self.ty, b1 + 1)
            own = np.arange(self.g0, self.g1)
            hit = self.vis[own] & (self.y0[own] < hi) & (self.y1[own] > lo)
            self.dest.append(own[hit])
        send = [len(d) for d in self.dest]
        assert send == [int(x) for x in matrix[rank]], "the count matrix disagrees with the slice's destinations"
        return self.bands, send, [int(x) for x in matrix[:, rank]]

    def pack(self, n_items):
        import torch
        buf = torch.zeros((n_items, sharding.PAYLOAD_FLOATS))
        ids = np.concatenate(self.dest) if self.dest else np.zeros(0, np.int64)
        assert len(ids) == n_items
        buf[:, 0] = torch.from_numpy(ids.astype(np.float32))
        self.order = ids
        return buf

    def band(self, payload, n, band, parts):
        import torch
        O = self.O
        ids = payload[:n, 0].numpy().astype(np.int64)
        assert np.all(np.diff(ids) > 0), "received ids are not strictly increasing"
        row0, row1 = band
        lo, hi = max(0, row0 - 1), min(self.ty, row1 + 1)
        touch = np.nonzero(self.vis & (self.y0 < hi) & (self.y1 > lo))[0]
        np.testing.assert_array_equal(ids, touch if row1 > row0 else np.zeros(0, np.int64))
        n_all = self.case.cfg.n
        dimg = self.ls["dL_dout_img"].copy()
        dimg[: row0 * 16] = 0.0
        dimg[row1 * 16:] = 0.0
        rb = O.rasterize_backward(n_all, self.bins, self.packed, self.fwd, self.cam, self.case.bg, dimg)
        rec = np.concatenate([rb["dL_dtransMat"], rb["dL_dopacity"], rb["dL_dcolors"], rb["dL_dnormal3D"]], 1)
        has = np.nonzero(np.any(rec != 0.0, axis=1))[0]
        assert np.isin(has, ids).all(), "a Gaussian with a gradient in the band was not routed to it"
        own = slice(row0 * 16, min(row1 * 16, self.cam.height))
        l1 = 0.8 * np.abs(self.fwd["out_img"][own] - self.case.gt[own]).astype(np.float64).sum()
        parts[:] = torch.tensor([l1 / (3 * self.cam.width * self.cam.height), 0.0, 0.0], dtype=torch.float64)
        self.received = ids
        return torch.from_numpy(np.ascontiguousarray(rec[ids], np.float32))

    def give_back(self, records, n_items):
        assert records.shape[0] == n_items == len(self.order)
        for k, i in enumerate(self.order):
            self.slice_grads[i - self.g0] += records[k]

    def adam(self):
        O, sl = self.O, slice(self.g0, self.g1)
        rec = self.slice_grads.numpy()
        deg = self.case.degree
        prm = self.params
        pb = O.project_backward(prm[0][sl], prm[1][sl], prm[2][sl], self.cam, self.p["radii"][sl],
                                np.ascontiguousarray(rec[:, 0:9]), np.ascontiguousarray(rec[:, 13:16]),
                                np.ascontiguousarray(rec[:, 10:13]), deg, deg, prm[4][sl])
        grads = [pb["dL_dmean3D"], pb["dL_dscale"], pb["dL_dquat"], pb["dL_dfeatures_dc"], pb["dL_dfeatures_rest"],
                 np.ascontiguousarray(rec[:, 9:10])]
        bc1 = np.float32(1.0 - float(np.float32(0.9)))
        bc2 = np.float32(1.0 - float(np.float32(0.999)))
        for k in range(6):
            if prm[k].size == 0:
                continue
            pk = np.ascontiguousarray(prm[k][sl])
            mk, vk = np.ascontiguousarray(self.m[k][sl]), np.ascontiguousarray(self.v[k][sl])
            O.fused_adam(pk, grads[k], mk, vk, np.float32(O.LR_INIT[k]) / bc1, 0.9, 0.999, float(np.sqrt(bc2)), 1e-8)
            prm[k][sl] = pk


def _rank_main(rank, ws, port, out_path):
    import torch.distributed as dist

    import torch
    from _cases import Case
    from oracle import oracle as O
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    O.set_threads(2)
    case = Case("sh3_small")
    cam = case.ocam
    plan = sharding.ShardPlan(case.cfg.n, (cam.height + 15) // 16, ws, rank)
    params = [np.array(a, np.float32) for a in (case.scene.means, case.scene.scales, case.scene.quats,
                                                 case.scene.f_dc, case.scene.f_rest,
                                                 case.scene.opacities.reshape(-1, 1))]
    m = [np.zeros_like(a) for a in params]
    v = [np.zeros_like(a) for a in params]
    calls = _OracleRouteCalls(case, plan, params, m, v)
    parts = torch.zeros(3, dtype=torch.float64)
    bands = sharding.routed_step(dist, plan, calls, parts)
    sl = slice(plan.g_begin, plan.g_end)
    np.savez(out_path + f".{rank}.npz", *[p[sl] for p in params], parts=parts.numpy(), bands=np.array(bands),
             g_begin=plan.g_begin, g_end=plan.g_end, row0=plan.row0, row1=plan.row1)
    dist.destroy_process_group()


def _band_cost(w, b0, b1):
    ty = len(w)
    if b1 <= b0:
        return 0
    return ROW_TENTHS * sum(w[b0:b1]) + (HALO_TENTHS * w[b0 - 1] if b0 > 0 else 0) + \
        (HALO_TENTHS * w[b1] if b1 < ty else 0)


def test_route_band_cuts_minimise_the_largest_band_cost():
    """The cuts cover every row with ordered bands and reach the least
    possible largest band cost (brute force over every cut placement)."""
    import itertools
    import random
    rng = random.Random(1)
    for _ in range(300):
        ty, world = rng.randint(1, 9), rng.randint(1, 4)
        w = [rng.randint(1, 1000) for _ in range(ty)]
        c = route_band_cuts(w, world)
        assert len(c) == world + 1 and c[0] == 0 and c[-1] == ty
        assert all(c[i] <= c[i + 1] for i in range(world))
        got = max(_band_cost(w, c[i], c[i + 1]) for i in range(world))
        best = min(max(_band_cost(w, cc[i], cc[i + 1]) for i in range(world))
                   for cc in ([0, *m, ty] for m in itertools.combinations_with_replacement(range(ty + 1), world - 1)))
        assert got == best, (w, world, c, got, best)


def _check(ws, tmp_path):
    import torch.multiprocessing as mp

    from _cases import Case
    from oracle import oracle as O
    out = str(tmp_path / f"route{ws}")
    mp.start_processes(_rank_main, args=(ws, _free_port(), out), nprocs=ws, start_method="spawn")
    res = [np.load(out + f".{r}.npz") for r in range(ws)]
    case = Case("sh3_small")
    tr = O.OracleTrainer(case.scene.params(), case.degree)
    ref = tr.step(case.ocam, case.gt, case.bg)
    ref_params = [tr.means, tr.scales, tr.quats, tr.f_dc, tr.f_rest, tr.opac]
    for r in range(1, ws):
        np.testing.assert_array_equal(res[0]["bands"], res[r]["bands"])
    bands = res[0]["bands"]
    for r in range(ws):
        assert (int(res[r]["row0"]), int(res[r]["row1"])) == (bands[r], bands[r + 1])
    assert bands[0] == 0 and bands[-1] == (case.ocam.height + 15) // 16 and np.all(np.diff(bands) >= 0)
    assert sum(int(res[r]["g_end"]) - int(res[r]["g_begin"]) for r in range(ws)) == case.cfg.n
    for k in range(6):
        got = np.concatenate([res[r][f"arr_{k}"] for r in range(ws)])
        ok = np.isclose(got, ref_params[k], rtol=1e-5, atol=1e-7)
        # a gradient that is zero up to rounding (summed in another order across
        # bands) can flip the sign of Adam's first step
        assert ok.mean() > 0.9995, (k, ok.mean())
    l1_total = 0.8 * np.abs(ref["out_img"] - case.gt).astype(np.float64).sum() / ref["out_img"].size
    for r in range(ws):
        assert abs(res[r]["parts"][0] - l1_total) < 1e-9


def test_two_gloo_ranks_routed_equal_one_oracle_step(tmp_path):
    _check(2, tmp_path)


def test_three_gloo_ranks_routed_equal_one_oracle_step(tmp_path):
    _check(3, tmp_path)

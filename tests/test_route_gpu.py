"""The routed exchange's entry points (msplat_route_*) on one GPU, through the
C ABI.

A slice's summary must hold the oracle's uncapped tile counts of the slice
(summed over slices: the oracle's) and the histograms of its tile
rectangles' first and last rows; the bands must be the least-maximum-cost
cover over the row work (min(count, 2048) + 430 per tile; halo rows at
0.4) and the send and receive counts the count matrix restated from the
histograms; every projected Gaussian must be packed for exactly the ranks
whose band plus a one-tile-row halo its rectangle meets, in increasing id
order. A routed step of `world` ranks, emulated on one GPU by running the
ranks' calls one after another (the payloads and returned records are
handed over in device memory instead of an all-to-all), must equal the
single-GPU fused step: the bands are rasterised over exactly the Gaussians
that touch them, in the same order.
"""
import numpy as np
import pytest

from _cases import Case
from test_binning_chunks import _tile_rects
from test_routed_gloo import route_band_cuts, route_matrix, route_row_work

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

CAP = 2048
ROW_WORK_PER_TILE = 430
PAYLOAD = 32


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")


def _B():
    from msplat import _backend as B
    B.load()
    return B


def _slices(n, world):
    chunk = -(-n // world)
    return [(min(r * chunk, n), min((r + 1) * chunk, n)) for r in range(world)]


@pytest.mark.parametrize("name", ["sh3_small", "overflow", "thin", "sh1_odd", "dense"])
def test_route_summaries_bands_and_payloads(name):
    case = Case(name)
    B = _B()
    g = B.DeviceGaussians(*case.scene.params(), sh_degree=case.degree)
    cam = B.camera_from_oracle(case.ocam)
    n = case.cfg.n
    p, bins, _, _ = case.oracle_forward()
    tx, ty = (case.cfg.width + 15) // 16, (case.cfg.height + 15) // 16
    tiles = tx * ty
    L = B.route_summary_len(cam)
    assert L == tiles + 2 * (ty + 1)
    x0, x1, y0, y1, vis = _tile_rects(p, tx, ty)
    world = 3
    slices = _slices(n, world)
    summaries = torch.full((world, L), -7, dtype=torch.int32, device="cuda")
    for r, (a, b) in enumerate(slices):
        B.route_project(g, cam, case.degree, a, b, summaries[r])
        want = np.zeros((ty, tx), np.int64)
        sel = np.nonzero(vis[a:b])[0] + a
        for i in sel:
            want[y0[i]:y1[i], x0[i]:x1[i]] += 1
        got = summaries[r].cpu().numpy()
        np.testing.assert_array_equal(got[:tiles].reshape(ty, tx), want)
        np.testing.assert_array_equal(got[tiles:tiles + ty + 1], np.bincount(y0[sel], minlength=ty + 1))
        np.testing.assert_array_equal(got[tiles + ty + 1:], np.bincount(y1[sel], minlength=ty + 1))
    sm = summaries.cpu().numpy().astype(np.int64)
    np.testing.assert_array_equal(sm[:, :tiles].sum(0), bins["raw_counts"])
    work = route_row_work(bins["raw_counts"].reshape(ty, tx).astype(np.int64))
    want_bands = route_band_cuts(work, world)
    matrix = route_matrix(sm[:, tiles:tiles + ty + 1], sm[:, tiles + ty + 1:], want_bands, ty)
    for r, (a, b) in enumerate(slices):
        B.route_project(g, cam, case.degree, a, b, torch.zeros(L, dtype=torch.int32, device="cuda"))
        bands, send, recv = B.route_plan(summaries, cam, world, r)
        assert bands == want_bands
        assert send == [int(x) for x in matrix[r]] and recv == [int(x) for x in matrix[:, r]]
        buf = torch.full((sum(send), PAYLOAD), float("nan"), device="cuda")
        B.route_pack(buf)
        got = buf.cpu().numpy()
        ids = got[:, 31].view(np.int32)
        off = 0
        for q in range(world):
            b0, b1 = bands[q], bands[q + 1]
            own = np.arange(a, b)
            if b1 > b0:
                lo, hi = max(0, b0 - 1), min(ty, b1 + 1)
                want_ids = own[vis[a:b] & (y0[a:b] < hi) & (y1[a:b] > lo)]
            else:
                want_ids = np.zeros(0, np.int64)
            assert send[q] == len(want_ids)
            np.testing.assert_array_equal(ids[off:off + send[q]], want_ids)
            np.testing.assert_array_equal(got[off:off + send[q], 30], p["depths"][want_ids])
            off += send[q]


def _routed_step_one_gpu(B, case, g, cam, adam, gt, world):
    """One routed step of `world` ranks run one after another on this GPU;
    returns the summed (l1, ssim, distortion) parts and the bands."""
    n, deg = case.cfg.n, case.degree
    slices = _slices(n, world)
    L = B.route_summary_len(cam)
    summaries = torch.zeros((world, L), dtype=torch.int32, device="cuda")
    for r, (a, b) in enumerate(slices):
        B.route_project(g, cam, deg, a, b, summaries[r])

    def send(r):
        a, b = slices[r]
        B.route_project(g, cam, deg, a, b, torch.zeros(L, dtype=torch.int32, device="cuda"))
        bands, counts, _ = B.route_plan(summaries, cam, world, r)
        buf = torch.empty((sum(counts), PAYLOAD), device="cuda")
        B.route_pack(buf)
        return bands, counts, buf

    sent = [send(r) for r in range(world)]
    bands = sent[0][0]
    parts_sum = torch.zeros(3, dtype=torch.float64, device="cuda")
    back = [[None] * world for _ in range(world)]
    for q in range(world):
        segs = []
        for r in range(world):
            counts, buf = sent[r][1], sent[r][2]
            off = sum(counts[:q])
            segs.append(buf[off:off + counts[q]])
        recv = torch.cat(segs).contiguous()
        m = recv.shape[0]
        grads = torch.empty((max(m, 1), 16), device="cuda")
        parts = torch.zeros(3, dtype=torch.float64, device="cuda")
        B.route_band(cam, g.sh_degree, recv, m, (bands[q], bands[q + 1]), case.bg, gt, 0.8, 0.0, 0.2, grads, parts)
        parts_sum += parts
        off = 0
        for r in range(world):
            k = sent[r][1][q]
            back[r][q] = grads[off:off + k].clone()
            off += k
    adam.step += 1
    for r, (a, b) in enumerate(slices):
        _, counts, _ = send(r)  # restores the slice's projection and packing order
        ret = torch.cat(back[r]).contiguous()
        sg = torch.zeros((max(b - a, 1), 16), device="cuda")
        B.route_return(ret, ret.shape[0], sg)
        B.route_project_backward_adam(g, cam, deg, sg, adam)
    torch.cuda.synchronize()
    return parts_sum.cpu().numpy(), bands


@pytest.mark.parametrize("name,world", [("sh3_small", 1), ("sh3_small", 3), ("overflow", 2), ("sh1_odd", 4),
                                        ("sh3_small", 8)])
def test_routed_step_equals_fused_step(name, world):
    from msplat import sharding
    case = Case(name)
    B = _B()
    cam = B.camera_from_oracle(case.ocam)
    gt = torch.as_tensor(case.gt).cuda()
    g = B.DeviceGaussians(*case.scene.params(), sh_degree=case.degree)
    adam = B.AdamState(g)
    parts, bands = _routed_step_one_gpu(B, case, g, cam, adam, gt, world)
    assert bands[0] == 0 and bands[-1] == (case.cfg.height + 15) // 16
    g1 = B.DeviceGaussians(*case.scene.params(), sh_degree=case.degree)
    a1 = B.AdamState(g1)
    loss_dev = torch.zeros(1, device="cuda")
    B.train_step_fused(g1, cam, case.degree, case.bg, gt, 0.8, 0.0, 0.2, a1, loss_dev=loss_dev)
    got = [t.detach().cpu().numpy() for t in g.groups()]
    want = [t.detach().cpu().numpy() for t in g1.groups()]
    for k in range(6):
        if want[k].size == 0:
            continue
        frac = np.isclose(got[k], want[k], rtol=1e-5, atol=1e-7).mean()
        # Adam's first step moves by about +-lr whatever the gradient's size: a
        # gradient that is zero up to rounding (summed over bands in another
        # order) may flip sign
        assert frac > 0.999, (k, frac)
    loss = sharding.loss_from_parts(parts, 0.2, case.cfg.width, case.cfg.height)
    ref = float(loss_dev.cpu()[0])
    assert abs(loss - ref) <= 1e-4 * abs(ref), (loss, ref)

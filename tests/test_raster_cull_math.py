"""CPU check of the forward rasteriser's cull (the cull record written by the
projection, project.cu cull_record, and the per-warp block test,
rasterize.cu block_hit), restated with numpy: for every tile-list entry and
every 8x4 warp block of its tile, a block that holds a pixel whose falloff
min(rho3d, rho2d) is within the surfel's rejection bound rmax must pass the
test. The pixel side is evaluated in float32 as the rasteriser does; the
record is computed in float64 from the same closed forms and rounded to
float32, and the block test runs in float32. (The GPU tests check the same
property end to end: a skipped blending pair would break the bit-exact
image.)"""
import numpy as np
import pytest

from _cases import Case
from oracle import oracle as O

RHO_SCALE = 1.002   # kCullRhoScale
MARGIN = 0.25       # kCullMargin (pixels)
MAX_ASPECT = 1.0e4  # kCullMaxAspect
f32 = np.float32


def _cull_records(T, rmax):
    """(c0, c1) per entry: centre, factors s1, t1, s2, conditional minimisers
    and the squared disc radius, as cull_record computes them."""
    r = rmax.astype(np.float64) * float(f32(RHO_SCALE))
    Tu, Tv, Tw = (T[:, k].astype(np.float64) for k in range(3))
    m0 = np.cross(Tv, Tw)
    m1 = np.cross(Tw, Tu)
    w = np.stack([np.ones_like(r), np.ones_like(r), -r], 1)
    qa, qb, qc = (m0 * m0 * w).sum(1), (m0 * m1 * w).sum(1), (m1 * m1 * w).sum(1)
    det_t = (Tu * m0).sum(1)
    dd = r * (Tw[:, 0] ** 2 + Tw[:, 1] ** 2) - Tw[:, 2] ** 2
    det_a = det_t * det_t * -dd
    ok = (rmax > 0) & (dd < 0) & (det_t != 0) & (qa > 0) & ((qa + qc) ** 2 <= MAX_ASPECT ** 2 * det_a)
    with np.errstate(all="ignore"):
        cx = (r * (Tu[:, 0] * Tw[:, 0] + Tu[:, 1] * Tw[:, 1]) - Tu[:, 2] * Tw[:, 2]) / dd
        cy = (r * (Tv[:, 0] * Tw[:, 0] + Tv[:, 1] * Tw[:, 1]) - Tv[:, 2] * Tw[:, 2]) / dd
        sc = -dd / (r * det_t * det_t)
        s1 = np.sqrt(qa * sc)
        vals = [cx, cy, s1, qb * sc / s1, np.sqrt(det_a * sc / qa), -qb / qc, -qb / qa]
    vals = [np.where(ok, v, 0.0).astype(f32) for v in vals]
    rd = (np.sqrt(f32(0.5) * rmax * f32(RHO_SCALE)) + f32(MARGIN)).astype(f32)
    rd2 = np.where(rmax > 0, rd * rd, f32(-1)).astype(f32)
    return vals, rd2


def _block_hit(vals, rd2, mx, my, x0, x1, y0, y1):
    cx, cy, s1, t1, s2, kx, ky = vals
    ddx = np.maximum(f32(0), np.maximum(x0 - mx, mx - x1))
    ddy = np.maximum(f32(0), np.maximum(y0 - my, my - y1))
    lox, hix, loy, hiy = x0 - cx, x1 - cx, y0 - cy, y1 - cy
    dx = np.minimum(np.maximum(f32(0), lox), hix)
    dy = np.minimum(np.maximum(f32(0), loy), hiy)
    dy1 = np.minimum(np.maximum(kx * dx, loy), hiy)
    dx2 = np.minimum(np.maximum(ky * dy, lox), hix)
    h1, g1 = s1 * dx + t1 * dy1, s2 * dy1
    h2, g2 = s1 * dx2 + t1 * dy, s2 * dy
    q = np.minimum(h1 * h1 + g1 * g1, h2 * h2 + g2 * g2)
    return (rd2 >= 0) & ((q <= f32(1)) | (ddx * ddx + ddy * ddy <= rd2))


@pytest.mark.parametrize("name,cam_index", [("thin", 0), ("thin", 1), ("sh3_small", 0), ("sh1_odd", 0)])
def test_block_cull_never_skips_a_reachable_block(name, cam_index):
    case = Case(name, cam_index=cam_index)
    p, bins, packed, _ = case.oracle_forward()
    tx, _ = O.tiles(case.ocam)
    W, H = case.cfg.width, case.cfg.height
    tb = bins["tile_bins"]
    gid = bins["gaussian_ids"][: bins["kept"]]
    tile = np.repeat(np.arange(len(tb)), tb[:, 1] - tb[:, 0])
    T = p["transmats"][gid].reshape(-1, 3, 3).astype(f32)
    xy = p["xys"][gid].astype(f32)
    opac = packed["packed_normal_opac"][: bins["kept"], 3].astype(f32)
    with np.errstate(all="ignore"):
        rmax = np.where(opac > 0, f32(2) * np.log(f32(255) * opac).astype(f32) + f32(0.01), f32(-1)).astype(f32)
    vals, rd2 = _cull_records(T, rmax)
    hits = needed = missed = 0
    for warp in range(8):
        bx = ((tile % tx) * 16 + (warp & 1) * 8).astype(f32)
        by = ((tile // tx) * 16 + (warp >> 1) * 4).astype(f32)
        hit = _block_hit(vals, rd2, xy[:, 0], xy[:, 1], bx - f32(MARGIN), bx + f32(7 + MARGIN),
                         by - f32(MARGIN), by + f32(3 + MARGIN))
        need = np.zeros(len(gid), bool)
        for q in range(32):
            px, py = bx + f32(q & 7), by + f32(q >> 3)
            inside = (px < W) & (py < H)
            dxp, dyp = xy[:, 0] - px, xy[:, 1] - py
            rho2d = f32(2) * (dxp * dxp + dyp * dyp)
            k = [px * T[:, 2, j] - T[:, 0, j] for j in range(3)]
            l = [py * T[:, 2, j] - T[:, 1, j] for j in range(3)]
            pxx = k[1] * l[2] - k[2] * l[1]
            pyy = k[2] * l[0] - k[0] * l[2]
            pzz = k[0] * l[1] - k[1] * l[0]
            with np.errstate(all="ignore"):
                u, v = pxx / pzz, pyy / pzz
                rho3d = u * u + v * v
            rho = np.where(rho2d < rho3d, rho2d, rho3d)
            need |= inside & (pzz != 0) & (rho <= rmax)
        hits += int(hit.sum())
        needed += int(need.sum())
        missed += int((need & ~hit).sum())
    assert needed > 1000
    assert missed == 0, f"{missed} reachable blocks culled (of {needed})"
    # the test is tight: far fewer blocks pass than the tile lists hold
    assert hits < 1.5 * needed, (hits, needed)

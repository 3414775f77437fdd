"""Densification (Model::afterTrain, core/src/model.cpp:240-306; msplat_densify,
core/metal/msplat_metal.mm:1339-1594; kernels msplat_metal.metal:3231-3491).

CPU: the oracle's staged restatement against an independent numpy restatement
of the same stages, and the library's split samples against the oracle's.
GPU: msplat_densify_plan / msplat_densify_apply against the oracle, bit for bit.
"""
import math

import numpy as np
import pytest

from oracle import oracle as O

LOG_SIZE_FAC = float(np.float32(math.log(1.6)))


def _args(check_screen=1, check_huge=1, half_max_dim=256.0):
    return dict(grad_thresh=0.0002, size_thresh=0.01, screen_thresh=0.05, check_screen=check_screen,
                cull_alpha_thresh=0.1, cull_scale_thresh=0.5, cull_screen_size=0.15, check_huge=check_huge,
                half_max_dim=half_max_dim, log_size_fac=LOG_SIZE_FAC)


def _state(n, degree, seed=0):
    """Parameters, moments and statistics that exercise every branch: size
    splits, screen splits (which also duplicate), duplicates, faint and huge
    culls, and Gaussians never seen (vis_counts 0)."""
    rng = np.random.default_rng(seed)
    K = (degree + 1) ** 2 - 1
    means = rng.normal(0, 1, (n, 3)).astype(np.float32)
    scales = rng.uniform(np.log(0.002), np.log(0.8), (n, 2)).astype(np.float32)
    quats = rng.normal(0, 1, (n, 4)).astype(np.float32)
    f_dc = rng.normal(0, 0.5, (n, 3)).astype(np.float32)
    f_rest = rng.normal(0, 0.05, (n, K, 3)).astype(np.float32)
    opac = rng.normal(0, 2, (n, 1)).astype(np.float32)
    groups = [means, scales, quats, f_dc, f_rest, opac]
    m = [rng.normal(0, 1e-3, g.shape).astype(np.float32) for g in groups]
    v = [np.abs(rng.normal(0, 1e-6, g.shape)).astype(np.float32) for g in groups]
    vis = rng.integers(0, 4, n).astype(np.float32)
    grad = (rng.uniform(0, 3e-6, n) * np.maximum(vis, 1)).astype(np.float32)
    max2d = rng.uniform(0, 0.25, n).astype(np.float32)
    return groups, m, v, (grad, vis, max2d)


def _numpy_densify(groups, m, v, degree, stats, a, samples):
    """The reference's stages restated with numpy (float32 arithmetic)."""
    f32 = np.float32
    ex = np.vectorize(lambda x: f32(O.det_exp(float(x))), otypes=[np.float32])
    n = groups[0].shape[0]
    K = (degree + 1) ** 2 - 1
    widths = [3, 2, 4, 3, 3 * K, 1]
    grad, vis, max2d = stats
    P = [np.array(g, np.float32).reshape(n, w) for g, w in zip(groups, widths)]
    Mm = [np.array(x, np.float32).reshape(n, w) for x, w in zip(m, widths)]
    Vv = [np.array(x, np.float32).reshape(n, w) for x, w in zip(v, widths)]
    ms = np.fmax(ex(P[1][:, 0]), ex(P[1][:, 1]))
    seen = vis > 0
    avg = np.where(seen, (grad / np.where(seen, vis, f32(1))) * f32(a["half_max_dim"]), f32(0))
    high = seen & (avg > f32(a["grad_thresh"]))
    large = ms > f32(a["size_thresh"])
    split = large.copy()
    if a["check_screen"]:
        split |= max2d > f32(a["screen_thresh"])
    split &= high
    dup = (~large) & high
    S, D = int(split.sum()), int(dup.sum())
    lsf = f32(a["log_size_fac"])
    rows = [[P[g][i].copy() for i in range(n)] for g in range(6)]
    mom = [[Mm[g][i].copy() for i in range(n)] for g in range(6)]
    vel = [[Vv[g][i].copy() for i in range(n)] for g in range(6)]
    children = []
    for o, i in enumerate(np.nonzero(split)[0]):
        q = P[2][i].astype(np.float32)
        qlen = np.sqrt(q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3], dtype=np.float32)
        qw, qx, qy, qz = q[0] / qlen, q[1] / qlen, q[2] / qlen, q[3] / qlen
        sx, sy = ex(P[1][i, 0]), ex(P[1][i, 1])
        for k in range(2):
            r = samples[(o * 2 + k) * 3:(o * 2 + k) * 3 + 3]
            r0, r1, r2 = r[0] * sx, r[1] * sy, r[2] * f32(0)
            two, one = f32(2), f32(1)
            v0 = (one - two * (qy * qy + qz * qz)) * r0 + two * (qx * qy - qw * qz) * r1 + two * (qx * qz + qw * qy) * r2
            v1 = two * (qx * qy + qw * qz) * r0 + (one - two * (qx * qx + qz * qz)) * r1 + two * (qy * qz - qw * qx) * r2
            v2 = two * (qx * qz - qw * qy) * r0 + two * (qy * qz + qw * qx) * r1 + (one - two * (qx * qx + qy * qy)) * r2
            child = [P[0][i] + np.array([v0, v1, v2], np.float32), P[1][i] - lsf] + [P[g][i].copy() for g in (2, 3, 4, 5)]
            children.append(child)
        rows[1][i] = P[1][i] - lsf  # the parent shrinks before duplicates copy it
    dups = [[rows[g][i].copy() for g in range(6)] for i in np.nonzero(dup)[0]]
    grown = [[rows[g][i] for g in range(6)] for i in range(n)] + children + dups
    zeros = [np.zeros(w, np.float32) for w in widths]
    grown_m = [[mom[g][i] for g in range(6)] for i in range(n)] + [zeros] * (2 * S + D)
    grown_v = [[vel[g][i] for g in range(6)] for i in range(n)] + [zeros] * (2 * S + D)
    keep = []
    for idx, row in enumerate(grown):
        sig = f32(1) / (f32(1) + ex(-row[5][0]))
        cull = sig < f32(a["cull_alpha_thresh"])
        if idx < n and split[idx]:
            cull = True
        if a["check_huge"]:
            if np.fmax(ex(row[1][0]), ex(row[1][1])) > f32(a["cull_scale_thresh"]):
                cull = True
            if a["check_screen"] and idx < n and max2d[idx] > f32(a["cull_screen_size"]):
                cull = True
        keep.append(not cull)
    sel = [i for i, k in enumerate(keep) if k]

    def stack(rowsets):
        return [np.stack([rowsets[i][g] for i in sel]) if sel else np.zeros((0, widths[g]), np.float32)
                for g in range(6)]
    return stack(grown), stack(grown_m), stack(grown_v), S, D


@pytest.mark.parametrize("degree", [3, 0])
def test_oracle_densify_matches_numpy_restatement(degree):
    n = 400
    groups, m, v, stats = _state(n, degree, seed=degree)
    a = _args()
    samples = O.normal_samples(600, 6 * n)
    got = O.densify(groups, m, v, degree, stats, a, samples)
    want = _numpy_densify(groups, m, v, degree, stats, a, samples)
    assert got[3] == want[3] and got[4] == want[4]
    assert got[3] > 5 and got[4] > 5, "the case must exercise splits and duplicates"
    assert got[0][0].shape[0] not in (0, n)
    for k in range(3):
        for g in range(6):
            if got[k][g].size == 0 and want[k][g].size == 0:
                continue
            np.testing.assert_array_equal(got[k][g], want[k][g].reshape(got[k][g].shape))


def test_split_and_duplicate_of_one_gaussian_copies_the_shrunk_parent():
    """A small Gaussian that is large on screen both splits and duplicates; the
    duplicate carries the parent's shrunk scale (the split kernel runs first)."""
    groups, m, v, stats = _state(3, 0, seed=5)
    groups[1][:] = np.log(0.005)            # small: not is_large
    groups[5][:] = 2.0                      # opaque: never culled as faint
    stats = (np.full(3, 1.0, np.float32), np.ones(3, np.float32), np.array([0.1, 0.0, 0.0], np.float32))
    a = _args(check_screen=1, check_huge=0)
    out = O.densify(groups, m, v, 0, stats, a, O.normal_samples(1, 18))
    assert out[3] == 1 and out[4] == 3
    # survivors: originals 1, 2; children of 0; duplicates of 0, 1, 2
    assert out[0][0].shape[0] == 2 + 2 + 3
    np.testing.assert_array_equal(out[0][1][4], (groups[1][0] - np.float32(LOG_SIZE_FAC)))
    np.testing.assert_array_equal(out[0][1][5], groups[1][1])


def test_library_split_samples_match_the_oracle():
    from msplat import _backend as B
    np.testing.assert_array_equal(B.normal_samples(1200, 999), O.normal_samples(1200, 999))


def _device_state(groups, m, v, degree):
    import torch
    from msplat import _backend as B
    g = B.DeviceGaussians(*[np.asarray(x) for x in (groups[0], groups[1], groups[2], groups[5].reshape(-1),
                                                     groups[3], groups[4])], sh_degree=degree)
    adam = B.AdamState(g)
    order = [0, 1, 2, 3, 4, 5]
    for k in order:
        adam.m[k].copy_(torch.from_numpy(np.asarray(m[k], np.float32).reshape(adam.m[k].shape)))
        adam.v[k].copy_(torch.from_numpy(np.asarray(v[k], np.float32).reshape(adam.v[k].shape)))
    return g, adam


@pytest.mark.gpu
@pytest.mark.parametrize("degree,check_huge", [(3, 1), (0, 1), (3, 0)])
def test_gpu_densify_matches_oracle(degree, check_huge):
    import torch
    from msplat import _backend as B
    n = 5000
    groups, m, v, stats = _state(n, degree, seed=10 + degree)
    a = _args(check_huge=check_huge)
    g, adam = _device_state(groups, m, v, degree)
    dstats = [torch.from_numpy(s).cuda() for s in stats]
    seed = 700
    new_g, new_adam, plan = B.densify(g, adam, dstats, a, seed)
    torch.cuda.synchronize()
    want = O.densify(groups, m, v, degree, stats, a, O.normal_samples(seed, 6 * n))
    assert plan["num_splits"] == want[3] and plan["num_dups"] == want[4]
    assert plan["new_count"] == want[0][0].shape[0]
    got_groups = [t.cpu().numpy() for t in new_g.groups()]
    for k in range(6):
        np.testing.assert_array_equal(got_groups[k].reshape(want[0][k].shape), want[0][k])
        np.testing.assert_array_equal(new_adam.m[k].cpu().numpy().reshape(want[1][k].shape), want[1][k])
        np.testing.assert_array_equal(new_adam.v[k].cpu().numpy().reshape(want[2][k].shape), want[2][k])


@pytest.mark.gpu
def test_gpu_densify_without_candidates_keeps_everything_in_order():
    import torch
    from msplat import _backend as B
    n = 3000
    groups, m, v, stats = _state(n, 1, seed=3)
    groups[5][:] = 3.0  # nothing faint
    groups[1][:] = np.log(0.05)  # nothing huge
    zero = (np.zeros(n, np.float32), np.zeros(n, np.float32), np.zeros(n, np.float32))
    g, adam = _device_state(groups, m, v, 1)
    new_g, new_adam, plan = B.densify(g, adam, [torch.from_numpy(s).cuda() for s in zero], _args(), 1)
    assert plan == {"num_splits": 0, "num_dups": 0, "new_count": n}
    for a_, b_ in zip(new_g.groups(), g.groups()):
        assert torch.equal(a_, b_)


@pytest.mark.gpu
def test_gpu_reset_opacity_clamps_and_zeroes_moments():
    import torch
    from msplat import _backend as B
    op = torch.tensor([-3.0, -1.0, 0.5, 4.0], device="cuda")
    mm = torch.ones(4, device="cuda")
    vv = torch.ones(4, device="cuda")
    limit = -1.3862943611198906
    B.reset_opacity(op, mm, vv, limit)
    torch.cuda.synchronize()
    assert op.cpu().tolist() == pytest.approx([-3.0, limit, limit, limit])
    assert float(mm.abs().sum()) == 0.0 and float(vv.abs().sum()) == 0.0

"""Camera setup (Model::prepareCam, core/src/model.cpp:500-544) through the
library's C ABI (msplat_prepare_camera, host code) equals the checker's
restatement bit for bit on every ring camera of the five workload
configurations, so that GPU parity tests may build their cameras either way."""
import numpy as np
import pytest

from msplat import synthetic as S
from oracle import oracle as O


def _fields(c):
    return (np.array(c.viewmat[:], np.float32), np.array(c.projmat[:], np.float32),
            np.array([c.fx, c.fy, c.cx, c.cy], np.float32), np.array(c.cam_pos[:], np.float32),
            (c.width, c.height))


@pytest.mark.parametrize("cfg_id", sorted(S.CONFIGS))
def test_prepare_camera_bit_exact_on_ring_cameras(cfg_id):
    from msplat import _backend as B
    cfg = S.CONFIGS[cfg_id]
    fx, fy, cx, cy = cfg.focal, cfg.focal, cfg.width / 2.0, cfg.height / 2.0
    # 32 ring cameras for every configuration (config 3's count), not only the
    # ones a configuration trains with
    for m in S.ring_cameras(32):
        got = _fields(B.prepare_camera(m, fx, fy, cx, cy, cfg.width, cfg.height))
        want = _fields(O.prepare_cam(m, fx, fy, cx, cy, cfg.width, cfg.height))
        for g, w in zip(got[:4], want[:4]):
            assert np.array_equal(g.view(np.uint32), w.view(np.uint32))
        assert got[4] == want[4]


def test_oracle_tile_helpers_match_full_binning():
    """The count-only and per-tile helpers the config-4 parity test uses give
    the same raw counts and kept ids as the full binning on a case with
    overfull tiles."""
    from _cases import Case
    case = Case("overflow")
    p = O.project_forward(*case.scene.params(), case.degree, case.degree, case.ocam)
    bins = O.bin_and_sort(p, case.ocam)
    raw = O.tile_counts(p, case.ocam)
    assert np.array_equal(raw, bins["raw_counts"])
    over = np.flatnonzero(raw > 2048)
    assert over.size > 0
    pick = np.concatenate([over[:6], np.flatnonzero((raw > 0) & (raw <= 2048))[:4]])
    kept = O.tile_kept_ids(p, case.ocam, pick)
    tb = bins["tile_bins"]
    for t in pick:
        want = bins["gaussian_ids"][tb[t, 0]:tb[t, 1]]
        assert np.array_equal(kept[int(t)], want)

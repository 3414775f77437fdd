"""The id-chunk rule of the binning (binning.cu k_tile_select, k_emit_keys):
intersections are counted per tile in 32 contiguous id chunks; a tile over
the 2048 cap emits only the chunks up to the first one at which its
cumulative count reaches 2048. That must never drop a kept intersection: the
oracle's kept ids of every overfull tile (its 2048 lowest ids) lie below the
tile's id bound, and the emitted set holds at least 2048 intersections.
Tile rectangles are restated from the projection (get_tile_bbox,
core/metal/msplat_metal.metal:77-92)."""
import numpy as np

from _cases import Case
from oracle import oracle as O

ID_CHUNKS = 32
CAP = 2048


def _tile_rects(p, tx, ty):
    f32 = np.float32
    tcx = p["xys"][:, 0].astype(f32) / f32(16)
    tcy = p["xys"][:, 1].astype(f32) / f32(16)
    tr = p["radii"].astype(f32) / f32(16)
    x0 = np.clip(np.trunc(tcx - tr).astype(np.int64), 0, tx)
    x1 = np.clip(np.trunc(tcx + tr + f32(1)).astype(np.int64), 0, tx)
    y0 = np.clip(np.trunc(tcy - tr).astype(np.int64), 0, ty)
    y1 = np.clip(np.trunc(tcy + tr + f32(1)).astype(np.int64), 0, ty)
    vis = (p["radii"] > 0) & (x1 > x0) & (y1 > y0)
    return x0, x1, y0, y1, vis


def test_overfull_tiles_keep_only_ids_from_emitted_chunks():
    case = Case("overflow")
    p, bins, _, _ = case.oracle_forward()
    tx, ty = O.tiles(case.ocam)
    n = case.cfg.n
    id_chunk = max(1, -(-n // ID_CHUNKS))
    x0, x1, y0, y1, vis = _tile_rects(p, tx, ty)
    counts = np.zeros((ID_CHUNKS, ty, tx), np.int64)
    for i in np.nonzero(vis)[0]:
        counts[i // id_chunk, y0[i]:y1[i], x0[i]:x1[i]] += 1
    counts = counts.reshape(ID_CHUNKS, -1)
    raw = counts.sum(0)
    np.testing.assert_array_equal(raw, bins["raw_counts"])
    over = np.nonzero(raw > CAP)[0]
    assert len(over) >= 5
    cum = np.cumsum(counts, 0)
    for t in over:
        cut = int(np.argmax(cum[:, t] >= CAP))
        limit = (cut + 1) * id_chunk
        assert cum[cut, t] >= CAP
        s, e = bins["tile_bins"][t]
        kept = bins["gaussian_ids"][s:e]
        assert e - s == CAP and kept.max() < limit

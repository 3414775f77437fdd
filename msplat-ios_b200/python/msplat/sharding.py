"""Tile-row sharding of the training step across GPUs (one process per GPU).

Every rank holds the full parameter set and projects all Gaussians; rank r
bins, sorts and rasterises the tile rows [row0, row1) (plus a one-tile-row
halo that the 11x11 SSIM window needs: 16 px >= the 10 px forward+backward
reach), evaluates the loss and the backward on its own rows, and leaves
per-Gaussian raster-space gradient records [N, 16]. Those are summed across
ranks with one reduce-scatter, so that rank r receives the records of the
Gaussian slice [g_begin, g_end); it runs the projection VJP and Adam on that
slice, and the six parameter groups are all-gathered in place. Adam moments
stay sharded (each rank only touches its slice). The three loss partial sums
(l1, ssim, distortion) are all-reduced for reporting.

The exchange is written once (`sharded_step`) over two callables, so the same
collective sequence runs with NCCL on GPUs (the C ABI does the compute) and
with gloo on CPU in the tests (the oracle does the compute).
"""
from __future__ import annotations

import dataclasses

GRAD_STRIDE = 16  # floats per Gaussian in the raster-gradient record


@dataclasses.dataclass
class ShardPlan:
    """Tile rows and the Gaussian slice owned by `rank` of `world` ranks.

    Tile rows are split into equal contiguous bands. The Gaussian index range
    is padded to world * chunk (chunk a multiple of 256) so that the
    reduce-scatter and all-gather move equal-sized pieces.
    """
    n: int
    tiles_y: int
    world: int
    rank: int

    def __post_init__(self):
        if not (0 <= self.rank < self.world):
            raise ValueError("rank out of range")
        rows = -(-self.tiles_y // self.world)
        self.row0 = min(self.rank * rows, self.tiles_y)
        self.row1 = min((self.rank + 1) * rows, self.tiles_y)
        chunk = -(-self.n // self.world)
        self.chunk = -(-chunk // 256) * 256
        self.padded = self.chunk * self.world
        self.g_begin = min(self.rank * self.chunk, self.n)
        self.g_end = min((self.rank + 1) * self.chunk, self.n)

    def slice_rows(self):
        """Rows of a [padded, ...] buffer that this rank contributes to all-gathers."""
        return slice(self.rank * self.chunk, (self.rank + 1) * self.chunk)


def pad_gaussians(g, padded: int):
    """Re-home each parameter group of a DeviceGaussians in a [padded, ...]
    buffer (rows >= n stay zero) so that all-gathers can run in place; g keeps
    contiguous [n] views for the compute."""
    import torch
    n = g.n
    g.full = []
    for name in ("means", "scales", "quats", "f_dc", "f_rest", "opacities"):
        t = getattr(g, name)
        full = torch.zeros((padded,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        full[:n].copy_(t)
        setattr(g, name, full[:n])
        g.full.append(full)
    return g


COLOR_GROUPS = (3, 4)  # features_dc, features_rest in Model group order


class PeerParams:
    """The parameter groups of a DeviceGaussians re-homed in [padded, ...]
    buffers that every rank maps through CUDA IPC (msplat_ipc_*): rank q
    owns and updates rows [q * chunk, (q + 1) * chunk) of its own buffers;
    the geometry groups are still all-gathered (every rank projects every
    Gaussian), but the colour groups are read from their owner after binning
    for just the Gaussians of the rank's band, so they are never gathered. `struct` is the MsplatPeerParams view;
    when any rank cannot map its peers, `ok` is False on every rank and the
    buffers remain usable as the [padded, ...] buffers of the NCCL
    all-gather exchange (g.full). close() must run on every rank (it
    synchronises and barriers before unmapping and freeing)."""

    def __init__(self, B, dist, plan: ShardPlan, g):
        import torch
        if plan.world > B.MAX_PEER_RANKS:
            raise ValueError("too many ranks for the peer view")
        self.B, self.dist = B, dist
        self.own, self.mapped = [], []
        n, dev = g.n, g.means.device
        names = ("means", "scales", "quats", "f_dc", "f_rest", "opacities")
        g.full = []
        for name in names:
            t = getattr(g, name)
            shape = (plan.padded,) + tuple(t.shape[1:])
            row = 1
            for d in t.shape[1:]:
                row *= int(d)
            ptr = B.device_alloc(plan.padded * max(row, 1) * 4)
            self.own.append(ptr)
            full = torch.as_tensor(B.DeviceArray(ptr, shape), device=dev)
            full[:n].copy_(t)
            setattr(g, name, full[:n])
            g.full.append(full)
        torch.cuda.synchronize()
        handles = [B.ipc_handle(p) for p in self.own]
        everyone = [None] * plan.world
        dist.all_gather_object(everyone, handles)
        st = B.MsplatPeerParams()
        st.world, st.chunk = plan.world, plan.chunk
        self.error = ""
        try:
            for q in range(plan.world):
                for k in range(6):
                    if q == plan.rank:
                        ptr = self.own[k]
                    else:
                        ptr = B.ipc_open(everyone[q][k])
                        self.mapped.append(ptr)
                    st.base[k][q] = ptr
        except Exception as e:  # e.g. no peer access between these GPUs
            self.error = str(e)
        # every rank must agree before anyone reads a peer buffer
        ok = torch.tensor([0 if self.error else 1], device=dev, dtype=torch.int32)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        self.ok = bool(ok.item())
        if not self.ok:
            for p in self.mapped:
                B.ipc_close(p)
            self.mapped = []
            self.error = self.error or "a peer could not map this rank's buffers"
        self.struct = st if self.ok else None
        dist.barrier()

    def close(self):
        import torch
        torch.cuda.synchronize()
        self.dist.barrier()  # no rank reads a peer buffer any more
        for p in self.mapped:
            self.B.ipc_close(p)
        self.mapped = []
        self.dist.barrier()  # no rank maps this rank's buffers any more
        for p in self.own:
            self.B.device_free(p)
        self.own = []


def sharded_step(dist, plan: ShardPlan, forward_backward, project_adam, rg, rg_shard, param_fulls, parts,
                 side_stream=None, skip_color=False, colors_next=None, rgb_full=None, marks=None):
    """One training step across ranks.

    forward_backward(plan, rg, parts): fills rg [padded, 16] with this rank's
        raster gradients (rows >= n zero) and parts [3] with its loss sums; it
        may rebalance plan.row0/plan.row1.
    project_adam(g_begin, g_end, rg_shard): projection VJP + Adam on the slice,
        rg_shard [chunk, 16] holding the summed records of Gaussians
        g_begin .. g_end - 1 in its first rows.
    param_fulls: the [padded, ...] parameter buffers to all-gather in place.
    side_stream: with a CUDA stream, the colour groups (features_dc,
        features_rest: 48 of the 58 floats per Gaussian) are gathered on it
        after everything else, and the returned event marks their arrival;
        the next step's forward_backward binds the geometry while the
        transfer runs and waits for the event only before its colour pass.
    skip_color: the colour groups are not gathered at all (the ranks read
        them from their owners, PeerParams, or exchange colours instead,
        below); the geometry all-gather and the loss all-reduce after Adam
        order every owner's update before the next step's reads.
    colors_next(g_begin, g_end), rgb_full [padded, 3]: colour exchange. After
        Adam the owner writes the clamped colours of its slice for the next
        step's camera into rgb_full (msplat_shard_colors); rgb_full is
        all-gathered on side_stream (12 B per Gaussian instead of the 192 B of
        colour coefficients) and the returned event marks its arrival. Use
        with skip_color=True.
    marks(name): optional, called on the host after each phase is enqueued
        ("forward_backward", "reduce_scatter", "project_adam", "all_gather",
        "all_reduce"), e.g. to record CUDA events between the phases.
    Every rank issues the collectives in the same order.
    """
    mark = marks if marks is not None else (lambda name: None)
    forward_backward(plan, rg, parts)
    mark("forward_backward")
    dist.reduce_scatter_tensor(rg_shard, rg, op=dist.ReduceOp.SUM)
    mark("reduce_scatter")
    project_adam(plan.g_begin, plan.g_end, rg_shard)
    rows = plan.slice_rows()
    if colors_next is not None:
        colors_next(plan.g_begin, plan.g_end)
    mark("project_adam")
    late = [rgb_full] if rgb_full is not None else []
    for k, full in enumerate(param_fulls):
        if full.numel() == 0 or (skip_color and k in COLOR_GROUPS):
            continue
        if side_stream is not None and k in COLOR_GROUPS:
            late.append(full)
            continue
        dist.all_gather_into_tensor(full, full[rows])
    mark("all_gather")
    dist.all_reduce(parts)
    mark("all_reduce")
    if not late:
        return None
    if side_stream is None:
        for full in late:
            dist.all_gather_into_tensor(full, full[rows])
        return None
    import torch
    adam_done = torch.cuda.Event()
    adam_done.record()
    side_stream.wait_event(adam_done)
    ready = torch.cuda.Event()
    with torch.cuda.stream(side_stream):
        for full in late:
            dist.all_gather_into_tensor(full, full[rows])
        ready.record(side_stream)
    return ready


def loss_from_parts(parts, lambda_dssim: float, width: int, height: int) -> float:
    """Loss of the whole image from the all-reduced (l1, ssim, distortion) sums."""
    l1, ssim, dist_term = (float(x) for x in parts)
    inv_num = 1.0 / (3.0 * width * height)
    return l1 + dist_term + lambda_dssim * (1.0 - ssim * inv_num)


def gpu_step_fns(B, g, cam, degree, bg, gt, lambda_l1, lambda_dist, lambda_dssim, adam, stats, balance=True,
                 features_ready=None, split_color=False, peers=None, rgb=None):
    """The two callables of sharded_step bound to the C ABI (msplat_shard_*).
    With balance the library picks work-balanced tile-row bands each step;
    with split_color the colour pass waits for features_ready (the event the
    previous sharded_step returned); with peers (a PeerParams) the projection
    reads every Gaussian from its owner rank; with rgb ([padded, 3], gathered
    colours for this camera) the colour pass copies them, after
    features_ready."""
    def forward_backward(plan, rg, parts):
        if rgb is not None:
            kw = dict(world=plan.world, rank=plan.rank) if balance else dict(rows=(plan.row0, plan.row1))
            plan.row0, plan.row1 = B.shard_forward_backward_rgb(g, cam, degree, bg, gt, lambda_l1, lambda_dist,
                                                                lambda_dssim, rg, parts, rgb, rgb_ready=features_ready,
                                                                **kw)
            return
        if peers is not None:
            plan.row0, plan.row1 = B.shard_forward_backward_peers(g, peers.struct, cam, degree, bg, gt, lambda_l1,
                                                                  lambda_dist, lambda_dssim, rg, parts,
                                                                  world=plan.world, rank=plan.rank)
            return
        kw = dict(features_ready=features_ready, split_color=split_color)
        if balance:
            plan.row0, plan.row1 = B.shard_forward_backward(g, cam, degree, bg, gt, lambda_l1, lambda_dist,
                                                            lambda_dssim, rg, parts, world=plan.world, rank=plan.rank,
                                                            **kw)
        else:
            B.shard_forward_backward(g, cam, degree, bg, gt, lambda_l1, lambda_dist, lambda_dssim, rg, parts,
                                     rows=(plan.row0, plan.row1), **kw)

    def project_adam(g0, g1, rg_shard):
        # the kernel indexes records by global Gaussian id: offset the base
        B.shard_project_backward_adam(g, cam, degree, rg_shard.data_ptr() - g0 * GRAD_STRIDE * 4, g0, g1, adam,
                                      stats=stats, count_step=False)

    return forward_backward, project_adam


def colors_fn(B, g, cam_next, degree, rgb_full):
    """The colors_next callable of sharded_step: the clamped colours of the
    owner's slice for the next step's camera (msplat_shard_colors)."""
    def colors_next(g0, g1):
        B.shard_colors(g, cam_next, degree, g0, g1, rgb_full)
    return colors_next


# ---------------------------------------------------------------- routed exchange
PAYLOAD_FLOATS = 32  # 128 bytes per routed Gaussian


def routed_step(dist, plan: ShardPlan, calls, parts, marks=None, between=None):
    """One training step with the routed exchange (msplat_route_*): each rank
    projects only its own Gaussians and sends each projected Gaussian to the
    ranks whose tile-row band (plus a one-row halo) it touches; every rank
    rasterises its band over what it received and sends the per-Gaussian
    gradient records back to their owners, which run the projection VJP and
    Adam on their slice. Nothing is gathered: each rank reads only its own
    slice of the parameters.

    calls (objects with these methods; bound to the C ABI by gpu_route_calls,
    or to a CPU stand-in in the tests):
      project()                  -> the slice's summary (int32 tensor [L]):
                                    per-tile intersection counts and the
                                    histograms of its rectangles' first and
                                    last tile rows
      plan(summaries)            -> (bands [world + 1], items sent to each
                                    rank [world], items received from each
                                    rank [world]) from all ranks' summaries
                                    ([world, L], rank order)
      pack(n_items)              -> payload tensor [n_items, 32] grouped by
                                    destination, increasing id per group
      band(payload, n, band, parts) -> raster-gradient records [n, 16] of the
                                    received Gaussians; parts [3] loss sums
      give_back(records, n_items) -> adds the returned records per own
                                    Gaussian (packing order)
      adam()                     -> projection VJP + Adam on the slice
    between(): optional, called on every rank after the payloads are
    exchanged and before the band is enqueued (e.g. to enqueue a collective
    that should run under the band's compute).
    Returns the bands. Every rank issues the collectives in the same order:
    one all-gather of the summaries, two all-to-alls (or two one-element
    all-reduces with peer stores), one all-reduce.
    """
    import torch
    mark = marks if marks is not None else (lambda name: None)
    peers = getattr(calls, "peers", None)
    summary = calls.project()
    gathered = torch.empty((plan.world, summary.numel()), dtype=summary.dtype, device=summary.device)
    if dist.get_backend() == "nccl":
        dist.all_gather_into_tensor(gathered, summary)
    else:  # gloo has no all_gather_into_tensor
        dist.all_gather(list(gathered.unbind(0)), summary)
    bands, send_counts, recv_counts = calls.plan(gathered)
    mark("project_plan")
    n_send, n_recv = sum(send_counts), sum(recv_counts)
    if peers is not None:
        # payloads stored straight into the destinations' inboxes; a
        # one-element all-reduce orders every rank's pack before any band
        calls.pack_peers()
        dist.all_reduce(peers.fence)
        recv_buf = peers.inbox_view(n_recv)
    else:
        send_buf = calls.pack(n_send)
        recv_buf = torch.empty((n_recv, PAYLOAD_FLOATS), dtype=send_buf.dtype, device=send_buf.device)
        dist.all_to_all_single(recv_buf, send_buf, output_split_sizes=recv_counts, input_split_sizes=send_counts)
    mark("route")
    if between is not None:
        between()
    grads = calls.band(recv_buf, n_recv, (bands[plan.rank], bands[plan.rank + 1]), parts)
    mark("band")
    if peers is not None:
        calls.push(grads[:n_recv])
        dist.all_reduce(peers.fence)
        back = peers.returnbox_view(n_send)
    else:
        back = torch.empty((n_send, GRAD_STRIDE), dtype=grads.dtype, device=grads.device)
        dist.all_to_all_single(back, grads[:n_recv], output_split_sizes=send_counts, input_split_sizes=recv_counts)
    mark("return")
    calls.give_back(back, n_send)
    calls.adam()
    mark("project_adam")
    dist.all_reduce(parts)
    mark("all_reduce")
    plan.row0, plan.row1 = bands[plan.rank], bands[plan.rank + 1]
    return bands


class RoutePeers:
    """Inboxes and return boxes of the routed exchange that every rank maps
    through CUDA IPC (msplat_route_pack_peers / msplat_route_push_peers).
    Rank q's inbox holds up to n_total 128-byte payloads (a band receives a
    Gaussian at most once); its return box up to world * chunk 64-byte
    records (each own Gaussian goes to at most every band). When any rank
    cannot map its peers, `ok` is False on every rank and routed_step keeps
    the NCCL all-to-alls. close() must run on every rank."""

    def __init__(self, B, dist, plan: ShardPlan, n_total: int, device):
        import torch
        if plan.world > B.MAX_PEER_RANKS:
            raise ValueError("too many ranks for the peer view")
        self.B, self.dist = B, dist
        self.inbox_items = max(int(n_total), 1)
        self.returnbox_items = max(plan.chunk * plan.world, 1)
        self.own = [B.device_alloc(self.inbox_items * PAYLOAD_FLOATS * 4),
                    B.device_alloc(self.returnbox_items * GRAD_STRIDE * 4)]
        self.mapped = []
        self.inbox = torch.as_tensor(B.DeviceArray(self.own[0], (self.inbox_items, PAYLOAD_FLOATS)), device=device)
        self.returnbox = torch.as_tensor(B.DeviceArray(self.own[1], (self.returnbox_items, GRAD_STRIDE)),
                                         device=device)
        self.fence = torch.zeros(1, dtype=torch.int32, device=device)
        torch.cuda.synchronize()
        handles = [B.ipc_handle(p) for p in self.own]
        everyone = [None] * plan.world
        dist.all_gather_object(everyone, handles)
        st = B.MsplatRoutePeers()
        st.world, st.rank = plan.world, plan.rank
        st.inbox_items, st.returnbox_items = self.inbox_items, self.returnbox_items
        self.error = ""
        try:
            for q in range(plan.world):
                for k, field in enumerate((st.inbox, st.returnbox)):
                    if q == plan.rank:
                        ptr = self.own[k]
                    else:
                        ptr = B.ipc_open(everyone[q][k])
                        self.mapped.append(ptr)
                    field[q] = ptr
        except Exception as e:  # e.g. no peer access between these GPUs
            self.error = str(e)
        ok = torch.tensor([0 if self.error else 1], device=device, dtype=torch.int32)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        self.ok = bool(ok.item())
        if not self.ok:
            for p in self.mapped:
                B.ipc_close(p)
            self.mapped = []
            self.error = self.error or "a peer could not map this rank's boxes"
        self.struct = st if self.ok else None
        dist.barrier()

    def inbox_view(self, n):
        return self.inbox[:n]

    def returnbox_view(self, n):
        return self.returnbox[:n]

    def close(self):
        import torch
        torch.cuda.synchronize()
        self.dist.barrier()  # no rank writes into a peer box any more
        for p in self.mapped:
            self.B.ipc_close(p)
        self.mapped = []
        self.dist.barrier()  # no rank maps this rank's boxes any more
        self.inbox = self.returnbox = None
        for p in self.own:
            self.B.device_free(p)
        self.own = []


class gpu_route_calls:
    """The callables of routed_step bound to the C ABI (msplat_route_*);
    with `peers` (a RoutePeers whose mapping succeeded) the payloads and the
    returned records move by peer stores instead of NCCL all-to-alls."""

    def __init__(self, B, g, cam, degree, bg, gt, lambda_l1, lambda_dist, lambda_dssim, adam_state, stats,
                 shard_plan, tiles=None, peers=None):
        import torch
        self.peers = peers if (peers is not None and peers.ok) else None
        self.B, self.g, self.cam, self.degree, self.bg, self.gt = B, g, cam, degree, bg, gt
        self.l1, self.ld, self.lds = lambda_l1, lambda_dist, lambda_dssim
        self.adam_state, self.stats, self.shard_plan = adam_state, stats, shard_plan
        dev = g.means.device
        self.dev = dev
        self.summary = torch.zeros(B.route_summary_len(cam), dtype=torch.int32, device=dev)
        self.slice_grads = torch.zeros((max(shard_plan.g_end - shard_plan.g_begin, 1), GRAD_STRIDE), device=dev)

    def project(self):
        p = self.shard_plan
        self.B.route_project(self.g, self.cam, self.degree, p.g_begin, p.g_end, self.summary)
        return self.summary

    def plan(self, summaries):
        return self.B.route_plan(summaries, self.cam, self.shard_plan.world, self.shard_plan.rank)

    def pack(self, n_items):
        import torch
        buf = torch.empty((n_items, PAYLOAD_FLOATS), device=self.dev)
        self.B.route_pack(buf)
        return buf

    def band(self, payload, n, band, parts):
        import torch
        grads = torch.empty((max(n, 1), GRAD_STRIDE), device=self.dev)
        self.B.route_band(self.cam, self.g.sh_degree, payload, n, band, self.bg, self.gt, self.l1, self.ld,
                          self.lds, grads, parts)
        return grads

    def pack_peers(self):
        self.B.route_pack_peers(self.peers.struct)

    def push(self, grads):
        self.B.route_push_peers(self.peers.struct, grads)

    def give_back(self, records, n_items):
        self.B.route_return(records, n_items, self.slice_grads)

    def adam(self):
        self.B.route_project_backward_adam(self.g, self.cam, self.degree, self.slice_grads, self.adam_state,
                                           stats=self.stats)

"""Z-slab partition of a voxel set over ranks, with a two-plane halo.

Multi-GPU runs of the residual stack (one process per GPU) split the voxels,
ordered by the packed ``(b, z, y, x)`` key, into contiguous z-slabs whose
boundaries balance each rank's work, owned + local rows (a thin surface
leaves most uniform z-slabs empty).  Submanifold convs and the per-voxel LayerNorm only reach
one z-plane across a slab boundary, so each rank holds, besides its own
voxels, the voxels of the two z-planes on either side that belong to its
neighbours:

    local rows = [owned (global order) | halo below | halo above]

Before every residual block each rank sends the two boundary z-planes of
its owned features to each neighbour and receives its halos (one exchange
per block).  A block then runs over all local rows: conv1 is exact on the
owned rows and on the inner halo plane (whose neighbours, the outer halo
plane and the owned rows, are local), so conv2 is exact on the owned rows;
outputs on halo rows are discarded by the next exchange.

The reference has no multi-node path (its refiner is single-process,
src/sparse.cpp:1110-1300); this layout is what the sparse executor needs to
shard the refiner's levels across the GPUs of one node.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

HALO_PLANES = 2


@dataclass
class SlabPart:
    """One rank's share.  Row indices refer to the globally sorted voxel array."""
    rank: int
    lo: int                      # owned rows [lo, hi)
    hi: int
    halo_lo: np.ndarray          # global rows of the halo below (owned by lower ranks), sorted
    halo_hi: np.ndarray          # global rows of the halo above (owned by higher ranks), sorted
    send_lo: int                 # my first send_lo owned rows are rank-1's halo_hi
    send_hi: int                 # my last send_hi owned rows are rank+1's halo_lo

    @property
    def n_owned(self) -> int:
        return self.hi - self.lo

    @property
    def n_local(self) -> int:
        return self.n_owned + len(self.halo_lo) + len(self.halo_hi)

    def local_rows(self) -> np.ndarray:
        """Global row of every local row: owned, then halo below, then above."""
        return np.concatenate([np.arange(self.lo, self.hi), self.halo_lo, self.halo_hi]).astype(np.int64)


def _planes(coords: np.ndarray):
    """(plane id per row, first row of each plane, (b, z) of each plane) for
    rows sorted by (b, z, y, x)."""
    bz = coords[:, 3].astype(np.int64) * (1 << 20) + coords[:, 2].astype(np.int64)
    starts = np.flatnonzero(np.r_[True, bz[1:] != bz[:-1]])
    pid = np.repeat(np.arange(len(starts)), np.diff(np.r_[starts, len(bz)]))
    return pid, starts, bz[starts]


def partition(coords: np.ndarray, nranks: int, halo: int = HALO_PLANES) -> list[SlabPart]:
    """Splits rows sorted by (b, z, y, x) into nranks z-slabs on plane
    boundaries, placed so that every rank's work (owned + local rows) is
    about equal (a thin surface leaves most uniform z-slabs empty, and a cut
    through large planes gives both sides large halos).  Every slab must span
    more than `halo` z-planes of one sample, so that a halo belongs to the
    adjacent rank only."""
    n = coords.shape[0]
    if nranks < 1:
        raise ValueError("nranks must be >= 1")
    if n > 1:
        keys = _sort_keys(coords)
        if not np.all(keys[1:] > keys[:-1]):
            raise ValueError("coords must be unique and sorted by the packed (b, z, y, x) key")
    pid, starts, pbz = _planes(coords)
    nplanes = len(starts)
    if nranks > 1 and nplanes < nranks * (halo + 1):
        raise ValueError(f"{nplanes} z-planes cannot give {nranks} slabs of more than {halo} planes")
    cuts = _balanced_cuts(starts, pbz, n, nranks, halo)
    if cuts is None:
        # plane cut points: first plane whose start row reaches the quantile
        cuts = [0]
        for r in range(1, nranks):
            target = n * r / nranks
            p = int(np.searchsorted(starts, target, side="left"))
            p = max(p, cuts[-1] + halo + 1)
            cuts.append(p)
        cuts.append(nplanes)
    for r in range(nranks):
        if cuts[r + 1] - cuts[r] <= halo:
            raise ValueError("slab too thin for the halo; use fewer ranks")
    bound = [int(starts[c]) if c < nplanes else n for c in cuts]
    b = pbz >> 20
    z = pbz & ((1 << 20) - 1)
    parts = []
    for r in range(nranks):
        p0, p1 = cuts[r], cuts[r + 1]
        lo, hi = bound[r], bound[r + 1]

        def planes_near(edge_plane: int, below: bool) -> np.ndarray:
            # planes of the same sample within `halo` z of the slab edge, outside it
            if below:
                cand = range(max(0, edge_plane - halo), edge_plane)
                zref = z[edge_plane]
                ok = [q for q in cand if b[q] == b[edge_plane] and zref - z[q] <= halo]
            else:
                cand = range(edge_plane + 1, min(nplanes, edge_plane + 1 + halo))
                zref = z[edge_plane]
                ok = [q for q in cand if b[q] == b[edge_plane] and z[q] - zref <= halo]
            if not ok:
                return np.zeros(0, dtype=np.int64)
            a0 = int(starts[min(ok)])
            a1 = int(starts[max(ok) + 1]) if max(ok) + 1 < nplanes else n
            return np.arange(a0, a1, dtype=np.int64)

        hl = planes_near(p0, True) if r > 0 else np.zeros(0, dtype=np.int64)
        hh = planes_near(p1 - 1, False) if r < nranks - 1 else np.zeros(0, dtype=np.int64)
        parts.append(SlabPart(r, lo, hi, hl, hh, 0, 0))
    for r in range(nranks):
        if r > 0:
            # rank r-1's halo above must be my first rows
            hh = parts[r - 1].halo_hi
            assert len(hh) == 0 or (hh[0] == parts[r].lo and hh[-1] < parts[r].hi)
            parts[r].send_lo = len(hh)
        if r < nranks - 1:
            hl = parts[r + 1].halo_lo
            assert len(hl) == 0 or (hl[-1] == parts[r].hi - 1 and hl[0] >= parts[r].lo)
            parts[r].send_hi = len(hl)
    return parts


def _cut_halos(starts: np.ndarray, pbz: np.ndarray, n: int, halo: int):
    """Halo rows a cut before plane c gives each side: below[c] = rows the
    upper rank copies from the planes under c, above[c] = rows the lower rank
    copies from plane c upwards (same sample, within `halo` z)."""
    nplanes = len(starts)
    sizes = np.diff(np.r_[starts, n]).astype(np.int64)
    b = pbz >> 20
    z = pbz & ((1 << 20) - 1)
    below = np.zeros(nplanes + 1, dtype=np.int64)
    above = np.zeros(nplanes + 1, dtype=np.int64)
    for c in range(1, nplanes):
        below[c] = sum(int(sizes[q]) for q in range(max(0, c - halo), c) if b[q] == b[c] and z[c] - z[q] <= halo)
        above[c] = sum(int(sizes[q]) for q in range(c, min(nplanes, c + halo))
                       if b[q] == b[c - 1] and z[q] - z[c - 1] <= halo)
    return below, above


def _balanced_cuts(starts: np.ndarray, pbz: np.ndarray, n: int, nranks: int, halo: int):
    """Plane cuts that even out the ranks' residual-block work, taken as
    owned + local rows (conv2 runs over the owned rows, conv1 and the operand
    preparation over owned and halo rows): the smallest bound C for which a
    greedy sweep (each rank takes planes while its work stays within C) gives
    every rank more than `halo` planes.  None when no cut is needed or found."""
    nplanes = len(starts)
    if nranks == 1:
        return [0, nplanes]
    below, above = _cut_halos(starts, pbz, n, halo)
    row_at = np.r_[starts, n].astype(np.int64)

    def work(s, e):
        rows = int(row_at[e] - row_at[s])
        return 2 * rows + (int(below[s]) if s > 0 else 0) + (int(above[e]) if e < nplanes else 0)

    def sweep(bound):
        cuts, s = [0], 0
        for r in range(nranks - 1):
            last = nplanes - (nranks - 1 - r) * (halo + 1)   # leave room for the ranks above
            best = -1
            for e in range(s + halo + 1, last + 1):
                if 2 * int(row_at[e] - row_at[s]) > bound:
                    break
                if work(s, e) <= bound:
                    best = e
            if best < 0:
                return None
            cuts.append(best)
            s = best
        if nplanes - s <= halo or work(s, nplanes) > bound:
            return None
        cuts.append(nplanes)
        return cuts

    lo, hi = 2 * n // nranks, 4 * n
    if sweep(hi) is None:
        return None
    while lo < hi:
        mid = (lo + hi) // 2
        if sweep(mid) is None:
            lo = mid + 1
        else:
            hi = mid
    return sweep(hi)


def _sort_keys(coords: np.ndarray) -> np.ndarray:
    from .synth import pack_keys
    return pack_keys(coords)


class SlabExchange:
    """Halo exchange of a rank's local feature rows ([n_local, C], row-major)
    with its z-neighbours over torch.distributed point-to-point (NCCL on
    GPUs, gloo on CPU).  Owned rows go out straight from the local array and
    halos land in place: the boundary planes are contiguous row ranges in
    both layouts."""

    def __init__(self, part: SlabPart, world: int, group=None):
        self.p = part
        self.world = world
        self.group = group

    def exchange(self, x) -> None:
        import torch.distributed as dist
        p, r = self.p, self.p.rank
        own = p.n_owned
        nlo, nhi = len(p.halo_lo), len(p.halo_hi)
        ops = []
        if r > 0:
            if p.send_lo:
                ops.append(dist.P2POp(dist.isend, x[:p.send_lo], r - 1, self.group))
            if nlo:
                ops.append(dist.P2POp(dist.irecv, x[own:own + nlo], r - 1, self.group))
        if r < self.world - 1:
            if p.send_hi:
                ops.append(dist.P2POp(dist.isend, x[own - p.send_hi:own], r + 1, self.group))
            if nhi:
                ops.append(dist.P2POp(dist.irecv, x[own + nlo:own + nlo + nhi], r + 1, self.group))
        if ops:
            for req in dist.batch_isend_irecv(ops):
                req.wait()


class PeerSlab:
    """One rank's shard on the fused-exchange path (``msc_slab_*``): the
    residual blocks run over the local rows and each block's second conv
    writes the boundary rows straight into the neighbours' halo rows (CUDA
    IPC memory over NVLink); no collective call per block.  The handles of
    the two feature buffers are exchanged once, here, with an all-gather over
    ``torch.distributed``."""

    def __init__(self, ex, part: SlabPart, world: int, channels: int = 128, group=None):
        import ctypes as C
        from . import lib as L
        self.ex, self.lib, self.p, self.world, self.c = ex, ex.lib, part, world, channels
        d = L.SlabDesc(part.rank, world, channels, part.n_local, part.n_owned, len(part.halo_lo), len(part.halo_hi),
                       part.send_lo, part.send_hi)
        h = C.c_void_p()
        L.check(self.lib.msc_slab_create(ex.ctx, C.byref(d), C.byref(h)))
        self.h = h
        buf = C.create_string_buffer(L.SLAB_HANDLE_BYTES)
        L.check(self.lib.msc_slab_get_handle(self.h, buf))
        mine = buf.raw
        if world > 1:
            import torch.distributed as dist
            allh = [None] * world
            dist.all_gather_object(allh, mine, group=group)
        else:
            allh = [mine]
        r = part.rank
        lower = C.create_string_buffer(allh[r - 1], L.SLAB_HANDLE_BYTES) if r > 0 else None
        upper = C.create_string_buffer(allh[r + 1], L.SLAB_HANDLE_BYTES) if r < world - 1 else None
        L.check(self.lib.msc_slab_connect(self.h, lower, upper))

    def _stream(self):
        import ctypes as C
        import torch
        return C.c_void_p(torch.cuda.current_stream().cuda_stream)

    def set_level(self, coords) -> None:
        import ctypes as C
        from . import lib as L
        L.check(self.lib.msc_slab_set_level(self.h, C.c_void_p(coords.data_ptr()), self._stream()))

    def put_features(self, x) -> None:
        import ctypes as C
        from . import lib as L
        L.check(self.lib.msc_slab_put_features(self.h, C.c_void_p(x.data_ptr()), self._stream()))

    def get_features(self, out) -> None:
        """The owned rows of the current features into out [n_owned, C]."""
        import ctypes as C
        from . import lib as L
        L.check(self.lib.msc_slab_get_features(self.h, C.c_void_p(out.data_ptr()), self._stream()))

    def res_block(self, blk: dict) -> None:
        import ctypes as C
        from . import lib as L
        p = lambda t: None if t is None else C.c_void_p(t.data_ptr())
        L.check(self.lib.msc_slab_res_block(self.h, p(blk.get("norm_w")), p(blk.get("norm_b")), p(blk["w1"].blob),
                                            p(blk.get("b1")), p(blk["w2"].blob), p(blk.get("b2")), self._stream()))

    def close(self):
        if self.h:
            self.lib.msc_slab_destroy(self.h)
            self.h = None

"""z-slab partition of one sparse voxel set across ranks, with halo exchange.

The reference is single-device; this is the multi-GPU layout of the same
SubM conv. Voxels are cut into P slabs along coordinate column 3 (z) with
about equal voxel counts. Rank r owns the voxels with z in [z_lo, z_hi) and
keeps, after them, the halo: the neighbours' voxels in the `depth` planes
below z_lo and above z_hi - 1 (depth = dilation * (kernel // 2); 1 for the
3^3 decoder convs). A conv on (own + halo) rows with outputs for own rows
only (t2sc_coords_create_halo) equals the global conv restricted to the
rank's rows, because every neighbour of an own row is own or halo.

Local row order, chosen so that every exchange is a contiguous slice and
the rows that need no halo come first:
    [interior | own rows in the low boundary planes | own rows in the high
     boundary planes | halo from below | halo from above]
Own rows keep their global (lexicographic) order inside each group. A layer
can then convolve the interior rows (targets [0, n_int)) while the halo is
in flight, and the boundary rows (targets [n_int, n_own)) after it lands.
"""
import numpy as np


class Slab:
    """One rank's share: index arrays into the global row order."""

    def __init__(self, rank, world, z_lo, z_hi, own, lo_send, hi_send, halo_lo, halo_hi):
        self.rank, self.world, self.z_lo, self.z_hi = rank, world, z_lo, z_hi
        self.own = own            # global rows, local order (interior, boundary-low, boundary-high)
        self.lo_send = lo_send    # slice of own rows sent to rank - 1
        self.hi_send = hi_send    # slice of own rows sent to rank + 1
        self.halo_lo = halo_lo    # global rows received from rank - 1 (its hi_send, same order)
        self.halo_hi = halo_hi    # global rows received from rank + 1 (its lo_send, same order)
        self.n_int = lo_send.start if lo_send.stop > lo_send.start else (
            hi_send.start if hi_send.stop > hi_send.start else len(own))  # interior rows come first

    @property
    def n_own(self):
        return len(self.own)

    @property
    def rows(self):
        """Global row of every local row (own, then halo)."""
        return np.concatenate([self.own, self.halo_lo, self.halo_hi])


def z_cuts(z, world, min_planes):
    """Cut points z_0 < ... < z_P so that slabs hold about equal voxel counts
    (prefix sum of the z histogram) and every slab spans >= min_planes planes."""
    zmin, zmax = int(z.min()), int(z.max()) + 1
    if zmax - zmin < world * min_planes:
        raise ValueError(f"{zmax - zmin} z planes cannot give {world} slabs of >= {min_planes} planes")
    hist = np.bincount(z - zmin, minlength=zmax - zmin)
    cum = np.concatenate([[0], np.cumsum(hist)])
    cuts = [zmin]
    for r in range(1, world):
        i = int(np.searchsorted(cum, cum[-1] * r / world))
        i = max(i, cuts[-1] - zmin + min_planes)            # this slab thick enough
        i = min(i, (zmax - zmin) - (world - r) * min_planes)  # room for the rest
        cuts.append(zmin + i)
    cuts.append(zmax)
    return cuts


def partition(coords, world, depth=1):
    """Slabs for every rank (all ranks compute the same partition). Every
    slab spans at least 2*depth planes, so its low and high boundary bands
    are disjoint."""
    coords = np.asarray(coords)
    z = coords[:, 3].astype(np.int64)
    n = len(coords)
    e = np.zeros(0, np.int64)
    if world == 1:
        return [Slab(0, 1, 0, 0, np.arange(n), slice(0, 0), slice(0, 0), e, e)]
    cuts = z_cuts(z, world, 2 * depth)
    parts = []
    for r in range(world):
        lo, hi = cuts[r], cuts[r + 1]
        rows = np.nonzero((z >= lo) & (z < hi))[0]
        zr = z[rows]
        in_lo = (zr < lo + depth) if r > 0 else np.zeros(len(rows), bool)
        in_hi = (zr >= hi - depth) if r < world - 1 else np.zeros(len(rows), bool)
        interior = rows[~in_lo & ~in_hi]
        own = np.concatenate([interior, rows[in_lo], rows[in_hi]])
        n_int, n_lo, n_hi = len(interior), int(in_lo.sum()), int(in_hi.sum())
        parts.append((lo, hi, own, slice(n_int, n_int + n_lo), slice(n_int + n_lo, n_int + n_lo + n_hi)))
    slabs = []
    for r in range(world):
        lo, hi, own, lo_send, hi_send = parts[r]
        halo_lo = parts[r - 1][2][parts[r - 1][4]] if r > 0 else e
        halo_hi = parts[r + 1][2][parts[r + 1][3]] if r < world - 1 else e
        slabs.append(Slab(r, world, lo, hi, own, lo_send, hi_send, halo_lo, halo_hi))
    return slabs


def start_halo(feats, slab, dist):
    """Issue the halo exchange of `feats` (see exchange_halo) and return the
    pending work; wait on it before reading the halo rows."""
    n_own, nlo = slab.n_own, len(slab.halo_lo)
    r, w = slab.rank, slab.world
    ops = []
    if r > 0:
        ops.append(dist.P2POp(dist.isend, feats[slab.lo_send], r - 1))
        ops.append(dist.P2POp(dist.irecv, feats[n_own:n_own + nlo], r - 1))
    if r < w - 1:
        ops.append(dist.P2POp(dist.isend, feats[slab.hi_send], r + 1))
        ops.append(dist.P2POp(dist.irecv, feats[n_own + nlo:], r + 1))
    return dist.batch_isend_irecv(ops) if ops else []


def exchange_halo(feats, slab, dist):
    """Fill the halo rows of `feats` [n_own + n_halo, C] (a torch tensor on
    any backend torch.distributed supports) from the z-neighbours: rank r
    sends its low boundary rows to r - 1 and its high boundary rows to
    r + 1, as one grouped batch (ncclGroupStart/End under NCCL)."""
    for q in start_halo(feats, slab, dist):
        q.wait()


# ---- the same partition and exchange through the C ABI (what a Mojo host calls) ----

class NativeSlab:
    """One rank's slab computed by t2sc_partition_zslab: `rows` are global
    rows in local order (own: interior, low band, high band; then the halo
    from rank - 1 and from rank + 1) and `counts` the six group sizes the
    exchange entry point takes."""

    def __init__(self, coords, world, rank, depth=1):
        import ctypes

        from ._lib import check, lib
        coords = np.ascontiguousarray(coords, np.int32)
        self.counts = np.zeros(6, np.int64)
        p = coords.ctypes.data_as(ctypes.c_void_p)
        cp = self.counts.ctypes.data_as(ctypes.c_void_p)
        check(lib.t2sc_partition_zslab(p, len(coords), world, rank, depth, None, 0, cp))
        total = int(self.counts[0] + self.counts[4] + self.counts[5])
        self.rows = np.empty(total, np.int64)
        check(lib.t2sc_partition_zslab(p, len(coords), world, rank, depth,
                                       self.rows.ctypes.data_as(ctypes.c_void_p), total, cp))
        self.rank, self.world = rank, world
        self.n_own, self.n_int = int(self.counts[0]), int(self.counts[1])
        self.own = self.rows[:self.n_own]


class Comm:
    """A NCCL communicator owned by libt2sc (t2sc_comm_*): the per-layer halo
    exchange runs inside the library on the context's stream."""

    ID_BYTES = 128

    @staticmethod
    def unique_id():
        import ctypes

        from ._lib import check, lib
        buf = ctypes.create_string_buffer(Comm.ID_BYTES)
        check(lib.t2sc_comm_unique_id(buf))
        return buf.raw

    def __init__(self, ctx, uid, nranks, rank, timeout_ms=120000):
        import ctypes

        from ._lib import check, lib
        if len(uid) != Comm.ID_BYTES:
            raise ValueError("Comm: the unique id must be 128 bytes")
        self.ctx = ctx
        h = ctypes.c_void_p()
        check(lib.t2sc_comm_create(ctx.handle, ctypes.create_string_buffer(bytes(uid), Comm.ID_BYTES), nranks, rank,
                                   timeout_ms, ctypes.byref(h)), ctx.handle)
        self.handle = h

    def exchange(self, feats, counts):
        """Halo rows of the device tensor feats [own + halo, C] from the
        z-neighbours (asynchronous on the context's stream)."""
        import ctypes

        from ._lib import check, lib
        counts = np.ascontiguousarray(counts, np.int64)
        row_bytes = feats.shape[1] * feats.element_size()
        check(lib.t2sc_halo_exchange_device(self.handle, ctypes.c_void_p(feats.data_ptr()), row_bytes,
                                            counts.ctypes.data_as(ctypes.c_void_p)), self.ctx.handle)

    def wait(self, timeout_ms=60000):
        from ._lib import check, lib
        check(lib.t2sc_comm_wait(self.handle, timeout_ms), self.ctx.handle)

    def close(self):
        from ._lib import lib
        if getattr(self, "handle", None):
            lib.t2sc_comm_destroy(self.handle)
            self.handle = None

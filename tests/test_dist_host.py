"""Host logic of the z-slab partition (CPU): neighbourhoods are complete
on every rank, sends and receives line up, and the halo exchange moves the
right rows between world-size-2 and -3 gloo ranks."""
import os

import numpy as np
import pytest


def _local_map_matches_global(oracle, coords, slabs):
    src, tgt, kidx = oracle.neighbor_map(coords)
    glob = {}
    for s_, t_, k_ in zip(src, tgt, kidx):
        glob.setdefault(int(t_), set()).add((int(s_), int(k_)))
    for sl in slabs:
        rows = sl.rows
        ls, lt, lk = oracle.neighbor_map(coords[rows])
        loc = {}
        for s_, t_, k_ in zip(ls, lt, lk):
            if t_ < sl.n_own:
                loc.setdefault(int(rows[t_]), set()).add((int(rows[s_]), int(k_)))
        for g in sl.own:
            assert loc.get(int(g), set()) == glob.get(int(g), set())


@pytest.mark.parametrize("world", [2, 3, 8])
def test_partition_neighbourhoods_complete(t2sc, oracle, world):
    from t2sc import dist
    coords = t2sc.synth.shell(*t2sc.synth.SHELLS["cfg1"])
    slabs = dist.partition(coords, world)
    own = np.concatenate([s.own for s in slabs])
    assert np.array_equal(np.sort(own), np.arange(len(coords)))
    sizes = [s.n_own for s in slabs]
    assert max(sizes) < 1.5 * len(coords) / world
    for r, s in enumerate(slabs):
        if r > 0:
            assert np.array_equal(s.halo_lo, slabs[r - 1].own[slabs[r - 1].hi_send])
        if r < world - 1:
            assert np.array_equal(s.halo_hi, slabs[r + 1].own[slabs[r + 1].lo_send])
    _local_map_matches_global(oracle, coords, slabs)
    # interior rows (first n_int) have no neighbour among the halo rows
    for sl in slabs:
        rows = sl.rows
        ls, lt, lk = oracle.neighbor_map(coords[rows])
        assert not np.any((lt < sl.n_int) & (ls >= sl.n_own))


def test_partition_rejects_too_thin(t2sc):
    from t2sc import dist
    with pytest.raises(ValueError):
        dist.partition(t2sc.synth.blob(3), 2)


def _worker(rank, world, port, q):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [os.path.dirname(here), os.path.join(os.path.dirname(here), "trellis2-mojo_b200")]
    import torch
    import torch.distributed as tdist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    tdist.init_process_group("gloo", rank=rank, world_size=world)
    from t2sc import dist, synth
    coords = synth.shell(*synth.SHELLS["cfg1"])
    glob = torch.from_numpy(synth.normal(5, (len(coords), 6)))
    sl = dist.partition(coords, world)[rank]
    rows = torch.from_numpy(sl.rows)
    local = torch.zeros((len(rows), 6))
    local[:sl.n_own] = glob[rows[:sl.n_own]]
    dist.exchange_halo(local, sl, tdist)
    q.put((rank, bool(torch.equal(local, glob[rows]))))
    tdist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_halo_exchange_gloo(world):
    import multiprocessing as mp
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in ps:
        p.join(timeout=60)
    assert all(res[r] for r in range(world))


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_native_partition_matches_host_mirror(t2sc, world):
    """t2sc_partition_zslab (the C ABI a Mojo host calls) gives every rank
    the same rows, order and group sizes as the Python partition."""
    from t2sc import dist
    for name in ("cfg1", "cfg2"):
        coords = t2sc.synth.shell(*t2sc.synth.SHELLS[name])
        for r, sl in enumerate(dist.partition(coords, world)):
            ns = dist.NativeSlab(coords, world, r)
            assert np.array_equal(ns.rows, sl.rows)
            assert ns.n_own == sl.n_own and ns.n_int == sl.n_int
            assert ns.counts[2] == sl.lo_send.stop - sl.lo_send.start
            assert ns.counts[3] == sl.hi_send.stop - sl.hi_send.start
            assert ns.counts[4] == len(sl.halo_lo) and ns.counts[5] == len(sl.halo_hi)


def test_native_partition_rejects_bad_arguments(t2sc):
    import ctypes
    from t2sc import _lib
    coords = t2sc.synth.blob(3)
    counts = np.zeros(6, np.int64)
    p, cp = coords.ctypes.data_as(ctypes.c_void_p), counts.ctypes.data_as(ctypes.c_void_p)
    L = _lib.lib
    assert L.t2sc_partition_zslab(p, len(coords), 2, 2, 1, None, 0, cp) == _lib.ERR_INVALID   # rank >= world
    assert L.t2sc_partition_zslab(p, len(coords), 4, 0, 1, None, 0, cp) == _lib.ERR_INVALID   # 3 planes, 4 slabs
    rows = np.empty(1, np.int64)
    assert L.t2sc_partition_zslab(p, len(coords), 1, 0, 1, rows.ctypes.data_as(ctypes.c_void_p), 1,
                                  cp) == _lib.ERR_CAPACITY


def test_comm_rejects_bad_arguments(t2sc):
    import ctypes
    from t2sc import _lib
    L = _lib.lib
    out = ctypes.c_void_p()
    assert L.t2sc_comm_create(None, None, 2, 0, 1000, ctypes.byref(out)) == _lib.ERR_INVALID
    assert L.t2sc_halo_exchange_device(None, None, 128, None) == _lib.ERR_INVALID
    assert L.t2sc_comm_wait(None, 10) == _lib.ERR_INVALID
    assert L.t2sc_comm_unique_id(None) == _lib.ERR_INVALID

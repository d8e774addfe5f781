"""GPU coordinate hash + neighbour map + CSR, bit-exact against the oracle
(the order of trellis2_mojo/sparse/conv.mojo:56-96 and :117-147)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def check_map(t2sc, O, coords, kernel=(3, 3, 3), dil=1):
    c = t2sc.Coords(t2sc.Context.default(), coords)
    src, tgt, kidx = c.neighbor_map(kernel, dil)
    osrc, otgt, okidx = O.neighbor_map(coords, kernel, dil)
    assert np.array_equal(src, osrc) and np.array_equal(tgt, otgt) and np.array_equal(kidx, okidx)
    rs, ss, ks = c.csr(kernel, dil)
    ors, oss, oks = O.csr(len(coords), osrc, otgt, okidx)
    assert np.array_equal(rs, ors) and np.array_equal(ss, oss) and np.array_equal(ks, oks)
    return len(src)


@pytest.mark.parametrize("side,dil", [(3, 1), (6, 1), (15, 1), (15, 2), (23, 1)])
def test_blob_maps(t2sc, oracle, side, dil):
    e = check_map(t2sc, oracle, t2sc.synth.blob(side), dil=dil)
    if dil == 1:
        assert e == (3 * side - 2) ** 3


@pytest.mark.parametrize("cfg", ["cfg1", "cfg2", "cfg3_parent"])
def test_shell_maps(t2sc, oracle, cfg):
    check_map(t2sc, oracle, t2sc.synth.shell(*t2sc.synth.SHELLS[cfg]))


def test_cfg4_full_size_map(t2sc, oracle):
    coords = t2sc.synth.shell(*t2sc.synth.SHELLS["cfg4"])
    e = check_map(t2sc, oracle, coords)
    assert abs(e / len(coords) - 10.35) < 0.01


def test_edge_cases(t2sc, oracle):
    # single voxel
    check_map(t2sc, oracle, np.array([[0, 7, 7, 7]], np.int32))
    # duplicates (the last row wins, as a Dict overwrite) across two batches
    c = np.array([[0, 1, 1, 1], [0, 1, 1, 1], [0, 1, 1, 2], [1, 1, 1, 1], [1, 1, 2, 1], [1, 1, 2, 1]], np.int32)
    check_map(t2sc, oracle, c)
    # extremes of the packable range: probes past the edge alias exactly as
    # the reference's key arithmetic does
    c = np.array([[0, -512, -512, -512], [0, 1535, 1535, 1535], [0, -512, -511, 1535], [0, -512, -512, 1535],
                  [2, 0, 0, 0]], np.int32)
    check_map(t2sc, oracle, c)
    # non-cubic and 1x1x1 kernels
    coords = t2sc.synth.blob(5)
    check_map(t2sc, oracle, coords, kernel=(1, 1, 1))
    check_map(t2sc, oracle, coords, kernel=(3, 1, 3), dil=2)
    check_map(t2sc, oracle, coords, kernel=(2, 2, 2))


def test_empty_coords(t2sc):
    c = t2sc.Coords(t2sc.Context.default(), np.zeros((0, 4), np.int32))
    src, tgt, kidx = c.neighbor_map()
    assert len(src) == 0
    rs, _, _ = c.csr()
    assert rs.tolist() == [0]


def test_out_of_range_rejected(t2sc):
    with pytest.raises(t2sc.T2SCError) as ei:
        t2sc.Coords(t2sc.Context.default(), np.array([[0, 1536, 0, 0]], np.int32))
    assert ei.value.code == 4
    with pytest.raises(t2sc.T2SCError):
        t2sc.Coords(t2sc.Context.default(), np.array([[-1, 0, 0, 0]], np.int32))
    # the context is still usable afterwards
    check = t2sc.Coords(t2sc.Context.default(), np.array([[0, 1, 1, 1]], np.int32))
    assert check.build_map() == 1

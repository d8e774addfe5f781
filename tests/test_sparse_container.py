"""The SparseTensor host container against the hand-computed expectations of
the reference's own tests (tests/parity/test_sparse_basic.mojo:28-44
make_sparse, :149-171 layout and contiguity, :229-243 replace shares the
spatial cache). No GPU needed: the container's checks run on the host."""
import numpy as np
import pytest


def _make_sparse(t2sc):
    # test_sparse_basic.mojo:28-44: 2 batches in a 2x2x2 grid, C = 2
    feats = np.arange(1, 11, dtype=np.float32).reshape(5, 2)
    coords = np.array([[0, 0, 0, 0], [0, 1, 0, 1], [1, 0, 1, 0], [1, 1, 1, 1], [1, 1, 0, 0]], np.int32)
    return t2sc.SparseTensor(feats, coords)


def test_layout_from_coords(t2sc):
    x = _make_sparse(t2sc)
    assert x.batch_size == 2
    assert x.seqlen(0) == 2 and x.seqlen(1) == 3
    assert x.spatial_shape() == [2, 2, 2]
    bm = x.batch_broadcast_map()
    assert bm[0] == 0 and bm[1] == 0 and bm[2] == 1 and bm[4] == 1
    assert x.offsets.tolist() == [0, 2, 5]


def test_contiguity_enforced(t2sc):
    coords = np.zeros((2, 4), np.int32)
    coords[0, 0] = 1  # batch 1 before batch 0 -> must raise
    with pytest.raises(ValueError):
        t2sc.SparseTensor(np.zeros((2, 1), np.float32), coords)


def test_replace_shares_cache(t2sc):
    x = _make_sparse(t2sc)
    x._cache["test_entry"] = [4, 4, 4]
    y = x.replace(x.feats + 1.0)
    assert y._cache.get("test_entry") == [4, 4, 4]
    y._cache["from_child"] = [4, 4, 4]
    assert "from_child" in x._cache  # writes on the derived tensor are visible on the parent
    assert np.array_equal(y.coords, x.coords) and y.feats[0, 0] == 2.0

"""GPU subdivision (child coordinates + mask compaction + feature rows)
bit-exact against the oracle (trellis2_mojo/sparse/spatial/basic.mojo:144-174,
spatial/spatial2channel.mojo:97-145, sparse_unet_vae.mojo:30-37)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_upsample_cfg3(t2sc, oracle):
    S = t2sc.synth
    coords = S.shell(*S.SHELLS["cfg3_parent"])
    n = len(coords)
    x = S.normal(1, (n, 128))
    mask = S.bernoulli(2, (n, 8))
    out = t2sc.SparseUpsample(2).forward_subdivision(t2sc.SparseTensor(x, coords), mask)
    idx, sidx, nc = oracle.subdivide(coords, mask)
    assert np.array_equal(out.coords, nc)
    assert np.array_equal(out.parent_idx, idx) and np.array_equal(out.subidx, sidx)
    assert np.array_equal(out.feats, oracle.select_rows(x, idx))
    assert abs(len(nc) / n - 4.0) < 0.05


@pytest.mark.parametrize("c", [2, 3, 8, 32])
def test_channel2spatial(t2sc, oracle, c):
    S = t2sc.synth
    coords = S.shell(*S.SHELLS["cfg1"])
    n = len(coords)
    x = S.normal(3, (n, 8 * c))
    mask = S.normal(4, (n, 8))  # signed values: != 0 keeps all, > 0 keeps about half
    out = t2sc.SparseChannel2Spatial(2).forward_subdivision(t2sc.SparseTensor(x, coords), mask)
    idx, sidx, nc = oracle.subdivide(coords, mask)
    assert np.array_equal(out.coords, nc) and np.array_equal(out.feats, oracle.c2s_unfold(x, idx, sidx))
    out = t2sc.SparseChannel2Spatial(2).forward_subdivision(t2sc.SparseTensor(x, coords), t2sc.binarize(mask))
    idx, sidx, nc = oracle.subdivide(coords, mask, positive=True)
    assert np.array_equal(out.coords, nc) and np.array_equal(out.feats, oracle.c2s_unfold(x, idx, sidx))


def test_edge_cases(t2sc, oracle):
    S = t2sc.synth
    coords = S.blob(3)
    x = S.normal(5, (27, 4))
    up = t2sc.SparseUpsample(2)
    out = up.forward_subdivision(t2sc.SparseTensor(x, coords), np.zeros((27, 8), np.float32))
    assert len(out.coords) == 0
    out = up.forward_subdivision(t2sc.SparseTensor(x, coords), np.ones((27, 8), np.float32))
    idx, sidx, nc = oracle.subdivide(coords, np.ones((27, 8), np.float32))
    assert len(out.coords) == 216 and np.array_equal(out.coords, nc)
    # two batches, negative coordinates
    c2 = np.array([[0, -3, 0, 5], [1, 2, -7, 1]], np.int32)
    m2 = np.array([[0, 1, 0, 0, 0, 0, 1, 0], [1, 0, 0, 0, 0, 0, 0, 1]], np.float32)
    out = up.forward_subdivision(t2sc.SparseTensor(np.ones((2, 3), np.float32), c2), m2)
    assert np.array_equal(out.coords, oracle.subdivide(c2, m2)[2])


def test_subdivide_then_conv_cfg3(t2sc, oracle):
    """cfg3: parents (C=128) -> subdivide + Bernoulli(0.5) -> 2 x (SubM 128->128 + SiLU), f32."""
    from _cases import F32_TOL, conv_inputs, oracle_conv, rel_err
    S = t2sc.synth
    coords = S.shell(64, 24.0, 0.9)  # a smaller parent shell keeps the oracle fast
    n = len(coords)
    x = S.normal(10, (n, 128))
    mask = S.bernoulli(11, (n, 8))
    up = t2sc.SparseUpsample(2).forward_subdivision(t2sc.SparseTensor(x, coords), mask)
    _, w1, b1 = conv_inputs(S, 1, 128, 128, seed=12)
    _, w2, b2 = conv_inputs(S, 1, 128, 128, seed=13)
    c1, c2 = t2sc.SparseConv3d(w1, b1), t2sc.SparseConv3d(w2, b2)
    y = c2.forward(c1.forward(up, silu=True), silu=True).feats
    idx, sidx, nc = oracle.subdivide(coords, mask)
    xu = oracle.select_rows(x, idx)
    edges = oracle.neighbor_map(nc)
    h = oracle_conv(oracle, nc, xu, w1, b1, silu=True, edges=edges)
    ref = oracle_conv(oracle, nc, h, w2, b2, silu=True, edges=edges)
    assert rel_err(y, ref) <= F32_TOL

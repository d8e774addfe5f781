"""Pipeline glue on the GPU against the oracle: fdg_head
(models/sc_vaes/fdg_vae.mojo:17-50), cascade_coords
(pipelines/image_to_3d.mojo:219-270) and grid_sample_trilinear
(meshing/vertex_attrs.mojo:46-104).

Tolerances: cascade coordinates and the intersected mask are bit-exact;
the sampler's f32 arithmetic is written out in the reference's order, so it
is compared at 2 ulp-scale (rtol 1e-6, atol 1e-6); fdg_head's exp/log
differ from libm's by a few ulp (rtol 2e-6, atol 2e-6)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _feats(t2sc, seed, shape, std=1.0):
    return t2sc.synth.normal(seed, shape, std)


def test_fdg_head_matches_oracle(t2sc, oracle):
    S = t2sc.synth
    coords = S.shell(*S.SHELLS["cfg1"])
    f = _feats(t2sc, 40, (len(coords), 7), 8.0)
    f[:5, 6] = [20.0, 20.5, -80.0, 19.99, 0.0]  # softplus branch edges
    f[:3, 3] = [0.0, -0.0, 1e-30]  # > 0 is strict
    h = t2sc.SparseTensor(f, coords)
    v, i, q = t2sc.fdg_head(h, 0.5)
    ov, oi, oq = oracle.fdg_head(f, 0.5)
    assert np.array_equal(i.feats, oi)
    np.testing.assert_allclose(v.feats, ov, rtol=2e-6, atol=2e-6)
    np.testing.assert_allclose(q.feats, oq, rtol=2e-6, atol=2e-6)
    assert np.array_equal(v.coords, coords)
    v2, _, _ = t2sc.fdg_head(h, 0.25)
    np.testing.assert_allclose(v2.feats, oracle.fdg_head(f, 0.25)[0], rtol=2e-6, atol=2e-6)


def test_fdg_head_empty_and_bad_shape(t2sc):
    import torch
    v, i, q = t2sc.fdg_head_device(torch.empty((0, 7), device="cuda"))
    assert v.shape == (0, 3) and i.shape == (0, 3) and q.shape == (0, 1)
    with pytest.raises(ValueError):
        t2sc.fdg_head_device(torch.zeros((4, 6), device="cuda"))


def _upsampled_512(t2sc):
    """Coordinates at resolution 512 as upsample_coords returns them: the
    cfg4 shell (503,562 voxels) in two batches (the second shifted)."""
    S = t2sc.synth
    c = S.shell(*S.SHELLS["cfg4"])
    c2 = c.copy()
    c2[:, 0] = 1
    c2[:, 1:] = (c2[:, 1:] + 37) % 512
    return np.concatenate([c, c2])


def test_cascade_coords_full_size(t2sc, oracle):
    hr = _upsampled_512(t2sc)
    got, res = t2sc.cascade_coords(hr, 512, 1024, 49152)
    want, wres = oracle.cascade_coords(hr, 512, 1024, 49152)
    assert res == wres == 1024
    assert np.array_equal(got, want)
    assert 0 < len(got) < len(hr)


@pytest.mark.parametrize("resolution,budget", [(1536, 30000), (1536, 1), (1408, 60000), (2048, 20000)])
def test_cascade_coords_token_budget(t2sc, oracle, resolution, budget):
    hr = _upsampled_512(t2sc)
    got, res = t2sc.cascade_coords(hr, 512, resolution, budget)
    want, wres = oracle.cascade_coords(hr, 512, resolution, budget)
    assert res == wres
    assert np.array_equal(got, want)


def test_cascade_coords_edges(t2sc, oracle):
    from t2sc import _lib
    # duplicates collapse, rows come back sorted
    hr = np.array([[0, 5, 5, 5], [0, 5, 5, 4], [0, 0, 0, 0], [1, 0, 0, 0], [0, 5, 5, 5]], np.int32)
    got, res = t2sc.cascade_coords(hr, 8, 1024, 100)
    want, _ = oracle.cascade_coords(hr, 8, 1024, 100)
    assert np.array_equal(got, want) and res == 1024
    got, _ = t2sc.cascade_coords(np.zeros((0, 4), np.int32), 512, 1024, 10)
    assert got.shape == (0, 4)
    ctx = t2sc.Context.default(0)
    with pytest.raises(_lib.T2SCError):
        t2sc.cascade_coords(np.array([[0, -1, 0, 0]], np.int32), 512, 1024, 10)
    with pytest.raises(_lib.T2SCError):
        t2sc.cascade_coords(hr, 512, 1024, 0)
    # a budget below 1024 that is never met: the reference would not stop
    with pytest.raises(_lib.T2SCError):
        t2sc.cascade_coords(hr, 8, 100, 1)
    # the context stays usable
    got, _ = t2sc.cascade_coords(hr, 8, 1024, 100)
    assert np.array_equal(got, want)
    ctx.synchronize()


def _queries(rng, l, grid):
    q = rng.uniform(-1.5, grid + 1.5, size=(l, 3)).astype(np.float32)
    q[: l // 4] = np.round(q[: l // 4] * 2) / 2  # exact half-voxel positions
    q[l // 4: l // 4 + 64] = rng.uniform(0, 0.5, size=(64, 3))  # p < 0.5: a neighbour counted twice
    return q


def test_grid_sample_small(t2sc, oracle):
    S = t2sc.synth
    c = S.shell(*S.SHELLS["cfg1"])
    xyz = np.ascontiguousarray(c[:, 1:])
    xyz = np.concatenate([xyz, xyz[:7]])  # repeated voxels: the last row wins
    feats = _feats(t2sc, 41, (len(xyz), 6))
    grid = int(xyz.max()) + 1
    rng = np.random.default_rng(0)
    # queries near the occupied voxels and anywhere in (and outside) the grid
    near = (xyz[rng.integers(0, len(xyz), 20000)] + rng.uniform(-1, 2, size=(20000, 3))).astype(np.float32)
    q = np.concatenate([near, _queries(rng, 20000, grid)])
    got = t2sc.grid_sample_trilinear(feats, xyz, grid, q)
    want = oracle.grid_sample_trilinear(feats, xyz, grid, q)
    np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-6)
    assert np.count_nonzero(np.abs(want).sum(1)) > 15000


def test_grid_sample_full_size(t2sc, oracle):
    """The cfg4 shell (503,562 voxels) sampled at 2M points, device form."""
    import torch
    S = t2sc.synth
    c = S.shell(*S.SHELLS["cfg4"])
    xyz = np.ascontiguousarray(c[:, 1:])
    feats = _feats(t2sc, 42, (len(xyz), 6))
    rng = np.random.default_rng(1)
    q = (xyz[rng.integers(0, len(xyz), 2_000_000)] + rng.uniform(-1, 2, size=(2_000_000, 3))).astype(np.float32)
    ctx = t2sc.Context.default(0)
    coords = t2sc.Coords(ctx, c)
    got = t2sc.grid_sample_trilinear_device(coords, torch.from_numpy(feats).cuda(), 512,
                                            torch.from_numpy(q).cuda()).cpu().numpy()
    want = oracle.grid_sample_trilinear(feats, xyz, 512, q)
    np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-6)


def test_grid_sample_rejects(t2sc):
    import torch
    from t2sc import _lib
    ctx = t2sc.Context.default(0)
    coords = t2sc.Coords(ctx, np.array([[0, 1, 1, 1]], np.int32))
    f = torch.zeros((1, 2), device="cuda")
    with pytest.raises(_lib.T2SCError):
        t2sc.grid_sample_trilinear_device(coords, f, 4096, torch.zeros((1, 3), device="cuda"))
    with pytest.raises(ValueError):
        t2sc.grid_sample_trilinear_device(coords, f, 4, torch.zeros((1, 3)))
    with pytest.raises(ValueError):
        t2sc.grid_sample_trilinear_device(coords, torch.zeros((2, 2), device="cuda"), 4,
                                          torch.zeros((1, 3), device="cuda"))
    out = t2sc.grid_sample_trilinear_device(coords, f + 3, 4, torch.tensor([[1.5, 1.5, 1.5]], device="cuda"))
    assert out.cpu().tolist() == [[3.0, 3.0]]

"""Every BASELINE configuration at its full size, GPU (through the C ABI)
against the oracle (sparse/conv.mojo:149-199, spatial/basic.mojo:144-174):

  cfg2  128^3 shell R=48 h=1.75 (101,422 voxels): SubM 256->256 -> SiLU ->
        SubM 256->256 + identity residual, f32 and f16-in / f32-acc;
  cfg3  51,982 parents at 128^3, C=128 -> subdivide with a Bernoulli(0.5)
        child mask -> 2 x (SubM 128->128 + SiLU), f32;
  cfg4  512^3 shell (503,562 voxels): all four SubM 64->64 + SiLU layers in
        bf16, intermediates rounded to bf16 between layers on both sides;
  cfg5  one shape (seed 0): subdivided 512^3 shell -> Bernoulli(0.5) ->
        ~2.0M voxels at 1024^3, 2 x (SubM 32->32 + SiLU) in bf16.

Child coordinates and neighbour maps bit-exact; features within max-rel-err
1e-4 (f32) / 1e-2 (16-bit)."""
import numpy as np
import pytest

from _cases import F16_TOL, F32_TOL, conv_inputs, oracle_chain, rel_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", ["f32", "f16", "f32_f16w"])
def test_cfg2_residual_block(t2sc, oracle, dtype):
    """f32_f16w: f32 activations with f16-exact weights, the reference's f16
    checkpoint storage (gpu/conv.mojo:32-36), passed to the f32 mode."""
    S = t2sc.synth
    coords = S.shell(*S.SHELLS["cfg2"])
    n, c = len(coords), 256
    assert n == 101422
    x, w1, b1 = conv_inputs(S, n, c, c, seed=200)
    _, w2, b2 = conv_inputs(S, 1, c, c, seed=210)
    if dtype == "f32_f16w":
        w1, w2 = (w.astype(np.float16).astype(np.float32) for w in (w1, w2))
        dtype = "f32"
    csr = oracle.csr(n, *oracle.neighbor_map(coords))
    convs = [t2sc.SparseConv3d(w1, b1, dtype=dtype), t2sc.SparseConv3d(w2, b2, dtype=dtype)]
    y = t2sc.conv_chain(convs, t2sc.SparseTensor(x, coords), [1, 2]).feats
    rm = None if dtype == "f32" else dtype
    ref = oracle_chain(oracle, n, x, [(w1, b1, True), (w2, b2, False)], csr, round_mode=rm, residual_last=x)
    assert rel_err(y, ref) <= (F32_TOL if dtype == "f32" else F16_TOL)


def test_cfg3_subdivide_then_two_convs(t2sc, oracle):
    S = t2sc.synth
    coords = S.shell(*S.SHELLS["cfg3_parent"])
    n = len(coords)
    assert n == 51982
    x = S.normal(300, (n, 128))
    mask = S.bernoulli(301, (n, 8))
    up = t2sc.SparseUpsample(2).forward_subdivision(t2sc.SparseTensor(x, coords), mask)
    idx, sidx, nc = oracle.subdivide(coords, mask)
    assert np.array_equal(up.coords, nc) and np.array_equal(up.parent_idx, idx)
    assert np.array_equal(up.feats, oracle.select_rows(x, idx))
    m = len(nc)
    _, w1, b1 = conv_inputs(S, 1, 128, 128, seed=310)
    _, w2, b2 = conv_inputs(S, 1, 128, 128, seed=320)
    c1, c2 = t2sc.SparseConv3d(w1, b1), t2sc.SparseConv3d(w2, b2)
    y = t2sc.conv_chain([c1, c2], up, [1, 1]).feats
    src, tgt, kidx = oracle.neighbor_map(nc)
    gs, gt, gk = up.device_coords.neighbor_map()
    assert np.array_equal(gs, src) and np.array_equal(gt, tgt) and np.array_equal(gk, kidx)
    ref = oracle_chain(oracle, m, up.feats, [(w1, b1, True), (w2, b2, True)], oracle.csr(m, src, tgt, kidx))
    assert rel_err(y, ref) <= F32_TOL


def test_cfg4_four_layers(t2sc, oracle):
    S = t2sc.synth
    coords = S.shell(*S.SHELLS["cfg4"])
    n = len(coords)
    assert n == 503562
    x = S.normal(400, (n, 64))
    layers = [(S.normal(401 + 3 * i, (64, 3, 3, 3, 64), std=(1.0 / (27 * 64)) ** 0.5),
               S.normal(402 + 3 * i, (64,), std=0.1), True) for i in range(4)]
    convs = [t2sc.SparseConv3d(w, b, dtype="bf16") for w, b, _ in layers]
    y = t2sc.conv_chain(convs, t2sc.SparseTensor(x, coords), [1] * 4).feats
    csr = oracle.csr(n, *oracle.neighbor_map(coords))
    ref = oracle_chain(oracle, n, x, layers, csr, round_mode="bf16")
    assert rel_err(y, ref) <= F16_TOL


def test_cfg5_one_shape(t2sc, oracle):
    S = t2sc.synth
    parents = S.shell(*S.SHELLS["cfg5_parent"], seed=0)
    npar = len(parents)
    mask = S.bernoulli(500, (npar, 8))
    x0 = S.normal(510, (npar, 32))
    up = t2sc.SparseUpsample(2).forward_subdivision(t2sc.SparseTensor(x0, parents), mask)
    idx, sidx, nc = oracle.subdivide(parents, mask)
    assert np.array_equal(up.coords, nc)
    m = len(nc)
    assert 1.9e6 < m < 2.2e6
    x = S.normal(520, (m, 32))
    layers = [(S.normal(521 + 3 * i, (32, 3, 3, 3, 32), std=(1.0 / (27 * 32)) ** 0.5),
               S.normal(522 + 3 * i, (32,), std=0.1), True) for i in range(2)]
    convs = [t2sc.SparseConv3d(w, b, dtype="bf16") for w, b, _ in layers]
    xt = up.replace(x)
    y = t2sc.conv_chain(convs, xt, [1, 1]).feats
    src, tgt, kidx = oracle.neighbor_map(nc)
    gs, gt, gk = xt.device_coords.neighbor_map()
    assert np.array_equal(gs, src) and np.array_equal(gt, tgt) and np.array_equal(gk, kidx)
    ref = oracle_chain(oracle, m, x, layers, oracle.csr(m, src, tgt, kidx), round_mode="bf16")
    assert rel_err(y, ref) <= F16_TOL

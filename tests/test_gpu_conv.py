"""GPU SubM conv vs the oracle (SparseConv3d.forward's CPU loop,
trellis2_mojo/sparse/conv.mojo:149-199), through the C ABI.

Bars: f32 mode max-rel-err <= 1e-4 (and the reference GPU test's absolute
atol 2e-4 / 5e-4 on its own cases); f16/bf16 modes max-rel-err <= 1e-2
against the oracle run on the 16-bit-rounded inputs and weights."""
import numpy as np
import pytest

from _cases import F16_TOL, F32_TOL, conv_inputs, oracle_conv, rel_err

pytestmark = pytest.mark.gpu


# the reference's Metal-vs-CPU cases, parity_wp11_gpu_conv.mojo:97-100
@pytest.mark.parametrize("side,ci,co,dil,seed,atol", [
    (15, 256, 256, 1, 41, 2e-4),
    (12, 128, 512, 1, 42, 2e-4),
    (12, 512, 256, 1, 43, 5e-4),
    (15, 256, 256, 2, 44, 2e-4),
])
def test_reference_blob_cases_f32(t2sc, oracle, side, ci, co, dil, seed, atol):
    S = t2sc.synth
    coords = S.blob(side)
    n = len(coords)
    x = S.lcg_fill((n, ci), seed, 1.0)
    w = S.lcg_fill((co, 3, 3, 3, ci), seed + 1, 0.05)
    b = S.lcg_fill((co,), seed + 2, 0.1)
    conv = t2sc.SparseConv3d(w, b, dilation=dil, dtype="f32")
    y = conv(t2sc.SparseTensor(x, coords)).feats
    ref = oracle_conv(oracle, coords, x, w, b, dil=dil)
    assert np.max(np.abs(y - ref)) <= atol
    assert rel_err(y, ref) <= F32_TOL


@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("ci,co", [(64, 64), (32, 32), (128, 128), (256, 256), (16, 48), (64, 512), (24, 40),
                                   (40, 64), (8, 16), (4, 16), (12, 32)])
def test_shell_modes(t2sc, oracle, dtype, ci, co):
    """Tile-shape coverage: 32/64/128-byte rows, partial Ci chunks, 1..4 Co
    tiles, and shapes that take the CUDA-core kernel (Co % 16 != 0, or Ci
    not a whole number of 16-byte vectors)."""
    S = t2sc.synth
    coords = S.shell(*S.SHELLS["cfg1"])
    x, w, b = conv_inputs(S, len(coords), ci, co, seed=100 + ci + co)
    conv = t2sc.SparseConv3d(w, b, dtype=dtype)
    y = conv(t2sc.SparseTensor(x, coords)).feats
    ref = oracle_conv(oracle, coords, x, w, b, round_mode=None if dtype == "f32" else dtype)
    assert rel_err(y, ref) <= (F32_TOL if dtype == "f32" else F16_TOL)


@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
def test_epilogue_flags(t2sc, oracle, dtype):
    S = t2sc.synth
    coords = S.shell(*S.SHELLS["cfg1"])
    x, w, b = conv_inputs(S, len(coords), 64, 64, seed=7)
    r = S.normal(99, (len(coords), 64))
    conv = t2sc.SparseConv3d(w, b, dtype=dtype)
    xt = t2sc.SparseTensor(x, coords)
    tol = F32_TOL if dtype == "f32" else F16_TOL
    rm = None if dtype == "f32" else dtype
    y = conv.forward(xt, silu=True).feats
    assert rel_err(y, oracle_conv(oracle, coords, x, w, b, silu=True, round_mode=rm)) <= tol
    y = conv.forward(xt, silu=True, residual=r).feats
    assert rel_err(y, oracle_conv(oracle, coords, x, w, b, silu=True, residual=r, round_mode=rm)) <= tol


def test_no_bias_and_dilation_16bit(t2sc, oracle):
    S = t2sc.synth
    coords = S.shell(*S.SHELLS["cfg1"])
    x, w, _ = conv_inputs(S, len(coords), 64, 64, seed=5)
    conv = t2sc.SparseConv3d(w, None, dilation=2, dtype="bf16")
    y = conv(t2sc.SparseTensor(x, coords)).feats
    ref = oracle_conv(oracle, coords, x, w, None, dil=2, round_mode="bf16")
    assert rel_err(y, ref) <= F16_TOL


def test_residual_block_chain(t2sc, oracle):
    """cfg2's block (conv -> SiLU -> conv + identity residual) on a smaller
    shell, f32 and f16-in/f32-acc, device-resident between the convs."""
    S = t2sc.synth
    coords = S.shell(64, 24.0, 1.75)
    n, c = len(coords), 128
    x, w1, b1 = conv_inputs(S, n, c, c, seed=21)
    _, w2, b2 = conv_inputs(S, n, c, c, seed=31)
    edges = oracle.neighbor_map(coords)
    for dtype, tol in (("f32", F32_TOL), ("f16", F16_TOL)):
        rm = None if dtype == "f32" else dtype
        convs = [t2sc.SparseConv3d(w1, b1, dtype=dtype), t2sc.SparseConv3d(w2, b2, dtype=dtype)]
        y = t2sc.conv_chain(convs, t2sc.SparseTensor(x, coords), [1, 2]).feats
        h = oracle_conv(oracle, coords, x, w1, b1, silu=True, round_mode=rm, edges=edges)
        if rm:
            h = oracle.round16(h, rm)
        ref = oracle_conv(oracle, coords, h, w2, b2, residual=x, round_mode=rm, edges=edges)
        assert rel_err(y, ref) <= tol, dtype


def test_cfg4_chain_sampled_rows(t2sc, oracle):
    """Full-size 512^3 shell, 4 x (SubM 64->64 + SiLU) in bf16: the first
    layer checked on 4096 sampled rows against the oracle, and the chain's
    output checked for finiteness and layer-by-layer consistency with the
    single-conv entry point."""
    S = t2sc.synth
    coords = S.shell(*S.SHELLS["cfg4"])
    n = len(coords)
    x, w, b = conv_inputs(S, n, 64, 64, seed=400)
    conv = t2sc.SparseConv3d(w, b, dtype="bf16")
    xt = t2sc.SparseTensor(x, coords)
    y1 = conv.forward(xt, silu=True).feats
    src, tgt, kidx = oracle.neighbor_map(coords)
    rows = np.random.default_rng(0).choice(n, 4096, replace=False)
    xr, wr = oracle.round16(x, "bf16").astype(np.float64), oracle.round16(w, "bf16").astype(np.float64)
    wk = wr.reshape(64, 27, 64)
    sel = np.isin(tgt, rows)
    ref = np.zeros((n, 64))
    for k in range(27):
        m = sel & (kidx == k)
        np.add.at(ref, tgt[m], xr[src[m]] @ wk[:, k, :].T)
    ref = ref[rows] + b
    ref = ref / (1 + np.exp(-ref))
    assert rel_err(y1[rows], ref) <= F16_TOL
    y4 = t2sc.conv_chain([conv] * 4, xt, [1] * 4).feats
    assert np.all(np.isfinite(y4))
    h = xt
    for _ in range(4):
        h = conv.forward(h, silu=True)
    assert np.array_equal(h.feats, y4)

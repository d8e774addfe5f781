"""The decoder's up block SparseResBlockC2S3d (sparse_unet_vae.mojo:67-133)
as one device call against the oracle's composition of the restated
pieces (oracle.c2s_block): child coordinates bit-exact, features within the
f32 bar (max-rel-err 1e-4), the predicted subdivision within 1e-4."""
import numpy as np
import pytest

from _cases import F32_TOL, rel_err

pytestmark = pytest.mark.gpu


def _weights(S, c, co, seed):
    norm1 = (1.0 + 0.1 * S.normal(seed, (c,)), 0.1 * S.normal(seed + 1, (c,)))
    conv1 = (S.normal(seed + 2, (8 * co, 3, 3, 3, c), std=(1.0 / (27 * c)) ** 0.5), S.normal(seed + 3, (8 * co,), std=0.1))
    conv2 = (S.normal(seed + 4, (co, 3, 3, 3, co), std=(1.0 / (27 * co)) ** 0.5), S.normal(seed + 5, (co,), std=0.1))
    to_sub = (S.normal(seed + 6, (8, c), std=(1.0 / c) ** 0.5), S.normal(seed + 7, (8,), std=0.1))
    return norm1, conv1, conv2, to_sub


@pytest.mark.parametrize("c,co", [(64, 32), (128, 64), (32, 16)])
def test_c2s_block_pred_subdiv_f32(t2sc, oracle, c, co):
    S = t2sc.synth
    coords = S.shell(*S.SHELLS["cfg1"])
    x = S.normal(700 + c, (len(coords), c))
    norm1, conv1, conv2, to_sub = _weights(S, c, co, 710 + c)
    blk = t2sc.SparseResBlockC2S3d(c, co, True, norm1, conv1, conv2, to_sub)
    h, sub = blk.forward(t2sc.SparseTensor(x, coords))
    nc, ref, ref_sub = oracle.c2s_block(coords, x, norm1, conv1, conv2, co, to_subdiv=to_sub)
    assert rel_err(sub, ref_sub) <= F32_TOL
    assert np.array_equal(h.coords, nc)
    assert rel_err(h.feats, ref) <= F32_TOL


def test_c2s_block_guided_and_16bit(t2sc, oracle):
    """forward_guided with a given subdivision (the texture decoder's path),
    in f32 and bf16 (inputs and weights rounded to bf16 on the oracle side)."""
    S = t2sc.synth
    coords = S.shell(*S.SHELLS["cfg1"])
    c, co = 64, 32
    x = S.normal(801, (len(coords), c))
    sub = S.normal(802, (len(coords), 8))
    norm1, conv1, conv2, _ = _weights(S, c, co, 810)
    blk = t2sc.SparseResBlockC2S3d(c, co, False, norm1, conv1, conv2)
    h = blk.forward_guided(t2sc.SparseTensor(x, coords), sub)
    nc, ref, _ = oracle.c2s_block(coords, x, norm1, conv1, conv2, co, subdiv=sub)
    assert np.array_equal(h.coords, nc) and rel_err(h.feats, ref) <= F32_TOL
    blk16 = t2sc.SparseResBlockC2S3d(c, co, False, norm1, conv1, conv2, dtype="bf16")
    h16 = blk16.forward_guided(t2sc.SparseTensor(x, coords), sub)
    assert np.array_equal(h16.coords, nc)
    assert rel_err(h16.feats, ref) <= 3e-2   # three 16-bit roundings of intermediates between f32 stages


def test_c2s_block_rejects_bad_shapes(t2sc):
    S = t2sc.synth
    norm1, conv1, conv2, to_sub = _weights(S, 64, 32, 900)
    with pytest.raises(t2sc.T2SCError):
        t2sc.SparseResBlockC2S3d(60, 32, True, (norm1[0][:60], norm1[1][:60]), conv1, conv2, to_sub)
    with pytest.raises(ValueError):
        t2sc.SparseResBlockC2S3d(64, 32, True, norm1, conv1, conv2, None)


def test_convnext_block_entry_point_f32(t2sc, oracle):
    """SparseConvNeXtBlock3d as one device call (conv -> LN -> lin1/SiLU ->
    lin2 + x) against oracle.convnext_block."""
    import torch
    S = t2sc.synth
    coords = S.shell(*S.SHELLS["cfg1"])
    c = 64
    x = S.normal(990, (len(coords), c))
    conv = (S.normal(991, (c, 3, 3, 3, c), std=(27 * c) ** -0.5), S.normal(992, (c,), std=0.1))
    norm = (1 + 0.1 * S.normal(993, (c,)), 0.1 * S.normal(994, (c,)))
    lin1 = (S.normal(995, (4 * c, c), std=c ** -0.5), S.normal(996, (4 * c,), std=0.1))
    lin2 = (S.normal(997, (c, 4 * c), std=(4 * c) ** -0.5), S.normal(998, (c,), std=0.1))
    blk = t2sc.SparseConvNeXtBlock3d(c, conv, norm, lin1, lin2)
    xt = t2sc.SparseTensor(x, coords)
    y = blk.forward_device(xt.device_coords, torch.from_numpy(x).cuda()).cpu().numpy()
    assert rel_err(y, oracle.convnext_block(coords, x, conv, norm, lin1, lin2)) <= F32_TOL
